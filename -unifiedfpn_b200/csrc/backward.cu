// Backward pass of the FPN neck's hot path (the training consumer of the same kernels).
//
// Reference: src/training/backward/lateral_conv_backward.cu:7-143 (1x1 lateral: grad input,
// grad weights, grad bias) and src/training/backward/upsample_backward.cu:4-80 (upsample-add:
// grad lateral = grad out, grad coarse = bilinear transpose of grad out).  The reference's
// kernels scatter with atomics (nondeterministic) and its upsample backward samples the
// coarse map without the forward's clamp of the source coordinate to [0, in-1] (so it is not
// the adjoint of its forward at the borders); everything here is the exact adjoint of this
// library's forward, computed deterministically:
//
//   * weight gradients, dW[o][tap][c] = sum_p dY[p][o] X[p + tap][c] (1x1: one tap; 3x3: the
//     nine taps of pad-1), are a tensor-core GEMM over pixels: fpn_dw_gemm_kernel, all 256
//     output channels (two M = 128 accumulators filling TMEM) x N = 256 input channels per CTA,
//     K = 64-pixel k-blocks fetched by TMA
//     as (64 channels x 64 pixels) boxes of the NHWC maps -- for both operands the channels
//     are contiguous, i.e. MN-major operands, read through MN-major 128-byte-swizzle
//     descriptors; the 3x3 taps shift the X box (TMA zero-fills outside the image = pad 1).
//     The pixel range is split over CTAs (split-K); each CTA writes its fp32 partial and
//     reduce_partials_kernel / reduce_partials_taps9_kernel add the partials in a fixed order.
//   * bias gradients: column sums of dY in fp32, per block then in a fixed order.
//   * input gradients reuse the forward kernels: the 1x1 lateral with the transposed weights
//     (one 256-channel slice of dX per launch) and the 3x3 with the weights transposed in
//     channels and flipped in space (dX = conv3x3(dY, W'), W'[c][8 - t][o] = W[o][t][c]).
//   * the top-down add's adjoint, upsample_adjoint_kernel, gathers for every coarse pixel the
//     bilinear weights of the fine pixels that tapped it (the forward's clamped taps), and P6's
//     adjoint adds dP6 into dP5's even pixels.
#include "kernels.h"
#include "tc_gemm.cuh"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>

namespace ufpn {

namespace {

// ------------------------------------------------------------------ weight gradient GEMM
constexpr int kDwStages = 3;
constexpr int kDwChunk = 64 * 128;         // one 64-channel x 64-pixel box, 16-bit: 8 KB
constexpr int kDwAStage = 4 * kDwChunk;    // 256 output channels (two M = 128 operands)
constexpr int kDwStaging = 32 * 128;       // epilogue: one 32 x 32 fp32 block (4 KB)
constexpr int kDwBStage = 4 * kDwChunk;    // 256 input channels
constexpr int kDwOffB = kDwStages * kDwAStage;
constexpr int kDwOffBars = kDwOffB + kDwStages * kDwBStage;
constexpr int kDwSmemBytes = kDwOffBars + 256 + 1024;
static_assert(kDwSmemBytes <= 232448, "dW smem");
static_assert(8 * 2 * kDwStaging <= kDwStages * kDwAStage, "epilogue staging reuses the A stages");
constexpr int kDevTimeoutDw = 0x106;

struct DwArgs {
  int tiles_x, tiles_y, N_img, kw, kh;  // 64-pixel k-blocks: kw x kh boxes over (W, H, N)
  int num_kb, per_kb, ksplit;
  int c_blocks, taps;
  int Cin;
  float* partial;  // [ksplit][taps][256][Cin]
  // bias gradient partials [ksplit][taps][256] (null: none): the idle epilogue warps of the
  // channel-block-0 CTAs also sum dY (plain loads of g, NHWC [N][H][W][256], mostly L2 hits
  // behind the operand TMA), the CTA of tap t over every taps-th k-block of its range from t
  float* db_partial;
  const void* g;
  int H, W;
  int* status;
};
constexpr int kDwEpiWarps = 8;  // warps 2..9

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_dw_gemm_kernel(const __grid_constant__ CUtensorMap map_g,
                       const __grid_constant__ CUtensorMap map_x,
                       const __grid_constant__ CUtensorMap map_p, const DwArgs a) {
  constexpr int S = kDwStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kDwOffB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDwOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* accf_bar = bars + 2 * S;
  uint64_t* done_bar = accf_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // work unit: (tap, 256-channel input block, pixel split); every unit covers all 256 outputs
  int r = static_cast<int>(blockIdx.x);
  const int split = r % a.ksplit;
  r /= a.ksplit;
  const int cb = r % a.c_blocks;
  const int tap = r / a.c_blocks;
  const int dy = a.taps == 9 ? tap / 3 - 1 : 0;
  const int dx = a.taps == 9 ? tap % 3 - 1 : 0;
  const int kb0 = split * a.per_kb;
  const int kb1 = min(a.num_kb, kb0 + a.per_kb);  // non-empty (host)
  // bias-gradient CTA: its epilogue warps sum dY over its share of the pixel range meanwhile
  const bool do_db = a.db_partial != nullptr && cb == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accf_bar, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_g);
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_p);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kTcBlockN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, a.status, kDevTimeoutDw)) break;
        const int tx = kb % a.tiles_x;
        const int t2 = kb / a.tiles_x;
        const int ty = t2 % a.tiles_y;
        const int n = t2 / a.tiles_y;
        const int x0 = tx * a.kw, y0 = ty * a.kh;
        mbar_arrive_expect_tx(&full_bar[stage], kDwAStage + kDwBStage);
        for (int j = 0; j < 4; ++j)
          tma_load_4d(smem_a + stage * kDwAStage + j * kDwChunk, &map_g, &full_bar[stage],
                      j * 64, x0, y0, n, kPolicyEvictFirst);
        for (int j = 0; j < 4; ++j)
          tma_load_4d(smem_b + stage * kDwBStage + j * kDwChunk, &map_x, &full_bar[stage],
                      cb * 256 + j * 64, x0 + dx, y0 + dy, n, kPolicyEvictFirst);
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      griddep_launch_dependents();
      for (int i = 0; i < S && i < issued; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait_drain(&full_bar[stage], phase);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // both operands MN-major: channels contiguous, pixels (K) across 128-byte rows
      constexpr uint32_t idesc =
          make_idesc(kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt, 1u, 1u);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, a.status, kDevTimeoutDw)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // A: output channels 0..127 (chunks 0, 1) and 128..255 (chunks 2, 3), one accumulator each
        const uint32_t a_addr = smem_u32(smem_a + stage * kDwAStage);
        const uint64_t adesc0 = sdesc_mnmajor_sw128(a_addr, kDwChunk);
        const uint64_t adesc1 = sdesc_mnmajor_sw128(a_addr + 2 * kDwChunk, kDwChunk);
        const uint64_t bdesc = sdesc_mnmajor_sw128(smem_u32(smem_b + stage * kDwBStage), kDwChunk);
#pragma unroll
        for (int k = 0; k < kMmaPerKb; ++k) {  // +16 pixel rows (2048 bytes) per MMA step
          const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
          tc_mma<T>(tmem_base, adesc0 + 128u * k, bdesc + 128u * k, idesc, acc);
          tc_mma<T>(tmem_base + kTcBlockN, adesc1 + 128u * k, bdesc + 128u * k, idesc, acc);
        }
        tc_commit(&empty_bar[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(accf_bar);
      tc_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // epilogue: accumulator `half` (output channels half*128..), TMEM lane = output channel,
    // column = input channel.  Each 32 x 32 fp32 block of partial rows is staged in shared
    // memory (the operand stages are idle once the accumulator is final; 128-byte swizzle:
    // 16-byte chunk j of row r at j ^ (r & 7)) and stored by one TMA store, two staging
    // buffers per warp.
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    const int row0 = (split * a.taps + tap) * 256 + half * 128 + quarter * 32;
    float db[8];
    if (do_db) {
      // thread e sums 16-byte group g16 (channels 8 g16 ..) of box pixels rl, rl + 8, ..,
      // rl + 56 of k-blocks kb0 + tap, kb0 + tap + taps, .. (the boxes the producer loads),
      // two k-blocks' loads in flight
      const int e = ew * 32 + lane;
      const int g16 = e & 31, rl = e >> 5;
      const uint4* gp = reinterpret_cast<const uint4*>(a.g) + g16;
#pragma unroll
      for (int i = 0; i < 8; ++i) db[i] = 0.f;
      for (int kb = kb0 + tap; kb < kb1; kb += 2 * a.taps) {
        uint4 u[16];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int k2 = kb + b * a.taps;
          const int tx = k2 % a.tiles_x;
          const int t2 = k2 / a.tiles_x;
          const int ty = t2 % a.tiles_y;
          const int n = t2 / a.tiles_y;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int p = rl + 8 * k;
            const int x = tx * a.kw + p % a.kw, y = ty * a.kh + p / a.kw;
            u[8 * b + k] = make_uint4(0u, 0u, 0u, 0u);
            if (k2 < kb1 && x < a.W && y < a.H)
              u[8 * b + k] = __ldg(gp + ((static_cast<size_t>(n) * a.H + y) * a.W + x) * 32);
          }
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint32_t w4[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = Pack<T>::unpack(w4[i]);
            db[2 * i] += f.x;
            db[2 * i + 1] += f.y;
          }
        }
      }
    }
    const bool ok = mbar_wait(accf_bar, 0, abort_flag, a.status, kDevTimeoutDw);
    if (do_db) {
      // every MMA is done: the B stages are free for the fixed-order sum of the 8 row lanes
      float* red = reinterpret_cast<float*>(smem_b);
      const int e = ew * 32 + lane;
#pragma unroll
      for (int i = 0; i < 8; ++i) red[(e >> 5) * 256 + (e & 31) * 8 + i] = db[i];
      asm volatile("bar.sync 1, %0;" ::"n"(kDwEpiWarps * 32) : "memory");
      float acc = 0.f;
      for (int r = 0; r < 8; ++r) acc += red[r * 256 + e];
      if (__all_sync(0xffffffffu, ok))
        a.db_partial[(static_cast<size_t>(split) * a.taps + tap) * 256 + e] = acc;
    }
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      uint8_t* const stage = smem + ew * 2 * kDwStaging;
#pragma unroll 1
      for (int h = 0; h < 8; ++h) {
        const int col = h * 32;
        const int c0 = cb * 256 + col;
        if (c0 >= a.Cin) break;  // (the map clips a block that ends beyond Cin)
        uint32_t v[32];
        tmem_ld32(tmem_base + static_cast<uint32_t>(half * kTcBlockN + col) +
                      (static_cast<uint32_t>(quarter * 32) << 16),
                  v);
        tmem_wait_ld();
        uint8_t* buf = stage + (h & 1) * kDwStaging;
        if (h >= 2) {
          if (lane == 0) bulk_wait_group_read<1>();  // this buffer's previous store read it
          __syncwarp();
        }
        const uint32_t base = smem_u32(buf) + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(base + ((j ^ (lane & 7)) << 4),
                       make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_p, buf, c0, row0);
          bulk_commit_group();
        }
      }
      if (lane == 0) bulk_wait_group<0>();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kTcBlockN);
  }
}

// Sum over s < n of v(s) in a fixed order: four running sums over s = 0, 4, 8, .. / 1, 5, .. /
// .., then (a0 + a1) + (a2 + a3).  Sixteen loads are issued before their adds (the sums keep
// that association), so a thread has 16 loads in flight instead of 4.
template <typename F>
__device__ __forceinline__ float fixed_order_sum(int n, F v) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int s = 0;
  for (; s + 16 <= n; s += 16) {
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = v(s + i);
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      a0 += t[i];
      a1 += t[i + 1];
      a2 += t[i + 2];
      a3 += t[i + 3];
    }
  }
  for (; s + 4 <= n; s += 4) {
    const float t0 = v(s), t1 = v(s + 1), t2 = v(s + 2), t3 = v(s + 3);
    a0 += t0;
    a1 += t1;
    a2 += t2;
    a3 += t3;
  }
  if (s < n) a0 += v(s);
  if (s + 1 < n) a1 += v(s + 1);
  if (s + 2 < n) a2 += v(s + 2);
  return (a0 + a1) + (a2 + a3);
}

// The same fixed order per element for a 16-byte vector of four outputs, spread over a group
// of four lanes: lane k sums the vectors s = k, k + 4, k + 8, .. in order (four loads in
// flight), then the group adds its chains as (c0 + c1) + (c2 + c3) -- fixed_order_sum's
// association, so every element comes out bitwise as from fixed_order_sum -- and lane 0 of
// the group holds the result.  All four lanes of a group must call it.
__device__ __forceinline__ float4 fixed_order_sum4(const float* p, long long stride, int n) {
  const int k = static_cast<int>(threadIdx.x) & 3;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](const float4 t) {
    a.x += t.x;
    a.y += t.y;
    a.z += t.z;
    a.w += t.w;
  };
  int s = k;
  for (; s + 12 < n; s += 16) {
    const float4 t0 = __ldg(reinterpret_cast<const float4*>(p + s * stride));
    const float4 t1 = __ldg(reinterpret_cast<const float4*>(p + (s + 4) * stride));
    const float4 t2 = __ldg(reinterpret_cast<const float4*>(p + (s + 8) * stride));
    const float4 t3 = __ldg(reinterpret_cast<const float4*>(p + (s + 12) * stride));
    add(t0);
    add(t1);
    add(t2);
    add(t3);
  }
  for (; s < n; s += 4) add(__ldg(reinterpret_cast<const float4*>(p + s * stride)));
  float4 b;
  b.x = __shfl_xor_sync(0xffffffffu, a.x, 1);
  b.y = __shfl_xor_sync(0xffffffffu, a.y, 1);
  b.z = __shfl_xor_sync(0xffffffffu, a.z, 1);
  b.w = __shfl_xor_sync(0xffffffffu, a.w, 1);
  a.x += b.x;  // lane 0: c0 + c1, lane 2: c2 + c3
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
  b.x = __shfl_xor_sync(0xffffffffu, a.x, 2);
  b.y = __shfl_xor_sync(0xffffffffu, a.y, 2);
  b.z = __shfl_xor_sync(0xffffffffu, a.z, 2);
  b.w = __shfl_xor_sync(0xffffffffu, a.w, 2);
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// 1x1 weight gradient: out[o * Cin + c] = sum over s of partial[s][o][c] in the fixed order,
// four lanes per 16-byte vector of outputs (Cin a multiple of 4).  With grad_b, the block
// after the last one sums the db_rows rows db_partial[r][o] the same way into grad_b[o].
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partial,
                                                              float* __restrict__ out, int ksplit,
                                                              int Cin,
                                                              const float* __restrict__ db_partial,
                                                              float* __restrict__ grad_b,
                                                              int db_rows) {
  const long long per = 256LL * Cin;
  const long long vblocks = (per / 4 + 63) / 64;
  if (static_cast<long long>(blockIdx.x) >= vblocks) {  // bias
    const int o = threadIdx.x;
    grad_b[o] = fixed_order_sum(db_rows, [&](int r) { return __ldg(db_partial + r * 256 + o); });
    return;
  }
  // (every lane takes part in the group's shuffles; a lane past the end sums nothing)
  const long long v = static_cast<long long>(blockIdx.x) * 64 + threadIdx.x / 4;
  const bool in = v * 4 < per;
  const float4 r = fixed_order_sum4(partial + (in ? v * 4 : 0), per, in ? ksplit : 0);
  if (in && (threadIdx.x & 3) == 0) {  // (scalar stores: grad_w need only be 4-byte aligned)
    out[v * 4 + 0] = r.x;
    out[v * 4 + 1] = r.y;
    out[v * 4 + 2] = r.z;
    out[v * 4 + 3] = r.w;
  }
}

// 3x3 weight gradient in [256 o][Cin c][9 t] order.  Block (o, 256-channel chunk) sums
// partial[s][t][o][chunk] for its 9 x 256 outputs: 576 items of (t, 16-byte vector of four
// channels), two per thread, each summed by its thread over s as four chains s = k, k + 4, ..
// added as (c0 + c1) + (c2 + c3) -- fixed_order_sum's association per element, so the sums are
// bitwise fixed_order_sum's -- with eight 16-byte loads in flight per thread; every warp reads
// 512 contiguous bytes of one (s, t) row.  The block stages its outputs as [c][t] and writes
// its 2304 contiguous outputs in order.  The last block (with grad_b) sums the bias partials.
// Cin a multiple of 4.
constexpr int kTaps9Chunk = 256;
__global__ void __launch_bounds__(288) reduce_partials_taps9_kernel(
    const float* __restrict__ partial, float* __restrict__ out, int ksplit, int Cin,
    const float* __restrict__ db_partial, float* __restrict__ grad_b, int db_rows) {
  __shared__ float tile[kTaps9Chunk * 9];
  const int chunks = (Cin + kTaps9Chunk - 1) / kTaps9Chunk;
  if (static_cast<int>(blockIdx.x) == 256 * chunks) {  // bias
    const int o = threadIdx.x;
    if (o < 256)
      grad_b[o] = fixed_order_sum(db_rows, [&](int r) { return __ldg(db_partial + r * 256 + o); });
    return;
  }
  const int o = static_cast<int>(blockIdx.x) / chunks;
  const int c0 = (static_cast<int>(blockIdx.x) % chunks) * kTaps9Chunk;
  const long long per = 9LL * 256 * Cin;
  const float* src[2];
  bool in[2];
  int t_of[2], v_of[2];
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int item = static_cast<int>(threadIdx.x) + it * 288;  // 0 .. 575
    t_of[it] = item / (kTaps9Chunk / 4);
    v_of[it] = item % (kTaps9Chunk / 4);
    in[it] = c0 + v_of[it] * 4 < Cin;
    src[it] = partial + (static_cast<size_t>(t_of[it]) * 256 + o) * Cin + c0 + v_of[it] * 4;
  }
  float4 acc[2][4];
#pragma unroll
  for (int it = 0; it < 2; ++it)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[it][k] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [](float4& a, const float4 t) {
    a.x += t.x;
    a.y += t.y;
    a.z += t.z;
    a.w += t.w;
  };
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  int s = 0;
  for (; s + 4 <= ksplit; s += 4) {
    float4 t[2][4];
#pragma unroll
    for (int it = 0; it < 2; ++it)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        t[it][k] = in[it] ? __ldg(reinterpret_cast<const float4*>(src[it] + (s + k) * per)) : zero;
#pragma unroll
    for (int it = 0; it < 2; ++it)
#pragma unroll
      for (int k = 0; k < 4; ++k) add(acc[it][k], t[it][k]);
  }
#pragma unroll
  for (int k = 0; k < 3; ++k)  // the tail: s + k < ksplit goes to chain k
    if (s + k < ksplit) {
#pragma unroll
      for (int it = 0; it < 2; ++it)
        if (in[it]) add(acc[it][k], __ldg(reinterpret_cast<const float4*>(src[it] + (s + k) * per)));
    }
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    if (!in[it]) continue;
    const float4 a = acc[it][0], b = acc[it][1], c = acc[it][2], d = acc[it][3];
    const float r[4] = {(a.x + b.x) + (c.x + d.x), (a.y + b.y) + (c.y + d.y),
                        (a.z + b.z) + (c.z + d.z), (a.w + b.w) + (c.w + d.w)};
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[(v_of[it] * 4 + j) * 9 + t_of[it]] = r[j];
  }
  __syncthreads();
  const int n_out = (Cin - c0 < kTaps9Chunk ? Cin - c0 : kTaps9Chunk) * 9;
  float* dst = out + (static_cast<size_t>(o) * Cin + c0) * 9;
  for (int j = threadIdx.x; j < n_out; j += 288) dst[j] = tile[j];
}

// ------------------------------------------------------------------ bias gradient
template <typename T>
__device__ __forceinline__ float bw_to_f(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float bw_to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float bw_to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T bw_from_f(float v);
template <>
__device__ __forceinline__ float bw_from_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half bw_from_f<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 bw_from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// part[b][c] = sum of g[p][c] over block b's contiguous run of pixels.  vt = C * sizeof(T) / 16
// threads cover a pixel's 16-byte vectors; the block's 256 / vt pixel lanes run through its
// pixels with that stride, four loads in flight each; the lanes' sums are then added in lane
// order (fixed: the result does not depend on timing).
template <typename T>
__global__ void __launch_bounds__(256) colsum_kernel(const T* __restrict__ g, long long pixels,
                                                     int C, long long per, float* __restrict__ part) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[256 * V];
  const int vt = C / V;
  const int lanes = 256 / vt;
  const int cv = threadIdx.x % vt;   // 16-byte vector: channels cv*V .. +V-1
  const int pl = threadIdx.x / vt;   // pixel lane
  const long long p0 = static_cast<long long>(blockIdx.x) * per;
  const long long p1 = min(pixels, p0 + per);
  float a[4][V];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int e = 0; e < V; ++e) a[q][e] = 0.f;
  const bool active = pl < lanes;
  long long p = p0 + pl;
  for (; active && p + 3 * lanes < p1; p += 4 * lanes) {
    union {
      uint4 u;
      T e[V];
    } x[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      x[q].u = __ldg(reinterpret_cast<const uint4*>(g + (p + q * lanes) * C) + cv);
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int e = 0; e < V; ++e) a[q][e] += bw_to_f(x[q].e[e]);
  }
  for (; active && p < p1; p += lanes) {
    union {
      uint4 u;
      T e[V];
    } x;
    x.u = __ldg(reinterpret_cast<const uint4*>(g + p * C) + cv);
#pragma unroll
    for (int e = 0; e < V; ++e) a[0][e] += bw_to_f(x.e[e]);
  }
  if (active) {
#pragma unroll
    for (int e = 0; e < V; ++e) red[pl * C + cv * V + e] = (a[0][e] + a[1][e]) + (a[2][e] + a[3][e]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float acc = 0.f;
    for (int l = 0; l < lanes; ++l) acc += red[l * C + c];
    part[static_cast<size_t>(blockIdx.x) * C + c] = acc;
  }
}
// out[c] = sum over r of part[r][c]: a block takes 32 channels, its 32 row lanes sum every
// 32nd row (four running sums each) and the lanes' sums are added in lane order (fixed order).
__global__ void __launch_bounds__(1024) sum_rows_kernel(const float* __restrict__ part, int rows,
                                                        int C, float* __restrict__ out) {
  __shared__ float red[32][33];
  const int cl = threadIdx.x & 31, lane = threadIdx.x >> 5;
  const int c = static_cast<int>(blockIdx.x) * 32 + cl;
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  if (c < C) {
    int r = lane;
    for (; r + 96 < rows; r += 128) {
#pragma unroll
      for (int q = 0; q < 4; ++q) a[q] += part[static_cast<size_t>(r + 32 * q) * C + c];
    }
    for (; r < rows; r += 32) a[0] += part[static_cast<size_t>(r) * C + c];
  }
  red[lane][cl] = (a[0] + a[1]) + (a[2] + a[3]);
  __syncthreads();
  if (lane == 0 && c < C) {
    float acc = 0.f;
    for (int l = 0; l < 32; ++l) acc += red[l][cl];
    out[c] = acc;
  }
}

// ------------------------------------------------------------------ top-down adjoint
__device__ __forceinline__ float bw_src(int o, int in, float scale) {
  const float s = (static_cast<float>(o) + 0.5f) * scale - 0.5f;
  return fminf(fmaxf(s, 0.f), static_cast<float>(in - 1));
}
// weight with which fine coordinate o (of `out`) taps coarse coordinate q (of `in`)
__device__ __forceinline__ float bw_tap_weight(int o, int q, int in, float scale) {
  const float s = bw_src(o, in, scale);
  const int a = static_cast<int>(s);
  const int b = min(a + 1, in - 1);
  const float w = s - static_cast<float>(a);
  return (a == q ? 1.f - w : 0.f) + (b == q ? w : 0.f);
}

// out[n, yc, xc, :] = base[n, yc, xc, :] (or 0) + sum over fine (y, x) of
// wy(y, yc) * wx(x, xc) * g[n, y, x, :]  -- NHWC, C a multiple of 16 / sizeof(T).
// One warp per coarse pixel, lanes over 16-byte channel vectors.
template <typename T>
__global__ void __launch_bounds__(256) upsample_adjoint_kernel(
    const T* __restrict__ g, const T* base, T* out, int N, int C, int Hc, int Wc, int H, int W,
    float sy, float sx) {
  constexpr int V = 16 / sizeof(T);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long pix = static_cast<long long>(blockIdx.x) * 8 + warp;
  if (pix >= static_cast<long long>(N) * Hc * Wc) return;
  const int xc = static_cast<int>(pix % Wc);
  const long long t = pix / Wc;
  const int yc = static_cast<int>(t % Hc);
  const int n = static_cast<int>(t / Hc);
  // fine rows / columns whose taps can reach (yc, xc): a superset, weights decide
  const float iy = 1.f / sy, ix = 1.f / sx;
  const int y_lo = max(0, static_cast<int>(floorf((yc - 1 + 0.5f) * iy - 0.5f)) - 1);
  const int y_hi = min(H - 1, static_cast<int>(ceilf((yc + 1 + 0.5f) * iy - 0.5f)) + 1);
  const int x_lo = max(0, static_cast<int>(floorf((xc - 1 + 0.5f) * ix - 0.5f)) - 1);
  const int x_hi = min(W - 1, static_cast<int>(ceilf((xc + 1 + 0.5f) * ix - 0.5f)) + 1);
  const bool y_edge = yc == Hc - 1, x_edge = xc == Wc - 1;  // clamped tails reach the edge
  const int y_end = y_edge ? H - 1 : y_hi;
  const int x_end = x_edge ? W - 1 : x_hi;
  const T* gn = g + static_cast<size_t>(n) * H * W * C;
  const size_t ob = (static_cast<size_t>(n) * Hc * Wc + static_cast<size_t>(yc) * Wc + xc) * C;
  for (int cv = lane; cv * V < C; cv += 32) {
    float acc[V];
#pragma unroll
    for (int e = 0; e < V; ++e) acc[e] = 0.f;
    for (int y = y_lo; y <= y_end; ++y) {
      const float wy = bw_tap_weight(y, yc, Hc, sy);
      if (wy == 0.f) continue;
      for (int x = x_lo; x <= x_end; ++x) {
        const float wx = bw_tap_weight(x, xc, Wc, sx);
        if (wx == 0.f) continue;
        const float w = wy * wx;
        union {
          uint4 u;
          T e[V];
        } v;
        v.u = __ldg(reinterpret_cast<const uint4*>(gn + (static_cast<size_t>(y) * W + x) * C) + cv);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = fmaf(bw_to_f(v.e[e]), w, acc[e]);
      }
    }
    union {
      uint4 u;
      T e[V];
    } o;
    if (base) {
      union {
        uint4 u;
        T e[V];
      } b;
      b.u = *(reinterpret_cast<const uint4*>(base + ob) + cv);
#pragma unroll
      for (int e = 0; e < V; ++e) o.e[e] = bw_from_f<T>(bw_to_f(b.e[e]) + acc[e]);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) o.e[e] = bw_from_f<T>(acc[e]);
    }
    *(reinterpret_cast<uint4*>(out + ob) + cv) = o.u;
  }
}

// fine rows (columns) whose taps can reach coarse row (column) q: [tap_lo, tap_hi], a superset
// of the nonzero ones (weights decide); the clamped tail of the last coarse index reaches the end
__device__ __forceinline__ int tap_lo(int q, float inv) {
  return max(0, static_cast<int>(floorf((q - 1 + 0.5f) * inv - 0.5f)) - 1);
}
__device__ __forceinline__ int tap_hi(int q, int in, int out, float inv) {
  return q == in - 1 ? out - 1 : min(out - 1, static_cast<int>(ceilf((q + 1 + 0.5f) * inv - 0.5f)) + 1);
}

constexpr int kUaTapsMax = 24;  // fine rows (columns) with a nonzero weight per coarse one
constexpr int kUaStripMax = 16;  // coarse columns per block
constexpr int kUaThreads = 256;

// 16 bytes of T <-> V floats with packed conversions (bf16: a shift or a mask per element)
template <typename T>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int V = 8;
  static __device__ __forceinline__ void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ uint4 pack(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <>
struct Vec16<__half> {
  static constexpr int V = 8;
  static __device__ __forceinline__ void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <>
struct Vec16<float> {
  static constexpr int V = 4;
  static __device__ __forceinline__ void unpack(const uint4& u, float (&f)[4]) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  static __device__ __forceinline__ uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

// acc += w * (16 bytes of T)
template <typename T, int V>
__device__ __forceinline__ void fma_vec(float (&acc)[V], const uint4& u, float w) {
  float f[V];
  Vec16<T>::unpack(u, f);
#pragma unroll
  for (int e = 0; e < V; ++e) acc[e] = fmaf(f[e], w, acc[e]);
}

// Same sum as upsample_adjoint_kernel, separably: a block takes coarse row yc of image n and a
// strip of up to TX coarse columns.  The fine rows that reach yc and the fine columns that reach
// each coarse column of the strip are listed once, with their weights, in shared memory (the
// scale is at most 8, so at most 2 * 8 + 1 of either have a nonzero weight).  Pass 1 sums the
// listed fine rows, weighted, into fp32 rows of shared memory, one per fine column the strip
// reaches (16-byte vectors; a thread keeps its vector and steps over fine columns, loads of
// four rows issued before their math, the first four rows' offsets and weights held in
// registers); pass 2 forms each coarse pixel of the strip from its listed fine columns there and
// adds `base`.  Each fine pixel is read once per coarse row it reaches (about twice at scale 2),
// not once per coarse pixel (four times).  In shared memory the four-float quarter q of channel
// vector cv of fine column j sits at j * C + (q * C / V + cv) * 4: a warp's 16-byte accesses are
// contiguous.  C / V <= 256.
template <typename T>
__global__ void __launch_bounds__(kUaThreads) upsample_adjoint_staged_kernel(
    const T* __restrict__ g, const T* base, T* out, int C, int Hc, int Wc, int H, int W, float sy,
    float sx, int TX) {
  constexpr int V = Vec16<T>::V;
  constexpr int Q = V / 4;  // float4 quarters per vector
  extern __shared__ float4 ua_smem[];
  float* R = reinterpret_cast<float*>(ua_smem);  // [span][C]
  __shared__ long long row_off[kUaTapsMax];      // element offset of the fine row in the image
  __shared__ float row_w[kUaTapsMax];
  __shared__ int nrows;
  __shared__ short col_x[kUaStripMax][kUaTapsMax];  // fine column - fx0
  __shared__ float col_w[kUaStripMax][kUaTapsMax];
  __shared__ int ncols[kUaStripMax];
  const int strips = (Wc + TX - 1) / TX;
  const int strip = static_cast<int>(blockIdx.x % strips);
  const int yc = static_cast<int>((blockIdx.x / strips) % Hc);
  const int n = static_cast<int>(blockIdx.x / strips / Hc);
  const int xc0 = strip * TX, xc1 = min(Wc, xc0 + TX) - 1;
  const float iy = 1.f / sy, ix = 1.f / sx;
  const int fx0 = tap_lo(xc0, ix);
  const int span = tap_hi(xc1, Wc, W, ix) - fx0 + 1;
  if (threadIdx.x == 0) {
    int k = 0;
    for (int y = tap_lo(yc, iy), ye = tap_hi(yc, Hc, H, iy); y <= ye; ++y) {
      const float w = bw_tap_weight(y, yc, Hc, sy);
      if (w != 0.f && k < kUaTapsMax) {
        row_off[k] = static_cast<long long>(y) * W * C;
        row_w[k] = w;
        ++k;
      }
    }
    nrows = k;
  } else if (threadIdx.x >= 32 && threadIdx.x < 32 + xc1 - xc0 + 1) {
    const int xl = threadIdx.x - 32, xc = xc0 + xl;
    int k = 0;
    for (int x = tap_lo(xc, ix), xe = tap_hi(xc, Wc, W, ix); x <= xe; ++x) {
      const float w = bw_tap_weight(x, xc, Wc, sx);
      if (w != 0.f && k < kUaTapsMax) {
        col_x[xl][k] = static_cast<short>(x - fx0);
        col_w[xl][k] = w;
        ++k;
      }
    }
    ncols[xl] = k;
  }
  const int cvn = C / V;
  const int jstep = kUaThreads / cvn;  // fine columns in flight per block
  const int cv = threadIdx.x % cvn, j0 = threadIdx.x / cvn;
  __syncthreads();
  const int nr = nrows;
  long long ro[4];
  float rwt[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    ro[q] = q < nr ? row_off[q] : 0;
    rwt[q] = q < nr ? row_w[q] : 0.f;
  }
  const T* gn = g + static_cast<size_t>(n) * H * W * C + cv * V;
  if (j0 < jstep) {
    for (int j = j0; j < span; j += jstep) {
      const T* src = gn + static_cast<size_t>(fx0 + j) * C;
      float acc[V];
#pragma unroll
      for (int e = 0; e < V; ++e) acc[e] = 0.f;
      uint4 v[4];
      if (nr >= 4) {
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = __ldg(reinterpret_cast<const uint4*>(src + ro[q]));
#pragma unroll
        for (int q = 0; q < 4; ++q) fma_vec<T, V>(acc, v[q], rwt[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 3; ++q)
          if (q < nr) v[q] = __ldg(reinterpret_cast<const uint4*>(src + ro[q]));
#pragma unroll
        for (int q = 0; q < 3; ++q)
          if (q < nr) fma_vec<T, V>(acc, v[q], rwt[q]);
      }
      for (int r = 4; r < nr; r += 4) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (r + q < nr) v[q] = __ldg(reinterpret_cast<const uint4*>(src + row_off[r + q]));
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (r + q < nr) fma_vec<T, V>(acc, v[q], row_w[r + q]);
      }
      float4* dst = reinterpret_cast<float4*>(R + static_cast<size_t>(j) * C) + cv;
#pragma unroll
      for (int q = 0; q < Q; ++q)
        dst[q * cvn] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    }
  }
  __syncthreads();
  if (j0 >= jstep) return;
  const size_t orow = (static_cast<size_t>(n) * Hc + yc) * Wc;
  for (int xl = j0; xl <= xc1 - xc0; xl += jstep) {
    float acc[V];
#pragma unroll
    for (int e = 0; e < V; ++e) acc[e] = 0.f;
    const int nc = ncols[xl];
    for (int k = 0; k < nc; ++k) {
      const float w = col_w[xl][k];
      const float4* r4 = reinterpret_cast<const float4*>(R + static_cast<size_t>(col_x[xl][k]) * C) + cv;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const float4 f = r4[q * cvn];
        acc[4 * q] = fmaf(f.x, w, acc[4 * q]);
        acc[4 * q + 1] = fmaf(f.y, w, acc[4 * q + 1]);
        acc[4 * q + 2] = fmaf(f.z, w, acc[4 * q + 2]);
        acc[4 * q + 3] = fmaf(f.w, w, acc[4 * q + 3]);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (orow + xc0 + xl) * C) + cv;
    if (base) {
      const uint4 b = *(reinterpret_cast<const uint4*>(base + (orow + xc0 + xl) * C) + cv);
      fma_vec<T, V>(acc, b, 1.f);
    }
    *dst = Vec16<T>::pack(acc);
  }
}

// dP5[n, 2y, 2x, :] += dP6[n, y, x, :] (NHWC, 16-byte vectors)
template <typename T>
__global__ void __launch_bounds__(256) p6_adjoint_kernel(const T* __restrict__ g6, T* g5, int N,
                                                         int C, int H5, int W5) {
  constexpr int V = 16 / sizeof(T);
  const int H6 = (H5 - 1) / 2 + 1, W6 = (W5 - 1) / 2 + 1;
  const long long total = static_cast<long long>(N) * H6 * W6 * (C / V);
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int cv = static_cast<int>(i % (C / V));
    const long long p = i / (C / V);
    const int x = static_cast<int>(p % W6);
    const long long q = p / W6;
    const int y = static_cast<int>(q % H6);
    const int n = static_cast<int>(q / H6);
    union {
      uint4 u;
      T e[V];
    } a, b;
    a.u = __ldg(reinterpret_cast<const uint4*>(g6 + (static_cast<size_t>(p) * C)) + cv);
    uint4* dst = reinterpret_cast<uint4*>(
                     g5 + ((static_cast<size_t>(n) * H5 + 2 * y) * W5 + 2 * x) * C) + cv;
    b.u = *dst;
#pragma unroll
    for (int e = 0; e < V; ++e) b.e[e] = bw_from_f<T>(bw_to_f(b.e[e]) + bw_to_f(a.e[e]));
    *dst = b.u;
  }
}

// ------------------------------------------------------------------ weight layouts
constexpr int kPrepMaxJobs = 16;
struct PrepArgs {
  int first_block[kPrepMaxJobs + 1];  // blocks of job j: [first_block[j], first_block[j + 1])
  const float* in[kPrepMaxJobs];
  void* out[kPrepMaxJobs];
  int kind[kPrepMaxJobs];
  int cin[kPrepMaxJobs];
  int vec[kPrepMaxJobs];  // kinds 0 / 1: in (and for kind 0 out) 16-byte aligned
  int num_jobs;
};

// One block per unit of a job (WeightPrepJob kinds), 256 threads; every thread reads adjacent
// fp32 words and every warp writes consecutive elements.
//   kind 0: unit = 2048 elements (vec: 8 per thread, two 16-byte loads and one 16-byte
//           store; else one output row o, out[o][c] = in[o][c])
//   kind 1: unit = 8 rows c0 .. c0+7; out[c][o] = in[o][c] (0 for c >= cin), thread o
//   kind 2: unit = output channel o;  out[o][t][c] = in[o][c][t], thread c
//   kind 3: unit = input channels c0 .. c0+3; out[c][t][o] = in[o][c][8 - t], thread o
template <typename T>
__global__ void __launch_bounds__(256) prepare_weights_kernel(const __grid_constant__ PrepArgs a) {
  int j = 0;
  while (j + 1 < a.num_jobs && static_cast<int>(blockIdx.x) >= a.first_block[j + 1]) ++j;
  const int u = static_cast<int>(blockIdx.x) - a.first_block[j];
  const float* in = a.in[j];
  T* out = static_cast<T*>(a.out[j]);
  const int cin = a.cin[j];
  const int t0 = threadIdx.x;
  switch (a.kind[j]) {
    case 0:
      if (a.vec[j]) {
        const size_t e = (static_cast<size_t>(u) * 256 + t0) * 8;
        const float4 lo = __ldg(reinterpret_cast<const float4*>(in + e));
        const float4 hi = __ldg(reinterpret_cast<const float4*>(in + e) + 1);
        const float f[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        *reinterpret_cast<uint4*>(out + e) = Vec16<T>::pack(f);
      } else {
        for (int c = t0; c < cin; c += 256)
          out[static_cast<size_t>(u) * cin + c] = bw_from_f<T>(in[static_cast<size_t>(u) * cin + c]);
      }
      break;
    case 1: {
      const int c0 = u * 8;
      float v[8];
      if (a.vec[j] && c0 + 8 <= cin) {
        const float4 lo = __ldg(reinterpret_cast<const float4*>(in + static_cast<size_t>(t0) * cin + c0));
        const float4 hi = __ldg(reinterpret_cast<const float4*>(in + static_cast<size_t>(t0) * cin + c0) + 1);
        v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w;
        v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = c0 + i < cin ? in[static_cast<size_t>(t0) * cin + c0 + i] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) out[static_cast<size_t>(c0 + i) * 256 + t0] = bw_from_f<T>(v[i]);
      break;
    }
    case 2: {
      const float* src = in + (static_cast<size_t>(u) * 256 + t0) * 9;
      float v[9];
#pragma unroll
      for (int t = 0; t < 9; ++t) v[t] = src[t];
#pragma unroll
      for (int t = 0; t < 9; ++t) out[(static_cast<size_t>(u) * 9 + t) * 256 + t0] = bw_from_f<T>(v[t]);
      break;
    }
    default: {
      // four input channels c0 .. c0+3: thread o reads its contiguous 36 words in[o][c0..][..]
      // (nine 16-byte loads when vec), every warp store covers 32 consecutive o
      const int c0 = u * 4;
      const float* src = in + (static_cast<size_t>(t0) * 256 + c0) * 9;
      float v[36];
      if (a.vec[j]) {
#pragma unroll
        for (int i = 0; i < 9; ++i) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(src) + i);
          v[4 * i] = q.x, v[4 * i + 1] = q.y, v[4 * i + 2] = q.z, v[4 * i + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 36; ++i) v[i] = src[i];
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
#pragma unroll
        for (int t = 0; t < 9; ++t)
          out[(static_cast<size_t>(c0 + cc) * 9 + t) * 256 + t0] = bw_from_f<T>(v[cc * 9 + 8 - t]);
      break;
    }
  }
}
// out[c][r] = in[r][c] for an R x C matrix (rows of out beyond C up to out_rows are zeroed)
template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T* __restrict__ in, T* __restrict__ out,
                                                        int R, int C, int out_rows) {
  const long long total = static_cast<long long>(out_rows) * R;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i % R);
    const int c = static_cast<int>(i / R);
    out[i] = c < C ? in[static_cast<size_t>(r) * C + c] : bw_from_f<T>(0.f);
  }
}
// packed 3x3 weights [256 o][9 t][256 c] -> [256 c][9 t'][256 o], t' = 8 - t
template <typename T>
__global__ void __launch_bounds__(256) flip_conv3x3_kernel(const T* __restrict__ in,
                                                           T* __restrict__ out) {
  const int total = 256 * 9 * 256;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int o = i % 256;
    const int tp = (i / 256) % 9;
    const int c = i / (256 * 9);
    out[i] = in[(static_cast<size_t>(o) * 9 + (8 - tp)) * 256 + c];
  }
}

// 64-pixel k-block shape with the fewest padded pixels
void dw_block_shape(int H, int W, int& kw, int& kh) {
  long long best = -1;
  for (int w : {64, 32, 16, 8}) {
    const int h = 64 / w;
    const long long area = static_cast<long long>((W + w - 1) / w) * w * ((H + h - 1) / h) * h;
    if (best < 0 || area < best) {
      best = area;
      kw = w;
      kh = h;
    }
  }
}

// Pixel split of the weight-gradient GEMM: about one wave of CTAs over all units (taps x
// input-channel blocks), at least 4 k-blocks per split, every split non-empty.
void dw_split(int num_kb, int units, int& per, int& ksplit) {
  int k = sm_count() / units;
  if (k < 1) k = 1;
  const int cap = num_kb / 4 > 0 ? num_kb / 4 : 1;
  if (k > cap) k = cap;
  per = (num_kb + k - 1) / k;
  ksplit = (num_kb + per - 1) / per;
}

int grid_for(long long work, int block) {
  const long long g = (work + block - 1) / block;
  return static_cast<int>(g < 148LL * 32 ? (g > 0 ? g : 1) : 148LL * 32);
}

}  // namespace

size_t dw_gemm_workspace_bytes(int N, int H, int W, int Cin, int taps) {
  if (N <= 0 || H <= 0 || W <= 0 || Cin <= 0 || (taps != 1 && taps != 9)) return 0;
  int kw = 64, kh = 1;
  dw_block_shape(H, W, kw, kh);
  const int num_kb = ((W + kw - 1) / kw) * ((H + kh - 1) / kh) * N;
  const int units = taps * ((Cin + 255) / 256);
  int per = 1, ksplit = 1;
  dw_split(num_kb, units, per, ksplit);
  // weight partials, then the bias partials [ksplit][taps][256]
  return static_cast<size_t>(ksplit) * taps * (static_cast<size_t>(256) * Cin + 256) * sizeof(float);
}

cudaError_t launch_dw_gemm(DType dt, const void* grad_out, const void* x, int N, int H, int W,
                           int Cin, int taps, float* grad_w, float* grad_b, float* workspace,
                           size_t ws_bytes, int* status, cudaStream_t s) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorNotSupported;
  if (N <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cin % 8 != 0 || (taps != 1 && taps != 9))
    return cudaErrorInvalidValue;
  if (!grad_out || !x || !grad_w || !workspace) return cudaErrorInvalidValue;
  DwArgs a;
  std::memset(&a, 0, sizeof(a));
  dw_block_shape(H, W, a.kw, a.kh);
  a.tiles_x = (W + a.kw - 1) / a.kw;
  a.tiles_y = (H + a.kh - 1) / a.kh;
  a.N_img = N;
  a.num_kb = a.tiles_x * a.tiles_y * N;
  a.c_blocks = (Cin + 255) / 256;
  a.taps = taps;
  a.Cin = Cin;
  const int units = taps * a.c_blocks;
  dw_split(a.num_kb, units, a.per_kb, a.ksplit);
  a.partial = workspace;
  a.status = status;
  const size_t wparts = static_cast<size_t>(a.ksplit) * taps * 256 * Cin;
  if ((wparts + static_cast<size_t>(a.ksplit) * taps * 256) * sizeof(float) > ws_bytes)
    return cudaErrorInvalidValue;
  a.db_partial = grad_b ? workspace + wparts : nullptr;
  a.g = grad_out;
  a.H = H;
  a.W = W;
  CUtensorMap map_g, map_x, map_p;
  cudaError_t e = encode_nhwc_map(&map_g, dt, grad_out, N, H, W, 256, 256, a.kw, a.kh);
  if (e != cudaSuccess) return e;
  if ((e = encode_nhwc_map(&map_x, dt, x, N, H, W, Cin, Cin, a.kw, a.kh)) != cudaSuccess) return e;
  if ((e = encode_rows_map(&map_p, DType::F32, workspace, Cin,
                           static_cast<long long>(a.ksplit) * taps * 256, 32, 32)) != cudaSuccess)
    return e;
  static std::atomic<bool> configured[2][64];  // per dtype and device
  const int ti = dt == DType::BF16 ? 0 : 1;
  auto kern = dt == DType::BF16 ? fpn_dw_gemm_kernel<__nv_bfloat16> : fpn_dw_gemm_kernel<__half>;
  if ((e = once_per_device(configured[ti], [&] {
         return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kDwSmemBytes);
       })) != cudaSuccess)
    return e;
  const int grid = units * a.ksplit;
  e = launch_ex(kern, dim3(grid), dim3(kTcThreads), kDwSmemBytes, s, LaunchOpts(), 1, map_g, map_x,
                map_p, a);
  if (e != cudaSuccess) return e;
  if (taps == 9) {
    // one block per (output channel, 256 input channels) + one for the bias
    const unsigned grid9 = static_cast<unsigned>(256 * ((Cin + 255) / 256) + (grad_b ? 1 : 0));
    return launch_ex(reduce_partials_taps9_kernel, dim3(grid9), dim3(288), 0, s, LaunchOpts(), 1,
                     static_cast<const float*>(workspace), grad_w, a.ksplit, Cin,
                     static_cast<const float*>(a.db_partial), grad_b, a.ksplit * taps);
  }
  // one block per 64 vectors of four outputs + one for the bias
  const long long vblocks = (64LL * Cin + 63) / 64;
  return launch_ex(reduce_partials_kernel, dim3(static_cast<unsigned>(vblocks + (grad_b ? 1 : 0))),
                   dim3(256), 0, s, LaunchOpts(), 1, static_cast<const float*>(workspace), grad_w,
                   a.ksplit, Cin, static_cast<const float*>(a.db_partial), grad_b,
                   a.ksplit * taps);
}

// Column sums: at most 4 blocks per SM (all resident at once), each over a contiguous run of at
// least 64 pixels.
static long long colsum_blocks(long long pixels) {
  const long long cap = 4LL * sm_count();
  const long long b = (pixels + 63) / 64;
  return b < 1 ? 1 : (b < cap ? b : cap);
}

size_t colsum_workspace_bytes(long long pixels, int C) {
  return static_cast<size_t>(colsum_blocks(pixels)) * C * sizeof(float);
}

cudaError_t launch_colsum(DType dt, const void* g, long long pixels, int C, float* out,
                          float* workspace, size_t ws_bytes, cudaStream_t s) {
  if (pixels <= 0 || C <= 0 || !g || !out || !workspace) return cudaErrorInvalidValue;
  // 16-byte vectors, at most one per thread, cover a pixel's channels
  if ((C * dtype_size(dt)) % 16 != 0 || C * dtype_size(dt) > 256 * 16 || !aligned16(g))
    return cudaErrorNotSupported;
  const long long blocks = colsum_blocks(pixels);
  const long long per = (pixels + blocks - 1) / blocks;
  const int nb = static_cast<int>((pixels + per - 1) / per);
  if (static_cast<size_t>(nb) * C * sizeof(float) > ws_bytes) return cudaErrorInvalidValue;
  cudaError_t e;
  switch (dt) {
    case DType::F32:
      e = launch_ex(colsum_kernel<float>, dim3(nb), dim3(256), 0, s, LaunchOpts(), 1,
                    static_cast<const float*>(g), pixels, C, per, workspace);
      break;
    case DType::F16:
      e = launch_ex(colsum_kernel<__half>, dim3(nb), dim3(256), 0, s, LaunchOpts(), 1,
                    static_cast<const __half*>(g), pixels, C, per, workspace);
      break;
    case DType::BF16:
      e = launch_ex(colsum_kernel<__nv_bfloat16>, dim3(nb), dim3(256), 0, s, LaunchOpts(), 1,
                    static_cast<const __nv_bfloat16*>(g), pixels, C, per, workspace);
      break;
    default:
      return cudaErrorNotSupported;
  }
  if (e != cudaSuccess) return e;
  return launch_ex(sum_rows_kernel, dim3((C + 31) / 32), dim3(1024), 0, s, LaunchOpts(), 1,
                   static_cast<const float*>(workspace), nb, C, out);
}

template <typename K, typename... Args>
cudaError_t launch_staged_adjoint(K kernel, long long blocks, size_t smem, cudaStream_t s,
                                  Args... args) {
  static std::atomic<bool> opted[64];
  cudaError_t e = once_per_device(opted, [&] {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kUaThreads), smem, s,
                   LaunchOpts(), 1, args...);
}

cudaError_t launch_prepare_weights(DType dt, const WeightPrepJob* jobs, int num_jobs,
                                   cudaStream_t s) {
  if (num_jobs < 1 || num_jobs > kPrepMaxJobs || !jobs) return cudaErrorInvalidValue;
  PrepArgs a;
  std::memset(&a, 0, sizeof(a));
  int blocks = 0;
  for (int j = 0; j < num_jobs; ++j) {
    const WeightPrepJob& jb = jobs[j];
    if (!jb.in || !jb.out || jb.kind < 0 || jb.kind > 3 || jb.cin <= 0) return cudaErrorInvalidValue;
    a.first_block[j] = blocks;
    a.in[j] = jb.in;
    a.out[j] = jb.out;
    a.kind[j] = jb.kind;
    a.cin[j] = jb.cin;
    // kind 0 vectorised: 2048-element units (256 * cin a multiple of 2048); kind 1: 8-row units
    // (kind 3: 4-channel units, 64 per job)
    a.vec[j] = aligned16(jb.in) && (jb.kind >= 2 || jb.cin % 8 == 0) &&
               (jb.kind != 0 || aligned16(jb.out));
    blocks += jb.kind == 1                 ? (jb.cin + 255) / 256 * 32
              : jb.kind == 0 && a.vec[j] ? jb.cin / 8
              : jb.kind == 3             ? 64
                                         : 256;
  }
  a.first_block[num_jobs] = blocks;
  a.num_jobs = num_jobs;
  const unsigned grid = static_cast<unsigned>(blocks);
  switch (dt) {
    case DType::BF16:
      return launch_ex(prepare_weights_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s,
                       LaunchOpts(), 1, a);
    case DType::F16:
      return launch_ex(prepare_weights_kernel<__half>, dim3(grid), dim3(256), 0, s, LaunchOpts(),
                       1, a);
    default:
      return cudaErrorNotSupported;
  }
}

cudaError_t launch_upsample_adjoint(DType dt, const void* grad_fine, const void* base, void* out,
                                    int N, int C, int Hc, int Wc, int H, int W, cudaStream_t s) {
  if (N <= 0 || C <= 0 || Hc <= 0 || Wc <= 0 || H <= 0 || W <= 0 || !grad_fine || !out)
    return cudaErrorInvalidValue;
  if (Hc > H || Wc > W) return cudaErrorNotSupported;  // the forward upsamples
  if (!aligned16(grad_fine) || !aligned16(out) || (base && !aligned16(base)))
    return cudaErrorMisalignedAddress;
  const int esz = dtype_size(dt);
  if ((C * esz) % 16 != 0) return cudaErrorInvalidValue;
  const float sy = static_cast<float>(Hc) / H, sx = static_cast<float>(Wc) / W;  // forward scales
  // Staged kernel: at most 8 fine rows / columns per coarse one (then at most 2 * 8 + 1 fine
  // rows or columns have a nonzero weight for a coarse one: their source coordinate lies in an
  // open interval of length 2), a strip of TX coarse columns whose fine span, bounded by
  // (TX + 1) W / Wc + 6, fits the shared-memory rows, and one 16-byte vector per thread.
  constexpr size_t kUaSmemMax = 160 * 1024;
  const double ratio = static_cast<double>(W) / Wc;
  auto span_bound = [&](int tx) { return static_cast<int>(std::ceil((tx + 1) * ratio)) + 6; };
  int TX = std::min(kUaStripMax, Wc);
  while (TX > 1 && static_cast<size_t>(span_bound(TX)) * C * 4 > 64 * 1024) --TX;
  const size_t smem = static_cast<size_t>(span_bound(TX)) * C * 4;
  const long long strips = (Wc + TX - 1) / TX;
  const long long blocks = static_cast<long long>(N) * Hc * strips;
  if (H <= 8 * Hc && W <= 8 * Wc && C / (16 / esz) <= kUaThreads && smem <= kUaSmemMax &&
      span_bound(TX) < 32768 && blocks < (1LL << 31)) {
    switch (dt) {
      case DType::F32:
        return launch_staged_adjoint(upsample_adjoint_staged_kernel<float>, blocks, smem, s,
                                     static_cast<const float*>(grad_fine),
                                     static_cast<const float*>(base), static_cast<float*>(out), C,
                                     Hc, Wc, H, W, sy, sx, TX);
      case DType::F16:
        return launch_staged_adjoint(upsample_adjoint_staged_kernel<__half>, blocks, smem, s,
                                     static_cast<const __half*>(grad_fine),
                                     static_cast<const __half*>(base), static_cast<__half*>(out), C,
                                     Hc, Wc, H, W, sy, sx, TX);
      case DType::BF16:
        return launch_staged_adjoint(upsample_adjoint_staged_kernel<__nv_bfloat16>, blocks, smem, s,
                                     static_cast<const __nv_bfloat16*>(grad_fine),
                                     static_cast<const __nv_bfloat16*>(base),
                                     static_cast<__nv_bfloat16*>(out), C, Hc, Wc, H, W, sy, sx, TX);
      default:
        return cudaErrorNotSupported;
    }
  }
  const long long pixels = static_cast<long long>(N) * Hc * Wc;
  const dim3 grid(static_cast<unsigned>((pixels + 7) / 8));
  switch (dt) {
    case DType::F32:
      return launch_ex(upsample_adjoint_kernel<float>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const float*>(grad_fine), static_cast<const float*>(base),
                       static_cast<float*>(out), N, C, Hc, Wc, H, W, sy, sx);
    case DType::F16:
      return launch_ex(upsample_adjoint_kernel<__half>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __half*>(grad_fine), static_cast<const __half*>(base),
                       static_cast<__half*>(out), N, C, Hc, Wc, H, W, sy, sx);
    case DType::BF16:
      return launch_ex(upsample_adjoint_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, LaunchOpts(),
                       1, static_cast<const __nv_bfloat16*>(grad_fine),
                       static_cast<const __nv_bfloat16*>(base),
                       static_cast<__nv_bfloat16*>(out), N, C, Hc, Wc, H, W, sy, sx);
    default:
      return cudaErrorNotSupported;
  }
}

cudaError_t launch_p6_adjoint(DType dt, const void* grad_p6, void* grad_p5, int N, int C, int H5,
                              int W5, cudaStream_t s) {
  if (N <= 0 || C <= 0 || H5 <= 0 || W5 <= 0 || !grad_p6 || !grad_p5) return cudaErrorInvalidValue;
  if (!aligned16(grad_p6) || !aligned16(grad_p5)) return cudaErrorMisalignedAddress;
  if ((C * dtype_size(dt)) % 16 != 0) return cudaErrorInvalidValue;
  const long long work =
      static_cast<long long>(N) * ((H5 - 1) / 2 + 1) * ((W5 - 1) / 2 + 1) * C * dtype_size(dt) / 16;
  const dim3 grid(grid_for(work, 256));
  switch (dt) {
    case DType::F32:
      return launch_ex(p6_adjoint_kernel<float>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const float*>(grad_p6), static_cast<float*>(grad_p5), N, C, H5, W5);
    case DType::F16:
      return launch_ex(p6_adjoint_kernel<__half>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __half*>(grad_p6), static_cast<__half*>(grad_p5), N, C, H5,
                       W5);
    case DType::BF16:
      return launch_ex(p6_adjoint_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __nv_bfloat16*>(grad_p6),
                       static_cast<__nv_bfloat16*>(grad_p5), N, C, H5, W5);
    default:
      return cudaErrorNotSupported;
  }
}

cudaError_t launch_transpose_weights(DType dt, const void* w, void* wt, int rows, int cols,
                                     int out_rows, cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || out_rows < cols || !w || !wt) return cudaErrorInvalidValue;
  const dim3 grid(grid_for(static_cast<long long>(out_rows) * rows, 256));
  switch (dt) {
    case DType::F16:
      return launch_ex(transpose_kernel<__half>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __half*>(w), static_cast<__half*>(wt), rows, cols, out_rows);
    case DType::BF16:
      return launch_ex(transpose_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(wt), rows,
                       cols, out_rows);
    default:
      return cudaErrorNotSupported;
  }
}

cudaError_t launch_flip_conv3x3_weights(DType dt, const void* w_packed, void* w_flipped,
                                        cudaStream_t s) {
  if (!w_packed || !w_flipped) return cudaErrorInvalidValue;
  const dim3 grid(grid_for(256LL * 9 * 256, 256));
  switch (dt) {
    case DType::F16:
      return launch_ex(flip_conv3x3_kernel<__half>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __half*>(w_packed), static_cast<__half*>(w_flipped));
    case DType::BF16:
      return launch_ex(flip_conv3x3_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, LaunchOpts(), 1,
                       static_cast<const __nv_bfloat16*>(w_packed),
                       static_cast<__nv_bfloat16*>(w_flipped));
    default:
      return cudaErrorNotSupported;
  }
}

}  // namespace ufpn
