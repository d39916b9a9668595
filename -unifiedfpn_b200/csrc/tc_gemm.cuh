// tcgen05 / TMEM / TMA implicit-GEMM engine shared by the two tensor-core FPN kernels.
//
//   Lateral (mode 0):  M_l[p, o] = sum_c C_l[p, c] * Wlat[o, c] + b[o]
//                                  + bilinear(M_{l+1})[p, o]      (optional)
//     Reference semantics: lib/kernels/compute/fpn_compute_kernels.cu:127-230
//     (1x1 conv, out = sum_c in * W[o,c] + bias[o]) followed by the top-down
//     upsample + add of lib/core/fpn_engine.cu:274-313 (bilinear, half-pixel,
//     scale = in/out), fused into the epilogue.
//
//   Conv3x3 (mode 1): P_l[p, o] = sum_{tap, c} M_l[p + tap, c] * W3[o, tap, c] + b[o]
//     K = 9 * 256.  The top level also emits P6 = max_pool2d(P5, k=1, s=2) = P5[::2, ::2].
//
// Both modes tile the output as tile_h x tile_w = 128 pixels of one image by all
// 256 output channels.  A (activations, NHWC) arrives through a 4-D TMA box
// (64 ch, tile_w, tile_h, 1) whose origin is shifted by the tap; TMA zero-fills
// coordinates outside the image, which is exactly the 3x3 conv's pad = 1 (and the
// ragged right/bottom tiles of both modes).  B (weights, [256][K] K-major) arrives
// as a 2-D box (64, 256).  Operands use the 128-byte swizzle.
//
// The fp32 accumulator lives in TMEM (two 256-column buffers, so the epilogue of
// tile i overlaps the main loop of tile i+1).  The epilogue reads TMEM, adds the
// bias (and, for the lateral, the bilinear sample of the coarser merged map,
// staged per tile in shared memory by TMA), converts, writes a 128-byte
// swizzled staging tile and stores it with a TMA tensor store (which also clips
// ragged tiles).
//
// One CTA per SM (persistent, static round-robin over tiles):
//   warp 0      : TMA producer (one lane)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one lane)
//   warps 2..9  : epilogue; warp w may access TMEM lanes 32*(w%4)..+31, and
//                 handles 128 of the 256 output channels ((w-2)/4 selects which)
#pragma once

#include "ptx.cuh"

namespace ufpn {

constexpr int kTcBlockM = 128;
constexpr int kTcBlockN = 256;
constexpr int kTcBlockK = 64;  // 16-bit elements in one 128-byte swizzled row
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 64 + kTcEpiWarps * 32;
constexpr int kTcAStage = kTcBlockM * 128;
constexpr int kTcBStage = kTcBlockN * 128;
constexpr int kTcTmemCols = 2 * kTcBlockN;
constexpr int kTcStagingPerWarp = 32 * 128;  // 32 rows x 64 channels (bf16/fp16)
constexpr int kTcCoarseMaxPix = 80;          // coarse pixels per staged 64-channel block

template <int kMode>
struct TcCfg {
  static constexpr int kStages = kMode == 0 ? 3 : 4;
  static constexpr int kCoarseBlk = kMode == 0 ? kTcCoarseMaxPix * 128 : 0;  // 1024-aligned
  static constexpr int kOffB = kStages * kTcAStage;
  static constexpr int kOffStaging = kOffB + kStages * kTcBStage;
  static constexpr int kOffCoarse = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kOffBars = kOffCoarse + 4 * kCoarseBlk;
  static constexpr int kSmemBytes = kOffBars + 256 + 1024 /*alignment slack*/;
};
static_assert(TcCfg<0>::kSmemBytes <= 232448, "lateral smem");
static_assert(TcCfg<1>::kSmemBytes <= 232448, "conv smem");

struct TcGemmArgs {
  int num_tiles;
  int num_kb;      // taps * cin_blocks
  int cin_blocks;  // ceil(Cin / 64)
  int N_img, H, W;
  int tile_w, tile_h, tiles_x, tiles_y;
  const float* bias;  // [256] fp32
  // lateral: coarser merged map M_{l+1}, NHWC [N][Hc][Wc][256]
  const void* coarse;  // null = no top-down add
  int Hc, Wc;
  float scale_y, scale_x;  // Hc / H, Wc / W
  int cbox_w, cbox_h;      // staged coarse box (0 = read the coarse map from global memory)
  // conv3x3 top level: P6 NHWC [N][H6][W6][256], or null
  void* p6;
  int H6, W6;
  int* status;  // device status word (0 = ok)
};

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t u) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(v);
  }
};
template <>
struct Pack<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t u) {
    __half2 v = *reinterpret_cast<__half2*>(&u);
    return __half22float2(v);
  }
};

__device__ __forceinline__ void tc_tile_origin(const TcGemmArgs& a, int tile, int& n, int& x0,
                                               int& y0) {
  const int tx = tile % a.tiles_x;
  const int t2 = tile / a.tiles_x;
  const int ty = t2 % a.tiles_y;
  n = t2 / a.tiles_y;
  x0 = tx * a.tile_w;
  y0 = ty * a.tile_h;
}

// Bilinear source index along one axis (half-pixel, clamped), identical on the
// producer side (coarse box origin) and in the epilogue.
__device__ __forceinline__ float tc_src(int o, float scale, int in) {
  const float s = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(o), 0.5f), scale), 0.5f);
  return fminf(fmaxf(s, 0.f), static_cast<float>(in - 1));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

template <int kMode, typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_out,
                       const __grid_constant__ CUtensorMap map_coarse, const TcGemmArgs args) {
  using Cfg = TcCfg<kMode>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + Cfg::kOffB;
  uint8_t* smem_stage = smem + Cfg::kOffStaging;
  uint8_t* smem_coarse = smem + Cfg::kOffCoarse;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* accf_bar = bars + 2 * S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint64_t* cfull_bar = done_bar + 1;
  uint64_t* cempty_bar = cfull_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cempty_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool coarse_smem = (kMode == 0) && args.coarse != nullptr && args.cbox_w > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], kTcEpiWarps * 32);
    }
    mbar_init(done_bar, 1);
    mbar_init(cfull_bar, 1);
    mbar_init(cempty_bar, kTcEpiWarps * 32);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    prefetch_tmap(&map_out);
    if (coarse_smem) prefetch_tmap(&map_coarse);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t cphase = 0;
      int issued = 0;
      bool ok = true;
      const uint32_t coarse_bytes = static_cast<uint32_t>(args.cbox_w * args.cbox_h * 128 * 4);
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        int n, x0, y0;
        tc_tile_origin(args, tile, n, x0, y0);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kTcAStage + kTcBStage);
          int dy = 0, dx = 0, cb = kb;
          if constexpr (kMode == 1) {
            const int tap = kb / args.cin_blocks;
            cb = kb - tap * args.cin_blocks;
            dy = tap / 3 - 1;
            dx = tap % 3 - 1;
          }
          tma_load_4d(smem_a + stage * kTcAStage, &map_a, &full_bar[stage], cb * kTcBlockK,
                      x0 + dx, y0 + dy, n, kMode == 0 ? kPolicyEvictFirst : kPolicyEvictLast);
          tma_load_2d(smem_b + stage * kTcBStage, &map_b, &full_bar[stage], kb * kTcBlockK, 0,
                      kPolicyEvictLast);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (coarse_smem) {
          // Coarse box for this tile, after its main-loop loads so those are not
          // held up by the previous tile's epilogue still reading the buffer.
          if (!mbar_wait(cempty_bar, cphase ^ 1u, abort_flag, args.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const int cy = static_cast<int>(tc_src(y0, args.scale_y, args.Hc));
          const int cx = static_cast<int>(tc_src(x0, args.scale_x, args.Wc));
          mbar_arrive_expect_tx(cfull_bar, coarse_bytes);
          for (int b = 0; b < 4; ++b)
            tma_load_4d(smem_coarse + b * Cfg::kCoarseBlk, &map_coarse, cfull_bar, b * 64, cx, cy,
                        n, kPolicyEvictLast);
          cphase ^= 1u;
        }
      }
      // Teardown: every copy this thread issued must land before the CTA exits
      // (matters only when another role aborted early).
      for (int i = 0; i < S && i < issued; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait_drain(&full_bar[stage], phase);
      }
      if (coarse_smem && issued > 0) mbar_wait_drain(cfull_bar, cphase ^ 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(kTcBlockM, kTcBlockN, Pack<T>::kFmt, Pack<T>::kFmt);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(smem_a + stage * kTcAStage));
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kTcBStage));
#pragma unroll
          for (int k = 0; k < kTcBlockK / 16; ++k) {
            // +32 bytes along K per 16-element MMA step (encoded >> 4).
            tc_mma_f16(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Wait for every MMA issued by this thread before TMEM can be released.
      tc_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter..+31
    const int chalf = ew >> 2;     // output channels chalf*128 .. +127
    const int row = quarter * 32 + lane;
    const int tw = args.tile_w;
    const uint32_t stage_addr = smem_u32(smem_stage + ew * kTcStagingPerWarp);
    const uint32_t coarse_addr = smem_u32(smem_coarse);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t cphase = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
      bool ok =
          mbar_wait(&accf_bar[acc], acc_phase, abort_flag, args.status, kDevTimeoutEpilogue);
      if (coarse_smem && ok)
        ok = mbar_wait(cfull_bar, cphase, abort_flag, args.status, kDevTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();

      int n, x0, y0;
      tc_tile_origin(args, tile, n, x0, y0);
      const int py = y0 + row / tw;
      const int px = x0 + row % tw;
      const bool valid = (py < args.H) && (px < args.W);

      // Bilinear corners in the coarser merged map (lateral mode).
      float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
      int r00 = 0, r01 = 0, r10 = 0, r11 = 0;  // staged-box rows
      bool corners_staged = false;
      const uint8_t* g00 = nullptr;
      const uint8_t* g01 = nullptr;
      const uint8_t* g10 = nullptr;
      const uint8_t* g11 = nullptr;
      if (kMode == 0 && args.coarse != nullptr) {
        const float sy = tc_src(min(py, args.H - 1), args.scale_y, args.Hc);
        const float sx = tc_src(min(px, args.W - 1), args.scale_x, args.Wc);
        const int ya = static_cast<int>(sy);
        const int xa = static_cast<int>(sx);
        const int yb = min(ya + 1, args.Hc - 1);
        const int xb = min(xa + 1, args.Wc - 1);
        const float wy = sy - static_cast<float>(ya);
        const float wx = sx - static_cast<float>(xa);
        w00 = (1.f - wy) * (1.f - wx);
        w01 = (1.f - wy) * wx;
        w10 = wy * (1.f - wx);
        w11 = wy * wx;
        if (coarse_smem) {
          const int cy0 = static_cast<int>(tc_src(y0, args.scale_y, args.Hc));
          const int cx0 = static_cast<int>(tc_src(x0, args.scale_x, args.Wc));
          corners_staged = (ya - cy0) >= 0 && (yb - cy0) < args.cbox_h && (xa - cx0) >= 0 &&
                           (xb - cx0) < args.cbox_w;
          r00 = (ya - cy0) * args.cbox_w + (xa - cx0);
          r01 = (ya - cy0) * args.cbox_w + (xb - cx0);
          r10 = (yb - cy0) * args.cbox_w + (xa - cx0);
          r11 = (yb - cy0) * args.cbox_w + (xb - cx0);
        }
        if (!corners_staged) {
          const size_t rowb = static_cast<size_t>(kTcBlockN) * sizeof(T);
          const uint8_t* cbase = static_cast<const uint8_t*>(args.coarse) +
                                 static_cast<size_t>(n) * args.Hc * args.Wc * rowb;
          g00 = cbase + (static_cast<size_t>(ya) * args.Wc + xa) * rowb;
          g01 = cbase + (static_cast<size_t>(ya) * args.Wc + xb) * rowb;
          g10 = cbase + (static_cast<size_t>(yb) * args.Wc + xa) * rowb;
          g11 = cbase + (static_cast<size_t>(yb) * args.Wc + xb) * rowb;
        }
      }
      const bool emit_p6 =
          (kMode == 1) && (args.p6 != nullptr) && valid && ((py & 1) == 0) && ((px & 1) == 0);
      uint8_t* p6_row = nullptr;
      if (emit_p6) {
        const size_t p6pix =
            (static_cast<size_t>(n) * args.H6 + (py >> 1)) * args.W6 + (px >> 1);
        p6_row = static_cast<uint8_t*>(args.p6) + p6pix * kTcBlockN * sizeof(T);
      }
      // Output box of this warp's 32 rows.
      const int wrow0 = quarter * 32;
      const int ox = x0 + (wrow0 % tw);
      const int oy = y0 + wrow0 / tw;

#pragma unroll 1
      for (int step = 0; step < 2; ++step) {
        const int col0 = chalf * 128 + step * 64;
        uint32_t r[64];
        __syncwarp();
        const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * kTcBlockN + col0) +
                               (static_cast<uint32_t>(quarter * 32) << 16);
        tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_wait_ld();
        if (step == 1) {
          // All of this tile's accumulator columns for this warp are in registers:
          // hand the TMEM buffer back to the MMA warp before the memory work.
          tc_fence_before();
          mbar_arrive(&acce_bar[acc]);
        }
        float v[64];
        const float4* b4 = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 bb = __ldg(b4 + i);
          v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + bb.x;
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
        }
        if (kMode == 0 && args.coarse != nullptr) {
          const int blk = col0 >> 6;  // 64-channel block of the staged coarse box
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 a, b, c, d;
            if (corners_staged) {
              const uint32_t base = coarse_addr + blk * Cfg::kCoarseBlk;
              a = ld_shared_v4(base + r00 * 128 + ((j ^ (r00 & 7)) << 4));
              b = ld_shared_v4(base + r01 * 128 + ((j ^ (r01 & 7)) << 4));
              c = ld_shared_v4(base + r10 * 128 + ((j ^ (r10 & 7)) << 4));
              d = ld_shared_v4(base + r11 * 128 + ((j ^ (r11 & 7)) << 4));
            } else {
              const size_t off = static_cast<size_t>(col0) * sizeof(T);
              a = __ldg(reinterpret_cast<const uint4*>(g00 + off) + j);
              b = __ldg(reinterpret_cast<const uint4*>(g01 + off) + j);
              c = __ldg(reinterpret_cast<const uint4*>(g10 + off) + j);
              d = __ldg(reinterpret_cast<const uint4*>(g11 + off) + j);
            }
            const uint32_t au[4] = {a.x, a.y, a.z, a.w};
            const uint32_t bu[4] = {b.x, b.y, b.z, b.w};
            const uint32_t cu[4] = {c.x, c.y, c.z, c.w};
            const uint32_t du[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 fa = Pack<T>::unpack(au[e]);
              const float2 fb = Pack<T>::unpack(bu[e]);
              const float2 fc = Pack<T>::unpack(cu[e]);
              const float2 fd = Pack<T>::unpack(du[e]);
              v[8 * j + 2 * e + 0] += w00 * fa.x + w01 * fb.x + w10 * fc.x + w11 * fd.x;
              v[8 * j + 2 * e + 1] += w00 * fa.y + w01 * fb.y + w10 * fc.y + w11 * fd.y;
            }
          }
        }
        // The previous TMA store from this warp's staging buffer must have read it.
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 o;
          o.x = Pack<T>::pack(v[8 * j + 0], v[8 * j + 1]);
          o.y = Pack<T>::pack(v[8 * j + 2], v[8 * j + 3]);
          o.z = Pack<T>::pack(v[8 * j + 4], v[8 * j + 5]);
          o.w = Pack<T>::pack(v[8 * j + 6], v[8 * j + 7]);
          st_shared_v4(stage_addr + lane * 128 + ((j ^ (lane & 7)) << 4), o);
          if (emit_p6)
            reinterpret_cast<uint4*>(p6_row + static_cast<size_t>(col0) * sizeof(T))[j] = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_4d(&map_out, smem_stage + ew * kTcStagingPerWarp, col0, ox, oy, n);
          bulk_commit_group();
        }
      }
      if (coarse_smem) mbar_arrive(cempty_bar);
      if (coarse_smem) cphase ^= 1u;
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

}  // namespace ufpn
