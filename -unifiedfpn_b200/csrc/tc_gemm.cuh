// tcgen05 / TMEM / TMA GEMM engine shared by the two tensor-core FPN kernels.
//
//   Lateral (mode 0):  M_l[p, o] = sum_c C_l[p, c] * Wlat[o, c] + b[o]
//                                  + bilinear(M_{l+1})[p, o]      (optional)
//     A = backbone feature C_l, NHWC viewed as [pixels, Cin] (K-major), 2-D TMA.
//     Reference semantics: lib/kernels/compute/fpn_compute_kernels.cu:127-230
//     (1x1 conv, out = sum_c in * W[o,c] + bias[o]) followed by the top-down
//     upsample + add of lib/core/fpn_engine.cu:274-313 (bilinear, half-pixel,
//     scale = in/out) fused into the epilogue.
//
//   Conv3x3 (mode 1): P_l[p, o] = sum_{tap, c} M_l[p + tap, c] * W3[o, tap, c] + b[o]
//     Implicit GEMM, K = 9 * 256.  A is fetched per (tap, 64-channel block) with a
//     4-D TMA box (64 ch, tile_w, tile_h, 1) whose origin is shifted by the tap;
//     TMA zero-fills out-of-image coordinates, which is exactly pad = 1.
//     The top level can also emit P6 = max_pool2d(P5, k=1, s=2) = P5[::2, ::2].
//
// One CTA per SM (persistent, static round-robin over tiles).  Tile = 128
// pixels x 256 output channels, fp32 accumulator in TMEM (two 256-column
// buffers so the epilogue of tile i overlaps the main loop of tile i+1).
//   warp 0      : TMA producer (one lane)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one lane)
//   warps 2..9  : epilogue (TMEM -> registers -> bias / upsample-add -> global)
#pragma once

#include "ptx.cuh"

namespace ufpn {

constexpr int kTcBlockM = 128;
constexpr int kTcBlockN = 256;
constexpr int kTcBlockK = 64;  // 16-bit elements in one 128-byte swizzled row
constexpr int kTcStages = 4;
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 64 + kTcEpiWarps * 32;
constexpr int kTcAStage = kTcBlockM * 128;
constexpr int kTcBStage = kTcBlockN * 128;
constexpr int kTcTmemCols = 2 * kTcBlockN;
constexpr int kTcSmemBytes = kTcStages * (kTcAStage + kTcBStage) + 1024 /*align*/ + 256;

struct TcGemmArgs {
  int num_tiles;
  int num_kb;      // 64-wide K blocks per tile
  int M;           // lateral: total pixels N*H*W
  int N_img, H, W;
  int tile_w, tile_h, tiles_x, tiles_y;  // conv3x3 spatial tiling (tile_w * tile_h = 128)
  int cin_blocks;  // conv3x3: input channels / 64
  const float* bias;    // [256] fp32
  void* out;            // NHWC [pixels][256]
  const void* coarse;   // lateral: NHWC [N][Hc][Wc][256] merged map of the coarser level, or null
  int Hc, Wc;
  float scale_y, scale_x;  // Hc / H, Wc / W
  void* p6;             // conv3x3 top level: NHWC [N][H6][W6][256], or null
  int H6, W6;
  int* status;          // device status word (0 = ok)
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

template <int kMode>
__device__ __forceinline__ void tc_tile_origin(const TcGemmArgs& a, int tile, int& m0, int& n,
                                               int& x0, int& y0) {
  if constexpr (kMode == 0) {
    m0 = tile * kTcBlockM;
    n = x0 = y0 = 0;
  } else {
    const int tx = tile % a.tiles_x;
    const int t2 = tile / a.tiles_x;
    const int ty = t2 % a.tiles_y;
    n = t2 / a.tiles_y;
    x0 = tx * a.tile_w;
    y0 = ty * a.tile_h;
    m0 = 0;
  }
}

template <int kMode, typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, const TcGemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kTcStages * kTcAStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_b + kTcStages * kTcBStage);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kTcStages;
  uint64_t* accf_bar = bars + 2 * kTcStages;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], kTcEpiWarps * 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
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
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        int m0, n, x0, y0;
        tc_tile_origin<kMode>(args, tile, m0, n, x0, y0);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kTcAStage + kTcBStage);
          if constexpr (kMode == 0) {
            tma_load_2d(smem_a + stage * kTcAStage, &map_a, &full_bar[stage], kb * kTcBlockK, m0,
                        kPolicyEvictFirst);
          } else {
            const int tap = kb / args.cin_blocks;
            const int cb = kb - tap * args.cin_blocks;
            const int dy = tap / 3 - 1;
            const int dx = tap % 3 - 1;
            tma_load_4d(smem_a + stage * kTcAStage, &map_a, &full_bar[stage], cb * kTcBlockK,
                        x0 + dx, y0 + dy, n, kPolicyEvictLast);
          }
          tma_load_2d(smem_b + stage * kTcBStage, &map_b, &full_bar[stage], kb * kTcBlockK, 0,
                      kPolicyEvictLast);
          ++issued;
          if (++stage == kTcStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Teardown: make sure every copy this thread issued has landed before the
      // CTA can exit (matters only when another role aborted early).
      for (int i = 0; i < kTcStages && i < issued; ++i) {
        if (--stage < 0) {
          stage = kTcStages - 1;
          phase ^= 1u;
        }
        mbar_wait_drain(&full_bar[stage], phase);
      }
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
          if (++stage == kTcStages) {
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
    const int quarter = warp & 3;  // TMEM lanes this warp may access: 32*quarter..+31
    const int chalf = ew >> 2;     // which 128 output channels this warp handles
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
      bool ok =
          mbar_wait(&accf_bar[acc], acc_phase, abort_flag, args.status, kDevTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();

      int m0, n, x0, y0;
      tc_tile_origin<kMode>(args, tile, m0, n, x0, y0);
      bool valid;
      long long pix;  // output pixel index (n*H + y)*W + x
      int py = 0, px = 0;
      if constexpr (kMode == 0) {
        pix = static_cast<long long>(m0) + row;
        valid = pix < args.M;
        const int hw = args.H * args.W;
        const int rem = static_cast<int>(pix % hw);
        n = static_cast<int>(pix / hw);
        py = rem / args.W;
        px = rem - py * args.W;
      } else {
        py = y0 + row / args.tile_w;
        px = x0 + row % args.tile_w;
        valid = (py < args.H) && (px < args.W);
        pix = (static_cast<long long>(n) * args.H + py) * args.W + px;
      }

      // Bilinear source corners in the coarser merged map (lateral mode).
      const uint8_t* c00 = nullptr;
      const uint8_t* c01 = nullptr;
      const uint8_t* c10 = nullptr;
      const uint8_t* c11 = nullptr;
      float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
      const bool fuse_up = (kMode == 0) && (args.coarse != nullptr);
      if (fuse_up) {
        float sy = (static_cast<float>(py) + 0.5f) * args.scale_y - 0.5f;
        float sx = (static_cast<float>(px) + 0.5f) * args.scale_x - 0.5f;
        sy = fminf(fmaxf(sy, 0.f), static_cast<float>(args.Hc - 1));
        sx = fminf(fmaxf(sx, 0.f), static_cast<float>(args.Wc - 1));
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
        const size_t rowb = static_cast<size_t>(kTcBlockN) * sizeof(T);
        const uint8_t* cbase = static_cast<const uint8_t*>(args.coarse) +
                               static_cast<size_t>(n) * args.Hc * args.Wc * rowb;
        c00 = cbase + (static_cast<size_t>(ya) * args.Wc + xa) * rowb;
        c01 = cbase + (static_cast<size_t>(ya) * args.Wc + xb) * rowb;
        c10 = cbase + (static_cast<size_t>(yb) * args.Wc + xa) * rowb;
        c11 = cbase + (static_cast<size_t>(yb) * args.Wc + xb) * rowb;
      }
      const bool emit_p6 =
          (kMode == 1) && (args.p6 != nullptr) && valid && ((py & 1) == 0) && ((px & 1) == 0);
      uint8_t* out_row =
          static_cast<uint8_t*>(args.out) + static_cast<size_t>(pix) * kTcBlockN * sizeof(T);
      uint8_t* p6_row = nullptr;
      if (emit_p6) {
        const size_t p6pix =
            (static_cast<size_t>(n) * args.H6 + (py >> 1)) * args.W6 + (px >> 1);
        p6_row = static_cast<uint8_t*>(args.p6) + p6pix * kTcBlockN * sizeof(T);
      }

#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col = chalf * 128 + c * 32;
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(tmem_base + static_cast<uint32_t>(acc * kTcBlockN + col) +
                      (static_cast<uint32_t>(quarter * 32) << 16),
                  r);
        tmem_wait_ld();
        float v[32];
        const float4* b4 = reinterpret_cast<const float4*>(args.bias + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 bb = __ldg(b4 + i);
          v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + bb.x;
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
        }
        if (fuse_up && valid) {
          const size_t off = static_cast<size_t>(col) * sizeof(T);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(c00 + off) + j);
            const uint4 b = __ldg(reinterpret_cast<const uint4*>(c01 + off) + j);
            const uint4 cc = __ldg(reinterpret_cast<const uint4*>(c10 + off) + j);
            const uint4 d = __ldg(reinterpret_cast<const uint4*>(c11 + off) + j);
            const uint32_t au[4] = {a.x, a.y, a.z, a.w};
            const uint32_t bu[4] = {b.x, b.y, b.z, b.w};
            const uint32_t cu[4] = {cc.x, cc.y, cc.z, cc.w};
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
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(out_row + static_cast<size_t>(col) * sizeof(T));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 o;
            o.x = Pack<T>::pack(v[8 * j + 0], v[8 * j + 1]);
            o.y = Pack<T>::pack(v[8 * j + 2], v[8 * j + 3]);
            o.z = Pack<T>::pack(v[8 * j + 4], v[8 * j + 5]);
            o.w = Pack<T>::pack(v[8 * j + 6], v[8 * j + 7]);
            dst[j] = o;
            if (emit_p6)
              reinterpret_cast<uint4*>(p6_row + static_cast<size_t>(col) * sizeof(T))[j] = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
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
