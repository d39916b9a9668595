// Bandwidth-bound FPN kernels (upsample-add, P6, layout conversion, weight
// packing) and the fp32 CUDA-core path (1x1 lateral + fused upsample-add, 3x3).
//
// Bilinear semantics follow the reference's host implementation
// benchmarks/upsample_benchmark.cu:24-108 and its device helper
// lib/kernels/compute/fpn_compute_kernels.cu:21-59: half-pixel source
// coordinate (o + 0.5) * in/out - 0.5 (or o * (in-1)/(out-1) with
// align_corners), clamped to [0, in-1], y1 = min(y0+1, in-1), weights
// (1-wy)(1-wx), (1-wy)wx, wy(1-wx), wy*wx.
#include "activation.cuh"
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace ufpn {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

struct BilinearTap {
  int y0, y1, x0, x1;
  float w00, w01, w10, w11;
};

__device__ __forceinline__ float src_coord(int o, int in, int out, float scale, int align_corners) {
  float s;
  if (align_corners) {
    s = out > 1 ? static_cast<float>(o) * scale : 0.f;
  } else {
    s = (static_cast<float>(o) + 0.5f) * scale - 0.5f;
  }
  return fminf(fmaxf(s, 0.f), static_cast<float>(in - 1));
}

__device__ __forceinline__ BilinearTap make_tap(int y, int x, int Hc, int Wc, int H, int W,
                                                float sy_scale, float sx_scale, int ac) {
  const float sy = src_coord(y, Hc, H, sy_scale, ac);
  const float sx = src_coord(x, Wc, W, sx_scale, ac);
  BilinearTap t;
  t.y0 = static_cast<int>(sy);
  t.x0 = static_cast<int>(sx);
  t.y1 = min(t.y0 + 1, Hc - 1);
  t.x1 = min(t.x0 + 1, Wc - 1);
  const float wy = sy - static_cast<float>(t.y0);
  const float wx = sx - static_cast<float>(t.x0);
  t.w00 = (1.f - wy) * (1.f - wx);
  t.w01 = (1.f - wy) * wx;
  t.w10 = wy * (1.f - wx);
  t.w11 = wy * wx;
  return t;
}

// Vector of 16 bytes viewed as elements of T.
template <typename T>
struct Vec16 {
  static constexpr int kN = 16 / sizeof(T);
  union {
    uint4 u;
    T e[kN];
  };
};

// Two 16-bit values in one 32-bit word <-> two floats, with one packed round-to-nearest
// conversion per pair (the same rounding as two scalar conversions).
template <typename T>
struct Pair16;
template <>
struct Pair16<__nv_bfloat16> {
  __device__ static __forceinline__ float2 unpack(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  // fp32 bits of the larger of two 16-bit magnitudes packed in m (|x| bits, order-preserving)
  __device__ static __forceinline__ uint32_t mag_to_f32_bits(uint32_t m) {
    return max(m & 0xFFFFu, m >> 16) << 16;
  }
};
template <>
struct Pair16<__half> {
  __device__ static __forceinline__ float2 unpack(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ uint32_t mag_to_f32_bits(uint32_t m) {
    const unsigned short mx = static_cast<unsigned short>(max(m & 0xFFFFu, m >> 16));
    return __float_as_uint(__half2float(__ushort_as_half(mx)));
  }
};

// |v| as fp32 bits (orders like an unsigned integer).
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// Warp-reduced atomicMax that skips the atomic when the published value is already as
// large (most warps, once the running maximum has settled), so one hot address sees
// few atomics.  Every lane of the warp must call it.
__device__ __forceinline__ void publish_amax(unsigned* amax, unsigned bits) {
  bits = __reduce_max_sync(0xffffffffu, bits);
  if ((threadIdx.x & 31) == 0 && bits > *reinterpret_cast<volatile unsigned*>(amax))
    atomicMax(amax, bits);
}
// Block-wide version (every thread of the block must call it; red: blockDim/32 words of
// shared memory): one guarded atomic per block.
__device__ __forceinline__ void publish_amax_block(unsigned* amax, unsigned bits,
                                                   unsigned* red) {
  bits = __reduce_max_sync(0xffffffffu, bits);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = bits;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned m = 0;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) m = max(m, red[i]);
    if (m > *reinterpret_cast<volatile unsigned*>(amax)) atomicMax(amax, m);
  }
  __syncthreads();
}

// ---------------------------------------------------------------- NHWC upsample-add
// out[n,y,x,c] = lat[n,y,x,c] (or 0) + bilinear(coarse)[n,y,x,c].
// A block takes one output row segment of 32 pixels: the row's vertical taps are
// computed once per block; warp w takes pixels x0 + 4w .. x0 + 4w + 3 and first issues
// all of their loads (4 coarse corners + the lateral, 16 bytes per lane each, every one a
// contiguous 512-byte segment per warp for C = 256 16-bit channels) and only then does
// the math and the stores, so each warp keeps 20 independent loads in flight and the
// per-pixel index arithmetic is a handful of 32-bit operations.  `out` may alias `lat`
// (in-place merge M_l = L_l + up(M_{l+1})): every element is read, then written, by the
// same lane.
constexpr int kUpPix = 4;  // pixels per warp
template <typename T, bool kVec>
__global__ void __launch_bounds__(256) upsample_add_nhwc_kernel(
    const T* __restrict__ coarse, const T* lat, T* out, int N, int C, int Hc, int Wc, int H,
    int W, float sy_scale, float sx_scale, int ac) {
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  constexpr int V = kVec ? Vec16<T>::kN : 1;
  const int cvs = C / V;  // channel vectors per pixel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int segs = (W + 8 * kUpPix - 1) / (8 * kUpPix);
  const int units = N * H * segs;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int r = u / segs;
    const int xb = (u - r * segs) * (8 * kUpPix) + warp * kUpPix;
    if (xb >= W) continue;
    const int n = r / H;
    const int y = r - n * H;
    const float sy = src_coord(y, Hc, H, sy_scale, ac);
    const int y0 = static_cast<int>(sy);
    const int y1 = min(y0 + 1, Hc - 1);
    const float wy = sy - static_cast<float>(y0);
    const T* c0 = coarse + (static_cast<size_t>(n) * Hc + y0) * Wc * C;
    const T* c1 = coarse + (static_cast<size_t>(n) * Hc + y1) * Wc * C;
    T* orow = out + static_cast<size_t>(r) * W * C;
    const T* lrow = lat ? lat + static_cast<size_t>(r) * W * C : nullptr;
    for (int cv = lane; cv < cvs; cv += 32) {
      const int e0 = cv * V;
      if constexpr (kVec) {
        Vec16<T> a[kUpPix], b[kUpPix], c[kUpPix], d[kUpPix], l[kUpPix];
        float wx[kUpPix];
#pragma unroll
        for (int k = 0; k < kUpPix; ++k) {
          const int x = min(xb + k, W - 1);  // clamped duplicates are not stored
          const float sx = src_coord(x, Wc, W, sx_scale, ac);
          const int x0 = static_cast<int>(sx);
          const int x1 = min(x0 + 1, Wc - 1);
          wx[k] = sx - static_cast<float>(x0);
          a[k].u = __ldg(reinterpret_cast<const uint4*>(c0 + static_cast<size_t>(x0) * C + e0));
          b[k].u = __ldg(reinterpret_cast<const uint4*>(c0 + static_cast<size_t>(x1) * C + e0));
          c[k].u = __ldg(reinterpret_cast<const uint4*>(c1 + static_cast<size_t>(x0) * C + e0));
          d[k].u = __ldg(reinterpret_cast<const uint4*>(c1 + static_cast<size_t>(x1) * C + e0));
          if (lrow) l[k].u = *reinterpret_cast<const uint4*>(lrow + static_cast<size_t>(x) * C + e0);
        }
#pragma unroll
        for (int k = 0; k < kUpPix; ++k) {
          if (xb + k >= W) break;
          const float w00 = (1.f - wy) * (1.f - wx[k]), w01 = (1.f - wy) * wx[k];
          const float w10 = wy * (1.f - wx[k]), w11 = wy * wx[k];
          Vec16<T> o;
#pragma unroll
          for (int e = 0; e < V; ++e) {
            float v = lrow ? to_f(l[k].e[e]) : 0.f;
            v = fmaf(to_f(a[k].e[e]), w00, v);
            v = fmaf(to_f(b[k].e[e]), w01, v);
            v = fmaf(to_f(c[k].e[e]), w10, v);
            v = fmaf(to_f(d[k].e[e]), w11, v);
            o.e[e] = from_f<T>(v);
          }
          *reinterpret_cast<uint4*>(orow + static_cast<size_t>(xb + k) * C + e0) = o.u;
        }
      } else {
        for (int k = 0; k < kUpPix && xb + k < W; ++k) {
          const int x = xb + k;
          const float sx = src_coord(x, Wc, W, sx_scale, ac);
          const int x0 = static_cast<int>(sx);
          const int x1 = min(x0 + 1, Wc - 1);
          const float wx = sx - static_cast<float>(x0);
          float v = lrow ? to_f(lrow[static_cast<size_t>(x) * C + e0]) : 0.f;
          v = fmaf(to_f(c0[static_cast<size_t>(x0) * C + e0]), (1.f - wy) * (1.f - wx), v);
          v = fmaf(to_f(c0[static_cast<size_t>(x1) * C + e0]), (1.f - wy) * wx, v);
          v = fmaf(to_f(c1[static_cast<size_t>(x0) * C + e0]), wy * (1.f - wx), v);
          v = fmaf(to_f(c1[static_cast<size_t>(x1) * C + e0]), wy * wx, v);
          orow[static_cast<size_t>(x) * C + e0] = from_f<T>(v);
        }
      }
    }
  }
}

// Fast path for 512-byte pixels (256 channels of a 16-bit type -- every FPN map).  A unit is
// 8 consecutive pixels of one output row, one per warp, lane = 16 bytes (8 channels).  A
// block takes a contiguous run of units and walks it kU units at a time, issuing the five
// 16-byte loads of every unit of the batch (lateral + 4 coarse corners) before any math, so
// each thread keeps 5 * kU independent loads in flight; the grid is sized to the blocks that
// are resident at once.  `out` may alias `lat`: each lane reads a lateral vector before it
// writes that vector, and the pixels of a batch are distinct.
// amax (optional): amax[n] = atomicMax of |out| of image n as fp32 bits (for a following
// per-image e4m3 quantisation), one block-reduced publication per image a run touches.
// out_s (optional): a second copy of out with channel c multiplied by
// 1 / (scale_a[0] * scale_w[c]) (the e4m3 P2 lateral adds this copy through its tensor-core
// top-down k-block before it scales its accumulator by the same factor).
// interleave (maps larger than L2): the blocks take chunks of kInterChunk units in turn
// (chunk blockIdx.x, + gridDim.x, ...) instead of one run each, so the resident blocks work
// on a band of a few dozen rows at a time and each coarse row is read from HBM about once
// (with runs, the blocks together touched the whole coarse map at every moment: a 498 MB
// merge read its 124 MB coarse map from HBM ~2.6 times).  Units of a chunk are walked as in
// a run (one division per chunk); batches of kU units interleaved across blocks were slower.
constexpr int kInterChunk = 16;
template <typename T, int kU>
__global__ void __launch_bounds__(256, 3) upsample_add_px512_kernel(
    const T* __restrict__ coarse, const T* lat, T* out, int N, int Hc, int Wc, int H, int W,
    int chunks, float sy_scale, float sx_scale, int ac, unsigned* amax, T* out_s,
    const float* scale_a, const float* scale_w, int units_per_block, int interleave) {
  static_assert(sizeof(T) == 2, "16-bit types");
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  __shared__ unsigned red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float inv[8];
  if (out_s) {
    const float sa = __ldg(scale_a);
#pragma unroll
    for (int e = 0; e < 8; ++e) inv[e] = __frcp_rn(sa * __ldg(scale_w + lane * 8 + e));
  }
  unsigned m = 0;
  int m_img = -1;  // image the running maximum m belongs to (block-uniform)
  const long long total = static_cast<long long>(N) * H * chunks;
  // one run of units_per_block units, or chunks of kInterChunk units every gridDim.x chunks
  const long long run = interleave ? kInterChunk : units_per_block;
  const long long rstep = interleave ? static_cast<long long>(gridDim.x) * kInterChunk : total;
  for (long long u0 = static_cast<long long>(blockIdx.x) * run; u0 < total; u0 += rstep) {
    const long long u1 = min(total, u0 + run);
    // position of the run's first unit (the only divisions); later units step from it
    int r = static_cast<int>(u0 / chunks);  // output row over all images
    int ci = static_cast<int>(u0 - static_cast<long long>(r) * chunks);
    int n = r / H;
    int y = r - n * H;
    for (long long ub = u0; ub < u1; ub += kU) {
      Vec16<T> l[kU], a[kU], b[kU], c[kU], d[kU];
      float wy[kU], wx[kU];
      size_t io[kU];
      int img[kU];
      bool live[kU];
#pragma unroll
      for (int k = 0; k < kU; ++k) {
        const bool in_run = ub + k < u1;
        const int x = ci * 8 + warp;
        live[k] = in_run && x < W;
        img[k] = n;
        const int xc = min(x, W - 1);
        const int rk = r, yk = y, nk = n;
        if (++ci == chunks) {  // step to the next unit
          ci = 0;
          ++r;
          if (++y == H) {
            y = 0;
            ++n;
          }
        }
        if (!in_run) continue;  // past the run: nothing loaded, nothing stored
        const float sy = src_coord(yk, Hc, H, sy_scale, ac);
        const float sx = src_coord(xc, Wc, W, sx_scale, ac);
        const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
        const int y1 = min(y0 + 1, Hc - 1), x1 = min(x0 + 1, Wc - 1);
        wy[k] = sy - static_cast<float>(y0);
        wx[k] = sx - static_cast<float>(x0);
        io[k] = (static_cast<size_t>(rk) * W + xc) * 256 + lane * 8;
        const T* cb = coarse + static_cast<size_t>(nk) * Hc * Wc * 256 + lane * 8;
        if (lat) l[k].u = *reinterpret_cast<const uint4*>(lat + io[k]);
        a[k].u = __ldg(reinterpret_cast<const uint4*>(cb + (static_cast<size_t>(y0) * Wc + x0) * 256));
        b[k].u = __ldg(reinterpret_cast<const uint4*>(cb + (static_cast<size_t>(y0) * Wc + x1) * 256));
        c[k].u = __ldg(reinterpret_cast<const uint4*>(cb + (static_cast<size_t>(y1) * Wc + x0) * 256));
        d[k].u = __ldg(reinterpret_cast<const uint4*>(cb + (static_cast<size_t>(y1) * Wc + x1) * 256));
      }
#pragma unroll
      for (int k = 0; k < kU; ++k) {
        if (ub + k >= u1) break;  // block-uniform
        if (amax && img[k] != m_img) {  // block-uniform: the image of a unit
          if (m_img >= 0) publish_amax_block(amax + m_img, m, red);
          m = 0;
          m_img = img[k];
        }
        if (!live[k]) continue;
        const float w00 = (1.f - wy[k]) * (1.f - wx[k]), w01 = (1.f - wy[k]) * wx[k];
        const float w10 = wy[k] * (1.f - wx[k]), w11 = wy[k] * wx[k];
        const uint32_t lw[4] = {l[k].u.x, l[k].u.y, l[k].u.z, l[k].u.w};
        const uint32_t aw[4] = {a[k].u.x, a[k].u.y, a[k].u.z, a[k].u.w};
        const uint32_t bw[4] = {b[k].u.x, b[k].u.y, b[k].u.z, b[k].u.w};
        const uint32_t cw[4] = {c[k].u.x, c[k].u.y, c[k].u.z, c[k].u.w};
        const uint32_t dw[4] = {d[k].u.x, d[k].u.y, d[k].u.z, d[k].u.w};
        uint32_t ow[4], mag = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // channel pairs: same fp32 chain per channel as ever
          const float2 fl = lat ? Pair16<T>::unpack(lw[e]) : make_float2(0.f, 0.f);
          const float2 fa = Pair16<T>::unpack(aw[e]), fb = Pair16<T>::unpack(bw[e]);
          const float2 fc = Pair16<T>::unpack(cw[e]), fd = Pair16<T>::unpack(dw[e]);
          float v0 = fmaf(fa.x, w00, fl.x), v1 = fmaf(fa.y, w00, fl.y);
          v0 = fmaf(fb.x, w01, v0);
          v1 = fmaf(fb.y, w01, v1);
          v0 = fmaf(fc.x, w10, v0);
          v1 = fmaf(fc.y, w10, v1);
          v0 = fmaf(fd.x, w11, v0);
          v1 = fmaf(fd.y, w11, v1);
          ow[e] = Pair16<T>::pack(v0, v1);
          mag = __vmaxu2(mag, ow[e] & 0x7FFF7FFFu);
        }
        if (amax) m = max(m, Pair16<T>::mag_to_f32_bits(mag));
        *reinterpret_cast<uint4*>(out + io[k]) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        if (out_s) {
          uint32_t sw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Pair16<T>::unpack(ow[e]);
            sw[e] = Pair16<T>::pack(f.x * inv[2 * e], f.y * inv[2 * e + 1]);
          }
          *reinterpret_cast<uint4*>(out_s + io[k]) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
        }
      }
    }
  }
  if (amax && m_img >= 0) publish_amax_block(amax + m_img, m, red);
}
// Units whose loads are issued together: 2 (80 registers, 3 resident blocks per SM; the bound
// above) measured 0.9 % faster end to end than 4 (128 registers, 2 blocks) on bf16 R50
// 800x1216 batch 2, the same on e4m3 640x640 batch 16.
constexpr int kPx512Batch = 2;

// Unit-per-warp form of the same merge, for maps that upsample along x (Wc / W <= 4 / 7): a
// warp owns a unit of 8 consecutive output pixels of one row.  It loads the unit's 8 lateral
// vectors into registers and the unit's coarse window -- 2 rows x kWinCols columns, which hold
// the taps of all 8 pixels -- into its own slice of shared memory with cp.async (each lane
// copies, and later reads, only its own 16 bytes of every pixel: no barrier), then computes
// the 8 pixels from there.  One load round trip per unit and 8 + 2 kWinCols loads of 16 bytes
// per lane, where one warp per pixel (above) makes 5 per pixel in several dependent rounds.
// The same fp32 chain per element as upsample_add_px512_kernel: bitwise the same output.  A
// tap outside the window (a larger ratio, or rounding at its edge) is read from global
// memory.  Warps take units with a grid stride, so the resident warps work on one band of
// rows at a time.
constexpr int kWinCols = 6;
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
template <typename T>
__global__ void __launch_bounds__(256) upsample_add_unit_kernel(
    const T* __restrict__ coarse, const T* lat, T* out, int N, int Hc, int Wc, int H, int W,
    int chunks, float sy_scale, float sx_scale, int ac, unsigned* amax, T* out_s,
    const float* scale_a, const float* scale_w) {
  static_assert(sizeof(T) == 2, "16-bit types");
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  __shared__ uint4 win[8][2 * kWinCols][32];  // per warp: row 0 columns, row 1 columns x lanes
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float inv[8];
  if (out_s) {
    const float sa = __ldg(scale_a);
#pragma unroll
    for (int e = 0; e < 8; ++e) inv[e] = __frcp_rn(sa * __ldg(scale_w + lane * 8 + e));
  }
  unsigned m = 0;
  int m_img = -1;  // image the running maximum m belongs to (warp-uniform)
  const int total = N * H * chunks;  // < 2^31 (host)
  for (int u = blockIdx.x * 8 + warp; u < total; u += gridDim.x * 8) {
    const int r = u / chunks;  // output row over all images
    const int xb = (u - r * chunks) * 8;
    const int n = r / H;
    const int y = r - n * H;
    const float sy = src_coord(y, Hc, H, sy_scale, ac);
    const int y0 = static_cast<int>(sy), y1 = min(y0 + 1, Hc - 1);
    const float wy = sy - static_cast<float>(y0);
    const int cx0 = static_cast<int>(src_coord(xb, Wc, W, sx_scale, ac));
    const T* cb = coarse + static_cast<size_t>(n) * Hc * Wc * 256 + lane * 8;
    const T* crow[2] = {cb + static_cast<size_t>(y0) * Wc * 256,
                        cb + static_cast<size_t>(y1) * Wc * 256};
#pragma unroll
    for (int j = 0; j < kWinCols; ++j) {
      const int col = min(cx0 + j, Wc - 1);
      cp_async16(&win[warp][j][lane], crow[0] + static_cast<size_t>(col) * 256);
      cp_async16(&win[warp][kWinCols + j][lane], crow[1] + static_cast<size_t>(col) * 256);
    }
    const size_t io0 = (static_cast<size_t>(r) * W + xb) * 256 + lane * 8;
    uint4 l[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      l[k] = (lat && xb + k < W) ? *reinterpret_cast<const uint4*>(lat + io0 + k * 256)
                                 : make_uint4(0u, 0u, 0u, 0u);
    cp_async_wait_all();
    if (amax && n != m_img) {  // warp-uniform
      if (m_img >= 0) publish_amax(amax + m_img, m);
      m = 0;
      m_img = n;
    }
    auto tap = [&](int row, int xc) -> uint4 {
      const int j = xc - cx0;
      return (j >= 0 && j < kWinCols)
                 ? win[warp][row * kWinCols + j][lane]
                 : __ldg(reinterpret_cast<const uint4*>(crow[row] + static_cast<size_t>(xc) * 256));
    };
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int x = xb + k;
      if (x >= W) break;  // warp-uniform
      const float sx = src_coord(x, Wc, W, sx_scale, ac);
      const int x0 = static_cast<int>(sx);
      const int x1 = min(x0 + 1, Wc - 1);
      const float wx = sx - static_cast<float>(x0);
      const float w00 = (1.f - wy) * (1.f - wx), w01 = (1.f - wy) * wx;
      const float w10 = wy * (1.f - wx), w11 = wy * wx;
      const uint4 a = tap(0, x0), b = tap(0, x1), c = tap(1, x0), d = tap(1, x1);
      const uint32_t lw[4] = {l[k].x, l[k].y, l[k].z, l[k].w};
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
      const uint32_t dw[4] = {d.x, d.y, d.z, d.w};
      uint32_t ow[4], mag = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fl = lat ? Pair16<T>::unpack(lw[e]) : make_float2(0.f, 0.f);
        const float2 fa = Pair16<T>::unpack(aw[e]), fb = Pair16<T>::unpack(bw[e]);
        const float2 fc = Pair16<T>::unpack(cw[e]), fd = Pair16<T>::unpack(dw[e]);
        float v0 = fmaf(fa.x, w00, fl.x), v1 = fmaf(fa.y, w00, fl.y);
        v0 = fmaf(fb.x, w01, v0);
        v1 = fmaf(fb.y, w01, v1);
        v0 = fmaf(fc.x, w10, v0);
        v1 = fmaf(fc.y, w10, v1);
        v0 = fmaf(fd.x, w11, v0);
        v1 = fmaf(fd.y, w11, v1);
        ow[e] = Pair16<T>::pack(v0, v1);
        mag = __vmaxu2(mag, ow[e] & 0x7FFF7FFFu);
      }
      if (amax) m = max(m, Pair16<T>::mag_to_f32_bits(mag));
      *reinterpret_cast<uint4*>(out + io0 + k * 256) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      if (out_s) {
        uint32_t sw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Pair16<T>::unpack(ow[e]);
          sw[e] = Pair16<T>::pack(f.x * inv[2 * e], f.y * inv[2 * e + 1]);
        }
        *reinterpret_cast<uint4*>(out_s + io0 + k * 256) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
      }
    }
  }
  if (amax && m_img >= 0) publish_amax(amax + m_img, m);
}

// ---------------------------------------------------------------- two-level merge
// M4 = L4 + up(M5) and M3 = L3 + up(M4) in ONE launch (NHWC, 256 channels of a 16-bit type,
// maps that upsample).  A block owns a kMergeTileH x kMergeTileW tile of M3 and
//   1. computes into shared memory every M4 pixel its tile's taps read, from L4 and four M5
//      taps, rounded to T exactly as the M4 map stores it; the M4 pixels it owns (the
//      rectangle [y0 H4 / H3, y1 H4 / H3) x [x0 W4 / W3, x1 W4 / W3), integer division, for
//      tile rows [y0, y1) and columns [x0, x1): these rectangles partition M4) also go to m4;
//   2. computes its M3 pixels from L3 (in place) and the shared M4 pixels.
// The arithmetic is that of two upsample_add_px512 passes (same taps, weights and fmaf
// order, one rounding per map), so the results are bitwise the same; the second pass's
// reads of M4 and the launch boundary between the passes disappear.  l4 must not alias m4
// (a block reads L4 pixels its neighbours own); l3 may alias m3.  The region computed in
// step 1 is the union of the tap rows / columns and the owned rectangle; reg_h x reg_w
// bounds it (host) and sizes the dynamic shared memory.
// Optional as in upsample_add_px512: amax4[n] / amax3[n] (|M4|, |M3| of image n, fp32 bits)
// and m3s, a copy of M3 with channel c scaled by 1 / (scale_a[0] * scale_w[c]).
constexpr int kMergeTileH = 8;
constexpr int kMergeTileW = 16;
template <typename T>
__global__ void __launch_bounds__(256, 3) merge_two_levels_kernel(
    const T* __restrict__ m5, const T* __restrict__ l4, T* __restrict__ m4, const T* l3, T* m3,
    int H5, int W5, int H4, int W4, int H3, int W3, float s54y, float s54x, float s43y,
    float s43x, int tiles_x, int tiles_y, int reg_h, int reg_w, unsigned* amax4,
    unsigned* amax3, T* m3s, const float* scale_a, const float* scale_w) {
  static_assert(sizeof(T) == 2, "16-bit types");
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  extern __shared__ uint4 merge_smem[];  // [reg_h * reg_w pixels][32 lanes] x 16 bytes
  __shared__ unsigned red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tx = static_cast<int>(blockIdx.x) % tiles_x;
  const int t2 = static_cast<int>(blockIdx.x) / tiles_x;
  const int ty = t2 % tiles_y;
  const int n = t2 / tiles_y;
  const int y0 = ty * kMergeTileH, x0 = tx * kMergeTileW;
  const int y1 = min(y0 + kMergeTileH, H3), x1 = min(x0 + kMergeTileW, W3);  // exclusive
  // owned M4 rectangle
  const int oy0 = static_cast<int>(static_cast<long long>(y0) * H4 / H3);
  const int oy1 = static_cast<int>(static_cast<long long>(y1) * H4 / H3);
  const int ox0 = static_cast<int>(static_cast<long long>(x0) * W4 / W3);
  const int ox1 = static_cast<int>(static_cast<long long>(x1) * W4 / W3);
  // region: tap rows / columns of the tile's pixels, united with the owned rectangle
  const int ry0 = min(static_cast<int>(src_coord(y0, H4, H3, s43y, 0)), oy0);
  const int ry1 = max(min(static_cast<int>(src_coord(y1 - 1, H4, H3, s43y, 0)) + 1, H4 - 1),
                      oy1 - 1);
  const int rx0 = min(static_cast<int>(src_coord(x0, W4, W3, s43x, 0)), ox0);
  const int rx1 = max(min(static_cast<int>(src_coord(x1 - 1, W4, W3, s43x, 0)) + 1, W4 - 1),
                      ox1 - 1);
  const int rh = ry1 - ry0 + 1, rw = rx1 - rx0 + 1;
  if (rh > reg_h || rw > reg_w) return;  // cannot happen for the host's bound (uniform exit)

  unsigned m = 0;
  // ---- 1. M4 region, kB pixels per warp at a time (all their loads issued first)
  constexpr int kB = 2;
  const T* m5n = m5 + static_cast<size_t>(n) * H5 * W5 * 256 + lane * 8;
  for (int i0 = warp; i0 < rh * rw; i0 += 8 * kB) {
    Vec16<T> l[kB], a[kB], b[kB], c[kB], d[kB];
    float wy[kB], wx[kB];
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int i = min(i0 + 8 * k, rh * rw - 1);  // clamped duplicates are not stored
      const int yy = ry0 + i / rw, xx = rx0 + i % rw;
      const float sy = src_coord(yy, H5, H4, s54y, 0);
      const float sx = src_coord(xx, W5, W4, s54x, 0);
      const int ya = static_cast<int>(sy), xa = static_cast<int>(sx);
      const int yb = min(ya + 1, H5 - 1), xb = min(xa + 1, W5 - 1);
      wy[k] = sy - static_cast<float>(ya);
      wx[k] = sx - static_cast<float>(xa);
      const size_t io = (static_cast<size_t>(n * H4 + yy) * W4 + xx) * 256 + lane * 8;
      l[k].u = __ldg(reinterpret_cast<const uint4*>(l4 + io));
      a[k].u = __ldg(reinterpret_cast<const uint4*>(m5n + (static_cast<size_t>(ya) * W5 + xa) * 256));
      b[k].u = __ldg(reinterpret_cast<const uint4*>(m5n + (static_cast<size_t>(ya) * W5 + xb) * 256));
      c[k].u = __ldg(reinterpret_cast<const uint4*>(m5n + (static_cast<size_t>(yb) * W5 + xa) * 256));
      d[k].u = __ldg(reinterpret_cast<const uint4*>(m5n + (static_cast<size_t>(yb) * W5 + xb) * 256));
    }
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int i = i0 + 8 * k;
      if (i >= rh * rw) break;
      const int yy = ry0 + i / rw, xx = rx0 + i % rw;
      const float w00 = (1.f - wy[k]) * (1.f - wx[k]), w01 = (1.f - wy[k]) * wx[k];
      const float w10 = wy[k] * (1.f - wx[k]), w11 = wy[k] * wx[k];
      Vec16<T> o;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = to_f(l[k].e[e]);
        v = fmaf(to_f(a[k].e[e]), w00, v);
        v = fmaf(to_f(b[k].e[e]), w01, v);
        v = fmaf(to_f(c[k].e[e]), w10, v);
        v = fmaf(to_f(d[k].e[e]), w11, v);
        o.e[e] = from_f<T>(v);
      }
      merge_smem[i * 32 + lane] = o.u;
      if (yy >= oy0 && yy < oy1 && xx >= ox0 && xx < ox1) {
        const size_t io = (static_cast<size_t>(n * H4 + yy) * W4 + xx) * 256 + lane * 8;
        *reinterpret_cast<uint4*>(m4 + io) = o.u;
        if (amax4) {
#pragma unroll
          for (int e = 0; e < 8; ++e) m = max(m, abs_bits(to_f(o.e[e])));
        }
      }
    }
  }
  if (amax4) publish_amax_block(amax4 + n, m, red);  // (also orders the shared M4 writes)
  else __syncthreads();

  // ---- 2. M3 tile
  float inv[8];
  if (m3s) {
    const float sa = __ldg(scale_a);
#pragma unroll
    for (int e = 0; e < 8; ++e) inv[e] = __frcp_rn(sa * __ldg(scale_w + lane * 8 + e));
  }
  m = 0;
  // the warp's pixels kPx at a time: their L3 loads first (each pixel is read, then
  // written, by the same lane, so an in-place M3 is safe), then the taps and the stores
  constexpr int kPx = 8;
#pragma unroll 1
  for (int p0 = warp; p0 < kMergeTileH * kMergeTileW; p0 += 8 * kPx) {
  Vec16<T> lt[kPx];
#pragma unroll
  for (int k = 0; k < kPx; ++k) {
    const int p = p0 + 8 * k;
    const int y = y0 + p / kMergeTileW, x = x0 + p % kMergeTileW;
    if (y < y1 && x < x1)
      lt[k].u = *reinterpret_cast<const uint4*>(
          l3 + (static_cast<size_t>(n * H3 + y) * W3 + x) * 256 + lane * 8);
  }
#pragma unroll
  for (int k = 0; k < kPx; ++k) {
    const int p = p0 + 8 * k;
    const int y = y0 + p / kMergeTileW, x = x0 + p % kMergeTileW;
    if (y >= y1 || x >= x1) continue;
    const float sy = src_coord(y, H4, H3, s43y, 0);
    const float sx = src_coord(x, W4, W3, s43x, 0);
    const int ya = static_cast<int>(sy), xa = static_cast<int>(sx);
    const int yb = min(ya + 1, H4 - 1), xb = min(xa + 1, W4 - 1);
    const float wy = sy - static_cast<float>(ya), wx = sx - static_cast<float>(xa);
    const size_t io = (static_cast<size_t>(n * H3 + y) * W3 + x) * 256 + lane * 8;
    Vec16<T> a, b, c, d;
    const Vec16<T>& l = lt[k];
    a.u = merge_smem[((ya - ry0) * rw + (xa - rx0)) * 32 + lane];
    b.u = merge_smem[((ya - ry0) * rw + (xb - rx0)) * 32 + lane];
    c.u = merge_smem[((yb - ry0) * rw + (xa - rx0)) * 32 + lane];
    d.u = merge_smem[((yb - ry0) * rw + (xb - rx0)) * 32 + lane];
    const float w00 = (1.f - wy) * (1.f - wx), w01 = (1.f - wy) * wx;
    const float w10 = wy * (1.f - wx), w11 = wy * wx;
    Vec16<T> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = to_f(l.e[e]);
      v = fmaf(to_f(a.e[e]), w00, v);
      v = fmaf(to_f(b.e[e]), w01, v);
      v = fmaf(to_f(c.e[e]), w10, v);
      v = fmaf(to_f(d.e[e]), w11, v);
      o.e[e] = from_f<T>(v);
      m = max(m, abs_bits(to_f(o.e[e])));
    }
    *reinterpret_cast<uint4*>(m3 + io) = o.u;
    if (m3s) {
      Vec16<T> os;
#pragma unroll
      for (int e = 0; e < 8; ++e) os.e[e] = from_f<T>(to_f(o.e[e]) * inv[e]);
      *reinterpret_cast<uint4*>(m3s + io) = os.u;
    }
  }
  }
  if (amax3) publish_amax_block(amax3 + n, m, red);
}

// ---------------------------------------------------------------- NCHW upsample-add
// One thread per output element; consecutive threads walk x of one plane.
template <typename T>
__global__ void __launch_bounds__(256) upsample_add_nchw_kernel(
    const T* __restrict__ coarse, const T* __restrict__ lat, T* __restrict__ out, int N, int C,
    int Hc, int Wc, int H, int W, float sy_scale, float sx_scale, int ac) {
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  const long long total = static_cast<long long>(N) * C * H * W;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % W);
    const long long t = i / W;
    const int y = static_cast<int>(t % H);
    const long long plane = t / H;  // n*C + c
    const BilinearTap tp = make_tap(y, x, Hc, Wc, H, W, sy_scale, sx_scale, ac);
    const T* cp = coarse + static_cast<size_t>(plane) * Hc * Wc;
    float r = to_f(__ldg(cp + tp.y0 * Wc + tp.x0)) * tp.w00 +
              to_f(__ldg(cp + tp.y0 * Wc + tp.x1)) * tp.w01 +
              to_f(__ldg(cp + tp.y1 * Wc + tp.x0)) * tp.w10 +
              to_f(__ldg(cp + tp.y1 * Wc + tp.x1)) * tp.w11;
    if (lat) r += to_f(lat[i]);
    out[i] = from_f<T>(r);
  }
}

// Vectorised NCHW upsample-add (W % 8 == 0, 16-byte aligned rows of a 16-bit type): a thread
// makes 8 consecutive outputs of one row -- one 16-byte lateral load and store, the row's
// source coordinate and its two coarse rows computed once per 8 outputs -- with the
// arithmetic of upsample_add_nchw_kernel element for element.  The scalar kernel did two
// 64-bit divisions per element and ran at 0.14 of HBM bandwidth on a 4x256x400x608 map.
template <typename T>
__global__ void __launch_bounds__(256) upsample_add_nchw_vec_kernel(
    const T* __restrict__ coarse, const T* __restrict__ lat, T* __restrict__ out, int N, int C,
    int Hc, int Wc, int H, int W, float sy_scale, float sx_scale, int ac) {
  static_assert(sizeof(T) == 2, "16-bit types");
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  const int vpr = W >> 3;  // 8-element vectors per row
  const long long total = static_cast<long long>(N) * C * H * vpr;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / vpr;
    const int x0v = static_cast<int>(i - row * vpr) * 8;
    const long long plane = row / H;
    const int y = static_cast<int>(row - plane * H);
    const float sy = src_coord(y, Hc, H, sy_scale, ac);
    const int ya = static_cast<int>(sy);
    const int yb = min(ya + 1, Hc - 1);
    const float wy = sy - static_cast<float>(ya);
    const T* c0 = coarse + (static_cast<size_t>(plane) * Hc + ya) * Wc;
    const T* c1 = coarse + (static_cast<size_t>(plane) * Hc + yb) * Wc;
    const size_t o = static_cast<size_t>(row) * W + x0v;
    Vec16<T> l, r;
    if (lat) l.u = __ldg(reinterpret_cast<const uint4*>(lat + o));
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sx = src_coord(x0v + e, Wc, W, sx_scale, ac);
      const int xa = static_cast<int>(sx);
      const int xb = min(xa + 1, Wc - 1);
      const float wx = sx - static_cast<float>(xa);
      float v = to_f(__ldg(c0 + xa)) * ((1.f - wy) * (1.f - wx)) +
                to_f(__ldg(c0 + xb)) * ((1.f - wy) * wx) +
                to_f(__ldg(c1 + xa)) * (wy * (1.f - wx)) + to_f(__ldg(c1 + xb)) * (wy * wx);
      if (lat) v += to_f(l.e[e]);
      r.e[e] = from_f<T>(v);
    }
    *reinterpret_cast<uint4*>(out + o) = r.u;
  }
}

// ---------------------------------------------------------------- P6
// P6 = max_pool2d(P5, kernel=1, stride=2): a single-element window, i.e. P5[::2, ::2].
template <typename T, bool kVec>
__global__ void __launch_bounds__(256) p6_nhwc_kernel(const T* __restrict__ in,
                                                      T* __restrict__ out, int N, int C, int H,
                                                      int W, int H6, int W6) {
  // Same walk as the NHWC upsample: blocks over output rows, warps over pixels,
  // lanes over 16-byte channel vectors (coalesced 512-byte rows), 32-bit indices.
  constexpr int V = kVec ? Vec16<T>::kN : 1;
  const int cvs = C / V;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = N * H6;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int n = r / H6;
    const int y = r - n * H6;
    const T* src_row = in + (static_cast<size_t>(n) * H + 2 * y) * W * C;
    T* dst_row = out + static_cast<size_t>(r) * W6 * C;
    if constexpr (kVec) {
      // The row's W6 x cvs 16-byte vectors, kB per thread per step: all kB loads are issued
      // before the first store (one load in flight per thread left the copy latency-bound).
      constexpr int kB = 4;
      const int items = W6 * cvs;
      for (int i0 = threadIdx.x; i0 < items; i0 += kB * 256) {
        uint4 v[kB];
        int dx[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          const int it = i0 + k * 256;
          dx[k] = -1;
          if (it < items) {
            const int x = it / cvs;
            const int cv = it - x * cvs;
            dx[k] = x * C + cv * V;
            v[k] = __ldg(reinterpret_cast<const uint4*>(src_row + static_cast<size_t>(2 * x) * C +
                                                        cv * V));
          }
        }
#pragma unroll
        for (int k = 0; k < kB; ++k)
          if (dx[k] >= 0) *reinterpret_cast<uint4*>(dst_row + dx[k]) = v[k];
      }
    } else {
      for (int x = warp; x < W6; x += 8) {
        const T* s = src_row + static_cast<size_t>(2 * x) * C;
        T* d = dst_row + static_cast<size_t>(x) * C;
        for (int cv = lane; cv < cvs; cv += 32) d[cv] = s[cv];
      }
    }
  }
}

// NCHW with W % 16 == 0 (16-bit, 16-byte aligned rows): a thread makes 8 outputs of one row
// from two 16-byte loads of the even input row (the even elements kept), one 16-byte store.
template <typename T>
__global__ void __launch_bounds__(256) p6_nchw_vec_kernel(const T* __restrict__ in,
                                                          T* __restrict__ out, int N, int C,
                                                          int H, int W, int H6, int W6) {
  static_assert(sizeof(T) == 2, "16-bit types");
  const int vpr = W6 >> 3;
  const long long total = static_cast<long long>(N) * C * H6 * vpr;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / vpr;  // (plane, y) of the output
    const int v = static_cast<int>(i - row * vpr);
    const long long plane = row / H6;
    const int y = static_cast<int>(row - plane * H6);
    const T* src = in + (static_cast<size_t>(plane) * H + 2 * y) * W + 16 * v;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(src + 8));
    // keep the low 16 bits of every 32-bit word (the even elements)
    uint4 o;
    o.x = __byte_perm(a.x, a.y, 0x5410);
    o.y = __byte_perm(a.z, a.w, 0x5410);
    o.z = __byte_perm(b.x, b.y, 0x5410);
    o.w = __byte_perm(b.z, b.w, 0x5410);
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * W6 + 8 * v) = o;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) p6_nchw_kernel(const T* __restrict__ in,
                                                      T* __restrict__ out, int N, int C, int H,
                                                      int W, int H6, int W6) {
  const long long total = static_cast<long long>(N) * C * H6 * W6;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % W6);
    const long long t = i / W6;
    const int y = static_cast<int>(t % H6);
    const long long plane = t / H6;
    out[i] = in[(static_cast<size_t>(plane) * H + 2 * y) * W + 2 * x];
  }
}

// ---------------------------------------------------------------- layout conversion
// NCHW -> NHWC through a 32x32 shared-memory tile (both sides coalesced).
template <typename T>
__global__ void __launch_bounds__(256) nchw_to_nhwc_kernel(const T* __restrict__ in,
                                                           T* __restrict__ out, int C, int HW) {
  __shared__ T tile[32][33];
  const int n = blockIdx.z;
  const int c0 = blockIdx.y * 32;
  const int p0 = blockIdx.x * 32;
  const T* src = in + static_cast<size_t>(n) * C * HW;
  T* dst = out + static_cast<size_t>(n) * C * HW;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int c = c0 + r, p = p0 + threadIdx.x;
    if (c < C && p < HW) tile[r][threadIdx.x] = src[static_cast<size_t>(c) * HW + p];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int p = p0 + r, c = c0 + threadIdx.x;
    if (c < C && p < HW) dst[static_cast<size_t>(p) * C + c] = tile[threadIdx.x][r];
  }
}

template <typename T>
__global__ void __launch_bounds__(256) nhwc_to_nchw_kernel(const T* __restrict__ in,
                                                           T* __restrict__ out, int C, int HW) {
  __shared__ T tile[32][33];
  const int n = blockIdx.z;
  const int c0 = blockIdx.y * 32;
  const int p0 = blockIdx.x * 32;
  const T* src = in + static_cast<size_t>(n) * C * HW;
  T* dst = out + static_cast<size_t>(n) * C * HW;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int p = p0 + r, c = c0 + threadIdx.x;
    if (c < C && p < HW) tile[r][threadIdx.x] = src[static_cast<size_t>(p) * C + c];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int c = c0 + r, p = p0 + threadIdx.x;
    if (c < C && p < HW) dst[static_cast<size_t>(c) * HW + p] = tile[threadIdx.x][r];
  }
}

// ---------------------------------------------------------------- weight packing
template <typename T>
__global__ void convert_kernel(const float* __restrict__ in, T* __restrict__ out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = from_f<T>(in[i]);
}

// [Cout][Cin][3][3] fp32 -> [Cout][9][Cin] T (K index = tap * Cin + c, K-major rows).
template <typename T>
__global__ void pack_conv3x3_kernel(const float* __restrict__ in, T* __restrict__ out, int Cout,
                                    int Cin) {
  const long long total = static_cast<long long>(Cout) * Cin * 9;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % Cin);
    const long long t = i / Cin;
    const int tap = static_cast<int>(t % 9);
    const int o = static_cast<int>(t / 9);
    out[i] = from_f<T>(in[(static_cast<size_t>(o) * Cin + c) * 9 + tap]);
  }
}

// ---------------------------------------------------------------- e4m3 quantisation
// Symmetric e4m3 with scale = amax / 448 (per tensor for activations, per output
// channel for weights):
//   amax > 0:  inv = 448 / amax,  scale = amax / 448;   amax == 0: inv = scale = 1
//   q = e4m3(x * inv), rounded to nearest even, saturated to +-448
// Every step is one correctly rounded fp32 operation, so a CPU restatement reproduces
// q and scale bit for bit.  The absmax travels as the bit pattern of a non-negative
// fp32, which orders like an unsigned integer (atomicMax).
__device__ __forceinline__ float e4m3_inv(unsigned amax_bits) {
  const float a = __uint_as_float(amax_bits);
  return a > 0.f ? __fdiv_rn(448.f, a) : 1.f;
}
__device__ __forceinline__ float e4m3_scale(unsigned amax_bits) {
  const float a = __uint_as_float(amax_bits);
  return a > 0.f ? __fdiv_rn(a, 448.f) : 1.f;
}
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d, float inv) {
  const uint32_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(a * inv, b * inv), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(c * inv, d * inv), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

// amax[g] = max |x| over group g = elements [g * per, (g + 1) * per).  Grid y = group;
// 16-byte vectors when the group start is aligned (vec), then the tail.
template <typename T>
__global__ void __launch_bounds__(256) absmax_kernel(const T* __restrict__ x, long long per,
                                                     int vec, unsigned* amax) {
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  constexpr int V = Vec16<T>::kN;
  const T* xg = x + static_cast<long long>(blockIdx.y) * per;
  unsigned m = 0;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nv = vec ? per / V : 0;
  for (long long i = tid; i < nv; i += stride) {
    Vec16<T> v;
    v.u = __ldg(reinterpret_cast<const uint4*>(xg) + i);
#pragma unroll
    for (int e = 0; e < V; ++e) m = max(m, abs_bits(to_f(v.e[e])));
  }
  for (long long i = nv * V + tid; i < per; i += stride) m = max(m, abs_bits(to_f(xg[i])));
  publish_amax(amax + blockIdx.y, m);
}

// q = e4m3(x * inv) per element, inv from the absmax of the element's group (grid y);
// block (0, g) also writes the group's dequantisation scale.
template <typename T>
__global__ void __launch_bounds__(256) quantize_e4m3_kernel(const T* __restrict__ x, long long per,
                                                            int vec, const unsigned* amax,
                                                            uint8_t* __restrict__ q,
                                                            float* scale_out) {
  griddep_wait();  // (programmatic launch) inputs written by the previous kernel
  griddep_launch_dependents();
  const unsigned a = amax[blockIdx.y];
  const float inv = e4m3_inv(a);
  if (scale_out && blockIdx.x == 0 && threadIdx.x == 0) scale_out[blockIdx.y] = e4m3_scale(a);
  x += static_cast<long long>(blockIdx.y) * per;
  q += static_cast<long long>(blockIdx.y) * per;
  const long long n = per;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  // 8 elements (8 output bytes) per step when x is 16-byte and q 8-byte aligned.
  const long long n8 = vec ? n / 8 : 0;
  for (long long i = tid; i < n8; i += stride) {
    float f[8];
    if constexpr (sizeof(T) == 4) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
      const float4 w = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
      f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
      f[4] = w.x; f[5] = w.y; f[6] = w.z; f[7] = w.w;
    } else {
      Vec16<T> v;
      v.u = __ldg(reinterpret_cast<const uint4*>(x) + i);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = to_f(v.e[e]);
    }
    uint2 o;
    o.x = e4m3x4(f[0], f[1], f[2], f[3], inv);
    o.y = e4m3x4(f[4], f[5], f[6], f[7], inv);
    reinterpret_cast<uint2*>(q)[i] = o;
  }
  for (long long i = n8 * 8 + tid; i < n; i += stride)
    q[i] = static_cast<uint8_t>(
        __nv_cvt_float_to_fp8(to_f(x[i]) * inv, __NV_SATFINITE, __NV_E4M3));
}

// Weights, one block per output channel (row): scale[row] = amax_row / 448 and
// q = e4m3(w * 448 / amax_row).  pack_cin > 0: the row is [pack_cin][3][3] and q is
// written tap-major, [9][pack_cin] (the K order of the 3x3 implicit GEMM).
__global__ void __launch_bounds__(256) quantize_rows_e4m3_kernel(const float* __restrict__ w,
                                                                 int cols, int pack_cin,
                                                                 uint8_t* __restrict__ q,
                                                                 float* __restrict__ scales) {
  __shared__ unsigned red[8];
  const float* row = w + static_cast<size_t>(blockIdx.x) * cols;
  unsigned m = 0;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) m = max(m, abs_bits(row[i]));
  m = __reduce_max_sync(0xffffffffu, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  unsigned a = 0;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) a = max(a, red[i]);
  const float inv = e4m3_inv(a);
  if (threadIdx.x == 0) scales[blockIdx.x] = e4m3_scale(a);
  uint8_t* qrow = q + static_cast<size_t>(blockIdx.x) * cols;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const int dst = pack_cin > 0 ? (i % 9) * pack_cin + i / 9 : i;
    qrow[dst] =
        static_cast<uint8_t>(__nv_cvt_float_to_fp8(row[i] * inv, __NV_SATFINITE, __NV_E4M3));
  }
}

// ---------------------------------------------------------------- fp32 CUDA-core GEMMs
// out[n, o, p] = sum_k Wt[o, k] * B(n, k, p) + bias[o] (+ bilinear(coarse)[n, o, p])
// with B either the NCHW input itself (1x1 conv, k = c) or its on-the-fly
// im2col (3x3 pad-1 conv, k = c*9 + ky*3 + kx, Wt in natural [Cout][Cin][3][3]).
// 64x64 output tile per CTA, 256 threads, 4x4 register block, K step 16.
constexpr int kSB = 64;
constexpr int kSK = 16;

template <bool kIm2col>
__global__ void __launch_bounds__(256) fp32_conv_gemm_kernel(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bias,
    const float* __restrict__ coarse, float* __restrict__ out, int Cin, int Cout, int H, int W,
    int Hc, int Wc, float sy_scale, float sx_scale, int act, float act_alpha) {
  __shared__ float sA[kSK][kSB + 4];  // [k][o]
  __shared__ float sB[kSK][kSB + 4];  // [k][p]
  const int HW = H * W;
  const int n = blockIdx.z;
  const int o0 = blockIdx.y * kSB;
  const int p0 = blockIdx.x * kSB;
  const int K = kIm2col ? Cin * 9 : Cin;
  const float* xn = x + static_cast<size_t>(n) * Cin * HW;
  const int tx = threadIdx.x & 15;  // pixel group
  const int ty = threadIdx.x >> 4;  // out-channel group
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kSK) {
    // A tile: 64 out x 16 k (4 loads per thread)
    for (int i = threadIdx.x; i < kSB * kSK; i += 256) {
      const int kk = i % kSK, oo = i / kSK;
      const int o = o0 + oo, k = k0 + kk;
      sA[kk][oo] = (o < Cout && k < K) ? __ldg(wt + static_cast<size_t>(o) * K + k) : 0.f;
    }
    // B tile: 16 k x 64 pixels
    for (int i = threadIdx.x; i < kSB * kSK; i += 256) {
      const int pp = i % kSB, kk = i / kSB;
      const int p = p0 + pp, k = k0 + kk;
      float v = 0.f;
      if (p < HW && k < K) {
        if constexpr (kIm2col) {
          const int c = k / 9, tap = k - c * 9;
          const int yy = p / W + tap / 3 - 1, xx = p % W + tap % 3 - 1;
          if (yy >= 0 && yy < H && xx >= 0 && xx < W)
            v = __ldg(xn + static_cast<size_t>(c) * HW + yy * W + xx);
        } else {
          v = __ldg(xn + static_cast<size_t>(k) * HW + p);
        }
      }
      sB[kk][pp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int o = o0 + ty * 4 + i;
    if (o >= Cout) continue;
    const float bo = bias ? __ldg(bias + o) : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = p0 + tx + 16 * j;
      if (p >= HW) continue;
      float r = acc[i][j] + bo;
      if (coarse) {
        const int y = p / W, xq = p % W;
        const BilinearTap tp = make_tap(y, xq, Hc, Wc, H, W, sy_scale, sx_scale, 0);
        const float* cp = coarse + (static_cast<size_t>(n) * Cout + o) * Hc * Wc;
        r += __ldg(cp + tp.y0 * Wc + tp.x0) * tp.w00 + __ldg(cp + tp.y0 * Wc + tp.x1) * tp.w01 +
             __ldg(cp + tp.y1 * Wc + tp.x0) * tp.w10 + __ldg(cp + tp.y1 * Wc + tp.x1) * tp.w11;
      }
      out[(static_cast<size_t>(n) * Cout + o) * HW + p] = epilogue_act(r, act, act_alpha);
    }
  }
}

int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// Blocks per group so the whole launch still covers about 16 blocks per SM.
int group_blocks(long long per, int groups, int elems_per_thread) {
  long long want = (per / elems_per_thread + 255) / 256;
  const long long cap = (148LL * 16 + groups - 1) / groups;
  if (want > cap) want = cap;
  return want < 1 ? 1 : static_cast<int>(want);
}

template <typename T>
cudaError_t absmax_t(const void* x, long long n, int groups, unsigned* amax, cudaStream_t s) {
  if (groups < 1 || groups > 65535 || n % groups != 0) return cudaErrorInvalidValue;
  const long long per = n / groups;
  const int vec =
      (aligned16(x) && (per * static_cast<long long>(sizeof(T))) % 16 == 0) ? 1 : 0;
  const dim3 grid(group_blocks(per, groups, Vec16<T>::kN), groups);
  absmax_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(x), per, vec, amax);
  return cudaGetLastError();
}

template <typename T>
cudaError_t upsample_add_t(const void* coarse, const void* lat, void* out, int N, int C, int Hc,
                           int Wc, int H, int W, int ac, Layout layout, cudaStream_t s,
                           unsigned* amax, const MergeScaledCopy* sc, LaunchOpts opts,
                           int units_per_block) {
  const float sy = (ac && H > 1) ? static_cast<float>(Hc - 1) / (H - 1)
                                 : static_cast<float>(Hc) / H;
  const float sx = (ac && W > 1) ? static_cast<float>(Wc - 1) / (W - 1)
                                 : static_cast<float>(Wc) / W;
  const T* c = static_cast<const T*>(coarse);
  const T* l = static_cast<const T*>(lat);
  T* o = static_cast<T*>(out);
  if (layout == Layout::NHWC) {
    constexpr int V = Vec16<T>::kN;
    const bool vec = (C % V == 0) && aligned16(coarse) && aligned16(out) &&
                     (lat == nullptr || aligned16(lat));
    if constexpr (sizeof(T) == 2) {
      if (vec && C == 256) {
        const int chunks = (W + 7) / 8;
        const long long units = static_cast<long long>(N) * H * chunks;
        // Maps whose lateral fills half of the L2 or more: interleaved chunks (coarse rows
        // stay in L2; 4 units per thread in flight instead of 2 measured 5 % slower there).
        const bool inter = static_cast<long long>(N) * H * W * 512 > l2_bytes() / 2;
        // units_per_block 0: one warp per 8-pixel unit where the map upsamples along x
        // (its taps then fit the unit's coarse window); -1 or > 0: one warp per pixel
        if (units_per_block == 0 && 7LL * Wc <= 4LL * W && units < (1LL << 31)) {
          auto ukern = upsample_add_unit_kernel<T>;
          static std::atomic<int> ures[64];
          int dev = 0;
          cudaGetDevice(&dev);
          const bool cached = dev >= 0 && dev < 64;
          int res = cached ? ures[dev].load(std::memory_order_relaxed) : 0;
          if (res == 0) {
            int per_sm = 0;
            cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ukern, 256, 0);
            if (e != cudaSuccess) return e;
            res = (per_sm > 0 ? per_sm : 1) * sm_count();
            if (cached) ures[dev].store(res, std::memory_order_relaxed);
          }
          const long long want = (units + 7) / 8;
          const int grid = static_cast<int>(want < res ? want : res);
          return launch_ex(ukern, dim3(grid), dim3(256), 0, s, opts, 1, c, l, o, N, Hc, Wc, H, W,
                           chunks, sy, sx, ac, amax, sc ? static_cast<T*>(sc->out) : nullptr,
                           sc ? sc->scale_a : nullptr, sc ? sc->scale_w : nullptr);
        }
        auto kern = upsample_add_px512_kernel<T, kPx512Batch>;
        // grid = the blocks resident at once, each with a contiguous run of units (or, when
        // interleaved, a chunk at a time)
        static std::atomic<int> resident[64];
        int dev = 0;
        cudaGetDevice(&dev);
        const bool cached = dev >= 0 && dev < 64;
        int res = cached ? resident[dev].load(std::memory_order_relaxed) : 0;
        if (res == 0) {
          int per_sm = 0;
          cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
          if (e != cudaSuccess) return e;
          res = (per_sm > 0 ? per_sm : 1) * sm_count();
          if (cached) resident[dev].store(res, std::memory_order_relaxed);
        }
        const long long g = units < res ? units : res;
        if (g <= 0) return cudaSuccess;
        const long long per =
            units_per_block > 0 ? units_per_block : (units + g - 1) / g;  // (-1: automatic)
        if (per >= (1LL << 31)) return cudaErrorInvalidValue;
        const int grid = static_cast<int>((units + per - 1) / per);
        return launch_ex(kern, dim3(grid), dim3(256), 0, s, opts, 1, c, l, o, N, Hc, Wc, H, W,
                         chunks, sy, sx, ac, amax, sc ? static_cast<T*>(sc->out) : nullptr,
                         sc ? sc->scale_a : nullptr, sc ? sc->scale_w : nullptr,
                         static_cast<int>(per), inter ? 1 : 0);
      }
    }
    if (sc) return cudaErrorNotSupported;  // the scaled copy exists on the 256-channel path
    const long long units =
        static_cast<long long>(N) * H * ((W + 8 * kUpPix - 1) / (8 * kUpPix));  // per block
    const int grid = units < 148 * 64 ? static_cast<int>(units) : 148 * 64;
    cudaError_t e0;
    if (vec)
      e0 = launch_ex(upsample_add_nhwc_kernel<T, true>, dim3(grid), dim3(256), 0, s, opts, 1, c, l,
                     o, N, C, Hc, Wc, H, W, sy, sx, ac);
    else
      e0 = launch_ex(upsample_add_nhwc_kernel<T, false>, dim3(grid), dim3(256), 0, s, opts, 1, c,
                     l, o, N, C, Hc, Wc, H, W, sy, sx, ac);
    if (e0 != cudaSuccess) return e0;
  } else {
    const long long work = static_cast<long long>(N) * C * H * W;
    if (sc) return cudaErrorNotSupported;
    cudaError_t e0;
    if constexpr (sizeof(T) == 2) {
      if (W % 8 == 0 && aligned16(out) && (lat == nullptr || aligned16(lat))) {
        e0 = launch_ex(upsample_add_nchw_vec_kernel<T>, dim3(grid_for(work / 8, 256)), dim3(256),
                       0, s, opts, 1, c, l, o, N, C, Hc, Wc, H, W, sy, sx, ac);
        if (e0 != cudaSuccess) return e0;
        e0 = cudaGetLastError();
        if (e0 == cudaSuccess && amax)
          e0 = absmax_t<T>(out, static_cast<long long>(N) * C * H * W, N, amax, s);
        return e0;
      }
    }
    e0 = launch_ex(upsample_add_nchw_kernel<T>, dim3(grid_for(work, 256)), dim3(256), 0, s, opts,
                   1, c, l, o, N, C, Hc, Wc, H, W, sy, sx, ac);
    if (e0 != cudaSuccess) return e0;
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && amax)
    e = absmax_t<T>(out, static_cast<long long>(N) * C * H * W, N, amax, s);
  return e;
}

template <typename T>
cudaError_t p6_t(const void* in, void* out, int N, int C, int H, int W, Layout layout,
                 cudaStream_t s) {
  const int H6 = (H - 1) / 2 + 1, W6 = (W - 1) / 2 + 1;
  const T* i = static_cast<const T*>(in);
  T* o = static_cast<T*>(out);
  if (layout == Layout::NHWC) {
    constexpr int V = Vec16<T>::kN;
    const bool vec = (C % V == 0) && aligned16(in) && aligned16(out);
    const int rows = N * H6;
    const int grid = rows < 148 * 8 ? rows : 148 * 8;
    if (vec)
      p6_nhwc_kernel<T, true><<<grid, 256, 0, s>>>(i, o, N, C, H, W, H6, W6);
    else
      p6_nhwc_kernel<T, false><<<grid, 256, 0, s>>>(i, o, N, C, H, W, H6, W6);
  } else {
    const long long work = static_cast<long long>(N) * C * H6 * W6;
    if constexpr (sizeof(T) == 2) {
      if (W % 16 == 0 && aligned16(in) && aligned16(out)) {
        p6_nchw_vec_kernel<T><<<grid_for(work / 8, 256), 256, 0, s>>>(i, o, N, C, H, W, H6, W6);
        return cudaGetLastError();
      }
    }
    p6_nchw_kernel<T><<<grid_for(work, 256), 256, 0, s>>>(i, o, N, C, H, W, H6, W6);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t transpose_t(const void* in, void* out, int N, int C, int HW, bool to_nhwc,
                        cudaStream_t s) {
  dim3 grid((HW + 31) / 32, (C + 31) / 32, N), block(32, 8);
  if (to_nhwc)
    nchw_to_nhwc_kernel<T>
        <<<grid, block, 0, s>>>(static_cast<const T*>(in), static_cast<T*>(out), C, HW);
  else
    nhwc_to_nchw_kernel<T>
        <<<grid, block, 0, s>>>(static_cast<const T*>(in), static_cast<T*>(out), C, HW);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_upsample_add(DType dt, const void* coarse, const void* lat, void* out, int N,
                                int C, int Hc, int Wc, int H, int W, int align_corners,
                                Layout layout, cudaStream_t s, unsigned* amax_out,
                                const MergeScaledCopy* scaled, LaunchOpts opts,
                                int units_per_block) {
  if (scaled && (!scaled->out || !scaled->scale_a || !scaled->scale_w || !aligned16(scaled->out)))
    return cudaErrorInvalidValue;
  if (units_per_block < -1) return cudaErrorInvalidValue;
  switch (dt) {
    case DType::F32:
      if (scaled) return cudaErrorNotSupported;
      return upsample_add_t<float>(coarse, lat, out, N, C, Hc, Wc, H, W, align_corners, layout, s,
                                   amax_out, nullptr, opts, units_per_block);
    case DType::F16:
      return upsample_add_t<__half>(coarse, lat, out, N, C, Hc, Wc, H, W, align_corners, layout,
                                    s, amax_out, scaled, opts, units_per_block);
    case DType::BF16:
      return upsample_add_t<__nv_bfloat16>(coarse, lat, out, N, C, Hc, Wc, H, W, align_corners,
                                           layout, s, amax_out, scaled, opts, units_per_block);
    default:
      return cudaErrorInvalidValue;
  }
}

namespace {
template <typename T>
cudaError_t merge_two_levels_t(const void* m5, const void* l4, void* m4, const void* l3, void* m3,
                               int N, int H5, int W5, int H4, int W4, int H3, int W3,
                               cudaStream_t s, unsigned* amax4, unsigned* amax3,
                               const MergeScaledCopy* sc, const LaunchOpts& opts) {
  // Region bound: the union of a tile's tap rows and its owned M4 rows spans at most
  // kMergeTileH * H4 / H3 + 3 rows (likewise columns); +4 keeps a margin for rounding.
  const int reg_h = static_cast<int>(static_cast<long long>(kMergeTileH) * H4 / H3) + 4;
  const int reg_w = static_cast<int>(static_cast<long long>(kMergeTileW) * W4 / W3) + 4;
  const size_t smem = static_cast<size_t>(reg_h) * reg_w * 512;
  if (smem > 200 * 1024) return cudaErrorNotSupported;
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(merge_two_levels_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  const int tiles_x = (W3 + kMergeTileW - 1) / kMergeTileW;
  const int tiles_y = (H3 + kMergeTileH - 1) / kMergeTileH;
  const long long blocks = static_cast<long long>(tiles_x) * tiles_y * N;
  if (blocks >= (1LL << 31)) return cudaErrorInvalidValue;
  // the scales of upsample_add_t (align_corners = 0)
  const float s54y = static_cast<float>(H5) / H4, s54x = static_cast<float>(W5) / W4;
  const float s43y = static_cast<float>(H4) / H3, s43x = static_cast<float>(W4) / W3;
  return launch_ex(merge_two_levels_kernel<T>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                   smem, s, opts, 1, static_cast<const T*>(m5), static_cast<const T*>(l4),
                   static_cast<T*>(m4), static_cast<const T*>(l3), static_cast<T*>(m3), H5, W5,
                   H4, W4, H3, W3, s54y, s54x, s43y, s43x, tiles_x, tiles_y, reg_h, reg_w, amax4,
                   amax3, sc ? static_cast<T*>(sc->out) : nullptr, sc ? sc->scale_a : nullptr,
                   sc ? sc->scale_w : nullptr);
}
}  // namespace

cudaError_t launch_merge_two_levels(DType dt, const void* m5, const void* l4, void* m4,
                                    const void* l3, void* m3, int N, int H5, int W5, int H4,
                                    int W4, int H3, int W3, cudaStream_t s, unsigned* amax4,
                                    unsigned* amax3, const MergeScaledCopy* m3_scaled,
                                    LaunchOpts opts) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorNotSupported;
  if (N <= 0 || H5 <= 0 || W5 <= 0 || H4 <= 0 || W4 <= 0 || H3 <= 0 || W3 <= 0)
    return cudaErrorInvalidValue;
  if (H5 > H4 || W5 > W4 || H4 > H3 || W4 > W3) return cudaErrorNotSupported;  // upsampling
  if (!m5 || !l4 || !m4 || !l3 || !m3) return cudaErrorInvalidValue;
  if (l4 == m4) return cudaErrorInvalidValue;
  if (!aligned16(m5) || !aligned16(l4) || !aligned16(m4) || !aligned16(l3) || !aligned16(m3))
    return cudaErrorMisalignedAddress;
  if (m3_scaled && (!m3_scaled->out || !m3_scaled->scale_a || !m3_scaled->scale_w ||
                    !aligned16(m3_scaled->out)))
    return cudaErrorInvalidValue;
  return dt == DType::BF16
             ? merge_two_levels_t<__nv_bfloat16>(m5, l4, m4, l3, m3, N, H5, W5, H4, W4, H3, W3,
                                                 s, amax4, amax3, m3_scaled, opts)
             : merge_two_levels_t<__half>(m5, l4, m4, l3, m3, N, H5, W5, H4, W4, H3, W3, s,
                                          amax4, amax3, m3_scaled, opts);
}

cudaError_t launch_p6(DType dt, const void* in, void* out, int N, int C, int H, int W,
                      Layout layout, cudaStream_t s) {
  switch (dt) {
    case DType::F32:
      return p6_t<float>(in, out, N, C, H, W, layout, s);
    case DType::F16:
      return p6_t<__half>(in, out, N, C, H, W, layout, s);
    case DType::BF16:
      return p6_t<__nv_bfloat16>(in, out, N, C, H, W, layout, s);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_transpose(DType dt, const void* in, void* out, int N, int C, int HW,
                             bool to_nhwc, cudaStream_t s) {
  switch (dt) {
    case DType::F32:
      return transpose_t<float>(in, out, N, C, HW, to_nhwc, s);
    case DType::F16:
      return transpose_t<__half>(in, out, N, C, HW, to_nhwc, s);
    case DType::BF16:
      return transpose_t<__nv_bfloat16>(in, out, N, C, HW, to_nhwc, s);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_convert_weights(DType dt, const float* in, void* out, long long n,
                                   cudaStream_t s) {
  const int g = grid_for(n, 256);
  switch (dt) {
    case DType::F32:
      return cudaMemcpyAsync(out, in, n * sizeof(float), cudaMemcpyDeviceToDevice, s);
    case DType::F16:
      convert_kernel<__half><<<g, 256, 0, s>>>(in, static_cast<__half*>(out), n);
      break;
    case DType::BF16:
      convert_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), n);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_pack_conv3x3(DType dt, const float* in, void* out, int Cout, int Cin,
                                cudaStream_t s) {
  const int g = grid_for(static_cast<long long>(Cout) * Cin * 9, 256);
  switch (dt) {
    case DType::F16:
      pack_conv3x3_kernel<__half><<<g, 256, 0, s>>>(in, static_cast<__half*>(out), Cout, Cin);
      break;
    case DType::BF16:
      pack_conv3x3_kernel<__nv_bfloat16>
          <<<g, 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), Cout, Cin);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_absmax(DType dt, const void* x, long long n, int groups, unsigned* amax_bits,
                          cudaStream_t s) {
  if (n <= 0 || !x || !amax_bits) return cudaErrorInvalidValue;
  switch (dt) {
    case DType::F32:
      return absmax_t<float>(x, n, groups, amax_bits, s);
    case DType::F16:
      return absmax_t<__half>(x, n, groups, amax_bits, s);
    case DType::BF16:
      return absmax_t<__nv_bfloat16>(x, n, groups, amax_bits, s);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_quantize_e4m3(DType dt, const void* x, long long n, int groups,
                                 const unsigned* amax_bits, void* q, float* scale_out,
                                 cudaStream_t s, LaunchOpts opts) {
  if (n <= 0 || !x || !q || !amax_bits) return cudaErrorInvalidValue;
  if (groups < 1 || groups > 65535 || n % groups != 0) return cudaErrorInvalidValue;
  const long long per = n / groups;
  const int vec = (aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0 && per % 8 == 0 &&
                   (per * dtype_size(dt)) % 16 == 0)
                      ? 1
                      : 0;
  const dim3 g(group_blocks(per, groups, 8), groups);
  n = per;
  uint8_t* qb = static_cast<uint8_t*>(q);
  switch (dt) {
    case DType::F32:
      return launch_ex(quantize_e4m3_kernel<float>, g, dim3(256), 0, s, opts, 1,
                       static_cast<const float*>(x), n, vec, amax_bits, qb, scale_out);
    case DType::F16:
      return launch_ex(quantize_e4m3_kernel<__half>, g, dim3(256), 0, s, opts, 1,
                       static_cast<const __half*>(x), n, vec, amax_bits, qb, scale_out);
    case DType::BF16:
      return launch_ex(quantize_e4m3_kernel<__nv_bfloat16>, g, dim3(256), 0, s, opts, 1,
                       static_cast<const __nv_bfloat16*>(x), n, vec, amax_bits, qb, scale_out);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_quantize_rows_e4m3(const float* w, int rows, int cols, int pack_cin, void* q,
                                      float* scales, cudaStream_t s) {
  if (!w || !q || !scales || rows <= 0 || cols <= 0) return cudaErrorInvalidValue;
  if (pack_cin > 0 && cols != 9 * pack_cin) return cudaErrorInvalidValue;
  quantize_rows_e4m3_kernel<<<rows, 256, 0, s>>>(w, cols, pack_cin, static_cast<uint8_t*>(q),
                                                 scales);
  return cudaGetLastError();
}

cudaError_t launch_fp32_lateral(const float* x, const float* w, const float* bias,
                                const float* coarse, float* out, int N, int Cin, int Cout, int H,
                                int W, int Hc, int Wc, cudaStream_t s) {
  dim3 grid((H * W + kSB - 1) / kSB, (Cout + kSB - 1) / kSB, N);
  const float sy = coarse ? static_cast<float>(Hc) / H : 0.f;
  const float sx = coarse ? static_cast<float>(Wc) / W : 0.f;
  fp32_conv_gemm_kernel<false>
      <<<grid, 256, 0, s>>>(x, w, bias, coarse, out, Cin, Cout, H, W, Hc, Wc, sy, sx, 0, 0.f);
  return cudaGetLastError();
}

cudaError_t launch_fp32_conv3x3(const float* x, const float* w, const float* bias, float* out,
                                int N, int Cin, int Cout, int H, int W, cudaStream_t s, int act,
                                float act_alpha) {
  if (act < 0 || act > 3) return cudaErrorInvalidValue;
  dim3 grid((H * W + kSB - 1) / kSB, (Cout + kSB - 1) / kSB, N);
  fp32_conv_gemm_kernel<true><<<grid, 256, 0, s>>>(x, w, bias, nullptr, out, Cin, Cout, H, W, 1,
                                                   1, 0.f, 0.f, act, act_alpha);
  return cudaGetLastError();
}

}  // namespace ufpn
