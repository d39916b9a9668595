// Host side of the tensor-core kernels: TMA descriptor encoding, tile
// planning and launch.  The device code lives in tc_gemm.cuh.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "conv_pair.cuh"
#include "kernels.h"
#include "lateral_group_pair.cuh"
#include "lateral_pair.cuh"
#include "neck_kernel.cuh"
#include "tc_gemm.cuh"

namespace ufpn {

static_assert(sizeof(TcGemmArgs) <= sizeof(TcPlan::args), "TcPlan::args too small");

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMapDataType tmap_dtype(DType dt) {
  switch (dt) {
    case DType::F16:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case DType::BF16:
      return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case DType::F32:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default:
      return CU_TENSOR_MAP_DATA_TYPE_UINT8;
  }
}

// rank-d tiled map with 128-byte swizzle (64-byte for a 64-byte inner box); dims/strides
// innermost first, strides in bytes.
cudaError_t encode(CUtensorMap* map, DType dt, int rank, const void* base, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box,
                   CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (!aligned16(base)) return cudaErrorMisalignedAddress;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16 != 0) return cudaErrorInvalidValue;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    if (box[i] < 1 || box[i] > 256) return cudaErrorInvalidValue;
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = fn(map, tmap_dtype(dt), rank, const_cast<void*>(base), d, st, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// NHWC activation map [N][H][W][C] with a (one 128-byte row of channels, bw, bh, 1) box, or
// with inner_bytes = 64 a 64-byte row of channels under the 64-byte swizzle (16-byte chunk c
// of box row r at chunk c ^ ((r >> 1) & 3)).  transposed: the map's (N, W, H, C) view --
// coordinate 1 runs down a column (stride W * C), coordinate 2 along a row (stride C), and a
// box of (bw, bh) covers bw rows of bh columns, stored column by column.
cudaError_t encode_nhwc(CUtensorMap* map, DType dt, const void* base, int N, int H, int W, int C,
                        int bw, int bh, int inner_bytes = 128, bool transposed = false) {
  const uint64_t esz = static_cast<uint64_t>(dtype_size(dt));
  const uint64_t pix = static_cast<uint64_t>(C) * esz, row = static_cast<uint64_t>(W) * pix;
  uint64_t dims[4] = {static_cast<uint64_t>(C), static_cast<uint64_t>(transposed ? H : W),
                      static_cast<uint64_t>(transposed ? W : H), static_cast<uint64_t>(N)};
  uint64_t strides[3] = {transposed ? row : pix, transposed ? pix : row,
                         static_cast<uint64_t>(H) * row};
  uint32_t box[4] = {static_cast<uint32_t>(inner_bytes / esz), static_cast<uint32_t>(bw),
                     static_cast<uint32_t>(bh), 1};
  return encode(map, dt, 4, base, dims, strides, box,
                inner_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

// Weights [256][K] K-major, (one 128-byte row of K, box_rows) box (256 rows, or 128 for
// the half k-blocks of a CTA pair).
cudaError_t encode_weights(CUtensorMap* map, DType dt, const void* base, int K,
                           int box_rows = kTcBlockN, int rows = kTcBlockN) {
  const uint64_t esz = static_cast<uint64_t>(dtype_size(dt));
  uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows)};
  uint64_t strides[1] = {static_cast<uint64_t>(K) * esz};
  uint32_t box[2] = {static_cast<uint32_t>(128 / esz), static_cast<uint32_t>(box_rows)};
  return encode(map, dt, 2, base, dims, strides, box);
}

// Host replay of the device's tc_src (every step rounded to fp32, no contraction).
float host_src(int o, float scale, int in) {
  volatile float a = static_cast<float>(o) + 0.5f;
  volatile float b = a * scale;
  volatile float c = b - 0.5f;
  float r = c;
  if (r < 0.f) r = 0.f;
  const float hi = static_cast<float>(in - 1);
  if (r > hi) r = hi;
  return r;
}

// Largest number of coarse rows (or columns) the bilinear taps of one tile of `tile`
// outputs can touch, over all tiles of an `out`-long axis.
int coarse_span(int out, int tile, float scale, int in) {
  int span = 0;
  for (int o0 = 0; o0 < out; o0 += tile) {
    const int lo = static_cast<int>(host_src(o0, scale, in));
    const int last = o0 + tile - 1 < out - 1 ? o0 + tile - 1 : out - 1;
    int hi = static_cast<int>(host_src(last, scale, in)) + 1;
    if (hi > in - 1) hi = in - 1;
    if (hi - lo + 1 > span) span = hi - lo + 1;
  }
  return span;
}

bool valid_tiling(Conv3x3Tiling t) {
  return t.tile_w >= 8 && t.tile_w <= 128 && (t.tile_w & (t.tile_w - 1)) == 0 &&
         t.tile_w * t.tile_h == kTcBlockM;
}

void fill_tiling(TcGemmArgs& a, int N, int H, int W, Conv3x3Tiling t) {
  a.N_img = N;
  a.H = H;
  a.W = W;
  a.tile_w = t.tile_w;
  a.tile_h = t.tile_h;
  a.tiles_x = (W + t.tile_w - 1) / t.tile_w;
  a.tiles_y = (H + t.tile_h - 1) / t.tile_h;
}

template <int kMode, typename T, bool kWideEpi = kMode == 0 && TcElem<T>::kFp8>
cudaError_t launch_t(const TcPlan& p, cudaStream_t s, LaunchOpts opts) {
  using Cfg = TcCfgT<kMode, T, kWideEpi>;
  auto kern = fpn_tc_gemm_kernel<kMode, T, kWideEpi>;
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  TcGemmArgs a;
  std::memcpy(&a, p.args, sizeof(a));
  return launch_ex(kern, dim3(p.grid), dim3(Cfg::kThreads),
                   Cfg::kSmemBytes, s, opts, 1, p.map_a, p.map_b, p.map_out,
                   p.map_coarse, a);
}

template <typename T>
cudaError_t launch_halo_t(const TcPlan& p, cudaStream_t s, LaunchOpts opts) {
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(fpn_conv3x3_halo_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, HaloCfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  TcGemmArgs a;
  std::memcpy(&a, p.args, sizeof(a));
  // (map_coarse of a single-CTA halo plan: the 128-row weight box of its channel-half items)
  return launch_ex(fpn_conv3x3_halo_kernel<T>, dim3(p.grid), dim3(kTcThreads),
                   HaloCfg::kSmemBytes, s, opts, 1, p.map_a, p.map_b, p.map_out, p.map_a2,
                   p.map_out2, p.map_coarse, a);
}

template <typename T, bool kCvt, bool kClaims>
cudaError_t launch_halo_pair_form(const TcPlan& p, const TcGemmArgs& a, cudaStream_t s,
                                  LaunchOpts opts) {
  auto kern = fpn_conv3x3_halo_pair_kernel<T, kCvt, kClaims>;
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                PairCfgT<kCvt>::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  // (map_coarse of a CTA-pair 3x3 plan: the 64-row weight box of its channel-half items)
  return launch_ex(kern, dim3(p.grid), dim3(PairCfgT<kCvt>::kThreads),
                   PairCfgT<kCvt>::kSmemBytes, s, opts, 2, p.map_a, p.map_b, p.map_out,
                   p.map_coarse, p.map_a2, p.map_out2, a);
}
template <typename T, bool kCvt = false>
cudaError_t launch_halo_pair_t(const TcPlan& p, cudaStream_t s, LaunchOpts opts) {
  TcGemmArgs a;
  std::memcpy(&a, p.args, sizeof(a));
  // run-time item claims: a separate instantiation, so the static form carries none of it
  return a.claim != nullptr ? launch_halo_pair_form<T, kCvt, true>(p, a, s, opts)
                            : launch_halo_pair_form<T, kCvt, false>(p, a, s, opts);
}

template <typename T>
cudaError_t launch_lateral_pair_t(const TcPlan& p, cudaStream_t s, LaunchOpts opts) {
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(fpn_lateral_pair_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, LpCfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  TcGemmArgs a;
  std::memcpy(&a, p.args, sizeof(a));
  return launch_ex(fpn_lateral_pair_kernel<T>, dim3(p.grid), dim3(kTcThreads), LpCfg::kSmemBytes,
                   s, opts, 2, p.map_a, p.map_b, p.map_out, p.map_coarse, a);
}

}  // namespace

int sm_count() {
  static std::atomic<int> counts[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev >= 0 && dev < 64;
  int n = cached ? counts[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (cached) counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

long long l2_bytes() {
  static std::atomic<long long> sizes[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev >= 0 && dev < 64;
  long long n = cached ? sizes[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev);
    n = v > 0 ? v : 126LL << 20;
    if (cached) sizes[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

Conv3x3Tiling default_tiling(int H, int W) {
  Conv3x3Tiling best;
  long long best_area = -1;
  for (int tw : {16, 8, 32, 64, 128}) {
    const int th = kTcBlockM / tw;
    const long long area = static_cast<long long>((W + tw - 1) / tw) * tw *
                           static_cast<long long>((H + th - 1) / th) * th;
    if (best_area < 0 || area < best_area) {
      best_area = area;
      best.tile_w = tw;
      best.tile_h = th;
    }
  }
  return best;
}

cudaError_t plan_tc_lateral(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, const void* coarse, void* out, int N, int Cin,
                            int H, int W, int Hc, int Wc, Conv3x3Tiling tiling, int* status,
                            int max_ctas, const TcScales& sc) {
  if (dt != DType::BF16 && dt != DType::F16 && dt != DType::E4M3) return cudaErrorInvalidValue;
  const bool fp8 = dt == DType::E4M3;
  const DType odt = fp8 ? DType::BF16 : dt;  // output / coarse element type
  const int kb_elems = 128 / dtype_size(dt);
  if (Cin <= 0 || (Cin * dtype_size(dt)) % 16 != 0 || N <= 0 || H <= 0 || W <= 0) return cudaErrorInvalidValue;
  if (!valid_tiling(tiling)) return cudaErrorInvalidValue;
  if (coarse && (Hc <= 0 || Wc <= 0)) return cudaErrorInvalidValue;
  if (fp8 && (!sc.ascale || !sc.wscale)) return cudaErrorInvalidValue;
  // (out_mode 2: each of the lateral's 16 epilogue warps stores its 64 channels as 64-byte
  // e4m3 rows through a map with a 64-byte box and the 64-byte swizzle.)
  if (sc.out_mode < 0 || sc.out_mode > 2 || (sc.out_mode == 1 && !sc.amax_out) ||
      (sc.out_mode == 2 && (!sc.qamax || !sc.qscale_out)))
    return cudaErrorInvalidValue;
  if (!aligned16(out) || (coarse && !aligned16(coarse)) || !aligned16(bias) ||
      (fp8 && !aligned16(sc.wscale)))
    return cudaErrorMisalignedAddress;
  TcGemmArgs a;
  std::memset(&a, 0, sizeof(a));
  fill_tiling(a, N, H, W, tiling);
  const long long tiles = static_cast<long long>(a.tiles_x) * a.tiles_y * N;
  if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
  a.num_tiles = static_cast<int>(tiles);
  a.cin_blocks = (Cin + kb_elems - 1) / kb_elems;
  a.num_kb = a.cin_blocks;
  a.bias = bias;
  a.status = status;
  a.ascale = sc.ascale;
  a.ascale_stride = sc.ascale_per_image ? 1 : 0;
  a.wscale = sc.wscale;
  a.amax_out = sc.amax_out;
  a.out_mode = sc.out_mode;
  a.qamax = sc.qamax;
  a.qscale_out = sc.qscale_out;
  cudaError_t e = encode_nhwc(&plan.map_a, dt, x, N, H, W, Cin, tiling.tile_w, tiling.tile_h);
  if (e != cudaSuccess) return e;
  if ((e = encode_weights(&plan.map_b, dt, w, Cin)) != cudaSuccess) return e;
  const int sw = tiling.tile_w < 32 ? tiling.tile_w : 32;
  if ((e = encode_nhwc(&plan.map_out, sc.out_mode == 2 ? DType::E4M3 : odt, out, N, H, W,
                       kTcBlockN, sw, 32 / sw, sc.out_mode == 2 ? 64 : 128)) != cudaSuccess)
    return e;
  plan.map_coarse = plan.map_out;  // unused unless a coarse map is staged
  if (coarse) {
    a.coarse = coarse;
    a.Hc = Hc;
    a.Wc = Wc;
    a.scale_y = static_cast<float>(Hc) / static_cast<float>(H);
    a.scale_x = static_cast<float>(Wc) / static_cast<float>(W);
    // Coarse box of the tensor-core top-down add: the exact span of the taps of any
    // tile (replaying the device arithmetic); must fit one 64-pixel k-block.  (e4m3:
    // the accumulator is scaled in the epilogue, so the taps are added there.)
    const int ch = coarse_span(H, tiling.tile_h, a.scale_y, Hc);
    const int cw = coarse_span(W, tiling.tile_w, a.scale_x, Wc);
    if ((!fp8 || sc.coarse_prescaled) && ch * cw <= kTcCoarseMaxPix) {
      a.cbox_h = ch;
      a.cbox_w = cw;
      if ((e = encode_nhwc(&plan.map_coarse, odt, coarse, N, Hc, Wc, kTcBlockN, cw, ch)) !=
          cudaSuccess)
        return e;
    }
  }
  std::memcpy(plan.args, &a, sizeof(a));
  plan.mode = 0;
  plan.dtype = dt;
  plan.num_tiles = a.num_tiles;
  const int cap = max_ctas > 0 ? max_ctas : sm_count();
  plan.grid = a.num_tiles < cap ? a.num_tiles : cap;
  return cudaSuccess;
}

cudaError_t plan_tc_lateral_pair(TcPlan& plan, DType dt, const void* x, const void* w,
                                 const float* bias, const void* coarse, void* out, int N,
                                 int Cin, int H, int W, int Hc, int Wc, Conv3x3Tiling tiling,
                                 int* status, int max_ctas) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorNotSupported;
  cudaError_t e = plan_tc_lateral(plan, dt, x, w, bias, coarse, out, N, Cin, H, W, Hc, Wc, tiling,
                                  status, max_ctas);
  if (e != cudaSuccess) return e;
  TcGemmArgs a;
  std::memcpy(&a, plan.args, sizeof(a));
  // resident weight halves must fit; a top-down add needs its staged coarse box
  if (a.num_kb > kLpMaxKb || (coarse && a.cbox_w <= 0)) return cudaErrorNotSupported;
  if ((e = encode_weights(&plan.map_b, dt, w, Cin, kTcBlockN / 2)) != cudaSuccess) return e;
  plan.mode = 5;
  const int units = (a.num_tiles + 1) / 2;
  const int cap = (max_ctas > 0 ? max_ctas : sm_count()) / 2;
  if (cap < 1) return cudaErrorInvalidValue;
  plan.grid = 2 * (units < cap ? units : cap);
  return cudaSuccess;
}

cudaError_t plan_tc_conv3x3(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, void* out, void* p6, int N, int H, int W,
                            Conv3x3Tiling tiling, int* status, int max_ctas,
                            const TcScales& sc, int* claim) {
  if (dt != DType::BF16 && dt != DType::F16 && dt != DType::E4M3) return cudaErrorInvalidValue;
  const bool fp8 = dt == DType::E4M3;
  const DType odt = fp8 ? DType::BF16 : dt;
  if (!valid_tiling(tiling)) return cudaErrorInvalidValue;
  if (N <= 0 || H <= 0 || W <= 0) return cudaErrorInvalidValue;
  // in_amax (e4m3 only): x is the bf16 map, quantised per image inside the kernel
  const bool cvt = fp8 && sc.in_amax != nullptr;
  if (fp8 && ((!sc.ascale && !cvt) || !sc.wscale || !tiling.halo)) return cudaErrorInvalidValue;
  if (cvt && !tiling.pair) return cudaErrorInvalidValue;
  if (!aligned16(out) || (p6 && !aligned16(p6)) || !aligned16(bias) ||
      (fp8 && !aligned16(sc.wscale)))
    return cudaErrorMisalignedAddress;
  const int C = kTcBlockN;
  // Transposed view: the kernel sees a W x H map (its tensor maps swap the two axes) and
  // mirrors each tap; only halo tilings, and not with the fused P6 (whose indexing is the
  // map's own).
  const bool tr = tiling.transposed;
  if (tr && (!tiling.halo || p6 != nullptr)) return cudaErrorInvalidValue;
  // Mixed tiling: the own view for rows [0, 16 floor(H/16)), the transposed view for the
  // strip of the remaining 1..8 rows.
  const bool mixed = tiling.mixed;
  if (mixed && (!tiling.halo || tr || p6 != nullptr || H < 16 || H % 16 == 0 || H % 16 > 8))
    return cudaErrorInvalidValue;
  TcGemmArgs a;
  std::memset(&a, 0, sizeof(a));
  fill_tiling(a, N, tr ? W : H, tr ? H : W, tiling);
  a.transposed = tr ? 1 : 0;
  long long tiles = static_cast<long long>(a.tiles_x) * a.tiles_y * N;
  if (mixed) {
    a.tiles_y = H / kHaloTileH;  // whole 16-row tile rows on the own view
    const long long own = static_cast<long long>(a.tiles_x) * a.tiles_y * N;
    if (tiling.pair && own % 2 != 0) return cudaErrorInvalidValue;
    a.strip_y0 = a.tiles_y * kHaloTileH;
    a.strip_tx = (W + kHaloTileH - 1) / kHaloTileH;
    tiles = own + static_cast<long long>(a.strip_tx) * N;
    if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
    a.strip_first = static_cast<int>(own);
  }
  if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
  a.num_tiles = static_cast<int>(tiles);
  a.cin_blocks = C / (128 / dtype_size(dt));
  a.num_kb = 9 * a.cin_blocks;
  a.bias = bias;
  a.p6 = p6;
  a.H6 = (H - 1) / 2 + 1;
  a.W6 = (W - 1) / 2 + 1;
  a.status = status;
  a.ascale = sc.ascale;
  a.ascale_stride = sc.ascale_per_image ? 1 : 0;
  a.wscale = sc.wscale;
  a.amax_out = sc.amax_out;
  a.in_amax = sc.in_amax;
  if (sc.act < 0 || sc.act > 3) return cudaErrorInvalidValue;
  a.act = sc.act;
  a.act_alpha = sc.act_alpha;
  const bool halo = tiling.halo;
  if (halo && (tiling.tile_w != kHaloTileW || tiling.tile_h != kHaloTileH))
    return cudaErrorInvalidValue;
  if (tiling.pair && !halo) return cudaErrorInvalidValue;
  // Halo path: one (tile_w + 2) x (tile_h + 2) box per channel block, origin (-1, -1)
  // (bf16 boxes of 64 channels when the kernel quantises its input itself).
  cudaError_t e = halo ? encode_nhwc(&plan.map_a, cvt ? DType::BF16 : dt, x, N, H, W, C,
                                     kHaloTileW + 2, kHaloTileH + 2, 128, tr)
                       : encode_nhwc(&plan.map_a, dt, x, N, H, W, C, tiling.tile_w, tiling.tile_h);
  if (e != cudaSuccess) return e;
  plan.map_a2 = plan.map_a;  // (unused unless mixed)
  if (mixed && (e = encode_nhwc(&plan.map_a2, cvt ? DType::BF16 : dt, x, N, H, W, C,
                                kHaloTileW + 2, kHaloTileH + 2, 128, true)) != cudaSuccess)
    return e;
  if ((e = encode_weights(&plan.map_b, dt, w, 9 * C, tiling.pair ? kTcBlockN / 2 : kTcBlockN)) !=
      cudaSuccess)
    return e;
  const int sw = tiling.tile_w < 32 ? tiling.tile_w : 32;
  if ((e = encode_nhwc(&plan.map_out, odt, out, N, H, W, kTcBlockN, sw, 32 / sw, 128, tr)) !=
      cudaSuccess)
    return e;
  plan.map_out2 = plan.map_out;
  if (mixed && (e = encode_nhwc(&plan.map_out2, odt, out, N, H, W, kTcBlockN, sw, 32 / sw, 128,
                                true)) != cudaSuccess)
    return e;
  plan.map_coarse = plan.map_out;
  plan.mode = cvt ? 4 : (tiling.pair ? 3 : (halo ? 2 : 1));
  plan.dtype = dt;
  plan.num_tiles = a.num_tiles;
  const int cap = max_ctas > 0 ? max_ctas : sm_count();
  if (tiling.pair) {
    a.claim = claim;
    // One (2,1,1) cluster per pair unit (two tiles), at most one CTA per SM.
    const int units = (a.num_tiles + 1) / 2;
    const int clusters = units < cap / 2 ? units : cap / 2;
    plan.grid = 2 * (clusters > 0 ? clusters : 1);
    // A last round of rem < clusters units: if its units split over the output channels fit
    // the pairs (2 rem <= clusters), run them as halves (N = 128), half as long a round.
    const int rem = clusters > 0 ? units % clusters : 0;
    if (tiling.tail_halves && rem > 0 && 2 * rem <= clusters) {
      a.pair_tail = rem;
      if ((e = encode_weights(&plan.map_coarse, dt, w, 9 * C, kTcBlockN / 4)) != cudaSuccess)
        return e;
    }
  } else {
    plan.grid = a.num_tiles < cap ? a.num_tiles : cap;
    // Halo tiles on single CTAs: the same for a last round of rem < grid tiles that fit the
    // CTAs as halves (2 rem <= grid; the halves' weight box has 128 rows).
    const int rem = plan.grid > 0 ? a.num_tiles % plan.grid : 0;
    if (halo && tiling.tail_halves && rem > 0 && 2 * rem <= plan.grid) {
      a.pair_tail = rem;
      if ((e = encode_weights(&plan.map_coarse, dt, w, 9 * C, kTcBlockN / 2)) != cudaSuccess)
        return e;
    }
  }
  std::memcpy(plan.args, &a, sizeof(a));
  return cudaSuccess;
}

size_t tc_wb_table_bytes(int H, int W, int Hc, int Wc, Conv3x3Tiling t) {
  if (!valid_tiling(t) || H <= 0 || W <= 0 || Hc <= 0 || Wc <= 0) return 0;
  const float sy = static_cast<float>(Hc) / static_cast<float>(H);
  const float sx = static_cast<float>(Wc) / static_cast<float>(W);
  const int ch = coarse_span(H, t.tile_h, sy, Hc);
  const int cw = coarse_span(W, t.tile_w, sx, Wc);
  if (ch * cw > kTcCoarseMaxPix) return 0;  // the lateral adds taps in its epilogue instead
  const size_t entries = static_cast<size_t>((W + t.tile_w - 1) / t.tile_w) *
                         static_cast<size_t>((H + t.tile_h - 1) / t.tile_h);
  return entries * kTcAStage;
}

cudaError_t tc_build_wb_table(DType dt, int H, int W, int Hc, int Wc, Conv3x3Tiling t,
                              void* table, cudaStream_t s) {
  const size_t bytes = tc_wb_table_bytes(H, W, Hc, Wc, t);
  if (bytes == 0 || !table || !aligned16(table)) return cudaErrorInvalidValue;
  TcGemmArgs a;
  std::memset(&a, 0, sizeof(a));
  fill_tiling(a, 1, H, W, t);
  a.Hc = Hc;
  a.Wc = Wc;
  a.scale_y = static_cast<float>(Hc) / static_cast<float>(H);
  a.scale_x = static_cast<float>(Wc) / static_cast<float>(W);
  a.cbox_h = coarse_span(H, t.tile_h, a.scale_y, Hc);
  a.cbox_w = coarse_span(W, t.tile_w, a.scale_x, Wc);
  const int entries = a.tiles_x * a.tiles_y;
  const size_t smem = kTcAStage + 1024;
  if (dt == DType::F16)
    tc_wb_table_kernel<__half><<<entries, 32, smem, s>>>(a, static_cast<uint8_t*>(table));
  else
    tc_wb_table_kernel<__nv_bfloat16><<<entries, 32, smem, s>>>(a, static_cast<uint8_t*>(table));
  return cudaGetLastError();
}

cudaError_t encode_nhwc_map(CUtensorMap* map, DType dt, const void* base, int N, int H, int W,
                            int C, int pix_stride, int bw, int bh) {
  if (N <= 0 || H <= 0 || W <= 0 || C <= 0 || pix_stride < C) return cudaErrorInvalidValue;
  const uint64_t esz = static_cast<uint64_t>(dtype_size(dt));
  uint64_t dims[4] = {static_cast<uint64_t>(C), static_cast<uint64_t>(W),
                      static_cast<uint64_t>(H), static_cast<uint64_t>(N)};
  uint64_t strides[3] = {static_cast<uint64_t>(pix_stride) * esz,
                         static_cast<uint64_t>(W) * pix_stride * esz,
                         static_cast<uint64_t>(H) * W * pix_stride * esz};
  uint32_t box[4] = {static_cast<uint32_t>(128 / esz), static_cast<uint32_t>(bw),
                     static_cast<uint32_t>(bh), 1};
  return encode(map, dt, 4, base, dims, strides, box);
}

cudaError_t encode_rows_map(CUtensorMap* map, DType dt, const void* base, int cols, long long rows,
                            int box_cols, int box_rows) {
  if (cols <= 0 || rows <= 0 || box_cols * dtype_size(dt) != 128) return cudaErrorInvalidValue;
  const uint64_t esz = static_cast<uint64_t>(dtype_size(dt));
  uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  uint64_t strides[1] = {static_cast<uint64_t>(cols) * esz};
  uint32_t box[2] = {static_cast<uint32_t>(box_cols), static_cast<uint32_t>(box_rows)};
  return encode(map, dt, 2, base, dims, strides, box);
}

cudaError_t tc_set_output_view(TcPlan& plan, void* out, int C, int pix_stride) {
  if (plan.mode != 0 || plan.dtype == DType::E4M3) return cudaErrorNotSupported;
  if (!aligned16(out)) return cudaErrorMisalignedAddress;
  TcGemmArgs a;
  std::memcpy(&a, plan.args, sizeof(a));
  if (C > kTcBlockN) return cudaErrorInvalidValue;
  const int sw = a.tile_w < 32 ? a.tile_w : 32;
  cudaError_t e = encode_nhwc_map(&plan.map_out, plan.dtype, out, a.N_img, a.H, a.W, C,
                                  pix_stride, sw, 32 / sw);
  if (e != cudaSuccess) return e;
  a.out_cols = C;
  std::memcpy(plan.args, &a, sizeof(a));
  return cudaSuccess;
}

cudaError_t tc_set_channel_slices(TcPlan& plan, const void* w, int K, int slices, void* out,
                                  int C) {
  if (plan.mode != 0 || plan.dtype == DType::E4M3) return cudaErrorNotSupported;
  if (!w || !out || slices < 1 || C <= 0 || C > slices * kTcBlockN ||
      C <= (slices - 1) * kTcBlockN)
    return cudaErrorInvalidValue;
  if (!aligned16(out) || !aligned16(w)) return cudaErrorMisalignedAddress;
  TcGemmArgs a;
  std::memcpy(&a, plan.args, sizeof(a));
  if (a.coarse != nullptr || a.out_mode != 0 || a.amax_out != nullptr || a.slices > 1)
    return cudaErrorNotSupported;
  const long long tiles = static_cast<long long>(a.num_tiles) * slices;
  if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
  const int kb_elems = 128 / dtype_size(plan.dtype);
  if (K <= (a.cin_blocks - 1) * kb_elems || K > a.cin_blocks * kb_elems) return cudaErrorInvalidValue;
  cudaError_t e = encode_weights(&plan.map_b, plan.dtype, w, K, kTcBlockN, slices * kTcBlockN);
  if (e != cudaSuccess) return e;
  const int sw = a.tile_w < 32 ? a.tile_w : 32;
  if ((e = encode_nhwc_map(&plan.map_out, plan.dtype, out, a.N_img, a.H, a.W, C, C, sw,
                           32 / sw)) != cudaSuccess)
    return e;
  a.out_cols = C;
  a.slices = slices;
  a.num_tiles = static_cast<int>(tiles);
  std::memcpy(plan.args, &a, sizeof(a));
  plan.num_tiles = a.num_tiles;
  const int cap = sm_count();
  plan.grid = a.num_tiles < cap ? a.num_tiles : cap;
  return cudaSuccess;
}

bool tc_use_wide_epilogue(TcPlan& plan) {
  if (plan.mode != 0 || (plan.dtype != DType::BF16 && plan.dtype != DType::F16)) return false;
  plan.mode = 6;
  return true;
}

bool tc_attach_wb_table(TcPlan& plan, const void* table) {
  TcGemmArgs a;
  std::memcpy(&a, plan.args, sizeof(a));
  if (plan.mode != 0 || !a.coarse || a.cbox_w <= 0 || !table) return false;
  a.wb_table = static_cast<const uint8_t*>(table);
  std::memcpy(plan.args, &a, sizeof(a));
  return true;
}

static_assert(sizeof(NeckParams) <= sizeof(NeckPlan::params), "NeckPlan::params too small");

int neck_lateral_tiles(int N, int H, int W, Conv3x3Tiling t) {
  if (!valid_tiling(t) || N <= 0 || H <= 0 || W <= 0) return 0;
  return ((W + t.tile_w - 1) / t.tile_w) * ((H + t.tile_h - 1) / t.tile_h) * N;
}

size_t neck_split_part_bytes(int N, int H, int W, Conv3x3Tiling t, int ksplit) {
  return static_cast<size_t>(neck_lateral_tiles(N, H, W, t)) * (ksplit > 1 ? ksplit : 0) *
         kTcBlockM * kTcBlockN * sizeof(float);
}

cudaError_t plan_neck_jobs(NeckPlan& plan, DType dt, int N, const NeckLevel* lv, void* p6,
                           const NeckJobSpec* specs, int num_specs, int* sched, int* status,
                           int max_ctas, unsigned long long* trace) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorInvalidValue;
  if (N <= 0 || !sched || num_specs < 1 || num_specs > kNeckMaxJobs) return cudaErrorInvalidValue;
  NeckParams* P = reinterpret_cast<NeckParams*>(plan.params);
  std::memset(plan.params, 0, sizeof(plan.params));
  int lat_tiles[4] = {};
  bool lat_in_launch[4] = {};
  for (int j = 0; j < num_specs; ++j) {
    const NeckJobSpec& s = specs[j];
    if (s.level < 0 || s.level > 3 || (s.mode != 0 && s.mode != 1)) return cudaErrorInvalidValue;
    if (s.mode == 0 && s.coarse && s.level == 3) return cudaErrorInvalidValue;
    const NeckLevel& L = lv[s.level];
    const Conv3x3Tiling t = s.mode == 0 ? L.lat_tiling : L.conv_tiling;
    if (!valid_tiling(t)) return cudaErrorInvalidValue;
    if (L.H <= 0 || L.W <= 0 || !aligned16(L.merged)) return cudaErrorInvalidValue;
    if (s.mode == 0) {
      if (L.Cin <= 0 || L.Cin % 8 != 0 || !aligned16(L.lat_b)) return cudaErrorInvalidValue;
      if (lat_in_launch[s.level]) return cudaErrorInvalidValue;
      if (s.ksplit != 1 && s.ksplit != 2 && s.ksplit != 4) return cudaErrorInvalidValue;
      if (s.nsplit != 1 && (s.nsplit != 2 || s.ksplit != 1 || s.coarse))
        return cudaErrorInvalidValue;
      const int cin_blocks = (L.Cin + kTcBlockK - 1) / kTcBlockK;
      if (s.ksplit > 1 && (cin_blocks < s.ksplit || !L.split_part || !L.split_sem ||
                           !aligned16(L.split_part)))
        return cudaErrorInvalidValue;
      lat_in_launch[s.level] = true;
      // (completions counted per publishing unit: a channel half publishes its own half)
      lat_tiles[s.level] =
          ((L.W + t.tile_w - 1) / t.tile_w) * ((L.H + t.tile_h - 1) / t.tile_h) * N * s.nsplit;
    } else if (s.ksplit != 1 || s.nsplit != 1) {
      return cudaErrorInvalidValue;
    } else if (!aligned16(L.out) || !aligned16(L.conv_b)) {
      return cudaErrorMisalignedAddress;
    }
  }
  int start = 0;
  for (int j = 0; j < num_specs; ++j) {
    const int mode = specs[j].mode, l = specs[j].level;
    const NeckLevel& L = lv[l];
    NeckJob& J = P->jobs[j];
    J.mode = mode;
    J.level = l;
    const Conv3x3Tiling t = mode == 0 ? L.lat_tiling : L.conv_tiling;
    J.N_img = N;
    J.H = L.H;
    J.W = L.W;
    J.tile_w = t.tile_w;
    J.tile_h = t.tile_h;
    J.tiles_x = (L.W + t.tile_w - 1) / t.tile_w;
    J.tiles_y = (L.H + t.tile_h - 1) / t.tile_h;
    J.num_tiles = J.tiles_x * J.tiles_y * N;
    J.tile_start = start;
    start += J.num_tiles;
    J.dep_level = -1;
    cudaError_t e;
    const int sw = t.tile_w < 32 ? t.tile_w : 32;
    if (mode == 0) {
      // Publish completions only if a later job of this launch waits on this level.
      for (int k = j + 1; k < num_specs; ++k)
        if ((specs[k].mode == 1 && specs[k].level == l) ||
            (specs[k].mode == 0 && specs[k].coarse && specs[k].level == l - 1))
          J.publish = 1;
      J.cin_blocks = (L.Cin + kTcBlockK - 1) / kTcBlockK;
      J.num_kb = J.cin_blocks;
      J.bias = L.lat_b;
      J.ksplit = specs[j].ksplit;
      J.nsplit = specs[j].nsplit;
      if (J.nsplit > 1) {
        start += J.num_tiles * (J.nsplit - 1);  // units = tiles x channel halves
        J.num_tiles *= J.nsplit;
      }
      if (J.ksplit > 1) {
        // ceil(num_kb / ksplit) k-blocks per unit; every unit gets at least one
        J.kb_per = (J.num_kb + J.ksplit - 1) / J.ksplit;
        while ((J.ksplit - 1) * J.kb_per >= J.num_kb) --J.kb_per;  // (never below 1: checked)
        J.part = L.split_part;
        J.sem = L.split_sem;
        start += J.num_tiles * (J.ksplit - 1);  // units = tiles x ksplit
        J.num_tiles *= J.ksplit;
      } else {
        J.kb_per = J.num_kb;
      }
      if ((e = encode_nhwc(&J.map_a, dt, L.x, N, L.H, L.W, L.Cin, t.tile_w, t.tile_h)) !=
          cudaSuccess)
        return e;
      if ((e = encode_weights(&J.map_b, dt, L.lat_w, L.Cin, kTcBlockN / J.nsplit)) !=
          cudaSuccess)
        return e;
      if ((e = encode_nhwc(&J.map_out, dt, L.merged, N, L.H, L.W, kTcBlockN, sw, 32 / sw)) !=
          cudaSuccess)
        return e;
      J.map_coarse = J.map_out;
      if (specs[j].coarse) {
        const NeckLevel& C = lv[l + 1];
        J.coarse = C.merged;
        J.Hc = C.H;
        J.Wc = C.W;
        J.scale_y = static_cast<float>(C.H) / static_cast<float>(L.H);
        J.scale_x = static_cast<float>(C.W) / static_cast<float>(L.W);
        // Wait for M_{l+1} only if its lateral runs in this launch (else it is complete).
        J.dep_count = lat_in_launch[l + 1] ? lat_tiles[l + 1] : 0;
        const int ch = static_cast<int>(std::ceil((t.tile_h - 1) * J.scale_y)) + 2;
        const int cw = static_cast<int>(std::ceil((t.tile_w - 1) * J.scale_x)) + 2;
        // (split-K tiles read their taps from global memory in the last unit's epilogue)
        if (J.ksplit <= 1 && ch * cw <= kTcCoarseMaxPix && ch <= 256 && cw <= 256) {
          J.cbox_h = ch;
          J.cbox_w = cw;
          if ((e = encode_nhwc(&J.map_coarse, dt, C.merged, N, C.H, C.W, kTcBlockN, cw, ch)) !=
              cudaSuccess)
            return e;
        }
      }
    } else {
      J.cin_blocks = kTcBlockN / kTcBlockK;
      J.num_kb = 9 * J.cin_blocks;
      J.kb_per = J.num_kb;
      J.ksplit = 1;
      J.nsplit = 1;
      J.bias = L.conv_b;
      if (L.act < 0 || L.act > 3) return cudaErrorInvalidValue;
      J.act = L.act;
      J.act_alpha = L.act_alpha;
      if (lat_in_launch[l]) {
        J.dep_level = l;
        J.dep_count = lat_tiles[l];
      }
      if ((e = encode_nhwc(&J.map_a, dt, L.merged, N, L.H, L.W, kTcBlockN, t.tile_w,
                           t.tile_h)) != cudaSuccess)
        return e;
      if ((e = encode_weights(&J.map_b, dt, L.conv_w, 9 * kTcBlockN)) != cudaSuccess) return e;
      if ((e = encode_nhwc(&J.map_out, dt, L.out, N, L.H, L.W, kTcBlockN, sw, 32 / sw)) !=
          cudaSuccess)
        return e;
      J.map_coarse = J.map_out;
      if (l == 3 && p6) {
        if (!aligned16(p6)) return cudaErrorMisalignedAddress;
        J.p6 = p6;
        J.H6 = (L.H - 1) / 2 + 1;
        J.W6 = (L.W - 1) / 2 + 1;
      }
    }
  }
  P->num_jobs = num_specs;
  P->total_tiles = start;
  for (int l = 0; l < 4; ++l) P->lat_tiles[l] = lat_tiles[l];
  P->trace = trace;
  P->sched = sched;
  P->status = status;
  plan.dtype = dt;
  plan.total_tiles = start;
  const int cap = max_ctas > 0 ? max_ctas : sm_count();
  plan.grid = start < cap ? start : cap;
  return cudaSuccess;
}

cudaError_t neck_plan_stall_dependency(NeckPlan& plan, int level, unsigned long long wait_ns) {
  NeckParams* P = reinterpret_cast<NeckParams*>(plan.params);
  if (wait_ns == 0 || level < 0 || level > 3) return cudaErrorInvalidValue;
  for (int j = 0; j < P->num_jobs; ++j) {
    NeckJob& J = P->jobs[j];
    if (J.mode == 1 && J.level == level && J.dep_level == level) {
      J.dep_count += 1;  // one more lateral tile than the level has: never reached
      P->dep_wait_ns = wait_ns;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidValue;  // no 3x3 of that level waits on its lateral in this plan
}

cudaError_t plan_neck(NeckPlan& plan, DType dt, int N, const NeckLevel* lv, void* p6,
                      int* sched, int* status, int max_ctas, unsigned long long* trace) {
  // Dispatch order: each job only depends on jobs before it.  All laterals go first:
  // their main loops depend on nothing, so every SM can work on them while the
  // top-down chain (lat5 -> lat4 -> lat3 -> lat2 epilogues) resolves; the 3x3 tiles,
  // the bulk of the FLOPs, follow and fill the machine.
  const NeckJobSpec specs[8] = {{0, 3, 0}, {0, 2, 1}, {0, 1, 1}, {0, 0, 1},
                                {1, 3, 0}, {1, 2, 0}, {1, 1, 0}, {1, 0, 0}};
  return plan_neck_jobs(plan, dt, N, lv, p6, specs, 8, sched, status, max_ctas, trace);
}

namespace {
template <typename T, int kStages, bool kCoarse>
cudaError_t launch_neck_cfg(const NeckPlan& p, cudaStream_t s, LaunchOpts opts) {
  using Cfg = NeckCfg<kStages, kCoarse>;
  auto kern = fpn_neck_kernel<T, kStages, kCoarse>;
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  const NeckParams* P = reinterpret_cast<const NeckParams*>(p.params);
  return launch_ex(kern, dim3(p.grid), dim3(kTcThreads), Cfg::kSmemBytes, s, opts, 1, *P);
}
template <typename T>
cudaError_t launch_neck_t(const NeckPlan& p, cudaStream_t s, LaunchOpts opts) {
  // Four operand stages when no job stages a coarse box (its buffer is not needed), else three.
  const NeckParams* P = reinterpret_cast<const NeckParams*>(p.params);
  bool coarse_box = false;
  for (int j = 0; j < P->num_jobs; ++j) coarse_box |= P->jobs[j].mode == 0 && P->jobs[j].cbox_w > 0;
  return coarse_box ? launch_neck_cfg<T, kNeckStages, true>(p, s, opts)
                    : launch_neck_cfg<T, kNeckStages + 1, false>(p, s, opts);
}
}  // namespace

static_assert(sizeof(LgParams) <= sizeof(LateralGroupPlan::params),
              "LateralGroupPlan::params too small");

cudaError_t plan_lateral_group_pair(LateralGroupPlan& plan, DType dt, int N,
                                    const NeckLevel* lv, const int* which, int count,
                                    int* status, int max_ctas, const int* nsplit) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorNotSupported;
  if (N <= 0 || count < 1 || count > kLgMaxJobs || !which) return cudaErrorInvalidValue;
  LgParams* P = reinterpret_cast<LgParams*>(plan.params);
  std::memset(plan.params, 0, sizeof(plan.params));
  // (job, units, k-blocks per unit, parts per unit)
  struct JobUnits {
    int job, units, kb, parts;
  };
  std::vector<JobUnits> ju;
  long long total_units = 0;
  for (int j = 0; j < count; ++j) {
    const int l = which[j];
    if (l < 0 || l > 3) return cudaErrorInvalidValue;
    const NeckLevel& L = lv[l];
    const Conv3x3Tiling t = L.lat_tiling;
    if (!valid_tiling(t) || L.H <= 0 || L.W <= 0 || L.Cin <= 0 || L.Cin % 8 != 0)
      return cudaErrorInvalidValue;
    if (!aligned16(L.merged) || !aligned16(L.lat_b)) return cudaErrorMisalignedAddress;
    LgJob& J = P->jobs[j];
    J.N_img = N;
    J.H = L.H;
    J.W = L.W;
    J.tile_w = t.tile_w;
    J.tile_h = t.tile_h;
    J.tiles_x = (L.W + t.tile_w - 1) / t.tile_w;
    J.tiles_y = (L.H + t.tile_h - 1) / t.tile_h;
    const long long tiles = static_cast<long long>(J.tiles_x) * J.tiles_y * N;
    if (tiles >= (1LL << 28)) return cudaErrorNotSupported;
    J.num_tiles = static_cast<int>(tiles);
    J.num_kb = (L.Cin + kTcBlockK - 1) / kTcBlockK;
    J.nsplit = nsplit ? nsplit[j] : 1;
    if (J.nsplit != 1 && J.nsplit != 2) return cudaErrorInvalidValue;
    J.bias = L.lat_b;
    cudaError_t e;
    if ((e = encode_nhwc(&J.map_a, dt, L.x, N, L.H, L.W, L.Cin, t.tile_w, t.tile_h)) !=
        cudaSuccess)
      return e;
    if ((e = encode_weights(&J.map_b, dt, L.lat_w, L.Cin, kTcBlockN / 2)) != cudaSuccess)
      return e;
    J.map_bh = J.map_b;
    if (J.nsplit > 1 &&
        (e = encode_weights(&J.map_bh, dt, L.lat_w, L.Cin, kTcBlockN / 4)) != cudaSuccess)
      return e;
    const int sw = t.tile_w < 32 ? t.tile_w : 32;
    if ((e = encode_nhwc(&J.map_out, dt, L.merged, N, L.H, L.W, kTcBlockN, sw, 32 / sw)) !=
        cudaSuccess)
      return e;
    const int units = (J.num_tiles + 1) / 2;
    if (units >= (1 << 12)) return cudaErrorNotSupported;
    ju.push_back({j, units, J.num_kb, J.nsplit});
    total_units += static_cast<long long>(units) * J.nsplit;
  }
  if (total_units > kLgMaxItems) return cudaErrorNotSupported;
  const int cap = (max_ctas > 0 ? max_ctas : sm_count()) / 2;
  const int pairs = static_cast<int>(std::min<long long>({total_units, cap, kLgMaxPairs}));
  if (pairs <= 0) return cudaErrorInvalidValue;
  // Longest first to the least-loaded pair (ties: the lowest pair).  Cost of an item: its
  // k-blocks, x 0.6 for a channel half (an N = 128 half of a unit measured ~0.6 of it).
  auto cost = [](const JobUnits& x) { return x.kb * (x.parts > 1 ? 6 : 10); };
  std::sort(ju.begin(), ju.end(), [&](const JobUnits& a, const JobUnits& b) {
    return cost(a) != cost(b) ? cost(a) > cost(b) : a.job < b.job;
  });
  std::vector<long long> load(pairs, 0);
  std::vector<std::vector<unsigned short>> lists(pairs);
  for (const JobUnits& x : ju)
    for (int u = 0; u < x.units; ++u)
      for (int part = x.parts > 1 ? 1 : 0; part <= (x.parts > 1 ? 2 : 0); ++part) {
        int best = 0;
        for (int p = 1; p < pairs; ++p)
          if (load[p] < load[best]) best = p;
        load[best] += cost(x);
        lists[best].push_back(static_cast<unsigned short>((x.job << 14) | (part << 12) | u));
      }
  int k = 0;
  for (int p = 0; p < pairs; ++p) {
    P->off[p] = static_cast<unsigned short>(k);
    for (unsigned short it : lists[p]) P->items[k++] = it;
  }
  P->off[pairs] = static_cast<unsigned short>(k);
  P->num_jobs = count;
  P->num_pairs = pairs;
  P->status = status;
  plan.dtype = dt;
  plan.grid = 2 * pairs;
  return cudaSuccess;
}

namespace {
template <typename T>
cudaError_t launch_lateral_group_pair_t(const LateralGroupPlan& p, cudaStream_t s,
                                        LaunchOpts opts) {
  auto kern = fpn_lateral_group_pair_kernel<T>;
  static std::atomic<bool> configured[64];
  cudaError_t e = once_per_device(configured, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                LgCfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  const LgParams* P = reinterpret_cast<const LgParams*>(p.params);
  return launch_ex(kern, dim3(p.grid), dim3(kTcThreads), LgCfg::kSmemBytes, s, opts, 2, *P);
}
}  // namespace

cudaError_t launch_lateral_group_pair(const LateralGroupPlan& plan, cudaStream_t s,
                                      LaunchOpts opts) {
  if (plan.grid <= 0) return cudaSuccess;
  return plan.dtype == DType::BF16 ? launch_lateral_group_pair_t<__nv_bfloat16>(plan, s, opts)
                                   : launch_lateral_group_pair_t<__half>(plan, s, opts);
}

cudaError_t launch_neck(const NeckPlan& plan, cudaStream_t s, LaunchOpts opts) {
  if (plan.grid <= 0) return cudaSuccess;
  return plan.dtype == DType::BF16 ? launch_neck_t<__nv_bfloat16>(plan, s, opts)
                                   : launch_neck_t<__half>(plan, s, opts);
}

cudaError_t launch_tc(const TcPlan& plan, cudaStream_t s, LaunchOpts opts) {
  if (plan.grid <= 0) return cudaSuccess;
  if (plan.dtype == DType::E4M3) {
    if (plan.mode == 0) return launch_t<0, __nv_fp8_e4m3>(plan, s, opts);
    if (plan.mode == 2) return launch_halo_t<__nv_fp8_e4m3>(plan, s, opts);
    if (plan.mode == 3) return launch_halo_pair_t<__nv_fp8_e4m3>(plan, s, opts);
    if (plan.mode == 4) return launch_halo_pair_t<__nv_fp8_e4m3, true>(plan, s, opts);
    return cudaErrorInvalidValue;
  }
  if (plan.mode == 3) {
    return plan.dtype == DType::BF16 ? launch_halo_pair_t<__nv_bfloat16>(plan, s, opts)
                                     : launch_halo_pair_t<__half>(plan, s, opts);
  }
  if (plan.mode == 5) {
    return plan.dtype == DType::BF16 ? launch_lateral_pair_t<__nv_bfloat16>(plan, s, opts)
                                     : launch_lateral_pair_t<__half>(plan, s, opts);
  }
  if (plan.mode == 0) {
    return plan.dtype == DType::BF16 ? launch_t<0, __nv_bfloat16>(plan, s, opts)
                                     : launch_t<0, __half>(plan, s, opts);
  }
  if (plan.mode == 6) {  // 16-bit lateral with the 16-warp epilogue
    return plan.dtype == DType::BF16 ? launch_t<0, __nv_bfloat16, true>(plan, s, opts)
                                     : launch_t<0, __half, true>(plan, s, opts);
  }
  if (plan.mode == 2) {
    return plan.dtype == DType::BF16 ? launch_halo_t<__nv_bfloat16>(plan, s, opts)
                                     : launch_halo_t<__half>(plan, s, opts);
  }
  return plan.dtype == DType::BF16 ? launch_t<1, __nv_bfloat16>(plan, s, opts)
                                   : launch_t<1, __half>(plan, s, opts);
}

}  // namespace ufpn
