// Host side of the tensor-core kernels: TMA descriptor encoding, tile
// planning and launch.  The device code lives in tc_gemm.cuh.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kernels.h"
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
    default:
      return CU_TENSOR_MAP_DATA_TYPE_UINT8;
  }
}

// rank-d tiled map with 128-byte swizzle; dims/strides innermost first, strides in bytes.
cudaError_t encode(CUtensorMap* map, DType dt, int rank, const void* base, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (!aligned16(base)) return cudaErrorMisalignedAddress;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16 != 0) return cudaErrorInvalidValue;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = fn(map, tmap_dtype(dt), rank, const_cast<void*>(base), d, st, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int kMode, typename T>
cudaError_t launch_t(const TcPlan& p, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fpn_tc_gemm_kernel<kMode, T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kTcSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  TcGemmArgs a;
  std::memcpy(&a, p.args, sizeof(a));
  fpn_tc_gemm_kernel<kMode, T><<<p.grid, kTcThreads, kTcSmemBytes, s>>>(p.map_a, p.map_b, a);
  return cudaGetLastError();
}

}  // namespace

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) dev = 63;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

cudaError_t plan_tc_lateral(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, const void* coarse, void* out, int N, int Cin,
                            int H, int W, int Hc, int Wc, int* status, int max_ctas) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorInvalidValue;
  if (Cin <= 0 || Cin % 8 != 0 || N <= 0 || H <= 0 || W <= 0) return cudaErrorInvalidValue;
  if (!aligned16(out) || (coarse && !aligned16(coarse)) || !aligned16(bias))
    return cudaErrorMisalignedAddress;
  const long long M = static_cast<long long>(N) * H * W;
  if (M >= (1LL << 31) - kTcBlockM) return cudaErrorInvalidValue;
  const int esz = 2;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(Cin), static_cast<uint64_t>(M)};
    uint64_t strides[1] = {static_cast<uint64_t>(Cin) * esz};
    uint32_t box[2] = {kTcBlockK, kTcBlockM};
    cudaError_t e = encode(&plan.map_a, dt, 2, x, dims, strides, box);
    if (e != cudaSuccess) return e;
  }
  {
    uint64_t dims[2] = {static_cast<uint64_t>(Cin), kTcBlockN};
    uint64_t strides[1] = {static_cast<uint64_t>(Cin) * esz};
    uint32_t box[2] = {kTcBlockK, kTcBlockN};
    cudaError_t e = encode(&plan.map_b, dt, 2, w, dims, strides, box);
    if (e != cudaSuccess) return e;
  }
  TcGemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.num_tiles = static_cast<int>((M + kTcBlockM - 1) / kTcBlockM);
  a.num_kb = (Cin + kTcBlockK - 1) / kTcBlockK;
  a.M = static_cast<int>(M);
  a.N_img = N;
  a.H = H;
  a.W = W;
  a.bias = bias;
  a.out = out;
  a.coarse = coarse;
  a.Hc = Hc;
  a.Wc = Wc;
  a.scale_y = coarse ? static_cast<float>(Hc) / static_cast<float>(H) : 0.f;
  a.scale_x = coarse ? static_cast<float>(Wc) / static_cast<float>(W) : 0.f;
  a.status = status;
  std::memcpy(plan.args, &a, sizeof(a));
  plan.mode = 0;
  plan.dtype = dt;
  plan.num_tiles = a.num_tiles;
  const int cap = max_ctas > 0 ? max_ctas : sm_count();
  plan.grid = a.num_tiles < cap ? a.num_tiles : cap;
  return cudaSuccess;
}

cudaError_t plan_tc_conv3x3(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, void* out, void* p6, int N, int H, int W,
                            Conv3x3Tiling tiling, int* status, int max_ctas) {
  if (dt != DType::BF16 && dt != DType::F16) return cudaErrorInvalidValue;
  if (tiling.tile_w * tiling.tile_h != kTcBlockM || tiling.tile_w < 1 || tiling.tile_w > 128)
    return cudaErrorInvalidValue;
  if (N <= 0 || H <= 0 || W <= 0) return cudaErrorInvalidValue;
  if (!aligned16(out) || (p6 && !aligned16(p6)) || !aligned16(bias))
    return cudaErrorMisalignedAddress;
  const int C = kTcBlockN;
  const int esz = 2;
  {
    uint64_t dims[4] = {static_cast<uint64_t>(C), static_cast<uint64_t>(W),
                        static_cast<uint64_t>(H), static_cast<uint64_t>(N)};
    uint64_t strides[3] = {static_cast<uint64_t>(C) * esz, static_cast<uint64_t>(W) * C * esz,
                           static_cast<uint64_t>(H) * W * C * esz};
    uint32_t box[4] = {kTcBlockK, static_cast<uint32_t>(tiling.tile_w),
                       static_cast<uint32_t>(tiling.tile_h), 1};
    cudaError_t e = encode(&plan.map_a, dt, 4, x, dims, strides, box);
    if (e != cudaSuccess) return e;
  }
  {
    uint64_t dims[2] = {static_cast<uint64_t>(9 * C), kTcBlockN};
    uint64_t strides[1] = {static_cast<uint64_t>(9 * C) * esz};
    uint32_t box[2] = {kTcBlockK, kTcBlockN};
    cudaError_t e = encode(&plan.map_b, dt, 2, w, dims, strides, box);
    if (e != cudaSuccess) return e;
  }
  TcGemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.tile_w = tiling.tile_w;
  a.tile_h = tiling.tile_h;
  a.tiles_x = (W + tiling.tile_w - 1) / tiling.tile_w;
  a.tiles_y = (H + tiling.tile_h - 1) / tiling.tile_h;
  const long long tiles = static_cast<long long>(a.tiles_x) * a.tiles_y * N;
  if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
  a.num_tiles = static_cast<int>(tiles);
  a.cin_blocks = C / kTcBlockK;
  a.num_kb = 9 * a.cin_blocks;
  a.N_img = N;
  a.H = H;
  a.W = W;
  a.bias = bias;
  a.out = out;
  a.p6 = p6;
  a.H6 = (H - 1) / 2 + 1;
  a.W6 = (W - 1) / 2 + 1;
  a.status = status;
  std::memcpy(plan.args, &a, sizeof(a));
  plan.mode = 1;
  plan.dtype = dt;
  plan.num_tiles = a.num_tiles;
  const int cap = max_ctas > 0 ? max_ctas : sm_count();
  plan.grid = a.num_tiles < cap ? a.num_tiles : cap;
  return cudaSuccess;
}

cudaError_t launch_tc(const TcPlan& plan, cudaStream_t s) {
  if (plan.grid <= 0) return cudaSuccess;
  if (plan.mode == 0) {
    return plan.dtype == DType::BF16 ? launch_t<0, __nv_bfloat16>(plan, s)
                                     : launch_t<0, __half>(plan, s);
  }
  return plan.dtype == DType::BF16 ? launch_t<1, __nv_bfloat16>(plan, s)
                                   : launch_t<1, __half>(plan, s);
}

}  // namespace ufpn
