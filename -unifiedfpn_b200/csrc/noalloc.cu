// ufpn_neck_forward_noalloc: the whole tensor-core neck in one call that
// allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc (or anything that does) on
// their hot path -- an inference server that owns every byte of device memory
// through its own fixed arena, a real-time loop that must not hit the driver's
// allocator (cudaMalloc can synchronise the device and can fail under memory
// pressure), or embedding code that must not create allocations the host
// framework does not track.  The regular engine (ufpn_core_*) allocates its
// workspace, packed weights and status word with cudaMalloc; this entry point
// takes every input, weight and output from the caller and keeps its own
// scratch -- the merged top-down maps M2..M5, the neck kernel's tile/level
// counters and a status word -- in the file-scope array below.
//
// That array is a module global: every GPU that loads this library holds its
// kNoAllocScratchBytes until the process exits, and every call on a device
// shares it.  A call keeps the previous call's contents, so each call clears
// the counters and the status word it relies on before its launch; calls whose
// executions overlap on the GPU (different streams, no ordering) race on the
// array and must be serialised by the caller.
//
// Host code must not pass the array's name to a kernel: in host code it names a
// host-side stand-in, not device memory.  The device address is obtained with
// cudaGetSymbolAddress the first time the entry point runs on a device (with
// that device current) and cached together with the identity of the device's
// context; that first call therefore performs a runtime query and should come
// before any stream capture.  If the context is replaced (cudaDeviceReset, or
// any teardown of the primary context), the module is loaded again at a new
// address: the next call sees the new context identity and looks it up again.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "kernels.h"
#include "unified_fpn_c.h"

namespace {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(UFPN_NOALLOC_SCRATCH_BYTES);
constexpr size_t kCountersBytes = 256;  // neck kernel schedule counters (8 used)
constexpr size_t kStatusBytes = 256;    // device status word (first int used)

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void* g_addr[64] = {};
unsigned long long g_ctx_id[64] = {};  // context the cached address belongs to (0 = none)

// Unique id of the calling thread's current context (ids are never reused within a
// process), or 0 when no context is current yet or the driver lacks the query.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of g_noalloc_scratch on the current device: looked up once per device and
// context (the set-up step), then served from the cache.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_addr_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_addr[dev] || ctx == 0 || ctx != g_ctx_id[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // creates the context if needed
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
    g_ctx_id[dev] = current_context_id();
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

namespace ufpn {
void set_last_error(const std::string& msg);  // capi.cpp: backs ufpn_last_error()
}

extern "C" int ufpn_neck_forward_noalloc(
    int dtype, const void* const* inputs, const void* const* lateral_w,
    const float* const* lateral_b, const void* const* output_w, const float* const* output_b,
    void* const* outputs, void* p6, int batch, const int* in_channels, const int* heights,
    const int* widths, int* status, void* stream) {
  using ufpn::DType;
  auto fail = [](int code, const std::string& m) {
    ufpn::set_last_error("ufpn_neck_forward_noalloc: " + m);
    return code;
  };
  if (dtype != UFPN_DTYPE_BF16 && dtype != UFPN_DTYPE_F16)
    return fail(UFPN_ERR_UNSUPPORTED, "dtype must be UFPN_DTYPE_BF16 or UFPN_DTYPE_F16");
  if (!inputs || !lateral_w || !lateral_b || !output_w || !output_b || !outputs ||
      !in_channels || !heights || !widths)
    return fail(UFPN_ERR_INVALID_ARG, "NULL argument array");
  if (batch <= 0) return fail(UFPN_ERR_INVALID_ARG, "batch must be positive");
  const DType dt = dtype == UFPN_DTYPE_BF16 ? DType::BF16 : DType::F16;
  // Scratch layout: counters | status | M2 | M3 | M4 | M5 (each map 256-byte aligned).
  size_t off[4];
  size_t need = kCountersBytes + kStatusBytes;
  for (int l = 0; l < 4; ++l) {
    if (!inputs[l] || !lateral_w[l] || !lateral_b[l] || !output_w[l] || !output_b[l] ||
        !outputs[l])
      return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
    if (in_channels[l] <= 0 || in_channels[l] % 8 != 0 || heights[l] <= 0 || widths[l] <= 0)
      return fail(UFPN_ERR_INVALID_ARG, "need Cin % 8 == 0 and positive sizes");
    if (l < 3 && (heights[l + 1] > heights[l] || widths[l + 1] > widths[l]))
      return fail(UFPN_ERR_INVALID_ARG, "levels must be ordered fine (C2) to coarse (C5)");
    off[l] = round_up(need, 256);
    need = off[l] + static_cast<size_t>(batch) * heights[l] * widths[l] * 256 * 2;
  }
  if (need > kNoAllocScratchBytes) {
    char buf[200];
    std::snprintf(buf, sizeof(buf),
                  "problem needs %zu bytes of scratch (merged maps M2..M5); this entry point "
                  "has a fixed %zu-byte scratch array",
                  need, kNoAllocScratchBytes);
    return fail(UFPN_ERR_INVALID_ARG, buf);
  }
  void* base = nullptr;
  cudaError_t e = scratch_address(&base);
  if (e != cudaSuccess)
    return fail(UFPN_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  unsigned char* s = static_cast<unsigned char*>(base);
  int* counters = reinterpret_cast<int*>(s);
  int* own_status = reinterpret_cast<int*>(s + kCountersBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the schedule counters and the
  // status word must start at zero.  A caller-owned status word is cleared as well, so that
  // it reports this call alone.
  e = cudaMemsetAsync(s, 0, kCountersBytes + kStatusBytes, st);
  if (e == cudaSuccess && status) e = cudaMemsetAsync(status, 0, sizeof(int), st);
  if (e != cudaSuccess)
    return fail(UFPN_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  ufpn::NeckLevel lv[4];
  for (int l = 0; l < 4; ++l) {
    lv[l].x = inputs[l];
    lv[l].lat_w = lateral_w[l];
    lv[l].lat_b = lateral_b[l];
    lv[l].conv_w = output_w[l];
    lv[l].conv_b = output_b[l];
    lv[l].merged = s + off[l];
    lv[l].out = outputs[l];
    lv[l].Cin = in_channels[l];
    lv[l].H = heights[l];
    lv[l].W = widths[l];
    lv[l].lat_tiling = ufpn::default_tiling(heights[l], widths[l]);
    lv[l].conv_tiling = lv[l].lat_tiling;
  }
  ufpn::NeckPlan plan;
  e = ufpn::plan_neck(plan, dt, batch, lv, p6, counters, status ? status : own_status, 0);
  if (e != cudaSuccess)
    return fail(UFPN_ERR_INVALID_ARG, std::string("plan: ") + cudaGetErrorString(e));
  e = ufpn::launch_neck(plan, st);
  if (e != cudaSuccess)
    return fail(UFPN_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return UFPN_OK;
}
