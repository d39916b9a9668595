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
// that device current) and cached; that first call therefore performs a
// runtime query and should come before any stream capture.
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

// Device address of g_noalloc_scratch on the current device (queried once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
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
  // status word must start at zero.
  e = cudaMemsetAsync(s, 0, kCountersBytes + kStatusBytes, st);
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
