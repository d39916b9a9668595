// extern "C" boundary of libunified_fpn_b200.so (declared in include/unified_fpn_c.h).
// Every entry point catches exceptions, stores a message for ufpn_last_error()
// and returns a status code; nothing here calls exit().
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "kernels.h"
#include "unified_fpn/core/engine.h"
#include "unified_fpn_c.h"

using ufpn::DType;
using ufpn::Layout;

struct ufpn_core {
  UnifiedFPNCore core;
  ufpn_core(int dev, size_t ws) : core(ws, dev) {}
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(UFPN_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool parse_dtype(int code, DType* out) {
  switch (code) {
    case UFPN_DTYPE_F32:
      *out = DType::F32;
      return true;
    case UFPN_DTYPE_F16:
      *out = DType::F16;
      return true;
    case UFPN_DTYPE_BF16:
      *out = DType::BF16;
      return true;
    default:
      return false;
  }
}
bool parse_layout(int code, Layout* out) {
  if (code == UFPN_LAYOUT_NCHW) {
    *out = Layout::NCHW;
    return true;
  }
  if (code == UFPN_LAYOUT_NHWC) {
    *out = Layout::NHWC;
    return true;
  }
  return false;
}

// One lazily allocated status word per device for the standalone tensor-core entry points.
std::mutex g_status_mu;
int* g_status[64] = {};
int* device_status_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, 256);
    g_status[dev] = p;
  }
  return g_status[dev];
}

template <typename F>
int guarded(F&& f) {
  try {
    return f();
  } catch (const std::exception& e) {
    return fail(UFPN_ERR_STATE, e.what());
  } catch (...) {
    return fail(UFPN_ERR_STATE, "unknown C++ exception");
  }
}

}  // namespace

namespace ufpn {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace ufpn

extern "C" {

const char* ufpn_last_error(void) { return g_last_error.c_str(); }

int ufpn_version(void) { return 100; }

int ufpn_set_peaks(double tensor_tflops, double fp32_tflops, double hbm_gbs) {
  if (!(tensor_tflops >= 0) || !(fp32_tflops >= 0) || !(hbm_gbs >= 0))
    return fail(UFPN_ERR_INVALID_ARG, "peaks must be >= 0 (0 keeps the current value)");
  ufpn::set_device_peaks(tensor_tflops * 1e12, fp32_tflops * 1e12, hbm_gbs * 1e9);
  return UFPN_OK;
}

int ufpn_get_peaks(double* out3) {
  if (!out3) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  double pk[3];
  ufpn::get_device_peaks(pk);
  out3[0] = pk[0] / 1e12;
  out3[1] = pk[1] / 1e12;
  out3[2] = pk[2] / 1e9;
  return UFPN_OK;
}

int ufpn_device_status(int reset, int* status_out) {
  int* w = device_status_word();
  if (!w) return fail(UFPN_ERR_CUDA, "could not allocate the device status word");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy");
  if (reset) cudaMemset(w, 0, sizeof(int));
  if (status_out) *status_out = v;
  return UFPN_OK;
}

// ------------------------------------------------------------------ engine
int ufpn_core_create(int device, size_t workspace_bytes, ufpn_core** out) {
  if (!out) return fail(UFPN_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  return guarded([&] {
    *out = new ufpn_core(device, workspace_bytes);
    return UFPN_OK;
  });
}

void ufpn_core_destroy(ufpn_core* core) { delete core; }

int ufpn_core_configure_levels(ufpn_core* core, int batch, const int* in_channels,
                               const int* heights, const int* widths, int output_channels,
                               int dtype, int layout) {
  if (!core || !in_channels || !heights || !widths) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  DType dt;
  Layout lay;
  if (!parse_dtype(dtype, &dt) && dtype != UFPN_DTYPE_E4M3)
    return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!parse_layout(layout, &lay)) return fail(UFPN_ERR_INVALID_ARG, "bad layout");
  return guarded([&] {
    std::vector<FPNDimensions> dims(4);
    for (int l = 0; l < 4; ++l) dims[l] = {batch, in_channels[l], heights[l], widths[l], 0};
    core->core.configure_levels(dims, output_channels, static_cast<FPNDataType>(dtype),
                                lay == Layout::NHWC ? FPNLayout::NHWC : FPNLayout::NCHW);
    return UFPN_OK;
  });
}

int ufpn_core_set_weights(ufpn_core* core, int level, const float* lateral_w,
                          const float* lateral_b, const float* output_w, const float* output_b) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  return guarded([&] {
    core->core.set_weights(level, lateral_w, lateral_b, output_w, output_b);
    return UFPN_OK;
  });
}

int ufpn_core_allocate_weights(ufpn_core* core, const int* in_channels, int output_channels) {
  if (!core || !in_channels) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return guarded([&] {
    core->core.allocate_weights(std::vector<int>(in_channels, in_channels + 4), output_channels);
    return UFPN_OK;
  });
}

int ufpn_core_forward(ufpn_core* core, const void* const* inputs, void* const* outputs, void* p6,
                      void* stream) {
  if (!core || !inputs || !outputs) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return guarded([&] {
    core->core.forward_raw(inputs, outputs, p6, static_cast<cudaStream_t>(stream));
    return UFPN_OK;
  });
}

int ufpn_core_forward_e4m3(ufpn_core* core, const void* const* inputs,
                           const float* const* input_scales, void* const* outputs, void* p6,
                           void* stream) {
  if (!core || !inputs || !input_scales || !outputs) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return guarded([&] {
    core->core.forward_raw_scaled(inputs, input_scales, outputs, p6,
                                  static_cast<cudaStream_t>(stream));
    return UFPN_OK;
  });
}

int ufpn_core_set_kernel_config(ufpn_core* core, int tile_size, int channels_per_thread,
                                int use_tensor_cores, int activation, int enable_graph_capture) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  return guarded([&] {
    FPNKernelConfig c = core->core.get_kernel_config();
    c.tile_size = tile_size;
    c.channels_per_thread = channels_per_thread;
    c.use_tensor_cores = use_tensor_cores != 0;
    c.activation = static_cast<FPNActivation>(activation);
    c.enable_graph_capture = enable_graph_capture != 0;
    core->core.set_kernel_config(c);
    return UFPN_OK;
  });
}

int ufpn_core_set_fp8_options(ufpn_core* core, int two_pass_p2) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  return guarded([&] {
    FPNKernelConfig c = core->core.get_kernel_config();
    c.fp8_two_pass_p2 = two_pass_p2 != 0;
    core->core.set_kernel_config(c);
    return UFPN_OK;
  });
}

int ufpn_core_set_activation(ufpn_core* core, int activation, float alpha) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  if (activation < 0 || activation > 3)
    return fail(UFPN_ERR_INVALID_ARG, "activation must be 0 (none), 1 (ReLU), 2 (LeakyReLU) or 3 (Swish)");
  return guarded([&] {
    FPNKernelConfig c = core->core.get_kernel_config();
    c.activation = static_cast<FPNActivation>(activation);
    c.activation_alpha = alpha;
    core->core.set_kernel_config(c);
    return UFPN_OK;
  });
}

int ufpn_fold_batch_norm(const float* conv_w, const float* conv_b, const float* gamma,
                         const float* beta, const float* mean, const float* var, float eps,
                         int Cout, long long K, float* out_w, float* out_b) {
  if (!conv_w || !mean || !var || !out_w || !out_b)
    return fail(UFPN_ERR_INVALID_ARG, "NULL pointer");
  if (Cout <= 0 || K <= 0 || !(eps >= 0.f)) return fail(UFPN_ERR_INVALID_ARG, "bad sizes or eps");
  for (int o = 0; o < Cout; ++o) {
    if (!(var[o] + static_cast<double>(eps) > 0.0))
      return fail(UFPN_ERR_INVALID_ARG, "var + eps must be positive");
  }
  for (int o = 0; o < Cout; ++o) {
    // BN(y) = (y - mean) / sqrt(var + eps) * gamma + beta, y = W x + b: scale the row of W by
    // s = gamma / sqrt(var + eps) and set b' = (b - mean) s + beta (double, rounded once).
    const double sc = (gamma ? gamma[o] : 1.0) / std::sqrt(static_cast<double>(var[o]) + eps);
    const float* wr = conv_w + static_cast<size_t>(o) * K;
    float* orow = out_w + static_cast<size_t>(o) * K;
    for (long long k = 0; k < K; ++k) orow[k] = static_cast<float>(wr[k] * sc);
    out_b[o] = static_cast<float>(((conv_b ? conv_b[o] : 0.0) - mean[o]) * sc + (beta ? beta[o] : 0.0));
  }
  return UFPN_OK;
}

int ufpn_core_trace_next_forward(ufpn_core* core) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  core->core.trace_next_forward();
  return UFPN_OK;
}

int ufpn_core_get_neck_trace(const ufpn_core* core, unsigned long long* out8) {
  if (!core || !out8) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  core->core.get_neck_trace(out8);
  return UFPN_OK;
}

int ufpn_core_set_schedule(ufpn_core* core, int fused_neck_kernel) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  if (fused_neck_kernel < 0 || fused_neck_kernel > 2)
    return fail(UFPN_ERR_INVALID_ARG, "schedule: 0 split (two streams), 1 fused, 2 split on one stream");
  return guarded([&] {
    FPNKernelConfig c = core->core.get_kernel_config();
    c.fused_neck_kernel = fused_neck_kernel == 1;
    c.single_stream = fused_neck_kernel == 2;
    core->core.set_kernel_config(c);
    return UFPN_OK;
  });
}

int ufpn_core_set_schedule_options(ufpn_core* core, int programmatic_launch, int chain_priority,
                                   int merge_two_levels) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  return guarded([&] {
    FPNKernelConfig c = core->core.get_kernel_config();
    c.programmatic_launch = programmatic_launch != 0;
    c.chain_priority = chain_priority != 0;
    c.merge_two_levels = merge_two_levels != 0;
    core->core.set_kernel_config(c);
    return UFPN_OK;
  });
}

int ufpn_core_set_option(ufpn_core* core, const char* name, int value) {
  if (!core || !name) return fail(UFPN_ERR_INVALID_ARG, "NULL core or name");
  try {
    core->core.set_option(name, value);
  } catch (const std::exception& e) {
    return fail(UFPN_ERR_INVALID_ARG, e.what());  // unknown name or value
  }
  return UFPN_OK;
}

int ufpn_core_get_option(const ufpn_core* core, const char* name, int* value) {
  if (!core || !name || !value) return fail(UFPN_ERR_INVALID_ARG, "NULL argument");
  try {
    *value = core->core.get_option(name);
  } catch (const std::exception& e) {
    return fail(UFPN_ERR_INVALID_ARG, e.what());
  }
  return UFPN_OK;
}

int ufpn_core_graph_stats(const ufpn_core* core, long long* out4) {
  if (!core || !out4) return fail(UFPN_ERR_INVALID_ARG, "NULL argument");
  core->core.graph_stats(out4);
  return UFPN_OK;
}

size_t ufpn_core_get_memory_usage(const ufpn_core* core) {
  return core ? core->core.get_memory_usage() : 0;
}

int ufpn_core_get_performance_metrics(const ufpn_core* core, float* kernel_times_ms,
                                      float* metrics) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  const FPNPerformanceMetrics& m = core->core.get_performance_metrics();
  if (kernel_times_ms) std::memcpy(kernel_times_ms, m.kernel_times_ms, sizeof(m.kernel_times_ms));
  if (metrics) {
    metrics[0] = m.forward_time_ms;
    metrics[1] = m.memory_bandwidth_gb_s;
    metrics[2] = m.compute_utilization;
    metrics[3] = static_cast<float>(m.peak_memory_usage_bytes) / (1024.f * 1024.f);
    metrics[4] = static_cast<float>(m.num_kernel_launches);
  }
  return UFPN_OK;
}

int ufpn_core_set_profiling(ufpn_core* core, int enable) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  core->core.set_profiling(enable != 0);
  return UFPN_OK;
}

int ufpn_core_autotune(ufpn_core* core, const void* const* inputs, void* const* outputs,
                       void* p6, void* stream, int iterations) {
  return ufpn_core_autotune_scaled(core, inputs, nullptr, outputs, p6, stream, iterations);
}

int ufpn_core_autotune_scaled(ufpn_core* core, const void* const* inputs,
                              const float* const* input_scales, void* const* outputs, void* p6,
                              void* stream, int iterations) {
  if (!core || !inputs || !outputs) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return guarded([&] {
    g_last_error = core->core.autotune(inputs, outputs, p6, static_cast<cudaStream_t>(stream),
                                       iterations, input_scales);
    return UFPN_OK;
  });
}

int ufpn_core_save_tuning(const ufpn_core* core, const char* path) {
  if (!core || !path) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return core->core.save_tuning(path) ? UFPN_OK : fail(UFPN_ERR_STATE, "cannot write file");
}

int ufpn_core_load_tuning(ufpn_core* core, const char* path) {
  if (!core || !path) return fail(UFPN_ERR_INVALID_ARG, "NULL");
  return core->core.load_tuning(path) ? UFPN_OK : fail(UFPN_ERR_STATE, "cannot read file");
}

int ufpn_core_device_status(ufpn_core* core, int reset, int* status_out) {
  if (!core) return fail(UFPN_ERR_INVALID_ARG, "NULL core");
  return guarded([&] {
    const int v = core->core.device_status(reset != 0);
    if (status_out) *status_out = v;
    return UFPN_OK;
  });
}

// ------------------------------------------------------------------ standalone ops
int ufpn_lateral_conv(int dtype, int layout, const void* x, const void* w, const float* bias,
                      const void* coarse, void* out, int N, int Cin, int H, int W, int Cout,
                      int Hc, int Wc, void* stream) {
  DType dt;
  Layout lay;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!parse_layout(layout, &lay)) return fail(UFPN_ERR_INVALID_ARG, "bad layout");
  if (!x || !w || !bias || !out) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (coarse && (Hc <= 0 || Wc <= 0 || Hc > H || Wc > W))
    return fail(UFPN_ERR_INVALID_ARG, "coarse map must be non-empty and not larger than output");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dt == DType::F32) {
    if (lay != Layout::NCHW) return fail(UFPN_ERR_UNSUPPORTED, "fp32 lateral takes NCHW");
    cudaError_t e = ufpn::launch_fp32_lateral(
        static_cast<const float*>(x), static_cast<const float*>(w), bias,
        static_cast<const float*>(coarse), static_cast<float*>(out), N, Cin, Cout, H, W,
        coarse ? Hc : 1, coarse ? Wc : 1, s);
    return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "fp32 lateral");
  }
  if (lay != Layout::NHWC) return fail(UFPN_ERR_UNSUPPORTED, "16-bit lateral takes NHWC");
  if (Cout != 256) return fail(UFPN_ERR_UNSUPPORTED, "the tensor-core lateral needs Cout = 256");
  if (Cin % 8 != 0) return fail(UFPN_ERR_UNSUPPORTED, "Cin must be a multiple of 8");
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || (coarse && !ufpn::aligned16(coarse)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  int* status = device_status_word();
  ufpn::TcPlan plan;
  cudaError_t e = ufpn::plan_tc_lateral(plan, dt, x, w, bias, coarse, out, N, Cin, H, W,
                                        coarse ? Hc : 0, coarse ? Wc : 0,
                                        ufpn::default_tiling(H, W), status, 0);
  if (e != cudaSuccess) return cuda_fail(e, "plan lateral");
  e = ufpn::launch_tc(plan, s);
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "lateral launch");
}

int ufpn_lateral_conv_pair(int dtype, const void* x, const void* w, const float* bias,
                           const void* coarse, void* out, int N, int Cin, int H, int W, int Hc,
                           int Wc, void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (dt != DType::BF16 && dt != DType::F16)
    return fail(UFPN_ERR_UNSUPPORTED, "the CTA-pair lateral takes bf16 or fp16");
  if (!x || !w || !bias || !out) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (coarse && (Hc <= 0 || Wc <= 0 || Hc > H || Wc > W))
    return fail(UFPN_ERR_INVALID_ARG, "coarse map must be non-empty and not larger than output");
  if (Cin % 8 != 0) return fail(UFPN_ERR_UNSUPPORTED, "Cin must be a multiple of 8");
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || (coarse && !ufpn::aligned16(coarse)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  ufpn::TcPlan plan;
  cudaError_t e = ufpn::plan_tc_lateral_pair(plan, dt, x, w, bias, coarse, out, N, Cin, H, W,
                                             coarse ? Hc : 0, coarse ? Wc : 0,
                                             ufpn::default_tiling(H, W), device_status_word(), 0);
  if (e == cudaErrorNotSupported)
    return fail(UFPN_ERR_UNSUPPORTED, "CTA-pair lateral: needs Cin <= 256 and a 64-pixel tap box");
  if (e != cudaSuccess) return cuda_fail(e, "plan lateral pair");
  e = ufpn::launch_tc(plan, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "lateral pair launch");
}

int ufpn_conv3x3(int dtype, const void* x, const void* w, const float* bias, void* out, void* p6,
                 int N, int H, int W, int tile_w, void* stream) {
  return ufpn_conv3x3_act(dtype, x, w, bias, out, p6, N, H, W, tile_w, 0, 0.01f, stream);
}

int ufpn_conv3x3_act(int dtype, const void* x, const void* w, const float* bias, void* out,
                     void* p6, int N, int H, int W, int tile_w, int activation, float alpha,
                     void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!x || !w || !bias || !out) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || H <= 0 || W <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (activation < 0 || activation > 3)
    return fail(UFPN_ERR_INVALID_ARG, "activation must be 0 (none), 1 (ReLU), 2 (LeakyReLU) or 3 (Swish)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dt == DType::F32) {
    cudaError_t e = ufpn::launch_fp32_conv3x3(static_cast<const float*>(x),
                                              static_cast<const float*>(w), bias,
                                              static_cast<float*>(out), N, 256, 256, H, W, s,
                                              activation, alpha);
    if (e == cudaSuccess && p6)
      e = ufpn::launch_p6(DType::F32, out, p6, N, 256, H, W, Layout::NCHW, s);
    return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "fp32 conv3x3");
  }
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || (p6 && !ufpn::aligned16(p6)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  ufpn::Conv3x3Tiling t = ufpn::halo_tiling();  // tile_w == 0: halo reuse, 8 x 16 tiles
  if (tile_w > 0) {
    if (tile_w > 128 || 128 % tile_w != 0)
      return fail(UFPN_ERR_INVALID_ARG, "tile_w must be 8, 16, 32, 64 or 128");
    t.tile_w = tile_w;
    t.tile_h = 128 / tile_w;
    t.halo = false;
  } else if (tile_w == -1 || tile_w == -3 || tile_w == -5) {
    t = ufpn::halo_pair_tiling();
  } else if (tile_w < -5) {
    return fail(UFPN_ERR_INVALID_ARG,
                "tile_w must be 0 (halo tiling), -1 (halo tiling on CTA pairs), -2 / -3 (the "
                "same on the map's transposed view), -4 / -5 (mixed) or 8..128");
  }
  t.transposed = tile_w == -2 || tile_w == -3;
  t.mixed = tile_w == -4 || tile_w == -5;
  if ((t.transposed || t.mixed) && p6)
    return fail(UFPN_ERR_INVALID_ARG, "transposed or mixed view: no fused P6");
  int* status = device_status_word();
  ufpn::TcPlan plan;
  ufpn::TcScales sc;
  sc.act = activation;
  sc.act_alpha = alpha;
  cudaError_t e = ufpn::plan_tc_conv3x3(plan, dt, x, w, bias, out, p6, N, H, W, t, status, 0, sc);
  if (e != cudaSuccess) return cuda_fail(e, "plan conv3x3");
  e = ufpn::launch_tc(plan, s);
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "conv3x3 launch");
}

int ufpn_upsample_add(int dtype, int layout, const void* coarse, const void* lateral, void* out,
                      int N, int C, int Hc, int Wc, int H, int W, int align_corners,
                      void* stream) {
  DType dt;
  Layout lay;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!parse_layout(layout, &lay)) return fail(UFPN_ERR_INVALID_ARG, "bad layout");
  if (!coarse || !out) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || C <= 0 || Hc <= 0 || Wc <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  cudaError_t e = ufpn::launch_upsample_add(dt, coarse, lateral, out, N, C, Hc, Wc, H, W,
                                            align_corners, lay, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "upsample_add");
}

int ufpn_merge_two_levels(int dtype, const void* m5, const void* l4, void* m4, void* l3_m3, int N,
                          int H5, int W5, int H4, int W4, int H3, int W3, void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (dt != DType::BF16 && dt != DType::F16)
    return fail(UFPN_ERR_UNSUPPORTED, "two-level merge: bf16 or fp16 maps");
  if (!m5 || !l4 || !m4 || !l3_m3) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (l4 == m4) return fail(UFPN_ERR_INVALID_ARG, "l4 must not alias m4");
  if (N <= 0 || H5 <= 0 || W5 <= 0 || H4 <= 0 || W4 <= 0 || H3 <= 0 || W3 <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (H5 > H4 || W5 > W4 || H4 > H3 || W4 > W3)
    return fail(UFPN_ERR_UNSUPPORTED, "two-level merge: each map must upsample to the next");
  cudaError_t e = ufpn::launch_merge_two_levels(dt, m5, l4, m4, l3_m3, l3_m3, N, H5, W5, H4, W4,
                                                H3, W3, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "merge_two_levels");
}

namespace {
// Stream-ordered scratch for one backward call, freed (stream-ordered) on scope exit.  The
// device's default pool keeps freed memory cached (release threshold raised once per device),
// so repeated calls reuse it instead of mapping and unmapping tens of MB every time.
struct StreamScratch {
  cudaStream_t s;
  void* p = nullptr;
  explicit StreamScratch(cudaStream_t st) : s(st) {}
  cudaError_t alloc(size_t bytes) {
    static std::atomic<bool> cached[64];
    ufpn::once_per_device(cached, [] {
      int dev = 0;
      cudaMemPool_t pool;
      cudaError_t e = cudaGetDevice(&dev);
      if (e == cudaSuccess) e = cudaDeviceGetDefaultMemPool(&pool, dev);
      uint64_t keep = UINT64_MAX;
      if (e == cudaSuccess) e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      return e;
    });
    return cudaMallocAsync(&p, bytes > 0 ? bytes : 16, s);
  }
  ~StreamScratch() {
    if (p) cudaFreeAsync(p, s);
  }
};
bool parse_16bit(int dtype, DType* dt) {
  return parse_dtype(dtype, dt) && (*dt == DType::BF16 || *dt == DType::F16);
}

// Per-level work of a training step on several streams.  A StreamFork makes its side streams
// wait for everything enqueued on `main` so far and, when it goes out of scope, makes `main`
// wait for them; `order(a, b)` makes stream b wait for what was enqueued on stream a so far.
//   * forward: one stream per level -- P5, P4, P3 on side streams, P2 (the largest) on `main`;
//   * backward: per level a chain stream (the device's greatest priority) for the work on the
//     critical path -- input gradients, the top-down adjoint, the lateral's gradients -- and
//     a weight-gradient stream (the least priority) for the 3x3's weight and bias gradients,
//     which nothing else reads: the chains' CTAs take SMs first as they free.
// The small levels' grids (20-70 CTAs) then share the GPU with the large ones instead of
// holding it alone; a captured step becomes one graph with the same fork and join.  The
// streams and events are made once per device (outside a capture: the first, eager step); if
// they cannot be made, everything runs on `main`.  One fork at a time per device (its lock is
// held until the join).
struct SideStreams {
  cudaStream_t fwd[3] = {};    // forward: P3..P5
  cudaStream_t chain[4] = {};  // backward: P2..P5, greatest priority
  cudaStream_t grads[4] = {};  // backward: P2..P5, least priority
  cudaEvent_t fork = nullptr, step = nullptr;
  cudaEvent_t join[8] = {};
  cudaEvent_t mark[4] = {};  // backward: dM_l final
  bool ready = false;
  std::mutex mu;
};
SideStreams* side_streams() {
  static SideStreams per_dev[64];
  static std::mutex create_mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStreams& ss = per_dev[dev];
  std::lock_guard<std::mutex> lk(create_mu);
  if (!ss.ready) {
    // (relaxed capture mode while creating them, so that a capture elsewhere in the
    // process does not refuse the calls; the thread's own mode is restored after)
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    int least = 0, greatest = 0;
    bool ok = cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess;
    for (auto& x : ss.fwd)
      ok = ok && cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking) == cudaSuccess;
    for (auto& x : ss.chain)
      ok = ok && cudaStreamCreateWithPriority(&x, cudaStreamNonBlocking, greatest) == cudaSuccess;
    for (auto& x : ss.grads)
      ok = ok && cudaStreamCreateWithPriority(&x, cudaStreamNonBlocking, least) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&ss.step, cudaEventDisableTiming) == cudaSuccess;
    for (auto& e : ss.join)
      ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
    for (auto& e : ss.mark)
      ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (!ok) {
      cudaGetLastError();  // (leaves no sticky error; everything then runs on `main`)
      return nullptr;
    }
    ss.ready = true;
  }
  return &ss;
}
class StreamFork {
 public:
  StreamFork(cudaStream_t main, bool backward) : main_(main), ss_(side_streams()) {
    if (!ss_) return;
    lock_ = std::unique_lock<std::mutex>(ss_->mu);
    if (backward) {
      for (int l = 0; l < 4; ++l) side_[n_++] = ss_->chain[l];
      for (int l = 0; l < 4; ++l) side_[n_++] = ss_->grads[l];
    } else {
      for (int l = 0; l < 3; ++l) side_[n_++] = ss_->fwd[l];
    }
    forked_ = cudaEventRecord(ss_->fork, main_) == cudaSuccess;
    for (int i = 0; forked_ && i < n_; ++i)
      forked_ = cudaStreamWaitEvent(side_[i], ss_->fork, 0) == cudaSuccess;
    backward_ = backward;
  }
  ~StreamFork() {
    if (!forked_) return;
    for (int i = 0; i < n_; ++i) {
      cudaEventRecord(ss_->join[i], side_[i]);
      cudaStreamWaitEvent(main_, ss_->join[i], 0);
    }
  }
  // level 0..3 = P2..P5: the forward's level streams, or the backward's chain streams
  cudaStream_t level(int l) const {
    if (!forked_) return main_;
    return backward_ ? ss_->chain[l] : l > 0 ? ss_->fwd[l - 1] : main_;
  }
  // the backward's weight-gradient streams
  cudaStream_t grads(int l) const { return forked_ && backward_ ? ss_->grads[l] : main_; }
  // Makes stream b wait for the work enqueued on stream a so far (one event, re-recorded: a
  // wait binds to the record before it, in eager mode and under capture alike).
  cudaError_t order(cudaStream_t a, cudaStream_t b) const {
    if (a == b) return cudaSuccess;
    cudaError_t e = cudaEventRecord(ss_->step, a);
    return e == cudaSuccess ? cudaStreamWaitEvent(b, ss_->step, 0) : e;
  }
  // Named points (i = 0..3, one record each per fork): `mark` records the work enqueued on
  // stream a so far, `after` makes stream b wait for that record, however much later it is
  // enqueued.
  cudaError_t mark(int i, cudaStream_t a) const {
    return forked_ ? cudaEventRecord(ss_->mark[i], a) : cudaSuccess;
  }
  cudaError_t after(int i, cudaStream_t b) const {
    return forked_ ? cudaStreamWaitEvent(b, ss_->mark[i], 0) : cudaSuccess;
  }

 private:
  cudaStream_t main_;
  SideStreams* ss_;
  std::unique_lock<std::mutex> lock_;
  cudaStream_t side_[8] = {};
  int n_ = 0;
  bool forked_ = false, backward_ = false;
};
}  // namespace

// Zero fp32 bias of the input-gradient launches (2048 floats, enough for Cin = 2048), one per
// device, made on first use (outside any stream capture: the first backward call).
const float* device_zeros() {
  static float* zeros[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!zeros[dev]) {
    float* p = nullptr;
    if (cudaMalloc(&p, 2048 * sizeof(float)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, 2048 * sizeof(float)) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    zeros[dev] = p;
  }
  return zeros[dev];
}

// Lateral backward; the input gradient uses w_t ([cblk * 256][256], w transposed with zero
// rows beyond Cin) if given, else transposes w into scratch.  ws: the caller's scratch (256-
// byte aligned, at least the call's need: a weight gradient's dw_gemm_workspace_bytes), or
// null to allocate on the stream what the call needs (nothing for an input gradient with w_t).
int lateral_backward(int dtype, const void* x, const void* w, const void* w_t,
                     const void* grad_out, void* grad_x, float* grad_w, float* grad_b, int N,
                     int Cin, int H, int W, void* stream, void* ws = nullptr) {
  DType dt;
  if (!parse_16bit(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "backward takes bf16 or fp16");
  if (!grad_out || (grad_x && !w && !w_t) || (grad_w && !x))
    return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (Cin % 8 != 0 || Cin > 2048) return fail(UFPN_ERR_UNSUPPORTED, "Cin must be a multiple of 8, at most 2048");
  if (!ufpn::aligned16(grad_out) || (x && !ufpn::aligned16(x)) || (w && !ufpn::aligned16(w)) ||
      (w_t && !ufpn::aligned16(w_t)) || (grad_x && !ufpn::aligned16(grad_x)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long pixels = static_cast<long long>(N) * H * W;
  const int cblk = (Cin + 255) / 256;
  const size_t esz = ufpn::dtype_size(dt);
  const size_t wt_bytes = grad_x && !w_t ? static_cast<size_t>(cblk) * 256 * 256 * esz : 0;
  const size_t dw_bytes = grad_w ? ufpn::dw_gemm_workspace_bytes(N, H, W, Cin, 1) : 0;
  // (the bias gradient comes out of the weight-gradient launch when both are asked for)
  const size_t cs_bytes = grad_b && !grad_w ? ufpn::colsum_workspace_bytes(pixels, 256) : 0;
  StreamScratch scratch(s);
  cudaError_t e = cudaSuccess;
  uint8_t* base = static_cast<uint8_t*>(ws);
  if (!base && wt_bytes + dw_bytes + cs_bytes > 0) {
    if ((e = scratch.alloc(wt_bytes + dw_bytes + cs_bytes)) != cudaSuccess)
      return cuda_fail(e, "backward scratch");
    base = static_cast<uint8_t*>(scratch.p);
  }
  if (grad_x) {
    const float* zero_bias = device_zeros();
    if (!zero_bias) return fail(UFPN_ERR_CUDA, "device zeros");
    const void* wt = w_t;
    if (!wt) {
      if ((e = ufpn::launch_transpose_weights(dt, w, base, 256, Cin, cblk * 256, s)) != cudaSuccess)
        return cuda_fail(e, "transpose weights");
      wt = base;
    }
    // grad_x[:, 256 cb .. +256) = grad_out . w^T[256 cb .. +256) for every slice cb: a
    // 256-channel lateral per slice, all slices in one launch
    ufpn::TcPlan plan;
    e = ufpn::plan_tc_lateral(plan, dt, grad_out, wt, zero_bias, nullptr, grad_x, N, 256, H, W,
                              0, 0, ufpn::default_tiling(H, W), device_status_word(), 0);
    if (e == cudaSuccess) e = ufpn::tc_set_channel_slices(plan, wt, 256, cblk, grad_x, Cin);
    if (e == cudaSuccess) e = ufpn::launch_tc(plan, s);
    if (e != cudaSuccess) return cuda_fail(e, "lateral input gradient");
  }
  if (grad_w) {
    float* ws = reinterpret_cast<float*>(base + wt_bytes);
    e = ufpn::launch_dw_gemm(dt, grad_out, x, N, H, W, Cin, 1, grad_w, grad_b, ws, dw_bytes,
                             device_status_word(), s);
    if (e != cudaSuccess) return cuda_fail(e, "lateral weight gradient");
  }
  if (grad_b && !grad_w) {
    float* ws = reinterpret_cast<float*>(base + wt_bytes + dw_bytes);
    e = ufpn::launch_colsum(dt, grad_out, pixels, 256, grad_b, ws, cs_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "bias gradient");
  }
  return UFPN_OK;
}

// 3x3 backward; the input gradient uses w_f ([256 c][9][256 o], the packed weights flipped)
// if given, else flips w into scratch.  ws: as for lateral_backward.
int conv3x3_backward(int dtype, const void* x, const void* w, const void* w_f,
                     const void* grad_out, void* grad_x, float* grad_w, float* grad_b, int N,
                     int H, int W, void* stream, void* ws = nullptr) {
  DType dt;
  if (!parse_16bit(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "backward takes bf16 or fp16");
  if (!grad_out || (grad_x && !w && !w_f) || (grad_w && !x))
    return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || H <= 0 || W <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (!ufpn::aligned16(grad_out) || (x && !ufpn::aligned16(x)) || (w && !ufpn::aligned16(w)) ||
      (w_f && !ufpn::aligned16(w_f)) || (grad_x && !ufpn::aligned16(grad_x)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long pixels = static_cast<long long>(N) * H * W;
  const size_t esz = ufpn::dtype_size(dt);
  const size_t wf_bytes = grad_x && !w_f ? 256ull * 9 * 256 * esz : 0;
  const size_t dw_bytes = grad_w ? ufpn::dw_gemm_workspace_bytes(N, H, W, 256, 9) : 0;
  // (the bias gradient comes out of the weight-gradient launch when both are asked for)
  const size_t cs_bytes = grad_b && !grad_w ? ufpn::colsum_workspace_bytes(pixels, 256) : 0;
  StreamScratch scratch(s);
  cudaError_t e = cudaSuccess;
  uint8_t* base = static_cast<uint8_t*>(ws);
  if (!base && wf_bytes + dw_bytes + cs_bytes > 0) {
    if ((e = scratch.alloc(wf_bytes + dw_bytes + cs_bytes)) != cudaSuccess)
      return cuda_fail(e, "backward scratch");
    base = static_cast<uint8_t*>(scratch.p);
  }
  if (grad_x) {
    const float* zero_bias = device_zeros();
    if (!zero_bias) return fail(UFPN_ERR_CUDA, "device zeros");
    const void* wf = w_f;
    if (!wf) {
      if ((e = ufpn::launch_flip_conv3x3_weights(dt, w, base, s)) != cudaSuccess)
        return cuda_fail(e, "flip weights");
      wf = base;
    }
    ufpn::TcPlan plan;
    // single-CTA halo tiles, as the forward engine runs its 3x3s (mixed tiling or the map's
    // transposed view where that needs fewer tiles; the same bits)
    ufpn::Conv3x3Tiling t = ufpn::halo_tiling();
    if (ufpn::halo_mixed_pays(N, H, W, false))
      t.mixed = true;
    else
      t.transposed = ufpn::halo_transpose_pays(H, W);
    e = ufpn::plan_tc_conv3x3(plan, dt, grad_out, wf, zero_bias, grad_x, nullptr, N, H, W, t,
                              device_status_word(), 0);
    if (e == cudaSuccess) e = ufpn::launch_tc(plan, s);
    if (e != cudaSuccess) return cuda_fail(e, "3x3 input gradient");
  }
  if (grad_w) {
    float* ws = reinterpret_cast<float*>(base + wf_bytes);
    e = ufpn::launch_dw_gemm(dt, grad_out, x, N, H, W, 256, 9, grad_w, grad_b, ws, dw_bytes,
                             device_status_word(), s);
    if (e != cudaSuccess) return cuda_fail(e, "3x3 weight gradient");
  }
  if (grad_b && !grad_w) {
    float* ws = reinterpret_cast<float*>(base + wf_bytes + dw_bytes);
    e = ufpn::launch_colsum(dt, grad_out, pixels, 256, grad_b, ws, cs_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "bias gradient");
  }
  return UFPN_OK;
}

int ufpn_lateral_conv_backward(int dtype, const void* x, const void* w, const void* grad_out,
                               void* grad_x, float* grad_w, float* grad_b, int N, int Cin, int H,
                               int W, void* stream) {
  return lateral_backward(dtype, x, w, nullptr, grad_out, grad_x, grad_w, grad_b, N, Cin, H, W,
                          stream);
}

int ufpn_lateral_conv_backward_t(int dtype, const void* x, const void* w_t, const void* grad_out,
                                 void* grad_x, float* grad_w, float* grad_b, int N, int Cin,
                                 int H, int W, void* stream) {
  if (grad_x && !w_t) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  return lateral_backward(dtype, x, nullptr, w_t, grad_out, grad_x, grad_w, grad_b, N, Cin, H, W,
                          stream);
}

int ufpn_conv3x3_backward(int dtype, const void* x, const void* w, const void* grad_out,
                          void* grad_x, float* grad_w, float* grad_b, int N, int H, int W,
                          void* stream) {
  return conv3x3_backward(dtype, x, w, nullptr, grad_out, grad_x, grad_w, grad_b, N, H, W, stream);
}

int ufpn_conv3x3_backward_f(int dtype, const void* x, const void* w_flipped, const void* grad_out,
                            void* grad_x, float* grad_w, float* grad_b, int N, int H, int W,
                            void* stream) {
  if (grad_x && !w_flipped) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  return conv3x3_backward(dtype, x, nullptr, w_flipped, grad_out, grad_x, grad_w, grad_b, N, H, W,
                          stream);
}

int ufpn_prepare_neck_weights(int dtype, int levels, const float* const* lat_w, const int* cin,
                              const float* const* conv_w, void* const* lat_out,
                              void* const* lat_t_out, void* const* conv_packed,
                              void* const* conv_flipped, void* stream) {
  DType dt;
  if (!parse_16bit(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "weights go to bf16 or fp16");
  if (levels < 1 || levels > 4 || !lat_w || !cin || !conv_w)
    return fail(UFPN_ERR_INVALID_ARG, "levels must be 1..4 with input arrays");
  ufpn::WeightPrepJob jobs[4 * 4];
  int nj = 0;
  for (int l = 0; l < levels; ++l) {
    if (cin[l] <= 0 || cin[l] % 8 != 0) return fail(UFPN_ERR_UNSUPPORTED, "Cin must be a multiple of 8");
    void* outs[4] = {lat_out ? lat_out[l] : nullptr, lat_t_out ? lat_t_out[l] : nullptr,
                     conv_packed ? conv_packed[l] : nullptr, conv_flipped ? conv_flipped[l] : nullptr};
    for (int k = 0; k < 4; ++k) {
      if (!outs[k]) continue;
      const float* in = k < 2 ? lat_w[l] : conv_w[l];
      if (!in) return fail(UFPN_ERR_INVALID_ARG, "NULL weight pointer");
      jobs[nj].kind = k;
      jobs[nj].cin = cin[l];
      jobs[nj].in = in;
      jobs[nj].out = outs[k];
      ++nj;
    }
  }
  if (nj == 0) return UFPN_OK;
  cudaError_t e = ufpn::launch_prepare_weights(dt, jobs, nj, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "prepare weights");
}

namespace {
// The grouped P5 / P4 / P3 lateral plan of the training forward, cached: planning costs the
// host ~25 us and its result depends only on the key below (the lateral tilings follow from
// H and W), which repeats from step to step as the caching allocators hand back the same
// buffers.  A few entries, replaced round robin; a miss plans again.
struct GroupPlanKey {
  int dev, dtype, N, cin[3], H[3], W[3];
  const void* x[3];
  const void* w[3];
  const float* b[3];
  void* m[3];
  int* status;
};
struct GroupPlanCache {
  std::mutex mu;
  GroupPlanKey key[4];
  ufpn::LateralGroupPlan plan[4];
  bool valid[4] = {};
  int next = 0;
};
cudaError_t grouped_lateral_plan(ufpn::LateralGroupPlan& out, ufpn::DType dt, int N,
                                 const ufpn::NeckLevel* lv, int* status) {
  static GroupPlanCache cache;
  GroupPlanKey k;
  std::memset(&k, 0, sizeof(k));  // (padding too: keys compare as bytes)
  if (cudaGetDevice(&k.dev) != cudaSuccess) k.dev = -1;
  k.dtype = static_cast<int>(dt);
  k.N = N;
  for (int i = 0; i < 3; ++i) {
    const ufpn::NeckLevel& l = lv[3 - i];
    k.cin[i] = l.Cin, k.H[i] = l.H, k.W[i] = l.W;
    k.x[i] = l.x, k.w[i] = l.lat_w, k.b[i] = l.lat_b, k.m[i] = l.merged;
  }
  k.status = status;
  {
    std::lock_guard<std::mutex> lk(cache.mu);
    for (int i = 0; i < 4; ++i)
      if (cache.valid[i] && std::memcmp(&cache.key[i], &k, sizeof(k)) == 0) {
        out = cache.plan[i];
        return cudaSuccess;
      }
  }
  const int which[3] = {3, 2, 1};
  const cudaError_t e = ufpn::plan_lateral_group_pair(out, dt, N, lv, which, 3, status, 0);
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lk(cache.mu);
    const int i = cache.next;
    cache.next = (i + 1) % 4;
    cache.key[i] = k;
    cache.plan[i] = out;
    cache.valid[i] = true;
  }
  return e;
}
}  // namespace

int ufpn_neck_train_forward(int dtype, int N, const int* cin, const int* H, const int* W,
                            const void* const* x, const float* const* lat_w,
                            const float* const* lat_b, const float* const* conv_w,
                            const float* const* conv_b, void* const* lat16, void* const* lat16_t,
                            void* const* packed, void* const* flipped, void* const* merged,
                            void* const* out, void* p6, void* stream) {
  DType dt;
  if (!parse_16bit(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "training runs on bf16 or fp16");
  if (N <= 0 || !cin || !H || !W || !x || !lat_w || !lat_b || !conv_w || !conv_b || !lat16 ||
      !packed || !merged || !out)
    return fail(UFPN_ERR_INVALID_ARG, "NULL argument");
  for (int l = 0; l < 4; ++l)
    if (!x[l] || !lat_w[l] || !lat_b[l] || !conv_w[l] || !conv_b[l] || !lat16[l] || !packed[l] ||
        !merged[l] || !out[l] || H[l] <= 0 || W[l] <= 0)
      return fail(UFPN_ERR_INVALID_ARG, "level arguments must be non-NULL with positive sizes");
  int rc = ufpn_prepare_neck_weights(dtype, 4, lat_w, cin, conv_w, lat16, lat16_t, packed,
                                     flipped, stream);
  if (rc != UFPN_OK) return rc;
  // Top-down on the caller's stream, M_l = lateral(C_l) + up(M_{l+1}); each level's 3x3 starts
  // on its own stream as soon as M_l is written (P5, P4, P3 on side streams beside the next
  // laterals, P2 on the caller's).  Where the maps upsample and the geometry fits its plan, as
  // the forward engine does: the raw P5 / P4 / P3 laterals in one launch on CTA pairs (L5 =
  // M5, L4 into scratch, L3 into M3's map), one launch for both merges (M4 = L4 + up(M5), M3 =
  // L3 + up(M4) in place), then the P2 lateral with the top-down add -- instead of a chain of
  // four laterals, each waiting for the one above.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StreamFork fork(s, false);
  StreamScratch l4(s);
  bool grouped = false;
  if (H[3] <= H[2] && W[3] <= W[2] && H[2] <= H[1] && W[2] <= W[1]) {
    ufpn::DType dt16;
    parse_16bit(dtype, &dt16);
    ufpn::NeckLevel lv[4] = {};
    for (int l = 0; l < 4; ++l) {
      lv[l].x = x[l];
      lv[l].lat_w = lat16[l];
      lv[l].lat_b = lat_b[l];
      lv[l].merged = merged[l];
      lv[l].Cin = cin[l];
      lv[l].H = H[l];
      lv[l].W = W[l];
      lv[l].lat_tiling = ufpn::default_tiling(H[l], W[l]);
    }
    cudaError_t e = l4.alloc(static_cast<size_t>(N) * H[2] * W[2] * 256 * ufpn::dtype_size(dt16));
    if (e != cudaSuccess) return cuda_fail(e, "train forward scratch");
    lv[2].merged = l4.p;
    ufpn::LateralGroupPlan lplan;
    e = grouped_lateral_plan(lplan, dt16, N, lv, device_status_word());
    if (e == cudaSuccess) {
      grouped = true;
      if ((e = ufpn::launch_lateral_group_pair(lplan, s)) != cudaSuccess)
        return cuda_fail(e, "grouped laterals");
      // (the P5 3x3 needs M5 = L5 only: its stream waits for the grouped launch, not the merge)
      if ((e = fork.order(s, fork.level(3))) != cudaSuccess) return cuda_fail(e, "level fork");
      if ((e = ufpn::launch_merge_two_levels(dt16, merged[3], l4.p, merged[2], merged[1],
                                             merged[1], N, H[3], W[3], H[2], W[2], H[1], W[1],
                                             s)) != cudaSuccess)
        return cuda_fail(e, "merge P4 and P3");
    } else if (e != cudaErrorNotSupported) {
      return cuda_fail(e, "plan grouped laterals");
    }
  }
  for (int l = 3; l >= 0; --l) {
    if (!grouped || l == 0) {
      rc = ufpn_lateral_conv(dtype, UFPN_LAYOUT_NHWC, x[l], lat16[l], lat_b[l],
                             l < 3 ? merged[l + 1] : nullptr, merged[l], N, cin[l], H[l], W[l],
                             256, l < 3 ? H[l + 1] : 0, l < 3 ? W[l + 1] : 0, stream);
      if (rc != UFPN_OK) return rc;
    }
    cudaError_t e = grouped && l == 3 ? cudaSuccess : fork.order(s, fork.level(l));
    if (e != cudaSuccess) return cuda_fail(e, "level fork");
    // 3x3s on single-CTA halo tiles, with the mixed tiling or the transposed view where that
    // needs fewer tiles (not with the fused P6): 2-5 % faster per training step than CTA pairs
    // on the own view
    const bool with_p6 = l == 3 && p6 != nullptr;
    const int tw = with_p6 ? 0
                   : ufpn::halo_mixed_pays(N, H[l], W[l], false)   ? -4
                   : ufpn::halo_transpose_pays(H[l], W[l])          ? -2
                                                                    : 0;
    rc = ufpn_conv3x3_act(dtype, merged[l], packed[l], conv_b[l], out[l], with_p6 ? p6 : nullptr,
                          N, H[l], W[l], tw, 0, 0.01f, fork.level(l));
    if (rc != UFPN_OK) return rc;
  }
  return UFPN_OK;
}

int ufpn_neck_train_backward(int dtype, int N, const int* cin, const int* H, const int* W,
                             const void* const* x, const void* const* merged,
                             const void* const* lat16_t, const void* const* flipped,
                             const void* const* grad_out, const void* grad_p6,
                             void* const* grad_x, float* const* grad_lat_w,
                             float* const* grad_lat_b, float* const* grad_conv_w,
                             float* const* grad_conv_b, void* stream) {
  DType dt;
  if (!parse_16bit(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "training runs on bf16 or fp16");
  if (N <= 0 || !cin || !H || !W || !x || !merged || !lat16_t || !flipped || !grad_out ||
      !grad_lat_w || !grad_lat_b || !grad_conv_w || !grad_conv_b)
    return fail(UFPN_ERR_INVALID_ARG, "NULL argument");
  for (int l = 0; l < 4; ++l)
    if (!x[l] || !merged[l] || !lat16_t[l] || !flipped[l] || !grad_lat_w[l] || !grad_lat_b[l] ||
        !grad_conv_w[l] || !grad_conv_b[l] || H[l] <= 0 || W[l] <= 0)
      return fail(UFPN_ERR_INVALID_ARG, "level arguments must be non-NULL with positive sizes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t esz = ufpn::dtype_size(dt);
  size_t map_bytes[4], off[6] = {0};
  for (int l = 0; l < 4; ++l) {
    map_bytes[l] = (static_cast<size_t>(N) * H[l] * W[l] * 256 * esz + 255) / 256 * 256;
    off[l + 1] = off[l] + map_bytes[l];
  }
  // scratch: dM2..dM5, then dP5 + P6's scatter (if dP6) or a zero map for an absent dP_l
  size_t zero_bytes = 0;
  for (int l = 0; l < 4; ++l)
    if (!grad_out[l] && map_bytes[l] > zero_bytes) zero_bytes = map_bytes[l];
  const size_t dp5_bytes = grad_p6 ? map_bytes[3] : 0;
  // then the eight weight gradients' split-K workspaces (they run concurrently on the level
  // streams, each in its own region; one allocation instead of one per launch)
  auto r256 = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t ws3[4], wsl[4], ws_bytes = 0;
  const size_t ws_base = off[4] + zero_bytes + dp5_bytes;
  for (int l = 0; l < 4; ++l) {
    ws3[l] = ws_base + ws_bytes;
    ws_bytes += r256(ufpn::dw_gemm_workspace_bytes(N, H[l], W[l], 256, 9));
    wsl[l] = ws_base + ws_bytes;
    ws_bytes += r256(ufpn::dw_gemm_workspace_bytes(N, H[l], W[l], cin[l], 1));
  }
  StreamScratch scratch(s);
  cudaError_t e = scratch.alloc(ws_base + ws_bytes + 16);
  if (e != cudaSuccess) return cuda_fail(e, "train backward scratch");
  uint8_t* base = static_cast<uint8_t*>(scratch.p);
  void* dm[4];
  for (int l = 0; l < 4; ++l) dm[l] = base + off[l];
  void* zeros = zero_bytes ? base + off[4] : nullptr;
  if (zeros && (e = cudaMemsetAsync(zeros, 0, zero_bytes, s)) != cudaSuccess)
    return cuda_fail(e, "memset");
  const void* dp[4];
  for (int l = 0; l < 4; ++l) dp[l] = grad_out[l] ? grad_out[l] : zeros;
  int rc;
  if (grad_p6) {  // dP5 += P6^T(dP6), into a copy (the caller's dP5 stays as given)
    void* dp5 = base + off[4] + zero_bytes;
    if ((e = cudaMemcpyAsync(dp5, dp[3], static_cast<size_t>(N) * H[3] * W[3] * 256 * esz,
                             cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
      return cuda_fail(e, "copy dP5");
    if ((rc = ufpn_p6_backward(dtype, grad_p6, dp5, N, 256, H[3], W[3], stream)) != UFPN_OK)
      return rc;
    dp[3] = dp5;
  }
  // Level l's chain stream: the 3x3 input gradient dM_l, then -- once the level below's dM
  // is final -- the top-down adjoint dM_l += up^T(dM_{l-1}), then the lateral's input
  // gradient dC_l and its weight and bias gradients (dM_l is final there; on the weight-
  // gradient stream they would queue behind the 3x3's weight gradient and its reduction,
  // measured 1.9 % slower).  Level l's weight-gradient stream: the 3x3's weight and bias
  // gradients.  Enqueued level by level (P5 first) with each level's 3x3 weight gradient right
  // after its input gradient, so that the weight gradients start early instead of forming the
  // step's tail (measured 1-2 % faster than enqueueing every chain first).
  StreamFork fork(s, true);
  for (int l = 3; l >= 0; --l) {
    rc = conv3x3_backward(dtype, nullptr, nullptr, flipped[l], dp[l], dm[l], nullptr, nullptr, N,
                          H[l], W[l], fork.level(l));
    if (rc != UFPN_OK) return rc;
    rc = conv3x3_backward(dtype, merged[l], nullptr, nullptr, dp[l], nullptr, grad_conv_w[l],
                          grad_conv_b[l], N, H[l], W[l], fork.grads(l), base + ws3[l]);
    if (rc != UFPN_OK) return rc;
  }
  if ((e = fork.mark(0, fork.level(0))) != cudaSuccess) return cuda_fail(e, "level fork");
  for (int l = 1; l < 4; ++l) {
    if ((e = fork.after(l - 1, fork.level(l))) != cudaSuccess) return cuda_fail(e, "level fork");
    rc = ufpn_upsample_add_backward(dtype, dm[l - 1], dm[l], dm[l], N, 256, H[l], W[l],
                                    H[l - 1], W[l - 1], fork.level(l));
    if (rc != UFPN_OK) return rc;
    if ((e = fork.mark(l, fork.level(l))) != cudaSuccess) return cuda_fail(e, "level fork");
  }
  for (int l = 3; l >= 0; --l) {
    if (grad_x) {
      rc = lateral_backward(dtype, nullptr, nullptr, lat16_t[l], dm[l], grad_x[l], nullptr,
                            nullptr, N, cin[l], H[l], W[l], fork.level(l));
      if (rc != UFPN_OK) return rc;
    }
    rc = lateral_backward(dtype, x[l], nullptr, nullptr, dm[l], nullptr, grad_lat_w[l],
                          grad_lat_b[l], N, cin[l], H[l], W[l], fork.level(l), base + wsl[l]);
    if (rc != UFPN_OK) return rc;
  }
  return UFPN_OK;
}

int ufpn_upsample_add_backward(int dtype, const void* grad_out, const void* base,
                               void* grad_coarse, int N, int C, int Hc, int Wc, int H, int W,
                               void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!grad_out || !grad_coarse) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || C <= 0 || Hc <= 0 || Wc <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (Hc > H || Wc > W) return fail(UFPN_ERR_UNSUPPORTED, "the coarse map must not be larger");
  cudaError_t e = ufpn::launch_upsample_adjoint(dt, grad_out, base, grad_coarse, N, C, Hc, Wc, H,
                                                W, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "upsample_add backward");
}

int ufpn_p6_backward(int dtype, const void* grad_p6, void* grad_p5, int N, int C, int H5, int W5,
                     void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!grad_p6 || !grad_p5) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || C <= 0 || H5 <= 0 || W5 <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  cudaError_t e = ufpn::launch_p6_adjoint(dt, grad_p6, grad_p5, N, C, H5, W5,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "p6 backward");
}

int ufpn_p6_maxpool(int dtype, int layout, const void* p5, void* p6, int N, int C, int H, int W,
                    void* stream) {
  DType dt;
  Layout lay;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!parse_layout(layout, &lay)) return fail(UFPN_ERR_INVALID_ARG, "bad layout");
  if (!p5 || !p6) return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  cudaError_t e = ufpn::launch_p6(dt, p5, p6, N, C, H, W, lay, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "p6");
}

int ufpn_pack_conv3x3_weights(int dtype, const float* w, void* out, int Cout, int Cin,
                              void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt) || dt == DType::F32)
    return fail(UFPN_ERR_UNSUPPORTED, "packing targets F16 or BF16");
  if (!w || !out || Cout <= 0 || Cin <= 0) return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  cudaError_t e =
      ufpn::launch_pack_conv3x3(dt, w, out, Cout, Cin, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "pack");
}

int ufpn_convert_weights(int dtype, const float* w, void* out, long long count, void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!w || !out || count <= 0) return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  cudaError_t e =
      ufpn::launch_convert_weights(dt, w, out, count, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "convert");
}

int ufpn_layout_convert(int dtype, const void* in, void* out, int N, int C, int H, int W,
                        int to_nhwc, void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!in || !out || N <= 0 || C <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  cudaError_t e = ufpn::launch_transpose(dt, in, out, N, C, H * W, to_nhwc != 0,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "layout convert");
}

// ------------------------------------------------------------------ e4m3 (FP8) path
int ufpn_absmax(int dtype, const void* x, long long count, int groups, unsigned* amax_bits,
                void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!x || !amax_bits || count <= 0) return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  if (groups < 1 || groups > 65535 || count % groups != 0)
    return fail(UFPN_ERR_INVALID_ARG, "groups must divide count (1..65535 groups)");
  cudaError_t e =
      ufpn::launch_absmax(dt, x, count, groups, amax_bits, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "absmax");
}

int ufpn_quantize_e4m3(int dtype, const void* x, long long count, int groups, unsigned* amax_ws,
                       void* q, float* scale_out, void* stream) {
  DType dt;
  if (!parse_dtype(dtype, &dt)) return fail(UFPN_ERR_UNSUPPORTED, "unsupported dtype");
  if (!x || !amax_ws || !q || !scale_out || count <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  if (groups < 1 || groups > 65535 || count % groups != 0)
    return fail(UFPN_ERR_INVALID_ARG, "groups must divide count (1..65535 groups)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax_ws, 0, sizeof(unsigned) * groups, s);
  if (e == cudaSuccess) e = ufpn::launch_absmax(dt, x, count, groups, amax_ws, s);
  if (e == cudaSuccess)
    e = ufpn::launch_quantize_e4m3(dt, x, count, groups, amax_ws, q, scale_out, s);
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "quantize e4m3");
}

int ufpn_quantize_e4m3_rows(const float* w, int rows, int cols, int pack_cin, void* q,
                            float* scales, void* stream) {
  if (!w || !q || !scales || rows <= 0 || cols <= 0 || pack_cin < 0)
    return fail(UFPN_ERR_INVALID_ARG, "bad arguments");
  if (pack_cin > 0 && cols != 9 * pack_cin)
    return fail(UFPN_ERR_INVALID_ARG, "packing a 3x3 kernel needs cols == 9 * pack_cin");
  cudaError_t e = ufpn::launch_quantize_rows_e4m3(w, rows, cols, pack_cin, q, scales,
                                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "quantize e4m3 rows");
}

int ufpn_lateral_conv_e4m3(const void* x, const float* x_scale, int x_scale_per_image,
                           const void* w, const float* w_scales, const float* bias,
                           const void* coarse, void* out, int N, int Cin, int H, int W, int Hc,
                           int Wc, unsigned* amax_out, void* stream) {
  if (!x || !x_scale || !w || !w_scales || !bias || !out)
    return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (coarse && (Hc <= 0 || Wc <= 0 || Hc > H || Wc > W))
    return fail(UFPN_ERR_INVALID_ARG, "coarse map must be non-empty and not larger than output");
  if (Cin % 16 != 0) return fail(UFPN_ERR_UNSUPPORTED, "Cin must be a multiple of 16");
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || !ufpn::aligned16(w_scales) ||
      (coarse && !ufpn::aligned16(coarse)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  ufpn::TcScales sc;
  sc.ascale = x_scale;
  sc.ascale_per_image = x_scale_per_image != 0;
  sc.wscale = w_scales;
  sc.amax_out = amax_out;
  ufpn::TcPlan plan;
  cudaError_t e = ufpn::plan_tc_lateral(plan, DType::E4M3, x, w, bias, coarse, out, N, Cin, H, W,
                                        coarse ? Hc : 0, coarse ? Wc : 0,
                                        ufpn::default_tiling(H, W), device_status_word(), 0, sc);
  if (e != cudaSuccess) return cuda_fail(e, "plan e4m3 lateral");
  e = ufpn::launch_tc(plan, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "e4m3 lateral launch");
}

int ufpn_conv3x3_e4m3(const void* x, const float* x_scale, int x_scale_per_image, const void* w,
                      const float* w_scales, const float* bias, void* out, void* p6, int N,
                      int H, int W, int tile_w, unsigned* amax_out, void* stream) {
  if (!x || !x_scale || !w || !w_scales || !bias || !out)
    return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || H <= 0 || W <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || !ufpn::aligned16(w_scales) || (p6 && !ufpn::aligned16(p6)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  ufpn::TcScales sc;
  sc.ascale = x_scale;
  sc.ascale_per_image = x_scale_per_image != 0;
  sc.wscale = w_scales;
  sc.amax_out = amax_out;
  if (tile_w > 0 || tile_w < -5)
    return fail(UFPN_ERR_INVALID_ARG,
                "e4m3 3x3: tile_w must be 0 (halo), -1 (halo, CTA pairs), -2 / -3 (the same "
                "on the map's transposed view) or -4 / -5 (mixed)");
  ufpn::Conv3x3Tiling t = tile_w == -1 || tile_w == -3 || tile_w == -5 ? ufpn::halo_pair_tiling()
                                                                      : ufpn::halo_tiling();
  t.transposed = tile_w == -2 || tile_w == -3;
  t.mixed = tile_w == -4 || tile_w == -5;
  if ((t.transposed || t.mixed) && p6)
    return fail(UFPN_ERR_INVALID_ARG, "transposed or mixed view: no fused P6");
  ufpn::TcPlan plan;
  cudaError_t e = ufpn::plan_tc_conv3x3(plan, DType::E4M3, x, w, bias, out, p6, N, H, W, t,
                                        device_status_word(), 0, sc);
  if (e != cudaSuccess) return cuda_fail(e, "plan e4m3 conv3x3");
  e = ufpn::launch_tc(plan, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "e4m3 conv3x3 launch");
}

int ufpn_conv3x3_e4m3_from_bf16(const void* x, const unsigned* amax_bits, const void* w,
                                const float* w_scales, const float* bias, void* out, void* p6,
                                int N, int H, int W, void* stream) {
  if (!x || !amax_bits || !w || !w_scales || !bias || !out)
    return fail(UFPN_ERR_INVALID_ARG, "NULL tensor pointer");
  if (N <= 0 || H <= 0 || W <= 0) return fail(UFPN_ERR_INVALID_ARG, "sizes must be positive");
  if (!ufpn::aligned16(x) || !ufpn::aligned16(w) || !ufpn::aligned16(out) ||
      !ufpn::aligned16(bias) || !ufpn::aligned16(w_scales) || (p6 && !ufpn::aligned16(p6)))
    return fail(UFPN_ERR_ALIGNMENT, "tensors must be 16-byte aligned");
  ufpn::TcScales sc;
  sc.wscale = w_scales;
  sc.in_amax = amax_bits;
  ufpn::TcPlan plan;
  cudaError_t e = ufpn::plan_tc_conv3x3(plan, DType::E4M3, x, w, bias, out, p6, N, H, W,
                                        ufpn::halo_pair_tiling(), device_status_word(), 0, sc);
  if (e != cudaSuccess) return cuda_fail(e, "plan e4m3 conv3x3");
  e = ufpn::launch_tc(plan, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? UFPN_OK : cuda_fail(e, "e4m3 conv3x3 launch");
}

// ------------------------------------------------------------------ reference C ABI
namespace {

// Times one upsample launch on the legacy stream with events and synchronises,
// as the reference's launchers did (fast_upsample_kernels.cu:482-496).
cudaError_t timed_upsample(DType dt, const void* in, void* out, int N, int C, int Hi, int Wi,
                           int Ho, int Wo, int ac, float* ms_out, float* gbs_out) {
  if (!in || !out || N <= 0 || C <= 0 || Hi <= 0 || Wi <= 0 || Ho <= 0 || Wo <= 0)
    return cudaErrorInvalidValue;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, 0);
  cudaError_t e = ufpn::launch_upsample_add(dt, in, nullptr, out, N, C, Hi, Wi, Ho, Wo, ac,
                                            Layout::NHWC, 0);
  cudaEventRecord(b, 0);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  float ms = 0.f;
  if (e == cudaSuccess) cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (ms_out) *ms_out = ms;
  if (gbs_out) {
    const double bytes = static_cast<double>(N) * C * (static_cast<double>(Hi) * Wi +
                                                        static_cast<double>(Ho) * Wo) *
                         ufpn::dtype_size(dt);
    *gbs_out = ms > 0 ? static_cast<float>(bytes / (ms * 1e-3) / 1e9) : 0.f;
  }
  return e;
}

struct UpsampleEngine {
  int device = 0;
  struct Rec {
    std::string name;
    float ms, gbs;
    size_t bytes;
  };
  std::vector<Rec> recs;
};

}  // namespace

cudaError_t launch_production_upsample_float(const float* input, float* output, int batch_size,
                                             int channels, int in_height, int in_width,
                                             int out_height, int out_width, int align_corners,
                                             float* kernel_time_ms, float* bandwidth_gb_s) {
  return timed_upsample(DType::F32, input, output, batch_size, channels, in_height, in_width,
                        out_height, out_width, align_corners, kernel_time_ms, bandwidth_gb_s);
}

cudaError_t launch_production_upsample_half(const void* input, void* output, int batch_size,
                                            int channels, int in_height, int in_width,
                                            int out_height, int out_width, int align_corners,
                                            float* kernel_time_ms, float* bandwidth_gb_s) {
  return timed_upsample(DType::F16, input, output, batch_size, channels, in_height, in_width,
                        out_height, out_width, align_corners, kernel_time_ms, bandwidth_gb_s);
}

cudaError_t launch_production_upsample_bfloat16(const void* input, void* output, int batch_size,
                                                int channels, int in_height, int in_width,
                                                int out_height, int out_width, int align_corners,
                                                float* kernel_time_ms, float* bandwidth_gb_s) {
  return timed_upsample(DType::BF16, input, output, batch_size, channels, in_height, in_width,
                        out_height, out_width, align_corners, kernel_time_ms, bandwidth_gb_s);
}

void* create_upsample_engine(int device_id) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device_id < 0 || device_id >= n) {
    g_last_error = "create_upsample_engine: invalid device";
    return nullptr;
  }
  auto* e = new UpsampleEngine;
  e->device = device_id;
  return e;
}

void destroy_upsample_engine(void* engine) { delete static_cast<UpsampleEngine*>(engine); }

int production_upsample_float(void* engine, const float* input, float* output, int batch_size,
                              int channels, int in_height, int in_width, int out_height,
                              int out_width, float scale_y, float scale_x, int align_corners,
                              float* metrics_out) {
  auto* eng = static_cast<UpsampleEngine*>(engine);
  if (!eng) return -1;
  (void)scale_y;  // the scale is derived from the sizes (in / out), as the kernels did
  (void)scale_x;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(eng->device);
  float ms = 0.f, gbs = 0.f;
  cudaError_t e = timed_upsample(DType::F32, input, output, batch_size, channels, in_height,
                                 in_width, out_height, out_width, align_corners, &ms, &gbs);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    g_last_error = std::string("production_upsample_float: ") + cudaGetErrorString(e);
    return -1;
  }
  const size_t bytes = static_cast<size_t>(batch_size) * channels *
                       (static_cast<size_t>(in_height) * in_width +
                        static_cast<size_t>(out_height) * out_width) * 4;
  eng->recs.push_back({"bilinear_upsample_f32", ms, gbs, bytes});
  if (metrics_out) {
    metrics_out[0] = ms;
    metrics_out[1] = gbs;
    metrics_out[2] = 0.f;
    metrics_out[3] = static_cast<float>(bytes);
  }
  return 0;
}

void print_upsample_profiling_summary(void* engine) {
  auto* eng = static_cast<UpsampleEngine*>(engine);
  if (!eng) return;
  double tot = 0;
  for (auto& r : eng->recs) tot += r.ms;
  std::printf("upsample engine (device %d): %zu calls, %.4f ms total\n", eng->device,
              eng->recs.size(), tot);
  for (auto& r : eng->recs)
    std::printf("  %-24s %9.4f ms %9.1f GB/s %12zu B\n", r.name.c_str(), r.ms, r.gbs, r.bytes);
}

int export_upsample_profiling_data(void* engine, const char* filename) {
  auto* eng = static_cast<UpsampleEngine*>(engine);
  if (!eng || !filename) return -1;
  std::ofstream f(filename);
  if (!f) return -1;
  f << "kernel,time_ms,bandwidth_gb_s,bytes\n";
  for (auto& r : eng->recs) f << r.name << "," << r.ms << "," << r.gbs << "," << r.bytes << "\n";
  return f ? 0 : -1;
}

// ------------------------------------------------------------------ autotuner C ABI
}  // extern "C"

namespace ufpn {
void record_lateral_tiling(DType dt, int N, int cin, int H, int W, int tile_w);  // engine.cu
}
namespace {
std::mutex g_tune_mu;
std::map<std::tuple<int, int, int, int, int>, TuningResult> g_tune_results;

// Seeded pseudo-random 16-bit values in [-1, 1) (hash of the index): tuning inputs that are
// not all zero, made on the device.
template <typename T>
__global__ void tune_fill_kernel(T* p, size_t n, uint32_t seed, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint32_t h = static_cast<uint32_t>(i) * 2654435761u ^ seed;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    p[i] = static_cast<T>((static_cast<float>(h & 0xFFFFu) / 32768.f - 1.f) * scale);
  }
}
template <typename T>
void tune_fill(void* p, size_t n, uint32_t seed, float scale, cudaStream_t s) {
  tune_fill_kernel<T><<<1024, 256, 0, s>>>(static_cast<T*>(p), n, seed, scale);
}
}  // namespace

extern "C" {

int ufpn_autotune_lateral(int dtype, int batch_size, int in_channels, int height, int width,
                          void* stream, TuningResult* out) {
  DType dt;
  if (!parse_dtype(dtype, &dt) || (dt != DType::BF16 && dt != DType::F16))
    return fail(UFPN_ERR_UNSUPPORTED, "the lateral tuner takes bf16 or fp16");
  if (!out || batch_size <= 0 || in_channels <= 0 || in_channels % 8 != 0 || height <= 0 || width <= 0)
    return fail(UFPN_ERR_INVALID_ARG, "need positive sizes, Cin % 8 == 0 and a result pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t px = static_cast<size_t>(batch_size) * height * width;
  void *x = nullptr, *w = nullptr, *o = nullptr;
  float* b = nullptr;
  TuningResult res{};
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  bool ok = cudaMalloc(&x, px * in_channels * 2) == cudaSuccess &&
            cudaMalloc(&w, static_cast<size_t>(256) * in_channels * 2) == cudaSuccess &&
            cudaMalloc(&o, px * 256 * 2) == cudaSuccess &&
            cudaMalloc(&b, 256 * sizeof(float)) == cudaSuccess &&
            cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
  float best = -1.f;
  if (ok) {
    if (dt == DType::BF16) {
      tune_fill<__nv_bfloat16>(x, px * in_channels, 1u, 1.f, s);
      tune_fill<__nv_bfloat16>(w, static_cast<size_t>(256) * in_channels, 2u, 0.05f, s);
    } else {
      tune_fill<__half>(x, px * in_channels, 1u, 1.f, s);
      tune_fill<__half>(w, static_cast<size_t>(256) * in_channels, 2u, 0.05f, s);
    }
    cudaMemsetAsync(b, 0, 256 * sizeof(float), s);
    // candidates: every lateral tile shape of 128 pixels (width 8..128) that is not mostly
    // padding, each timed on the caller's stream (10 launches after one warm-up)
    for (int tw : {8, 16, 32, 64, 128}) {
      if (tw > 2 * width && tw != 8) continue;
      ufpn::Conv3x3Tiling t;
      t.tile_w = tw;
      t.tile_h = 128 / tw;
      ufpn::TcPlan plan;
      if (ufpn::plan_tc_lateral(plan, dt, x, w, b, nullptr, o, batch_size, in_channels, height,
                                width, 0, 0, t, device_status_word(), 0) != cudaSuccess)
        continue;
      if (ufpn::launch_tc(plan, s) != cudaSuccess) break;
      cudaEventRecord(e0, s);
      for (int i = 0; i < 10; ++i) ufpn::launch_tc(plan, s);
      cudaEventRecord(e1, s);
      if (cudaEventSynchronize(e1) != cudaSuccess) break;
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      ms /= 10.f;
      if (best < 0 || ms < best) {
        best = ms;
        res.tile_w = tw;
        res.tile_h = 128 / tw;
        res.num_ctas = plan.grid;
      }
    }
    ok = best > 0;
  }
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFree(x);
  cudaFree(w);
  cudaFree(o);
  cudaFree(b);
  if (!ok) return fail(UFPN_ERR_CUDA, "lateral tuning: allocation or launch failed");
  res.time_ms = best;
  const double flops = 2.0 * px * 256 * in_channels;
  const double bytes = (px * (in_channels + 256) + 256.0 * in_channels) * 2;
  res.performance_gflops = static_cast<float>(flops / (best * 1e-3) / 1e9);
  res.memory_bandwidth_gb_s = static_cast<float>(bytes / (best * 1e-3) / 1e9);
  std::snprintf(res.architecture_name, sizeof(res.architecture_name), "sm_100a");
  // engines configured for this shape afterwards start from the tuned tile shape
  ufpn::record_lateral_tiling(dt, batch_size, in_channels, height, width, res.tile_w);
  *out = res;
  return UFPN_OK;
}

TuningResult* fpn_auto_tune_lateral_conv(int batch_size, int in_channels, int out_channels,
                                         int height, int width) {
  if (out_channels != 256 || batch_size <= 0 || in_channels <= 0 || in_channels % 8 != 0 ||
      height <= 0 || width <= 0) {
    g_last_error = "fpn_auto_tune_lateral_conv: need out_channels = 256, Cin % 8 == 0";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_tune_mu);
  auto key = std::make_tuple(batch_size, in_channels, out_channels, height, width);
  auto it = g_tune_results.find(key);
  if (it != g_tune_results.end()) return &it->second;
  TuningResult res{};
  // (the reference's signature has no stream: the calling thread's default stream)
  if (ufpn_autotune_lateral(UFPN_DTYPE_BF16, batch_size, in_channels, height, width,
                            cudaStreamPerThread, &res) != UFPN_OK)
    return nullptr;
  auto ins = g_tune_results.emplace(key, res);
  return &ins.first->second;
}

void fpn_auto_tune_save_results(const char* filename) {
  if (!filename) return;
  std::lock_guard<std::mutex> lk(g_tune_mu);
  std::ofstream f(filename);
  f << "batch,in_channels,out_channels,height,width,num_ctas,time_ms,gflops,gb_s,arch\n";
  for (auto& kv : g_tune_results) {
    const auto& k = kv.first;
    const auto& r = kv.second;
    f << std::get<0>(k) << "," << std::get<1>(k) << "," << std::get<2>(k) << ","
      << std::get<3>(k) << "," << std::get<4>(k) << "," << r.num_ctas << "," << r.time_ms << ","
      << r.performance_gflops << "," << r.memory_bandwidth_gb_s << "," << r.architecture_name
      << "\n";
  }
}

}  // extern "C"
