// UnifiedFPNCore: the FPN neck engine (C++ API).
//
// Replaces lib/core/fpn_engine.cu:10-416 of the reference with the same method
// names.  Differences a caller sees:
//   * forward() is stream-ordered on the caller's stream and never blocks the
//     host (the reference synchronised four private streams every call,
//     fpn_engine.cu:239-241).
//   * The neck computed is the standard one: M5 = lat(C5); M_l = lat(C_l) +
//     bilinear_up(M_{l+1}); P_l = conv3x3(M_l) (full 256->256 conv, bias, no
//     BN/ReLU); P6 = max_pool2d(P5, 1, 2).
//   * Inputs are C2..C5 (a fifth tensor, C6, is accepted and ignored).
//   * 16-bit inputs run on the tensor cores (tcgen05 + TMA), fp32 inputs on the
//     CUDA cores in full fp32.
//   * FP8_E4M3 inputs (NHWC, each with a per-tensor fp32 scale) run on the fp8
//     tensor cores: weights are quantised per output channel (absmax / 448) when
//     set, every merged map M_l is quantised per tensor before its 3x3, and the
//     outputs P2..P6 are bf16.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "unified_fpn/core/types.h"

class __attribute__((visibility("default"))) UnifiedFPNCore {
 public:
  explicit UnifiedFPNCore(size_t workspace_size = 512ull << 20, int device = -1);
  ~UnifiedFPNCore();
  UnifiedFPNCore(const UnifiedFPNCore&) = delete;
  UnifiedFPNCore& operator=(const UnifiedFPNCore&) = delete;

  // backbone_dims: C2..C5 (4 entries) or C2..C6 (5, the last ignored).
  // dtype: FLOAT32, FLOAT16, BFLOAT16 or FP8_E4M3 (NHWC only; bf16 outputs).
  // layout: layout of inputs and outputs.
  void configure_levels(const std::vector<FPNDimensions>& backbone_dims, int output_channels,
                        FPNDataType dtype = FPNDataType::FLOAT32,
                        FPNLayout layout = FPNLayout::NCHW);
  // backbone_channels: Cin of C2..C5 (4 entries) or the reference's 5-entry form
  // {unused, C2, C3, C4, C5}.
  void allocate_weights(const std::vector<int>& backbone_channels, int output_channels);
  // fp32 weights, host or device memory: lateral [256][Cin] (or [256][Cin][1][1]),
  // bias [256], output [256][256][3][3], bias [256].
  void set_weights(int level, const float* lateral_weights, const float* lateral_bias,
                   const float* output_weights, const float* output_bias);

  // inputs: C2..C5 (or C2..C6); outputs: P2..P5 (4) or P2..P6 (5).
  template <typename T>
  void forward(const std::vector<FPNTensor<T>>& backbone_features,
               std::vector<FPNTensor<T>>& output_features, cudaStream_t stream = nullptr);

  const FPNPerformanceMetrics& get_performance_metrics() const;
  void set_kernel_config(const FPNKernelConfig& config);
  FPNKernelConfig get_kernel_config() const;
  size_t get_memory_usage() const;

  // Graph cache counters: [0] pointer sets captured into a graph, [1] graph replays,
  // [2] forwards launched directly (a pointer set's first use), [3] graphs cached now.
  void graph_stats(long long* out4) const;
  // Time every kernel of the next forward() with CUDA events (serialises the
  // schedule; synchronises the stream at the end of that forward).
  void set_profiling(bool enable);
  // Named integer options of the schedule and of the per-level kernel shapes (the knobs the
  // autotuner sets; the C ABI's ufpn_core_set_option lists them).  Throws FPNException on an
  // unknown name or value.
  void set_option(const std::string& name, int value);
  int get_option(const std::string& name) const;
  // Record the fused neck kernel's device timeline during the next forward() (launched
  // directly, then the stream is synchronised).  get_neck_trace returns globaltimer ns:
  // [0] start, [1..4] P2..P5 laterals complete, [5] end, [6] first P2 3x3 tile started.
  void trace_next_forward();
  void get_neck_trace(unsigned long long* out8) const;
  // Tunes the schedule for the configured geometry with the given buffers: every knob
  // (per level: 3x3 tiling, lateral tile shape; the P2 lateral on CTA pairs, the grouped
  // lateral launch's top-down adds and split-K, the merge grid, programmatic launches, the
  // two-level merge; e4m3: the 3x3 pair / single CTA, the two-pass P2 lateral) is set to each
  // candidate in turn, each timed as the whole forward (graph replays on `stream`), keeping
  // the fastest (coordinate descent).  The result is kept for this geometry (save_tuning /
  // load_tuning) and applied; returns a human-readable report.  FP8_E4M3: input_scales as
  // for forward_raw_scaled.
  std::string autotune(const void* const* inputs, void* const* outputs, void* p6,
                       cudaStream_t stream, int iterations = 10,
                       const float* const* input_scales = nullptr);
  bool save_tuning(const std::string& path) const;
  bool load_tuning(const std::string& path);

  // Reads (and optionally clears) the device status word the kernels write on a
  // pipeline timeout.  Synchronises the device.
  int device_status(bool reset);

  // Untyped entry point used by the C ABI.
  void forward_raw(const void* const* inputs, void* const* outputs, void* p6,
                   cudaStream_t stream);
  // FP8_E4M3 inputs: input_scales[l] points to the device fp32 dequantisation scale of
  // C_{l+2} (x = q * scale).  Other dtypes accept input_scales == nullptr only.
  void forward_raw_scaled(const void* const* inputs, const float* const* input_scales,
                          void* const* outputs, void* p6, cudaStream_t stream);

  struct Impl;

 private:
  std::unique_ptr<Impl> impl_;
};
