// Public C++ types of the B200 FPN-neck library.
//
// Names, members and meanings follow the reference's public header
// include/unified_fpn/core/types.h so code written against it keeps compiling:
//   FPNException / FPN_THROW ............ types.h:24-46
//   CUDA_CHECK .......................... types.h:140-186 (throws, never exit())
//   FPNDataType ......................... types.h:208-223 (same ordinal values)
//   FPNActivation ....................... types.h:295-300
//   FPNDimensions ....................... types.h:302-308
//   FPNLevelConfig ...................... types.h:310-315
//   FPNTensor<T> ........................ types.h:317-333 (+ layout member)
//   FPNKernelConfig ..................... types.h:335-361 (subset that has meaning here)
//   FPNWeights .......................... types.h:363-376
//   FPNPerformanceMetrics ............... types.h:378-405
// The declared-but-never-defined reference classes (DeviceCapabilities,
// MemoryPool, AutoTuner, PrecisionConfig) are not carried over; the CUDA
// caching allocator of the caller and the measured autotuner of the engine
// (include/unified_fpn/core/engine.h) take their place.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <exception>
#include <string>

class FPNException : public std::exception {
 public:
  FPNException(const std::string& message, const char* file, int line, const char* function)
      : message_(message), file_(file), line_(line), function_(function) {
    full_message_ = "FPN Error in " + std::string(function) + " at " + std::string(file) + ":" +
                    std::to_string(line) + " - " + message;
  }
  const char* what() const noexcept override { return full_message_.c_str(); }
  const std::string& get_message() const { return message_; }
  const char* get_file() const { return file_; }
  int get_line() const { return line_; }
  const char* get_function() const { return function_; }

 private:
  std::string message_;
  std::string full_message_;
  const char* file_;
  int line_;
  const char* function_;
};

#define FPN_THROW(message) throw FPNException(message, __FILE__, __LINE__, __func__)

#define CUDA_CHECK(call)                                                            \
  do {                                                                              \
    cudaError_t fpn_err_ = (call);                                                  \
    if (fpn_err_ != cudaSuccess)                                                    \
      FPN_THROW(std::string("CUDA Error: ") + cudaGetErrorString(fpn_err_) +        \
                "\nCall: " #call);                                                  \
  } while (0)

enum class FPNDataType {
  FLOAT32,
  FLOAT16,
  BFLOAT16,
  INT8,
  INT4,
  TFLOAT32,
  FP8_E4M3,
  FP8_E5M2,
  DOUBLE,
  INT16,
  UINT8,
  COMPLEX64,
  BOOL,
  AUTO
};

// Memory layout of a 4-D feature map [N, C, H, W].  NCHW is the reference's
// (torch-contiguous) layout; NHWC is torch.channels_last, the layout the
// tensor-core path computes in.
enum class FPNLayout { NCHW = 0, NHWC = 1 };

enum class FPNActivation { NONE, RELU, LEAKY_RELU, SWISH };

struct FPNDimensions {
  int batch_size;
  int channels;
  int height;
  int width;
  size_t stride_bytes;
};

struct FPNLevelConfig {
  FPNDimensions input_dim;
  FPNDimensions output_dim;
  float scale_factor;
  bool enable_output_conv;
};

inline size_t fpn_element_size(FPNDataType t) {
  switch (t) {
    case FPNDataType::FLOAT32:
    case FPNDataType::TFLOAT32:
      return 4;
    case FPNDataType::FLOAT16:
    case FPNDataType::BFLOAT16:
    case FPNDataType::INT16:
      return 2;
    case FPNDataType::DOUBLE:
    case FPNDataType::COMPLEX64:
      return 8;
    default:
      return 1;
  }
}

template <typename T>
struct FPNTensor {
  T* data;
  FPNDimensions dims;
  FPNDataType dtype;
  bool is_device_memory;
  FPNLayout layout = FPNLayout::NCHW;

  size_t total_elements() const {
    return static_cast<size_t>(dims.batch_size) * dims.channels * dims.height * dims.width;
  }
  size_t size_bytes() const { return total_elements() * fpn_element_size(dtype); }
};

struct FPNKernelConfig {
  // 3x3 conv: 0 = automatic (tuned tiling if any, else 8 x 16 tiles with halo reuse on
  // CTA pairs); 8..128 = plain tiles of that width (tile height = 128 / width).
  int tile_size = 0;
  int channels_per_thread = 8;   // accepted for API compatibility
  int shared_mem_size = 0;       // accepted for API compatibility
  bool use_tensor_cores = true;  // false forces the fp32 CUDA-core path
  bool enable_async_copy = true; // TMA is always used on the tensor-core path
  // Output activation of every level's 3x3 (and so of P6), fused into its epilogue after the
  // bias: NONE (the standard neck), RELU, LEAKY_RELU (negative slope activation_alpha; the
  // reference's engine passes 0.01) or SWISH (v / (1 + exp(-v))).
  FPNActivation activation = FPNActivation::NONE;
  float activation_alpha = 0.01f;
  // e4m3 schedule: the P2 lateral runs twice -- once publishing only the per-image absmax of
  // its bf16-rounded output, once storing that output quantised to e4m3 -- instead of
  // storing bf16 M2 for a separate quantisation pass (same codes and scales).  Off: the
  // lateral is bound by its per-tile epilogue latency, not HBM, so the second pass costs
  // nearly a whole lateral (R50 640x640 batch 16: 30.3k against 32.4k images/s).
  bool fp8_two_pass_p2 = false;
  bool enable_graph_capture = true;  // replay the P5->P2 schedule as one CUDA graph
  // Tensor-core path: run all 4 laterals and 4 3x3 convs as ONE persistent kernel with
  // device-side level dependencies (true), or as 8 kernels on two streams (false, the
  // faster schedule at the R50 800x1216 batch-2 workload today).
  bool fused_neck_kernel = false;
  // Split schedule only: run every kernel on the caller's stream, one after the other
  // (false: each level's 3x3 on a second stream, overlapping the top-down chain).
  bool single_stream = false;
  // 16-bit split schedule: launch each kernel that follows another kernel on the main
  // stream as a programmatic dependent launch (it is scheduled during its predecessor's
  // tail, sets up and waits on the device for the predecessor's results), hiding launch
  // latency and prologues along the P5 -> P2 chain.  (Not used by the e4m3 schedule.)
  bool programmatic_launch = true;
  // 16-bit split schedule: launch the main-stream chain (laterals, merges, P2 3x3) at the
  // device's highest launch priority, the side streams' 3x3s at the default one.  Off:
  // measured 1.4% slower at the R50 800x1216 batch-2 workload (the chain's CTAs then take
  // every freed SM and the side 3x3s pile up behind the P2 3x3).
  bool chain_priority = false;
  // Tensor-core split schedules: merge M4 and M3 in one launch when the maps upsample
  // (merge_two_levels; set before the first forward of a geometry, which allocates its raw-L4
  // buffer), else per level in place.  Off: measured slower end to end at the R50 800x1216
  // batch-2 and 640x640 batch-16 workloads (one launch, but the P4 3x3 then waits for both
  // merges and the tiles form a single wave that other streams' CTAs cut short).
  bool merge_two_levels = false;
  // 16-bit split schedule: the grouped lateral launch (P5, P4, P3) also performs the top-down
  // adds M4 = L4 + up(M5) and M3 = L3 + up(M4) in its epilogues, ordered by device-side level
  // counters, instead of two merge kernels after it (false: raw laterals, then the merges).
  bool grouped_topdown = false;
  // Units per lateral tile over K in the grouped lateral launch, per level (P2..P5; the P2
  // lateral runs in its own kernel and ignores its entry): 1, 2 or 4.  A long K loop (the P5
  // lateral's 2048 channels) otherwise holds one SM per tile for its whole weight stream.
  int lateral_ksplit[4] = {1, 1, 1, 1};
  // Units per lateral tile over the output channels in the grouped lateral launch, per level
  // (P2..P5; P2 ignored): 1, or 2 (two N = 128 halves, each streaming half the weights; a
  // level with lateral_ksplit > 1 keeps whole-channel units).
  int lateral_nsplit[4] = {1, 1, 1, 1};
  // 3x3 on CTA pairs: run a short last round of pair units as channel halves (N = 128 each).
  bool conv3x3_tail_halves = true;
  // Halo 3x3s on the map's transposed view (tiles of 16 columns x 8 rows) wherever that
  // needs fewer tiles (200 x 304: 475 instead of 494 per image).  The same bits.
  bool conv3x3_transpose = true;
  // With conv3x3_transpose: where it needs no more tiles than the transposed view, a mixed
  // tiling -- the map's own view for the rows that fill whole 16-row tiles, the transposed
  // view only for the remaining strip of at most 8 rows (200 x 304: 456 + 19 tiles per
  // image).  The same bits.
  bool conv3x3_mixed = true;
  // 3x3s on CTA pairs claim their work items at run time (a device counter) instead of a
  // static round robin, so that pairs that reach an SM late, while other streams' CTAs hold
  // it, take fewer items.  Each item's results do not depend on which pair runs it.
  // Measured slower at R50 800x1216 x 2 (equal-sized items claimed greedily end less evenly
  // than the static deal's 6.5 rounds): off.
  bool conv3x3_dynamic = false;
  // 16-bit split schedule: the grouped raw P5 / P4 / P3 laterals on CTA pairs (each SM
  // streams half of every weight k-block; host-dealt static schedule).  Same bits as the
  // single-CTA grouped launch (false), which split-K, channel halves and top-down adds in
  // the launch still use.
  bool grouped_laterals_pair = true;
  // e4m3 schedule: the P2 3x3 (CTA pairs) quantises its bf16 input per image in shared
  // memory instead of a separate quantisation pass over M2 (the same bits).
  bool fp8_quantise_in_conv = false;
  // Self-test of the device's bounded waits (0 = off): on the fused schedule, the P2 3x3
  // waits for a lateral tile that never comes, with a limit of this many microseconds, so
  // the forward ends with status kDevTimeoutDependency (outputs undefined) and the engine
  // must recover after device_status(reset).  No fault, trap or hang is involved.
  int test_stall_dependency_us = 0;
  // 16-bit P2 lateral (one CTA per tile): 16 epilogue warps and 3 operand stages instead of 8
  // warps and 4 stages (bitwise the same results).
  bool lateral_wide_epilogue = false;
  // 16-bit split schedule: the P2 level (its lateral and 3x3) pipelined over this many groups
  // of images (0 or 1: one launch each for the whole batch).  Group g's 3x3 runs on a second
  // stream while group g + 1's lateral runs, so the P2 3x3 starts after one group's lateral
  // instead of the whole batch's.
  int p2_parts = 0;
};

struct FPNWeights {
  void* lateral_conv_weights[4];  // packed in the compute dtype, [256][Cin]
  float* lateral_conv_bias[4];
  void* output_conv_weights[4];   // packed in the compute dtype, [256][9][256]
  float* output_conv_bias[4];
  size_t lateral_weight_sizes[4];
  size_t output_weight_sizes[4];
  bool weights_initialized;
};

struct FPNPerformanceMetrics {
  float forward_time_ms;
  float memory_bandwidth_gb_s;
  float compute_utilization;  // achieved TFLOP/s / measured-peak TFLOP/s of the last timed forward
  size_t peak_memory_usage_bytes;
  int num_kernel_launches;  // counted, not estimated
  // Per-stage device times of the last profiled (serialised) forward.  Tensor-core path:
  // [laterals P5+P4+P3 (one grouped launch), 3x3 P5 (+P6), merge P4, 3x3 P4, merge P3,
  //  3x3 P3, lateral P2 (+fused top-down add), 3x3 P2];
  // fp32 path: [lat P5, 3x3 P5, lat P4, 3x3 P4, lat P3, 3x3 P3, lat P2, 3x3 P2].
  float kernel_times_ms[8];
};
