/* C ABI of the B200 FPN-neck library (libunified_fpn_b200.so).
 *
 * Plain pointers, sizes and status codes; no C++ or torch types.  Every entry
 * point enqueues work on the given CUDA stream (NULL = legacy default stream)
 * and returns without blocking the host unless stated otherwise.  On failure
 * an entry point returns a non-zero UFPN_ERR_* code and ufpn_last_error()
 * describes it; nothing here calls exit().
 *
 * Each declaration names the reference interface it replaces (paths are
 * relative to the sanowl/-UnifiedFPN source tree).
 */
#ifndef UNIFIED_FPN_C_H_
#define UNIFIED_FPN_C_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define UFPN_OK 0
#define UFPN_ERR_INVALID_ARG 1
#define UFPN_ERR_CUDA 2
#define UFPN_ERR_UNSUPPORTED 3
#define UFPN_ERR_DEVICE_TIMEOUT 4
#define UFPN_ERR_STATE 5
#define UFPN_ERR_ALIGNMENT 6

/* dtype codes: the ordinals of FPNDataType (include/unified_fpn/core/types.h:208-223) */
#define UFPN_DTYPE_F32 0
#define UFPN_DTYPE_F16 1
#define UFPN_DTYPE_BF16 2
#define UFPN_DTYPE_E4M3 6

/* Device status words (ufpn_device_status, ufpn_core_device_status): the first bounded wait
 * that gave up in a launch records which role it was; 0 = no error.  Each replaces one of
 * the reference's exit() paths (include/unified_fpn/core/types.h:140-206). */
#define UFPN_DEV_TIMEOUT_PRODUCER 0x101   /* TMA producer waiting for a free stage */
#define UFPN_DEV_TIMEOUT_MMA 0x102        /* MMA issuer waiting for operands / accumulator */
#define UFPN_DEV_TIMEOUT_EPILOGUE 0x103   /* epilogue waiting for an accumulator */
#define UFPN_DEV_TIMEOUT_DRAIN 0x104      /* teardown waiting for copies in flight */
#define UFPN_DEV_TIMEOUT_DEPENDENCY 0x105 /* one-launch neck: a level dependency not met */

#define UFPN_LAYOUT_NCHW 0 /* torch contiguous */
#define UFPN_LAYOUT_NHWC 1 /* torch channels_last */

/* Message of the last failing call on this thread ("" if none). */
const char* ufpn_last_error(void);
/* Library version, major * 10000 + minor * 100 + patch. */
int ufpn_version(void);
/* Peaks that utilisation figures (ufpn_core_get_performance_metrics, UnifiedFPN.benchmark)
 * are reported against: dense 16-bit tensor TFLOP/s (e4m3 counts twice it), fp32 CUDA-core
 * TFLOP/s, HBM GB/s.  Nominal B200 figures (2250, 80, 8000) until set; a value of 0 keeps
 * the current one.  No reference counterpart (the reference divided by fixed figures,
 * python/fpn_pytorch.cpp:160-166).  ufpn_get_peaks writes the three current values. */
int ufpn_set_peaks(double tensor_tflops, double fp32_tflops, double hbm_gbs);
int ufpn_get_peaks(double* out3);
/* Reads (and with reset != 0 clears) the status word the tensor-core kernels of
 * the standalone entry points write when a pipeline wait times out on the
 * current device; 0 = no error.  Synchronises the device. */
int ufpn_device_status(int reset, int* status_out);

/* ---------------------------------------------------------------- engine
 * Replaces class UnifiedFPNCore (lib/core/fpn_engine.cu:10-416) and the
 * PyTorchFPNWrapper state it is driven through (python/fpn_pytorch.cpp:9-137). */
typedef struct ufpn_core ufpn_core;

/* fpn_engine.cu:29-35 (UnifiedFPNCore(size_t workspace_size)) */
int ufpn_core_create(int device, size_t workspace_bytes, ufpn_core** out);
/* fpn_engine.cu:37-41 */
void ufpn_core_destroy(ufpn_core* core);
/* fpn_engine.cu:95-106 (configure_levels).  in_channels/heights/widths: C2..C5. */
int ufpn_core_configure_levels(ufpn_core* core, int batch, const int* in_channels,
                               const int* heights, const int* widths, int output_channels,
                               int dtype, int layout);
/* fpn_engine.cu:108-150 (allocate_weights).  in_channels: Cin of C2..C5. */
int ufpn_core_allocate_weights(ufpn_core* core, const int* in_channels, int output_channels);
/* fpn_engine.cu:169-189 (set_weights).  fp32, host or device memory. */
int ufpn_core_set_weights(ufpn_core* core, int level, const float* lateral_w,
                          const float* lateral_b, const float* output_w, const float* output_b);
/* fpn_engine.cu:191-245 (forward).  inputs: C2..C5 device pointers in the configured
 * dtype/layout; outputs: P2..P5; p6 may be NULL. */
int ufpn_core_forward(ufpn_core* core, const void* const* inputs, void* const* outputs,
                      void* p6, void* stream);
/* fpn_engine.cu:404-406 (set_kernel_config) via fpn_pytorch.cpp:189-209.
 * tile_size: 3x3 tile width (8..128, 0 = autotuned/heuristic); activation:
 * FPNActivation ordinal (only NONE is supported). */
int ufpn_core_set_kernel_config(ufpn_core* core, int tile_size, int channels_per_thread,
                                int use_tensor_cores, int activation, int enable_graph_capture);
/* Output activation of every level's 3x3 with its LeakyReLU slope (ufpn_core_set_kernel_config
 * sets the activation with alpha unchanged, 0.01 by default as the reference's engine passes at
 * fpn_engine.cu:356-358); 0 none, 1 ReLU, 2 LeakyReLU, 3 Swish. */
int ufpn_core_set_activation(ufpn_core* core, int activation, float alpha);
/* e4m3 schedule: two_pass_p2 = 1 runs the P2 lateral twice (per-image absmax, then the e4m3
 * store) instead of storing bf16 M2 and quantising it in a separate pass (0, the default:
 * measured faster); the same codes and scales either way. */
int ufpn_core_set_fp8_options(ufpn_core* core, int two_pass_p2);
/* Host-side BatchNorm folding into a conv: for each output channel o, s = gamma[o] /
 * sqrt(var[o] + eps), out_w[o][k] = conv_w[o][k] * s, out_b[o] = (conv_b[o] - mean[o]) * s +
 * beta[o] (conv_b, gamma, beta may be NULL: 0, 1, 0), so conv(out_w, out_b) equals
 * batch_norm_kernel applied to conv(conv_w, conv_b) (fpn_compute_kernels.cu:342-371, called
 * with eps 1e-5 at fpn_engine.cu:343-353).  K = weights per output channel (Cin * kh * kw);
 * host pointers; out_w / out_b may alias conv_w / conv_b. */
int ufpn_fold_batch_norm(const float* conv_w, const float* conv_b, const float* gamma,
                         const float* beta, const float* mean, const float* var, float eps,
                         int Cout, long long K, float* out_w, float* out_b);
/* Tensor-core schedule: 1 = one persistent kernel for the whole neck, 0 = per-level kernels
 * on two streams (default), 2 = the same kernels one after the other on the caller's stream.
 * No reference counterpart (its engine launched 16 kernels on four unordered streams,
 * fpn_engine.cu:191-245). */
int ufpn_core_set_schedule(ufpn_core* core, int fused_neck_kernel);
/* Split-schedule options (results are the same either way), 16-bit inputs:
 * programmatic_launch 1 (default) = kernels that follow a kernel on the main stream are
 * programmatic dependent launches (scheduled during the predecessor's tail, waiting on the
 * device for its results), 0 = ordinary stream order; chain_priority 1 = the main-stream
 * chain runs at the device's highest launch priority, 0 (default) = default priority;
 * every tensor-core input type: merge_two_levels 1 = the P4 and P3 top-down merges in one
 * launch when the maps upsample (set before the first forward of a geometry), 0 (default)
 * = one in-place merge per level. */
int ufpn_core_set_schedule_options(ufpn_core* core, int programmatic_launch, int chain_priority,
                                   int merge_two_levels);
/* fpn_engine.cu:408-415 (get_memory_usage) */
/* Named integer options of the schedule and of the per-level kernel shapes (no reference
 * counterpart; the reference's FPNKernelConfig had fixed fields, types.h:265-293).  Every
 * option keeps the results within the tolerances; each default is the measured faster choice
 * at the R50 800x1216 batch-2 workload, and the autotuner (ufpn_core_autotune) sets them per
 * geometry.  Per level (p2..p5):
 *   "lateral_tile_pN"   8/16/32/64/128  lateral tile width (height 128 / width); default the
 *                            shape with the fewest padded pixels, or fpn_auto_tune_lateral_conv's
 *   "conv3x3_pN"        -1/0/8..128  3x3 tiling: -1 8x16 halo tiles on CTA pairs, 0 halo tiles
 *                            on single CTAs, 8..128 plain tiles of that width
 * and for the whole neck:
 *   "p2_lateral_pair"   0/1  16-bit P2 lateral on CTA pairs with resident weight halves and
 *                            fp32 top-down taps (when Cin <= 256), else one CTA per tile with
 *                            the top-down add as a tensor-core k-block
 *   "p2_lateral_dynamic"  0/1  16-bit P2 lateral as a one-job fpn_neck_kernel launch: CTAs
 *                            claim tiles from a counter, top-down taps added in fp32 in the
 *                            epilogue
 *   "lateral_wide_epilogue"  0/1  16-bit P2 lateral with 16 epilogue warps and 3 operand stages
 *                            (the same bits)
 *   "p2_parts"          0..8  the P2 level (lateral + 3x3) pipelined over this many groups of
 *                            images (0 / 1: one launch each for the whole batch)
 *   "merge_units"     -1..256  form of the top-down merge kernels: 0 = automatic (one warp
 *                            per 8-pixel unit where the map upsamples along x, else one warp
 *                            per pixel), -1 = one warp per pixel with automatic runs, > 0 =
 *                            one warp per pixel with that many 8-pixel units per block
 *   "fp8_two_pass_p2"   0/1  as ufpn_core_set_fp8_options
 *   "grouped_topdown"   0/1  the grouped P5/P4/P3 lateral launch also does the top-down adds
 *                            of M4 and M3 (device-side level counters) instead of two merge
 *                            kernels after it (16-bit split schedule)
 *   "ksplit_p3", "ksplit_p4", "ksplit_p5"
 *                       1/2/4 units per lateral tile over K in that launch (a last-arriving
 *                            unit sums the fp32 partials in a fixed order: deterministic)
 *   "p2_lateral_ctas"  0..4096  CTAs of the 16-bit P2 lateral (0 = one per SM): fewer leave
 *                            SMs to the P3 / P4 3x3s running beside it.  Default: 128/148 of
 *                            the SMs when the P2 lateral has 4..10 tiles per SM, else 0
 *   "grouped_laterals_pair"  0/1  (default 1) the grouped raw P5 / P4 / P3 laterals on CTA
 *                            pairs, each SM streaming half of every weight k-block (the same
 *                            bits as 0, the single-CTA launch)
 *   "fp8_quantise_in_conv"  0/1  e4m3: the P2 3x3 quantises its bf16 input per image in
 *                            shared memory (no quantisation pass over M2; the same bits)
 *   "conv3x3_tail_halves"  0/1  (default 1) a 3x3 on CTA pairs runs a last round of at most
 *                            half as many units as pairs as channel halves (N = 128), in half
 *                            the time; the same bits
 *   "conv3x3_transpose"  0/1  (default 1) halo 3x3s run on the map's transposed view (16 x 8
 *                            tiles) where that needs fewer tiles (200 x 304: 475 instead of
 *                            494 per image); the same bits
 *   "conv3x3_ctas_p2" .. "conv3x3_ctas_p5"  0..4096  CTAs of that level's 3x3 (0 = one per
 *                            SM; a CTA-pair 3x3 takes pairs of them).  Default 0, except the
 *                            e4m3 P3 3x3 on 96/148 of the SMs (the quantisation of M2 then
 *                            starts beside it as soon as the P2 lateral ends)
 *   "conv3x3_mixed"      0/1  (default 1) with conv3x3_transpose: the map's own view for its
 *                            whole 16-row tile rows and the transposed view for the last
 *                            1..8 rows, where that needs no more tiles than the transposed
 *                            view (200 x 304: 456 + 19 tiles); the same bits
 *   "conv3x3_dynamic"    0/1  (default 0) 3x3s on CTA pairs claim their work items at run
 *                            time (a device counter) instead of a static round robin; the
 *                            same bits
 *   "nsplit_p3", "nsplit_p4", "nsplit_p5"
 *                         1/2  units per lateral tile over the output channels in that
 *                            launch (two N = 128 halves: half the weight stream per unit, the
 *                            same bits; ignored for a level with ksplit > 1 or a top-down add)
 *   "test_stall_dependency_us"  0..1000000  self-test of the device's bounded waits (0 =
 *                            off): on the fused schedule the P2 3x3 waits for a lateral tile
 *                            that never comes, for this many microseconds, then the forward
 *                            ends with device status 0x105 (outputs undefined); clear it with
 *                            ufpn_core_device_status(reset = 1)
 *   "programmatic_launch", "chain_priority", "merge_two_levels", "single_stream",
 *   "fused_neck_kernel" 0/1  as ufpn_core_set_schedule / ufpn_core_set_schedule_options
 * Unknown names and values return UFPN_ERR_INVALID_ARG. */
int ufpn_core_set_option(ufpn_core* core, const char* name, int value);
int ufpn_core_get_option(const ufpn_core* core, const char* name, int* value);

/* Graph cache of the forward (no reference counterpart; the reference launched every kernel
 * each call and synchronised the host, fpn_engine.cu:191-245).  A forward's pointer set
 * (inputs, outputs, P6, e4m3 scales) is captured into a CUDA graph on its second use and
 * replayed after that (up to 8 sets cached, oldest evicted); its first use launches the
 * kernels directly.  out4: [0] captures, [1] replays, [2] direct forwards, [3] cached now. */
int ufpn_core_graph_stats(const ufpn_core* core, long long* out4);

size_t ufpn_core_get_memory_usage(const ufpn_core* core);
/* fpn_pytorch.cpp:171-187 (get_performance_breakdown): kernel_times_ms[8], metrics[5] =
 * {forward_ms, GB/s, compute utilisation, peak MiB, kernel launches}. */
int ufpn_core_get_performance_metrics(const ufpn_core* core, float* kernel_times_ms,
                                      float* metrics);
/* Time each kernel of the next forward with events (serialised). */
int ufpn_core_set_profiling(ufpn_core* core, int enable);
/* Record the fused neck kernel's device timeline during the next forward (synchronises);
 * out8 (globaltimer ns): [0] start, [1..4] P2..P5 laterals complete, [5] end,
 * [6] first P2 3x3 tile started.  No reference counterpart. */
int ufpn_core_trace_next_forward(ufpn_core* core);
int ufpn_core_get_neck_trace(const ufpn_core* core, unsigned long long* out8);
/* lib/utils/auto_tuner.cu:213-275 (auto_tune_lateral_conv), for every level of the neck. */
int ufpn_core_autotune(ufpn_core* core, const void* const* inputs, void* const* outputs,
                       void* p6, void* stream, int iterations);
/* ufpn_core_autotune for any input type: FP8_E4M3 inputs pass their per-tensor device scales
 * (as ufpn_core_forward_e4m3); other types NULL.  Every knob of ufpn_core_set_option that
 * applies to the geometry is tried in turn, each candidate timed as the whole forward on
 * `stream`; the fastest values are applied, kept for the geometry (save / load_tuning) and
 * reported (ufpn_last_error holds the report). */
int ufpn_core_autotune_scaled(ufpn_core* core, const void* const* inputs,
                              const float* const* input_scales, void* const* outputs, void* p6,
                              void* stream, int iterations);
/* auto_tuner.cu:305-323 (save_tuning_results) plus the missing load. */
int ufpn_core_save_tuning(const ufpn_core* core, const char* path);
int ufpn_core_load_tuning(ufpn_core* core, const char* path);
int ufpn_core_device_status(ufpn_core* core, int reset, int* status_out);

/* ---------------------------------------------------------------- standalone ops */

/* 1x1 lateral conv + bias, optionally fused with the top-down bilinear
 * upsample-add of the coarser merged map: out = conv1x1(x) + b [+ up(coarse)].
 * Replaces fpn_lateral_conv (python/fpn_pytorch.cpp:293-326) and
 * lateral_conv_kernel (lib/kernels/compute/fpn_compute_kernels.cu:127-230).
 *   dtype F32: layout must be NCHW, w fp32 [Cout][Cin], CUDA-core fp32 path.
 *   dtype F16/BF16: layout must be NHWC, w in dtype [256][Cin], Cout = 256,
 *   tcgen05 path.  coarse: same dtype/layout, [N][Cout][Hc][Wc] logical, or NULL. */
int ufpn_lateral_conv(int dtype, int layout, const void* x, const void* w, const float* bias,
                      const void* coarse, void* out, int N, int Cin, int H, int W, int Cout,
                      int Hc, int Wc, void* stream);
/* The same 16-bit lateral (NHWC, Cout = 256) on CTA pairs with each SM's half of the weights
 * resident in shared memory (tcgen05 cta_group::2); needs Cin <= 256 and, with a coarse map,
 * a top-down tap box of at most 64 coarse pixels per tile (UFPN_ERR_UNSUPPORTED otherwise).
 * The top-down taps are added to the fp32 accumulator in the epilogue, so results agree with
 * ufpn_lateral_conv to within one bf16 rounding. */
int ufpn_lateral_conv_pair(int dtype, const void* x, const void* w, const float* bias,
                           const void* coarse, void* out, int N, int Cin, int H, int W, int Hc,
                           int Wc, void* stream);

/* 3x3 pad-1 output conv 256->256 (+ optional P6 = P5[::2, ::2]).
 * Replaces launch_output_conv / depthwise_conv_kernel (fpn_engine.cu:315-362,
 * fpn_compute_kernels.cu:277-340) with the full conv of the standard neck.
 *   dtype F16/BF16: NHWC x, w in dtype packed [256][9][256] (ufpn_pack_conv3x3_weights).
 *   dtype F32: NCHW x, w fp32 [256][256][3][3].
 * tile_w: 0 = 8 x 16 tiles with halo reuse (default: each 64-channel halo is loaded once
 * and shared by the nine taps); -1 = the same tiles on CTA pairs (tcgen05 cta_group::2:
 * two SMs share one M = 256 MMA stream and each streams half of the weights); -2 / -3 =
 * 0 / -1 on the map's transposed view (tiles of 16 columns x 8 rows: fewer tiles where H is
 * not a multiple of 16 but W is; the same bits; no P6); -4 / -5 = 0 / -1 with a mixed tiling
 * (the own view for the whole 16-row tile rows, the transposed view for the remaining 1..8
 * rows; H % 16 in 1..8; on CTA pairs N x ceil(W/8) x floor(H/16) even; no P6); 8..128 =
 * plain tiles of that width (one box per tap). */
int ufpn_conv3x3(int dtype, const void* x, const void* w, const float* bias, void* out,
                 void* p6, int N, int H, int W, int tile_w, void* stream);
/* ufpn_conv3x3 with an output activation fused into its epilogue after the bias (P6, if
 * asked for, is taken from the activated output): activation 0 none, 1 ReLU, 2 LeakyReLU
 * (negative slope alpha), 3 Swish (v / (1 + exp(-v))).  Replaces launch_output_conv's
 * separate activation_kernel pass (fpn_engine.cu:356-358; fpn_compute_kernels.cu:373-395). */
int ufpn_conv3x3_act(int dtype, const void* x, const void* w, const float* bias, void* out,
                     void* p6, int N, int H, int W, int tile_w, int activation, float alpha,
                     void* stream);

/* out = lateral + bilinear_upsample(coarse -> H x W); lateral may be NULL (pure upsample).
 * Replaces launch_upsample_and_add (fpn_engine.cu:274-313) = bilinear_upsample_kernel +
 * element_wise_add_kernel (fpn_compute_kernels.cu:232-275, 397-409). */
int ufpn_upsample_add(int dtype, int layout, const void* coarse, const void* lateral, void* out,
                      int N, int C, int Hc, int Wc, int H, int W, int align_corners,
                      void* stream);

/* Two iterations of the top-down loop in one launch (NHWC, 256 channels, bf16 / fp16, maps
 * that upsample): m4 = l4 + bilinear(m5), then m3 = l3 + bilinear(m4), written in place over
 * l3.  Bitwise equal to two ufpn_upsample_add calls.  l4 must not alias m4.  Replaces two
 * iterations of the loop of UnifiedFPNCore::forward (fpn_engine.cu:230-245) calling
 * launch_upsample_and_add (fpn_engine.cu:274-313). */
int ufpn_merge_two_levels(int dtype, const void* m5, const void* l4, void* m4, void* l3_m3, int N,
                          int H5, int W5, int H4, int W4, int H3, int W3, void* stream);

/* ---- Backward pass (training).  Replaces the reference's backward_lateral_conv_kernel
 * (src/training/backward/lateral_conv_backward.cu:7-143) and backward_upsample_add_kernel
 * (src/training/backward/upsample_backward.cu:4-80) with the exact adjoints of this library's
 * forward, computed deterministically (no atomics): weight gradients on the tensor cores
 * (a GEMM over pixels), input gradients through the forward kernels with transposed weights.
 * dtype BF16/F16, NHWC maps; weight and bias gradients are fp32; any output pointer may be
 * NULL to skip that gradient.  Scratch is allocated stream-ordered on `stream`. */
/* grad_x [N][H][W][Cin] = grad_out . w; grad_w [256][Cin] = sum_p grad_out^T x;
 * grad_b [256] = sum_p grad_out.  w is the packed lateral weight [256][Cin] in dtype;
 * Cin a multiple of 8, at most 2048. */
int ufpn_lateral_conv_backward(int dtype, const void* x, const void* w, const void* grad_out,
                               void* grad_x, float* grad_w, float* grad_b, int N, int Cin, int H,
                               int W, void* stream);
/* The same with w already transposed for the input gradient: w_t [ceil(Cin/256)*256][256]
 * (ufpn_prepare_neck_weights kind "lateral transposed"). */
int ufpn_lateral_conv_backward_t(int dtype, const void* x, const void* w_t, const void* grad_out,
                                 void* grad_x, float* grad_w, float* grad_b, int N, int Cin,
                                 int H, int W, void* stream);
/* 3x3 pad-1 conv 256 -> 256: grad_x = conv3x3(grad_out, w flipped and transposed);
 * grad_w [256][256][3][3] (output channel, input channel, ky, kx); grad_b [256].
 * w is the packed weight [256][9][256] (ufpn_pack_conv3x3_weights). */
int ufpn_conv3x3_backward(int dtype, const void* x, const void* w, const void* grad_out,
                          void* grad_x, float* grad_w, float* grad_b, int N, int H, int W,
                          void* stream);
/* The same with the weights already flipped for the input gradient: w_flipped
 * [256 c][9 t][256 o] = w[o][c][8 - t] (ufpn_prepare_neck_weights). */
int ufpn_conv3x3_backward_f(int dtype, const void* x, const void* w_flipped, const void* grad_out,
                            void* grad_x, float* grad_w, float* grad_b, int N, int H, int W,
                            void* stream);
/* Every per-step weight layout of the training path from the fp32 master weights in ONE
 * launch, for `levels` levels (1..4): lat_out[l] = lateral [256][cin[l]] in dtype, lat_t_out[l]
 * = its transpose [ceil(cin/256)*256][256] (zero rows from cin), conv_packed[l] = the 3x3
 * [256][9][256] as ufpn_pack_conv3x3_weights, conv_flipped[l] = [256 c][9][256 o] =
 * w[o][c][8 - t].  lat_w[l]: fp32 [256][cin[l]], conv_w[l]: fp32 [256][256][3][3]; any output
 * array, or entry, may be NULL to skip it. */
int ufpn_prepare_neck_weights(int dtype, int levels, const float* const* lat_w, const int* cin,
                              const float* const* conv_w, void* const* lat_out,
                              void* const* lat_t_out, void* const* conv_packed,
                              void* const* conv_flipped, void* stream);
/* Training step of the whole neck in two calls (C2..C5 = level 0..3, NHWC 16-bit, batch N,
 * level sizes H[l] x W[l], input channels cin[l]; fp32 master weights as for
 * ufpn_prepare_neck_weights, fp32 biases [256]).
 * Forward: prepares the weight layouts (lat16, lat16_t, packed, flipped: caller-allocated as
 * in ufpn_prepare_neck_weights; lat16_t / flipped may be NULL for inference), computes the
 * merged maps M2..M5 (merged[l], [N][H][W][256]) top-down and P2..P5 (out[l]) with P6 (p6, or
 * NULL) -- bitwise the outputs of UnifiedFPN's forward with the same weights.
 * Backward: from dP2..dP5 (grad_out[l], 16-bit NHWC; NULL = zero) and dP6 (grad_p6 or NULL) and
 * the forward's x, merged, lat16_t and flipped, writes dC_l (grad_x[l]; grad_x or an entry
 * NULL skips it) and the fp32 gradients of every weight ([256][cin] lateral, [256][256][3][3]
 * 3x3) and bias, deterministically (fixed-order sums, no atomics).  Both calls spread their
 * per-level work over the library's own side streams, which wait for `stream` on entry and
 * are joined back into it before the call returns, so work enqueued on `stream` afterwards
 * sees every result; their scratch (the backward's dM2..dM5 and split-K workspaces) is
 * stream-ordered on `stream`.  One such call at a time per device (calls from several threads
 * take turns). */
int ufpn_neck_train_forward(int dtype, int N, const int* cin, const int* H, const int* W,
                            const void* const* x, const float* const* lat_w,
                            const float* const* lat_b, const float* const* conv_w,
                            const float* const* conv_b, void* const* lat16, void* const* lat16_t,
                            void* const* packed, void* const* flipped, void* const* merged,
                            void* const* out, void* p6, void* stream);
int ufpn_neck_train_backward(int dtype, int N, const int* cin, const int* H, const int* W,
                             const void* const* x, const void* const* merged,
                             const void* const* lat16_t, const void* const* flipped,
                             const void* const* grad_out, const void* grad_p6,
                             void* const* grad_x, float* const* grad_lat_w,
                             float* const* grad_lat_b, float* const* grad_conv_w,
                             float* const* grad_conv_b, void* stream);
/* Top-down add: grad_coarse = base (or 0) + bilinear^T(grad_out) [N][Hc][Wc][C] (the lateral's
 * gradient is grad_out itself). */
int ufpn_upsample_add_backward(int dtype, const void* grad_out, const void* base,
                               void* grad_coarse, int N, int C, int Hc, int Wc, int H, int W,
                               void* stream);
/* P6 = P5[::2, ::2]: grad_p5 at even pixels += grad_p6 (in place). */
int ufpn_p6_backward(int dtype, const void* grad_p6, void* grad_p5, int N, int C, int H5, int W5,
                     void* stream);

/* P6 = max_pool2d(P5, kernel 1, stride 2).  No reference counterpart (the reference never
 * produces P6 although it takes C6, python/fpn_pytorch.cpp:84-86). */
int ufpn_p6_maxpool(int dtype, int layout, const void* p5, void* p6, int N, int C, int H, int W,
                    void* stream);

/* The whole tensor-core neck (P2..P5 and optional P6) in one call that allocates nothing.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc on
 * their hot path (servers that own all device memory through a fixed arena, real-time
 * loops that must not enter the driver's allocator, code embedded in a framework that
 * must not create untracked allocations).
 *   inputs: C2..C5, NHWC, dtype BF16/F16; lateral_w[l]: [256][Cin_l] and output_w[l]:
 *   [256][9][256] (ufpn_pack_conv3x3_weights) in the same dtype; biases fp32 [256];
 *   outputs: P2..P5 NHWC; p6 NHWC or NULL; levels ordered fine (C2) to coarse (C5).
 *   status: optional caller-owned device int.  The call zeroes it (stream-ordered) and the
 *   kernel writes a pipeline-timeout code into it if a bounded wait gives up, so after the
 *   stream is synchronised it reports this call alone (a caller that wants to watch several
 *   calls passes a different word to each).  With status = NULL a timeout is not reported
 *   anywhere the caller can read: the outputs of such a call are undefined.
 * Scratch (merged maps M2..M5 = batch * sum(H_l * W_l) * 512 bytes, plus 512 bytes of
 * counters) lives in a file-scope device array of UFPN_NOALLOC_SCRATCH_BYTES that every
 * GPU loading the library holds until exit; larger problems are rejected with
 * UFPN_ERR_INVALID_ARG.  The first call on a device (and the first after its context was
 * replaced, e.g. by cudaDeviceReset) looks the array's address up (cudaGetSymbolAddress)
 * and should come before any stream capture.  All calls share the array: each clears the
 * counters it needs, and calls that overlap on the GPU race. */
#define UFPN_NOALLOC_SCRATCH_BYTES (64u << 20)
int ufpn_neck_forward_noalloc(int dtype, const void* const* inputs,
                              const void* const* lateral_w, const float* const* lateral_b,
                              const void* const* output_w, const float* const* output_b,
                              void* const* outputs, void* p6, int batch, const int* in_channels,
                              const int* heights, const int* widths, int* status, void* stream);

/* fp32 [Cout][Cin][3][3] (device) -> dtype [Cout][9][Cin] K-major packing for ufpn_conv3x3. */
int ufpn_pack_conv3x3_weights(int dtype, const float* w, void* out, int Cout, int Cin,
                              void* stream);
/* fp32 (device) -> dtype element conversion (lateral weight packing). */
int ufpn_convert_weights(int dtype, const float* w, void* out, long long count, void* stream);
/* NCHW <-> NHWC layout conversion. */
int ufpn_layout_convert(int dtype, const void* in, void* out, int N, int C, int H, int W,
                        int to_nhwc, void* stream);

/* ---------------------------------------------------------------- e4m3 (FP8) path
 * The reference declares FPNDataType::FP8_E4M3 (include/unified_fpn/core/types.h:208-223)
 * but never computes in it; these entry points are the FP8 neck of the same ops.
 * Quantisation is symmetric with scale = absmax / 448:
 *   amax > 0: q = e4m3_rn_satfinite(x * (448 / amax)), scale = amax / 448
 *   amax = 0: q = 0, scale = 1
 * each step a single correctly rounded fp32 operation; x ~ q * scale.
 * Absmax values travel as the bit pattern of a non-negative fp32 in an unsigned word. */

/* The count elements form `groups` equal consecutive groups (e.g. images), each with its
 * own absmax and scale.  atomicMax of max|x| of group g (dtype F32/F16/BF16) into
 * amax_bits[g] (device; zero them first). */
int ufpn_absmax(int dtype, const void* x, long long count, int groups, unsigned* amax_bits,
                void* stream);
/* Quantisation of x (dtype F32/F16/BF16, count elements in `groups` equal groups) to e4m3 q
 * (count bytes).  amax_ws: device unsigned scratch [groups]; scale_out: device fp32
 * [groups], the dequantisation scales. */
int ufpn_quantize_e4m3(int dtype, const void* x, long long count, int groups, unsigned* amax_ws,
                       void* q, float* scale_out, void* stream);
/* Per-row (output channel) quantisation of fp32 weights [rows][cols] to e4m3 + scales[rows].
 * pack_cin > 0: each row is [pack_cin][3][3] (cols = 9 * pack_cin) and is written tap-major
 * [9][pack_cin], the K order of ufpn_conv3x3_e4m3; pack_cin = 0: lateral [rows][cols]. */
int ufpn_quantize_e4m3_rows(const float* w, int rows, int cols, int pack_cin, void* q,
                            float* scales, void* stream);
/* FP8 lateral 1x1 (+ optional top-down add), NHWC: x e4m3 [N][H][W][Cin] with device scale(s)
 * x_scale[0] (x_scale_per_image = 0) or x_scale[n]; w e4m3 [256][Cin] with scales [256];
 * coarse bf16 [N][Hc][Wc][256] or NULL; out bf16 = acc * (x_scale * w_scales[o]) + bias[o]
 * (+ bilinear(coarse)).  amax_out (device [N], may be NULL): per-image atomicMax of |out|.
 * Same roles as launch_lateral_conv / lateral_conv_kernel (fpn_engine.cu:248-272). */
int ufpn_lateral_conv_e4m3(const void* x, const float* x_scale, int x_scale_per_image,
                           const void* w, const float* w_scales, const float* bias,
                           const void* coarse, void* out, int N, int Cin, int H, int W, int Hc,
                           int Wc, unsigned* amax_out, void* stream);
/* FP8 3x3 pad-1 conv 256 -> 256 (8 x 16 halo tiles; tile_w -1: on CTA pairs, -2 / -3: the
 * map's transposed view, -4 / -5: mixed, as for ufpn_conv3x3), NHWC: x e4m3 [N][H][W][256]
 * with device scale(s) as above; w e4m3 packed [256][9][256] (ufpn_quantize_e4m3_rows with pack_cin =
 * 256) with scales [256]; out (and optional p6 = out[::2, ::2]) bf16; amax_out as above.
 * Same role as launch_output_conv (fpn_engine.cu:315-362). */
int ufpn_conv3x3_e4m3(const void* x, const float* x_scale, int x_scale_per_image, const void* w,
                      const float* w_scales, const float* bias, void* out, void* p6, int N,
                      int H, int W, int tile_w, unsigned* amax_out, void* stream);
/* The same FP8 3x3 (CTA pairs) on a bf16 input x [N][H][W][256] with per-image absmax
 * amax_bits[N] (fp32 bits): each halo is quantised in shared memory to exactly the codes
 * ufpn_quantize_e4m3 (groups = N) would store, and scaled by amax / 448. */
int ufpn_conv3x3_e4m3_from_bf16(const void* x, const unsigned* amax_bits, const void* w,
                                const float* w_scales, const float* bias, void* out, void* p6,
                                int N, int H, int W, void* stream);
/* fpn_engine.cu:191-245 (forward) for an engine configured with dtype UFPN_DTYPE_E4M3
 * (NHWC): inputs C2..C5 e4m3, input_scales[l] = device fp32 per-tensor scale of inputs[l];
 * outputs P2..P5 (and p6) bf16.  Each merged map M_l is quantised per image before its 3x3,
 * so an image's outputs do not depend on the rest of the batch. */
int ufpn_core_forward_e4m3(ufpn_core* core, const void* const* inputs,
                           const float* const* input_scales, void* const* outputs, void* p6,
                           void* stream);

/* ---------------------------------------------------------------- reference C ABI
 * Same names and argument meaning as the reference's exported functions.  NHWC
 * tensors (the layout of the reference's kernels).  These time the launch with
 * events and synchronise, like the originals. */

/* lib/kernels/memory/fast_upsample_kernels.cu:622-647 */
cudaError_t launch_production_upsample_float(const float* input, float* output, int batch_size,
                                             int channels, int in_height, int in_width,
                                             int out_height, int out_width, int align_corners,
                                             float* kernel_time_ms, float* bandwidth_gb_s);
/* fast_upsample_kernels.cu:649-674 (half = IEEE fp16, passed as uint16_t storage) */
cudaError_t launch_production_upsample_half(const void* input, void* output, int batch_size,
                                            int channels, int in_height, int in_width,
                                            int out_height, int out_width, int align_corners,
                                            float* kernel_time_ms, float* bandwidth_gb_s);
/* lib/kernels/memory/upsample_specializations.cu:492-539 */
cudaError_t launch_production_upsample_bfloat16(const void* input, void* output,
                                                int batch_size, int channels, int in_height,
                                                int in_width, int out_height, int out_width,
                                                int align_corners, float* kernel_time_ms,
                                                float* bandwidth_gb_s);

/* lib/kernels/memory/upsample_host_interface.cpp:516-522 */
void* create_upsample_engine(int device_id);
/* upsample_host_interface.cpp:527-531 */
void destroy_upsample_engine(void* engine);
/* upsample_host_interface.cpp:536-585; metrics_out[4] = {ms, GB/s, util, bytes} */
int production_upsample_float(void* engine, const float* input, float* output, int batch_size,
                              int channels, int in_height, int in_width, int out_height,
                              int out_width, float scale_y, float scale_x, int align_corners,
                              float* metrics_out);
/* upsample_host_interface.cpp:590-594 */
void print_upsample_profiling_summary(void* engine);
/* upsample_host_interface.cpp:599-609 (CSV) */
int export_upsample_profiling_data(void* engine, const char* filename);

/* lib/utils/auto_tuner.cu:8-25: the reference's TuningResult carries a std::string;
 * this C-layout version carries a fixed buffer instead. */
typedef struct {
  int tile_w;              /* chosen lateral tile width (128-pixel tiles, height 128 / width) */
  int tile_h;
  int num_ctas;            /* persistent CTAs launched */
  float time_ms;           /* measured */
  float performance_gflops;
  float memory_bandwidth_gb_s;
  char architecture_name[32];
} TuningResult;

/* Tunes the tensor-core lateral 1x1 (bf16 / fp16 dtype code) for one shape on seeded random
 * data: every 128-pixel tile shape (width 8..128) timed on `stream`; the fastest goes to
 * *out and into a process-wide table from which engines configuring a level of that shape
 * (batch, Cin, H, W, dtype) take their lateral tile shape.  No reference counterpart
 * (the stream-taking form of the entry point below). */
int ufpn_autotune_lateral(int dtype, int batch_size, int in_channels, int height, int width,
                          void* stream, TuningResult* out);
/* auto_tuner.cu:328-333: ufpn_autotune_lateral for bf16 on the calling thread's default
 * stream; out_channels must be 256.  Returns a pointer to a per-shape cached result (valid
 * until process exit), NULL on error. */
TuningResult* fpn_auto_tune_lateral_conv(int batch_size, int in_channels, int out_channels,
                                         int height, int width);
/* auto_tuner.cu:335-338 */
void fpn_auto_tune_save_results(const char* filename);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* UNIFIED_FPN_C_H_ */
