// Kernel-level C++ API of the B200 FPN-neck library: one launcher per kernel.
//
// Replaces the reference's kernel interface header
// include/unified_fpn/kernels/interface.h:5-109, which declared the raw
// __global__ templates (lateral_conv_kernel, bilinear_upsample_kernel,
// depthwise_conv_kernel, element_wise_add_kernel, ...).  Here the kernels stay
// private to the library and each is reached through a stream-ordered
// launcher taking plain device pointers; the tensor-core kernels additionally
// take a TcPlan built once per (pointers, shapes) so a launch is replayable
// (and capturable in a CUDA graph).
//   lateral_conv_kernel (:18-29)              -> plan_tc_lateral / launch_fp32_lateral
//   bilinear_upsample_kernel (:31-43)
//     + element_wise_add_kernel (:79-85)      -> launch_upsample_add
//   depthwise_conv_kernel (:45-56)            -> plan_tc_conv3x3 / launch_fp32_conv3x3
//   (no counterpart: P6)                      -> launch_p6
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ufpn {

// Values match FPNDataType in include/unified_fpn/core/types.h (FLOAT32 = 0, FLOAT16 = 1,
// BFLOAT16 = 2, FP8_E4M3 = 6) and the ufpn_dtype codes of the C ABI.
enum class DType : int { F32 = 0, F16 = 1, BF16 = 2, E4M3 = 6 };
enum class Layout : int { NCHW = 0, NHWC = 1 };

inline int dtype_size(DType d) {
  return d == DType::F32 ? 4 : (d == DType::E4M3 ? 1 : 2);
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch options of the launchers that take them.
//   pdl: programmatic dependent launch -- the kernel may be scheduled while the previous
//        kernel of stream s still runs; it sets up, then waits for that kernel's completion
//        before touching memory (griddepcontrol.wait).  Only for a launch whose predecessor
//        in the stream is a kernel.
//   priority: launch priority (cudaLaunchAttributePriority; lower = dispatched first when
//        CTAs of several kernels wait for SMs); 0 keeps the stream's.
struct LaunchOpts {
  bool pdl = false;
  int priority = 0;
};

// ---- bandwidth kernels (simt_kernels.cu)
// A second, per-channel scaled copy of an upsample-add result: out[c] / (scale_a[0] *
// scale_w[c]), same layout (NHWC, 256 channels of a 16-bit type only).
struct MergeScaledCopy {
  void* out = nullptr;
  const float* scale_a = nullptr;  // device scalar
  const float* scale_w = nullptr;  // device [256]
};
// amax_out (optional): amax_out[n] = atomicMax of |out| of image n as fp32 bits (the caller
// zeroes them first).  scaled (optional): also write the scaled copy.
// units_per_block (NHWC, 256 channels of a 16-bit type): 0 = automatic -- one warp per
// 8-pixel row unit (its lateral vectors and its coarse window loaded at once) where the map
// upsamples along x (Wc / W <= 4 / 7), else one warp per pixel with one wave of resident
// blocks, each walking a contiguous run of units; -1 = one warp per pixel, automatic runs;
// > 0 = one warp per pixel, that many units per block.  The same bits either way.
cudaError_t launch_upsample_add(DType dt, const void* coarse, const void* lat, void* out, int N,
                                int C, int Hc, int Wc, int H, int W, int align_corners,
                                Layout layout, cudaStream_t s, unsigned* amax_out = nullptr,
                                const MergeScaledCopy* scaled = nullptr,
                                LaunchOpts opts = LaunchOpts(), int units_per_block = 0);
// Two top-down merges in one launch (NHWC, 256 channels, bf16 / fp16, maps that upsample):
// M4 = L4 + up(M5) into m4 and M3 = L3 + up(M4) in place (l3 may alias m3; l4 must not
// alias m4).  Bitwise the same as launch_upsample_add for M4 then for M3 (the reference's
// top-down loop, fpn_engine.cu:274-313, two iterations).  amax4 / amax3 / m3_scaled: as
// amax_out / scaled of launch_upsample_add, for M4, M3 and M3.
cudaError_t launch_merge_two_levels(DType dt, const void* m5, const void* l4, void* m4,
                                    const void* l3, void* m3, int N, int H5, int W5, int H4,
                                    int W4, int H3, int W3, cudaStream_t s,
                                    unsigned* amax4 = nullptr, unsigned* amax3 = nullptr,
                                    const MergeScaledCopy* m3_scaled = nullptr,
                                    LaunchOpts opts = LaunchOpts());
// ---- e4m3 quantisation (simt_kernels.cu).  scale = amax / 448, q = e4m3_rn_satfinite(
// x * (448 / amax)) (amax == 0: scale = 1, q = 0); amax carried as fp32 bits.
// The n elements form `groups` equal consecutive groups (images), each with its own
// absmax amax_bits[g] and scale scale_out[g].
// atomicMax of max|x| of each group into amax_bits[g] (the caller zeroes them first).
cudaError_t launch_absmax(DType dt, const void* x, long long n, int groups, unsigned* amax_bits,
                          cudaStream_t s);
// Quantisation with the absmax values in amax_bits[groups]; writes the dequantisation
// scales to scale_out[groups] (device, may be null).
cudaError_t launch_quantize_e4m3(DType dt, const void* x, long long n, int groups,
                                 const unsigned* amax_bits, void* q, float* scale_out,
                                 cudaStream_t s, LaunchOpts opts = LaunchOpts());
// Per-row (output channel) quantisation of fp32 weights [rows][cols] -> e4m3 + scales[rows].
// pack_cin > 0: rows are [pack_cin][3][3] and q is written [9][pack_cin] (3x3 K order).
cudaError_t launch_quantize_rows_e4m3(const float* w, int rows, int cols, int pack_cin, void* q,
                                      float* scales, cudaStream_t s);
cudaError_t launch_p6(DType dt, const void* in, void* out, int N, int C, int H, int W,
                      Layout layout, cudaStream_t s);
cudaError_t launch_transpose(DType dt, const void* in, void* out, int N, int C, int HW,
                             bool to_nhwc, cudaStream_t s);
cudaError_t launch_convert_weights(DType dt, const float* in, void* out, long long n,
                                   cudaStream_t s);
cudaError_t launch_pack_conv3x3(DType dt, const float* in, void* out, int Cout, int Cin,
                                cudaStream_t s);
cudaError_t launch_fp32_lateral(const float* x, const float* w, const float* bias,
                                const float* coarse, float* out, int N, int Cin, int Cout, int H,
                                int W, int Hc, int Wc, cudaStream_t s);
cudaError_t launch_fp32_conv3x3(const float* x, const float* w, const float* bias, float* out,
                                int N, int Cin, int Cout, int H, int W, cudaStream_t s,
                                int act = 0, float act_alpha = 0.01f);

// ---- tensor-core kernels (tc_kernels.cu)
// Spatial tiling of the 3x3 implicit GEMM: tile_w * tile_h = 128 output pixels.
struct Conv3x3Tiling {
  int tile_w = 16;
  int tile_h = 8;
  // 3x3 only: 8 x 16 tiles whose (18 x 10) halo is loaded once per 64-channel block
  // and shared by the nine taps (instead of one shifted box per tap).
  bool halo = false;
  // Halo tiles on CTA pairs (tcgen05 cta_group::2, M = 256 per MMA): each CTA streams
  // half of every weight k-block.
  bool pair = false;
  // CTA pairs: a last round with at most half as many units as pairs runs each of its
  // units as two halves over the output channels (N = 128), in half the time (same bits).
  bool tail_halves = true;
  // Halo tiles only: run the conv on the map's transposed view (rows and columns swapped in
  // the tensor maps, taps mirrored), so that a tile covers 16 columns x 8 rows.  Maps whose
  // height is not a multiple of 16 but whose width is (200 x 304) then tile without padded
  // rows.  Each output element accumulates the same k-blocks in the same order: the results
  // are bitwise those of the untransposed conv.  Not with a fused P6 output.
  bool transposed = false;
  // Halo tiles only (not with transposed, not with a fused P6 output): a mixed tiling -- the
  // map's own view for the rows that fill whole 16-row tiles and the transposed view for the
  // remaining strip of at most 8 rows (200 x 304: 12 rows of 38 tiles + 19 strip tiles, 475
  // per image, as the transposed view, but most tiles keep the own view's row-order boxes).
  // The same bits.  CTA pairs need an even number of own-view tiles (N x ceil(W/8) x
  // floor(H/16)).
  bool mixed = false;
};
// The 3x3 default: halo reuse with 8 x 16 tiles.
inline Conv3x3Tiling halo_tiling() {
  Conv3x3Tiling t;
  t.tile_w = 8;
  t.tile_h = 16;
  t.halo = true;
  return t;
}
// Whether an H x W map needs fewer 8 x 16 halo tiles on its transposed view.
inline bool halo_transpose_pays(int H, int W) {
  const long long plain = static_cast<long long>((W + 7) / 8) * ((H + 15) / 16);
  const long long trans = static_cast<long long>((H + 7) / 8) * ((W + 15) / 16);
  return trans < plain;
}
// Whether the mixed tiling applies to N images of H x W (pair: on CTA pairs) and needs fewer
// halo tiles than the map's own view, and no more than the transposed view.
inline bool halo_mixed_pays(int N, int H, int W, bool pair) {
  const int rem = H % 16;
  if (H < 16 || rem == 0 || rem > 8) return false;
  const long long own_rows = static_cast<long long>((W + 7) / 8) * (H / 16);
  if (pair && (own_rows * N) % 2 != 0) return false;
  const long long mixed = own_rows + (W + 15) / 16;
  const long long plain = static_cast<long long>((W + 7) / 8) * ((H + 15) / 16);
  const long long trans = static_cast<long long>((H + 7) / 8) * ((W + 15) / 16);
  return mixed < plain && mixed <= trans;
}
inline Conv3x3Tiling halo_pair_tiling() {
  Conv3x3Tiling t = halo_tiling();
  t.pair = true;
  return t;
}

// Everything one tensor-core launch needs, built on the host once per
// (pointers, shapes) and replayable: the TMA descriptors (A, B, output,
// coarse map) plus the kernel argument block.
struct TcPlan {
  alignas(64) CUtensorMap map_a;
  alignas(64) CUtensorMap map_b;
  alignas(64) CUtensorMap map_out;
  alignas(64) CUtensorMap map_coarse;
  // halo 3x3 with a mixed tiling: input and output maps of the strip's transposed view
  alignas(64) CUtensorMap map_a2;
  alignas(64) CUtensorMap map_out2;
  unsigned char args[256];  // TcGemmArgs, opaque outside tc_kernels.cu
  int mode = 0;  // 0 lateral, 1 conv3x3, 2 conv3x3 halo, 3 halo on CTA pairs, 4 the same + e4m3
                 // quantisation of a bf16 input in shared memory, 5 lateral on CTA pairs,
                 // 6 16-bit lateral with a 16-warp epilogue
  DType dtype = DType::BF16;
  int grid = 0;
  int num_tiles = 0;
};

// Device-resident scale operands of one tensor-core launch.  dtype E4M3 (x and w e4m3,
// coarse / out / p6 bf16): out = acc * (ascale[n or 0] * wscale[o]) + bias[o]; both
// required.  amax_out (any dtype, optional): amax_out[n] = atomicMax of |stored output| of
// image n as fp32 bits, for a following per-image e4m3 quantisation of the output.
struct TcScales {
  const float* ascale = nullptr;  // activation scale(s) (device)
  bool ascale_per_image = false;  // ascale[n] per image, else ascale[0] for the tensor
  const float* wscale = nullptr;  // per-output-channel weight scales [256], 16-byte aligned
  unsigned* amax_out = nullptr;   // [N] (device), zeroed by the caller
  // E4M3 lateral with a coarse map: the coarse map is already divided by (ascale[0] *
  // wscale[c]) per channel (MergeScaledCopy), so the top-down add can run as a tensor-core
  // k-block on the unscaled accumulator.  Otherwise the epilogue adds it from global memory.
  bool coarse_prescaled = false;
  // Lateral output: 0 = store the 16-bit map; 1 = store nothing (amax_out only); 2 = store
  // it quantised to e4m3 per image with the absmax in qamax[n] (out is then e4m3), writing
  // the dequantisation scales to qscale_out[n].  1 then 2 = a two-pass lateral whose
  // quantised output equals quantising the stored 16-bit map.
  int out_mode = 0;
  const unsigned* qamax = nullptr;
  float* qscale_out = nullptr;
  // E4M3 3x3 on CTA pairs only: x is the bf16 map and in_amax[n] its per-image absmax
  // (fp32 bits); the kernel quantises each halo itself (e4m3(x * 448 / amax), the same
  // codes as launch_quantize_e4m3) and scales by amax / 448 (ascale unused).
  const unsigned* in_amax = nullptr;
  // 3x3 only: output activation after the bias, numbered as FPNActivation (0 none, 1 ReLU,
  // 2 LeakyReLU with act_alpha, 3 Swish); P6 is taken from the activated output.
  int act = 0;
  float act_alpha = 0.01f;
};

// Lateral 1x1 (+ optional fused bilinear upsample-add of the coarser merged map).
//   x: NHWC [N][H][W][Cin]; w: [256][Cin] (dtype, K-major); bias fp32 [256];
//   coarse: NHWC [N][Hc][Wc][256] or null; out: NHWC [N][H][W][256].
cudaError_t plan_tc_lateral(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, const void* coarse, void* out, int N, int Cin,
                            int H, int W, int Hc, int Wc, Conv3x3Tiling tiling, int* status,
                            int max_ctas, const TcScales& scales = TcScales());
// 3x3 pad-1 conv, 256 -> 256: x NHWC [N][H][W][256]; w: [256][9][256]; out NHWC;
// p6 (optional) NHWC [N][ceil(H/2)][ceil(W/2)][256].  E4M3 requires the halo tiling.
// The 16-bit lateral on CTA pairs (lateral_pair.cuh): each CTA keeps half of the weights
// resident (Cin <= 256) and adds the top-down taps from a staged coarse box in its epilogue
// (the box must fit 64 coarse pixels).  cudaErrorNotSupported when those do not hold.
cudaError_t plan_tc_lateral_pair(TcPlan& plan, DType dt, const void* x, const void* w,
                                 const float* bias, const void* coarse, void* out, int N,
                                 int Cin, int H, int W, int Hc, int Wc, Conv3x3Tiling tiling,
                                 int* status, int max_ctas = 0);
// claim (CTA-pair tilings only; else ignored): two device ints, zero before the first launch,
// through which the pairs claim their work items at run time (the launch leaves them zero
// again); null = static round robin.  At most one launch in flight per claim pair.
cudaError_t plan_tc_conv3x3(TcPlan& plan, DType dt, const void* x, const void* w,
                            const float* bias, void* out, void* p6, int N, int H, int W,
                            Conv3x3Tiling tiling, int* status, int max_ctas,
                            const TcScales& scales = TcScales(), int* claim = nullptr);
// Precomputed bilinear-weight table of the lateral's tensor-core top-down add (one 16 KB
// entry per tile position of an H x W map upsampled from Hc x Wc with tiling t; the same
// for every image).  Bytes needed (0 when that lateral adds the taps in its epilogue),
// building it (dt: the lateral's input dtype), and attaching it to a lateral plan (false
// if the plan has no tensor-core top-down add).  A plan without a table builds its weights
// per tile in the producer warp.
size_t tc_wb_table_bytes(int H, int W, int Hc, int Wc, Conv3x3Tiling t);
cudaError_t tc_build_wb_table(DType dt, int H, int W, int Hc, int Wc, Conv3x3Tiling t,
                              void* table, cudaStream_t s);
bool tc_attach_wb_table(TcPlan& plan, const void* table);
// 16-bit lateral plans: 16 epilogue warps (64 output channels each) and 3 operand stages
// instead of 8 warps and 4 stages; same results bitwise.  Returns false (plan unchanged)
// for other plans.
bool tc_use_wide_epilogue(TcPlan& plan);
// Tiled NHWC tensor map with 128-byte swizzle: dims (C, W, H, N), pixel stride pix_stride
// elements (>= C), box (one 128-byte row of channels, bw, bh, 1).
cudaError_t encode_nhwc_map(CUtensorMap* map, DType dt, const void* base, int N, int H, int W,
                            int C, int pix_stride, int bw, int bh);
// 16-bit lateral plans only: store the output into channels [0, C) of a map whose pixels are
// pix_stride elements apart (out = that channel slice's first element).  Used to write the
// 256-channel slices of a wider tensor (the input gradient of a Cin > 256 lateral).
cudaError_t tc_set_output_view(TcPlan& plan, void* out, int C, int pix_stride);
// Row-major [rows][cols] map with a (box_cols, box_rows) box whose inner extent is one
// 128-byte row (128-byte swizzle): row tiles staged in shared memory, stored by TMA.
cudaError_t encode_rows_map(CUtensorMap* map, DType dt, const void* base, int cols, long long rows,
                            int box_cols, int box_rows);
// One launch of a 16-bit lateral plan (no top-down add, plain output) for `slices` output
// channel slices of 256: weights w [slices * 256][K] row-major (K = the plan's input
// channels), bias [slices * 256], output NHWC with C channels (256 (slices - 1) < C <= 256
// slices) at the plan's geometry.  Slice s writes channels [256 s, min(C, 256 s + 256)).
cudaError_t tc_set_channel_slices(TcPlan& plan, const void* w, int K, int slices, void* out, int C);
// Tiling with the fewest padded pixels for an H x W map (ties: 16 wide).
Conv3x3Tiling default_tiling(int H, int W);

// Peaks the profiled forward reports its utilisation against (engine.cu): dense 16-bit
// tensor FLOP/s, fp32 FLOP/s, HBM bytes/s; values <= 0 keep the current one.
void set_device_peaks(double tensor_flops, double fp32_flops, double hbm_bytes);
void get_device_peaks(double* out3);

// ---- whole-neck persistent kernel (one launch for all 4 laterals and 4 3x3 convs)
struct NeckLevel {
  const void* x;        // C_l, NHWC [N][H][W][Cin]
  const void* lat_w;    // [256][Cin] in the compute dtype
  const float* lat_b;   // [256]
  const void* conv_w;   // [256][9][256] in the compute dtype
  const float* conv_b;  // [256]
  void* merged;         // M_l workspace, NHWC [N][H][W][256]
  void* out;            // P_l, NHWC [N][H][W][256]
  int Cin, H, W;
  Conv3x3Tiling lat_tiling, conv_tiling;
  int act = 0;  // the level's 3x3: output activation as TcScales::act, with act_alpha
  float act_alpha = 0.01f;
  // Split-K lateral of this level (NeckJobSpec::ksplit > 1): fp32 partials
  // (neck_split_part_bytes) and one arrival counter per lateral tile (neck_lateral_tiles ints,
  // zero before the first launch; every launch leaves them zero again).
  float* split_part = nullptr;
  int* split_sem = nullptr;
};
// Lateral tiles of a level's map (one per 128-pixel tile and image).
int neck_lateral_tiles(int N, int H, int W, Conv3x3Tiling lat_tiling);
// Bytes of the fp32 partials of a split-K lateral: ksplit x 128 x 256 x 4 per tile.
size_t neck_split_part_bytes(int N, int H, int W, Conv3x3Tiling lat_tiling, int ksplit);
struct NeckPlan {
  alignas(64) unsigned char params[6144];  // NeckParams, opaque outside tc_kernels.cu
  DType dtype = DType::BF16;
  int grid = 0;
  int total_tiles = 0;
};
// levels[0..3] = P2..P5; p6 (NHWC, optional) = P5[::2, ::2].  sched: 8 device ints,
// zero before the first launch (each launch leaves them zero again).
// trace (optional, 8 device u64): [0] = ~0 and the rest 0 before the launch; receives the
// launch's timeline in globaltimer ns (see NeckParams in neck_kernel.cuh).
cudaError_t plan_neck(NeckPlan& plan, DType dt, int N, const NeckLevel* levels, void* p6,
                      int* sched, int* status, int max_ctas,
                      unsigned long long* trace = nullptr);
// General form: any subset of the 8 jobs, in dispatch order (a job may only depend on
// jobs before it).  mode 0 = lateral of `level` (coarse = 1: fused top-down add of
// level+1's merged map), mode 1 = 3x3 of `level`.  A job waits on a level only if that
// level's lateral runs in the same launch; otherwise its input must be complete before.
// ksplit (laterals): 1, 2 or 4 units per tile over K, each at least one k-block long; > 1
// needs the level's split_part / split_sem workspace.  nsplit (laterals without a top-down
// add, ksplit 1): 1, or 2 units per tile over the output channels (128 each).
struct NeckJobSpec {
  int mode;
  int level;
  int coarse;
  int ksplit = 1;
  int nsplit = 1;
};
cudaError_t plan_neck_jobs(NeckPlan& plan, DType dt, int N, const NeckLevel* levels, void* p6,
                           const NeckJobSpec* specs, int num_specs, int* sched, int* status,
                           int max_ctas, unsigned long long* trace = nullptr);
cudaError_t launch_neck(const NeckPlan& plan, cudaStream_t s, LaunchOpts opts = LaunchOpts());
// The raw laterals (no top-down add) of levels[0..count) in one launch on CTA pairs (two
// tiles of a level per tcgen05 cta_group::2 MMA stream, each CTA streaming half of every
// weight k-block), pair units dealt on the host longest first.  nsplit (optional, per
// entry, 1 or 2): 2 runs that level's units as two N = 128 halves each.  Bitwise the same
// outputs as plan_neck_jobs with those lateral jobs.  cudaErrorNotSupported: not 16-bit, or
// more work items than a plan holds (2048; 4095 pair units per level).
struct LateralGroupPlan {
  alignas(64) unsigned char params[8192];  // opaque outside tc_kernels.cu
  DType dtype = DType::BF16;
  int grid = 0;
};
cudaError_t plan_lateral_group_pair(LateralGroupPlan& plan, DType dt, int N,
                                    const NeckLevel* levels, const int* which, int count,
                                    int* status, int max_ctas, const int* nsplit = nullptr);
cudaError_t launch_lateral_group_pair(const LateralGroupPlan& plan, cudaStream_t s,
                                      LaunchOpts opts = LaunchOpts());
// Self-test of the bounded waits: in a planned launch, the 3x3 job of `level` waits for one
// more lateral tile than its level has (a count nothing reaches) with a wait limit of
// wait_ns; its tiles then give up, record kDevTimeoutDependency (0x105) in the status word
// and the kernel ends normally (copies drained, TMEM freed, schedule counters reset).
cudaError_t neck_plan_stall_dependency(NeckPlan& plan, int level, unsigned long long wait_ns);
cudaError_t launch_tc(const TcPlan& plan, cudaStream_t s, LaunchOpts opts = LaunchOpts());

// ---- backward pass (backward.cu).  Reference: src/training/backward/lateral_conv_backward.cu
// :7-143 and upsample_backward.cu:4-80; here the exact adjoints of the forward, deterministic.
// Weight gradient dW[o][c][t] = sum_p dY[p][o] X[p + shift(t)][c] (fp32, [256][Cin][taps];
// taps 1 = the 1x1 lateral, 9 = the pad-1 3x3 with shift(t) = (t / 3 - 1, t % 3 - 1)) of
// NHWC dY [N][H][W][256] and X [N][H][W][Cin] (16-bit): a tensor-core GEMM over pixels with
// fp32 split-K partials in `workspace` (dw_gemm_workspace_bytes) added in a fixed order.
size_t dw_gemm_workspace_bytes(int N, int H, int W, int Cin, int taps);
// With grad_b (nullable), grad_b[o] = sum_p dY[p][o] comes out of the same launch: the idle
// epilogue warps of the channel-block-0 CTAs sum dY (fixed-order partials, reduced with dW).
cudaError_t launch_dw_gemm(DType dt, const void* grad_out, const void* x, int N, int H, int W,
                           int Cin, int taps, float* grad_w, float* grad_b, float* workspace,
                           size_t ws_bytes, int* status, cudaStream_t s);
// Per-step weight layouts of the training path from fp32 master weights, all in one launch.
// kind 0: lateral [256][cin] -> 16-bit [256][cin]; 1: the same transposed, [cblk * 256][256]
// (cblk = ceil(cin / 256), zero rows from cin); 2: 3x3 [256 o][256 c][3][3] -> packed
// [256 o][9 t][256 c]; 3: the same flipped for the input gradient, [256 c][9 t][256 o] holding
// w[o][c][8 - t].  Rounding as launch_pack_conv3x3 (to nearest even).
struct WeightPrepJob {
  int kind = 0;
  int cin = 0;
  const float* in = nullptr;
  void* out = nullptr;
};
cudaError_t launch_prepare_weights(DType dt, const WeightPrepJob* jobs, int num_jobs,
                                   cudaStream_t s);
// out[c] = sum over the pixels of g[p][c] (fp32; per block, then in a fixed order).
size_t colsum_workspace_bytes(long long pixels, int C);
cudaError_t launch_colsum(DType dt, const void* g, long long pixels, int C, float* out,
                          float* workspace, size_t ws_bytes, cudaStream_t s);
// Adjoint of launch_upsample_add's bilinear (NHWC, align_corners = false):
// out = base (or 0) + up^T(grad_fine), out and base [N][Hc][Wc][C].
cudaError_t launch_upsample_adjoint(DType dt, const void* grad_fine, const void* base, void* out,
                                    int N, int C, int Hc, int Wc, int H, int W, cudaStream_t s);
// Adjoint of P6 = P5[::2, ::2]: grad_p5 at even pixels += grad_p6 (NHWC, in place).
cudaError_t launch_p6_adjoint(DType dt, const void* grad_p6, void* grad_p5, int N, int C, int H5,
                              int W5, cudaStream_t s);
// wt[c][r] = w[r][c] for a rows x cols matrix; rows cols..out_rows-1 of wt are zeroed.
cudaError_t launch_transpose_weights(DType dt, const void* w, void* wt, int rows, int cols,
                                     int out_rows, cudaStream_t s);
// Packed 3x3 weights [256 o][9 t][256 c] -> [256 c][9 t'][256 o] with t' = 8 - t: the weights
// of the 3x3 that computes the input gradient.
cudaError_t launch_flip_conv3x3_weights(DType dt, const void* w_packed, void* w_flipped,
                                        cudaStream_t s);

// Number of SMs on the current device (cached).
int sm_count();
// L2 size of the current device in bytes (cached per device).
long long l2_bytes();

}  // namespace ufpn
