// UnifiedFPNCore: the FPN neck engine.
//
// Reference: lib/core/fpn_engine.cu:10-416 (class UnifiedFPNCore).  The
// reference ran a 4-level lateral loop then a top-down loop on four private
// streams with no ordering between level l+1's output and level l's upsample
// (fpn_engine.cu:223-235) and a blocking host sync every call (:239-241).
// This engine instead enqueues, on the caller's stream:
//
//   main stream:  lat5 -> lat4 -> lat3 -> lat2          (each lateral epilogue
//                  |       |       |       |             reads M_{l+1} written
//   side stream:  3x3_5   3x3_4   3x3_3   3x3_2 (+P6)   by the previous one)
//
// i.e. the top-down chain stays on one stream (true data dependence) while each
// level's 3x3 output conv runs on a side stream as soon as its merged map M_l
// exists, overlapping the next lateral.  The whole schedule is captured once
// per (pointer set) into a CUDA graph on a private stream and replayed with a
// single cudaGraphLaunch on the caller's stream.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <mutex>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "kernels.h"
#include "unified_fpn/core/engine.h"

using ufpn::Conv3x3Tiling;
using ufpn::DType;
using ufpn::Layout;
using ufpn::TcPlan;

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

DType to_dtype(FPNDataType t) {
  switch (t) {
    case FPNDataType::FLOAT32:
      return DType::F32;
    case FPNDataType::FLOAT16:
      return DType::F16;
    case FPNDataType::BFLOAT16:
      return DType::BF16;
    case FPNDataType::FP8_E4M3:
      return DType::E4M3;
    default:
      FPN_THROW("unsupported dtype: the neck runs in FLOAT32, FLOAT16, BFLOAT16 or FP8_E4M3");
  }
}

// 3x3 tiling from its tuning code: -1 = halo tiles on CTA pairs (the default for large
// maps), 0 = halo reuse with 8 x 16 tiles on single CTAs, 8..128 = plain tiles of that width
// (one shifted box per tap).
constexpr int kDefaultTilingCode = -1;
int tiling_code(const Conv3x3Tiling& t) { return t.pair ? -1 : (t.halo ? 0 : t.tile_w); }
Conv3x3Tiling tiling_from_code(int tw) {
  if (tw == -1) return ufpn::halo_pair_tiling();
  if (tw <= 0) return ufpn::halo_tiling();
  Conv3x3Tiling t;
  t.tile_w = tw;
  t.tile_h = 128 / tw;
  return t;
}

}  // namespace

namespace ufpn {
// Peaks the profiled forward's utilisation figures are reported against (set_device_peaks):
// dense 16-bit tensor FLOP/s (e4m3 counts twice that), fp32 CUDA-core FLOP/s, HBM bytes/s.
// Nominal B200 figures until a caller sets measured ones.
namespace {
std::atomic<double> g_peak_tensor{2.25e15}, g_peak_fp32{8.0e13}, g_peak_hbm{8.0e12};
}
void set_device_peaks(double tensor_flops, double fp32_flops, double hbm_bytes) {
  if (tensor_flops > 0) g_peak_tensor.store(tensor_flops);
  if (fp32_flops > 0) g_peak_fp32.store(fp32_flops);
  if (hbm_bytes > 0) g_peak_hbm.store(hbm_bytes);
}
void get_device_peaks(double* out3) {
  out3[0] = g_peak_tensor.load();
  out3[1] = g_peak_fp32.load();
  out3[2] = g_peak_hbm.load();
}

// Lateral tile shapes chosen by the standalone lateral tuner (fpn_auto_tune_lateral_conv),
// process-wide, keyed by (dtype, batch, Cin, H, W); an engine configuring that geometry
// starts from them (its own whole-neck tuning, when present, takes precedence).
namespace {
std::mutex g_lat_mu;
std::map<std::string, int> g_lat_tuned;  // key -> tile width
std::string lat_key(DType dt, int N, int cin, int H, int W) {
  std::ostringstream k;
  k << static_cast<int>(dt) << "/" << N << "x" << cin << "x" << H << "x" << W;
  return k.str();
}
}  // namespace
void record_lateral_tiling(DType dt, int N, int cin, int H, int W, int tile_w) {
  std::lock_guard<std::mutex> lk(g_lat_mu);
  g_lat_tuned[lat_key(dt, N, cin, H, W)] = tile_w;
}
bool lateral_tiling_for(DType dt, int N, int cin, int H, int W, Conv3x3Tiling* t) {
  std::lock_guard<std::mutex> lk(g_lat_mu);
  auto it = g_lat_tuned.find(lat_key(dt, N, cin, H, W));
  if (it == g_lat_tuned.end()) return false;
  t->tile_w = it->second;
  t->tile_h = 128 / it->second;
  t->halo = t->pair = false;
  return true;
}
}  // namespace ufpn

struct UnifiedFPNCore::Impl {
  int device = 0;
  size_t workspace_cap = 0;
  int cout = 256;
  DType dtype = DType::F32;
  Layout layout = Layout::NCHW;
  int batch = 0;
  int cin[4] = {};
  int H[4] = {};
  int W[4] = {};
  bool configured = false;
  int w_cin[4] = {};  // Cin the weight buffers were allocated for
  bool weights_allocated = false;
  bool weights_set[4] = {};
  float* lat_w32[4] = {};
  float* lat_b[4] = {};
  float* out_w32[4] = {};
  float* out_b[4] = {};
  void* lat_wp[4] = {};
  void* out_wp[4] = {};
  float* lat_ws[4] = {};  // e4m3: per-output-channel weight scales
  float* out_ws[4] = {};
  DType packed_dtype = DType::F32;
  void* merged[4] = {};   // M_l in the compute dtype (bf16 for e4m3 inputs)
  void* qmerged[4] = {};  // e4m3: M_l quantised per image (input of the 3x3)
  void* m3_scaled = nullptr;  // e4m3: M3 / (scale(C2) * lateral-P2 weight scale), per channel
  // Raw P4 lateral L4 when the P4 and P3 merges run as one launch (which reads L4 around
  // each tile while it writes M4, so L4 cannot be merged in place); null: merge per level.
  void* lat4_raw = nullptr;
  void* wb_table = nullptr;   // P2 lateral's precomputed top-down (bilinear) weights
  // Split-K grouped laterals: fp32 partials per level and per-tile arrival counters (one
  // allocation: counters first), sized for split_alloc[l] units per tile.
  float* split_part[4] = {};
  int* split_sem = nullptr;
  int split_sem_off[4] = {};
  int split_alloc[4] = {1, 1, 1, 1};
  Conv3x3Tiling split_tiling[4];  // lateral tilings the split workspace was sized for
  size_t split_bytes = 0;
  const float* in_scale[4] = {};  // e4m3: scales of the current forward's inputs
  unsigned* fp8_amax = nullptr;   // e4m3: [4][N] per-image absmax of M_l (fp32 bits)
  float* fp8_scale = nullptr;     // e4m3: [4][N] per-image dequantisation scale of M_l
  void* nhwc_in[4] = {};
  void* nhwc_out[5] = {};
  size_t workspace_bytes = 0;
  size_t weight_bytes = 0;
  int* d_status = nullptr;
  int* d_sched = nullptr;  // neck-kernel tile counter + level completion counters
  unsigned long long* d_trace = nullptr;  // neck-kernel timeline (same allocation)
  bool trace_next = false;
  unsigned long long last_trace[8] = {};
  cudaStream_t side = nullptr;
  cudaStream_t p2_side = nullptr;  // the P2 3x3s of an image-pipelined P2 level
  static constexpr int kMaxP2Parts = 8;
  cudaEvent_t ev_p2[kMaxP2Parts] = {};
  cudaEvent_t ev_p2_join = nullptr;
  cudaStream_t lat_side[2] = {};  // e4m3: the P4 and P3 laterals beside the P5 one
  cudaEvent_t ev_lat_done[2] = {};
  cudaStream_t capture = nullptr;
  cudaStream_t setup = nullptr;
  cudaEvent_t ev_fork = nullptr;
  cudaEvent_t ev_lat[4] = {};
  cudaEvent_t ev_join = nullptr;
  cudaEvent_t ev_join_lat[2] = {};  // joins of the P4 / P3 3x3 streams
  int chain_priority_value = 0;     // greatest launch priority of the device
  cudaEvent_t prof[10] = {};
  FPNKernelConfig cfg;
  Conv3x3Tiling tiling[4];
  bool tiling_tuned[4] = {};
  Conv3x3Tiling lat_tiling[4];  // lateral tile shape per level (tuned or the least padding)
  int wb_tile_w = 0;            // lateral tile width the Wb table was built for
  bool p2_pair = false;         // 16-bit P2 lateral on CTA pairs (resident weight halves)
  int merge_units = 0;  // merge kernel form / units per block (launch_upsample_add)
  int p2_lateral_ctas = 0;      // CTAs of the 16-bit P2 lateral (0: one per SM)
  int conv_ctas[4] = {0, 0, 0, 0};  // CTAs of each level's 3x3 (0: one per SM)
  bool p2_lateral_dynamic = false;  // 16-bit P2 lateral as a one-job neck launch (tile claims)
  // Options set through UnifiedFPNCore::set_option, by name, re-applied after every
  // (re)configuration so that a choice made before the first forward -- or kept across a new
  // geometry -- is not replaced by the geometry's defaults.  autotune() drops the entries of
  // the knobs it tunes (its choice replaces them).
  std::map<std::string, int> explicit_options;
  void apply_explicit_options();
  bool profiling = false;
  FPNPerformanceMetrics metrics{};
  struct GraphEntry {
    const void* in[4];
    const float* scale[4];
    void* out[4];
    void* p6;
    cudaGraphExec_t exec;
    int launches;
  };
  std::vector<GraphEntry> graphs;
  // Pointer sets seen once and not captured (capture happens on a set's second use).
  struct SeenKey {
    const void* in[4];
    const float* scale[4];
    void* out[4];
    void* p6;
  };
  std::vector<SeenKey> seen_once;
  long long stat_captures = 0, stat_replays = 0, stat_direct = 0;
  std::map<std::string, std::pair<int, float>> tuning_db;  // v1: key -> (3x3 tile_w, ms)
  // v2 (whole-neck tuning): geometry key -> knob values and the tuned forward time
  std::map<std::string, std::pair<std::map<std::string, int>, float>> tuning_db2;

  ~Impl() { release_all(); }

  void release_graphs() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.exec);
    graphs.clear();
    seen_once.clear();
  }
  void free_workspace() {
    for (int l = 0; l < 4; ++l) {
      cudaFree(merged[l]);
      cudaFree(qmerged[l]);
      cudaFree(nhwc_in[l]);
      merged[l] = qmerged[l] = nhwc_in[l] = nullptr;
    }
    for (int l = 0; l < 5; ++l) {
      cudaFree(nhwc_out[l]);
      nhwc_out[l] = nullptr;
    }
    cudaFree(fp8_amax);  // one allocation with fp8_scale
    fp8_amax = nullptr;
    fp8_scale = nullptr;
    cudaFree(m3_scaled);
    m3_scaled = nullptr;
    cudaFree(lat4_raw);
    lat4_raw = nullptr;
    cudaFree(wb_table);
    wb_table = nullptr;
    free_split();
    workspace_bytes = 0;
  }
  void free_split() {
    cudaFree(split_sem);  // one allocation with the partials
    split_sem = nullptr;
    for (int l = 0; l < 4; ++l) {
      split_part[l] = nullptr;
      split_alloc[l] = 1;
    }
    workspace_bytes -= split_bytes;
    split_bytes = 0;
  }
  // The P2 lateral's top-down weights (tensor-core k-block) depend only on the geometry and
  // the lateral's tile shape: built at configuration and again when the tile shape changes.
  size_t wb_bytes = 0;
  void build_wb_table() {
    cudaFree(wb_table);
    wb_table = nullptr;
    workspace_bytes -= wb_bytes;
    wb_bytes = 0;
    wb_tile_w = 0;
    if (!configured || !tensor_core_path()) return;
    const size_t tb = ufpn::tc_wb_table_bytes(H[0], W[0], H[1], W[1], lat_tiling[0]);
    wb_tile_w = lat_tiling[0].tile_w;
    if (tb == 0) return;  // taps beyond one box: the lateral reads them from global memory
    check(cudaMalloc(&wb_table, tb), "workspace");
    check(ufpn::tc_build_wb_table(dtype, H[0], W[0], H[1], W[1], lat_tiling[0], wb_table, setup),
          "build bilinear weight table");
    check(cudaStreamSynchronize(setup), "build bilinear weight table");
    wb_bytes = tb;
    workspace_bytes += tb;
  }
  // Buffers the current knob settings need, allocated before any capture.
  void ensure_plan_buffers() {
    if (!tensor_core_path()) return;
    if (wb_tile_w != lat_tiling[0].tile_w) {
      release_graphs();
      build_wb_table();
    }
    if (cfg.merge_two_levels && !lat4_raw && H[3] <= H[2] && W[3] <= W[2] && H[2] <= H[1] &&
        W[2] <= W[1]) {
      release_graphs();
      const size_t bytes = static_cast<size_t>(batch) * H[2] * W[2] * cout * 2;
      check(cudaMalloc(&lat4_raw, bytes), "workspace");
      workspace_bytes += bytes;
    }
    ensure_split_workspace();
  }
  // Key of this geometry in the whole-neck tuning cache: dtype, layout, batch, every level's
  // shape, the SM count and the driver version.
  std::string geometry_key() const {
    std::ostringstream k;
    int drv = 0;
    cudaDriverGetVersion(&drv);
    k << "neck/dt" << static_cast<int>(dtype) << "/lay" << static_cast<int>(layout) << "/b" << batch;
    for (int l = 0; l < 4; ++l) k << "/" << cin[l] << "x" << H[l] << "x" << W[l];
    k << "/sm" << ufpn::sm_count() << "/drv" << drv;
    return k.str();
  }
  void apply_tuning_db2();  // (defined with the option table)

  // Units per tile of level l's lateral in the grouped launch (1 when the level does not
  // split or its K loop is too short for the configured split).
  int lateral_ksplit(int l) const {
    if (l < 1 || l > 3) return 1;
    const int ks = cfg.lateral_ksplit[l];
    const int kbs = (cin[l] + 63) / 64;
    return (ks == 2 || ks == 4) && kbs >= ks ? ks : 1;
  }
  // Allocates (before any capture) the split-K workspace the current configuration needs.
  void ensure_split_workspace() {
    if (!tensor_core_path() || dtype == DType::E4M3) return;
    bool same = split_sem != nullptr || (lateral_ksplit(1) == 1 && lateral_ksplit(2) == 1 &&
                                         lateral_ksplit(3) == 1);
    for (int l = 1; l < 4 && same && split_sem; ++l)
      same = split_alloc[l] == lateral_ksplit(l) && split_tiling[l].tile_w == lat_tiling[l].tile_w;
    if (same) return;
    release_graphs();
    free_split();
    size_t sem_ints = 0, part_bytes = 0;
    size_t off[4] = {};
    for (int l = 1; l < 4; ++l) {
      const ufpn::Conv3x3Tiling t = lat_tiling[l];
      split_sem_off[l] = static_cast<int>(sem_ints);
      sem_ints += static_cast<size_t>(ufpn::neck_lateral_tiles(batch, H[l], W[l], t));
      off[l] = part_bytes;
      part_bytes += ufpn::neck_split_part_bytes(batch, H[l], W[l], t, lateral_ksplit(l));
    }
    const size_t sem_bytes = (sem_ints * sizeof(int) + 255) / 256 * 256;
    void* p = nullptr;
    check(cudaMalloc(&p, sem_bytes + part_bytes), "workspace");
    check(cudaMemset(p, 0, sem_bytes), "workspace");
    split_sem = static_cast<int*>(p);
    for (int l = 1; l < 4; ++l) {
      split_alloc[l] = lateral_ksplit(l);
      split_tiling[l] = lat_tiling[l];
      split_part[l] = split_alloc[l] > 1
                          ? reinterpret_cast<float*>(static_cast<char*>(p) + sem_bytes + off[l])
                          : nullptr;
    }
    split_bytes = sem_bytes + part_bytes;
    workspace_bytes += split_bytes;
  }
  void free_weights() {
    for (int l = 0; l < 4; ++l) {
      cudaFree(lat_w32[l]);
      cudaFree(lat_b[l]);
      cudaFree(out_w32[l]);
      cudaFree(out_b[l]);
      cudaFree(lat_wp[l]);
      cudaFree(out_wp[l]);
      cudaFree(lat_ws[l]);
      cudaFree(out_ws[l]);
      lat_w32[l] = lat_b[l] = out_w32[l] = out_b[l] = lat_ws[l] = out_ws[l] = nullptr;
      lat_wp[l] = out_wp[l] = nullptr;
      weights_set[l] = false;
    }
    weights_allocated = false;
    weight_bytes = 0;
  }
  void release_all() {
    DeviceGuard g(device);
    release_graphs();
    free_workspace();
    free_weights();
    cudaFree(d_status);
    d_status = nullptr;
    d_sched = nullptr;  // same allocation
    if (side) cudaStreamDestroy(side);
    if (p2_side) cudaStreamDestroy(p2_side);
    p2_side = nullptr;
    for (auto& e : ev_p2)
      if (e) cudaEventDestroy(e);
    if (ev_p2_join) cudaEventDestroy(ev_p2_join);
    ev_p2_join = nullptr;
    if (capture) cudaStreamDestroy(capture);
    if (setup) cudaStreamDestroy(setup);
    side = capture = setup = nullptr;
    for (int i = 0; i < 2; ++i) {
      if (lat_side[i]) cudaStreamDestroy(lat_side[i]);
      if (ev_lat_done[i]) cudaEventDestroy(ev_lat_done[i]);
      lat_side[i] = nullptr;
      ev_lat_done[i] = nullptr;
    }
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    for (auto& e : ev_join_lat)
      if (e) cudaEventDestroy(e);
    for (auto& e : ev_lat)
      if (e) cudaEventDestroy(e);
    for (auto& e : prof)
      if (e) cudaEventDestroy(e);
  }

  // Stage-timing event of the profiled forward.  That forward is captured into a graph, and
  // only an external event record (not the dependency-only node a plain record becomes
  // during capture) can be timed after the replay.
  void prof_record(int k, cudaStream_t st) {
    cudaEventRecordWithFlags(prof[k], st, cudaEventRecordExternal);
  }

  bool tensor_core_path() const { return dtype != DType::F32 && cfg.use_tensor_cores; }
  int act() const { return static_cast<int>(cfg.activation); }
  ufpn::TcScales act_scales() const {
    ufpn::TcScales sc;
    sc.act = act();
    sc.act_alpha = cfg.activation_alpha;
    return sc;
  }

  std::string tuning_key(int l) const {
    std::ostringstream k;
    k << "conv3x3/" << static_cast<int>(dtype) << "/" << batch << "x" << H[l] << "x" << W[l]
      << "/sm" << ufpn::sm_count();
    return k.str();
  }

  Conv3x3Tiling tiling_for(int l) const {
    if (cfg.tile_size > 0 && 128 % cfg.tile_size == 0 && cfg.tile_size <= 128) {
      Conv3x3Tiling t;
      t.tile_w = cfg.tile_size;
      t.tile_h = 128 / cfg.tile_size;
      return t;
    }
    Conv3x3Tiling t = tiling[l];
    t.tail_halves = cfg.conv3x3_tail_halves;
    return t;
  }
  // Claim counters of level l's 3x3 (used when it runs on CTA pairs): two ints of the
  // schedule area per level, zero between launches (device_status(true) clears them after
  // an abort).
  int* conv_claim(int l) const { return cfg.conv3x3_dynamic ? d_sched + 32 + 2 * l : nullptr; }
  // The 3x3 tiling of level l launched on its own: halo tiles on the map's transposed view
  // where that needs fewer tiles (conv3x3_transpose), except with the fused P6 output.
  // (conv3x3_mixed: the own view for the whole 16-row tile rows and the transposed view for
  // the remaining strip, where that needs no more tiles than the transposed view.)
  Conv3x3Tiling conv_tiling_for(int l, Conv3x3Tiling t, bool with_p6, int images) const {
    t.transposed = false;
    t.mixed = false;
    if (!t.halo || with_p6 || !cfg.conv3x3_transpose) return t;
    if (cfg.conv3x3_mixed && ufpn::halo_mixed_pays(images, H[l], W[l], t.pair))
      t.mixed = true;
    else
      t.transposed = ufpn::halo_transpose_pays(H[l], W[l]);
    return t;
  }

  void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) FPN_THROW(std::string(what) + ": " + cudaGetErrorString(e));
  }

  void ensure_weight_packing() {
    if (!tensor_core_path() || packed_dtype == dtype) return;
    for (int l = 0; l < 4; ++l) {
      cudaFree(lat_wp[l]);
      cudaFree(out_wp[l]);
      cudaFree(lat_ws[l]);
      cudaFree(out_ws[l]);
      lat_wp[l] = out_wp[l] = nullptr;
      lat_ws[l] = out_ws[l] = nullptr;
      const size_t esz = ufpn::dtype_size(dtype);
      check(cudaMalloc(&lat_wp[l], static_cast<size_t>(cout) * w_cin[l] * esz), "cudaMalloc");
      check(cudaMalloc(&out_wp[l], static_cast<size_t>(cout) * cout * 9 * esz), "cudaMalloc");
      if (dtype == DType::E4M3) {
        check(cudaMalloc(&lat_ws[l], cout * sizeof(float)), "cudaMalloc");
        check(cudaMalloc(&out_ws[l], cout * sizeof(float)), "cudaMalloc");
      }
      if (weights_set[l]) pack_level(l);
    }
    packed_dtype = dtype;
  }

  void pack_level(int l) {
    if (!tensor_core_path()) return;
    if (dtype == DType::E4M3) {
      // Per output channel: scale = absmax / 448, e4m3 codes; 3x3 packed tap-major.
      check(ufpn::launch_quantize_rows_e4m3(lat_w32[l], cout, w_cin[l], 0, lat_wp[l], lat_ws[l],
                                            setup),
            "quantise lateral weights");
      check(ufpn::launch_quantize_rows_e4m3(out_w32[l], cout, cout * 9, cout, out_wp[l],
                                            out_ws[l], setup),
            "quantise 3x3 weights");
      check(cudaStreamSynchronize(setup), "weight quantisation");
      return;
    }
    check(ufpn::launch_convert_weights(dtype, lat_w32[l], lat_wp[l],
                                       static_cast<long long>(cout) * w_cin[l], setup),
          "pack lateral weights");
    check(ufpn::launch_pack_conv3x3(dtype, out_w32[l], out_wp[l], cout, cout, setup),
          "pack 3x3 weights");
    check(cudaStreamSynchronize(setup), "weight packing");
  }

  // ------------------------------------------------------------ the schedule
  // Enqueues the whole neck on `main`; returns the number of kernels launched.
  int enqueue(const void* const* in, void* const* out, void* p6, cudaStream_t main,
              bool prof_events) {
    int launches = 0;
    auto ok = [&](cudaError_t e, const char* what) {
      check(e, what);
      ++launches;
    };
    if (!tensor_core_path()) {
      // fp32 CUDA-core path, NCHW, all on one stream.
      if (prof_events) prof_record(0, main);
      for (int l = 3; l >= 0; --l) {
        const float* coarse = l < 3 ? static_cast<const float*>(merged[l + 1]) : nullptr;
        ok(ufpn::launch_fp32_lateral(static_cast<const float*>(in[l]), lat_w32[l], lat_b[l],
                                     coarse, static_cast<float*>(merged[l]), batch, cin[l], cout,
                                     H[l], W[l], l < 3 ? H[l + 1] : 1, l < 3 ? W[l + 1] : 1, main),
           "fp32 lateral");
        if (prof_events) prof_record(1 + 2 * (3 - l), main);
        ok(ufpn::launch_fp32_conv3x3(static_cast<const float*>(merged[l]), out_w32[l], out_b[l],
                                     static_cast<float*>(out[l]), batch, cout, cout, H[l], W[l],
                                     main, act(), cfg.activation_alpha),
           "fp32 conv3x3");
        if (l == 3 && p6)
          ok(ufpn::launch_p6(DType::F32, out[3], p6, batch, cout, H[3], W[3], Layout::NCHW, main),
             "p6");
        if (prof_events) prof_record(2 + 2 * (3 - l), main);
      }
      return launches;
    }

    if (dtype == DType::E4M3) return enqueue_e4m3(in, out, p6, main, prof_events);
    const bool nchw = layout == Layout::NCHW;
    const void* x[4];
    void* o[4];
    void* o6 = p6 ? (nchw ? nhwc_out[4] : p6) : nullptr;
    for (int l = 0; l < 4; ++l) {
      o[l] = nchw ? nhwc_out[l] : out[l];
      x[l] = in[l];
    }
    if (prof_events) prof_record(0, main);
    if (nchw) {
      for (int l = 3; l >= 0; --l) {
        ok(ufpn::launch_transpose(dtype, in[l], nhwc_in[l], batch, cin[l], H[l] * W[l], true,
                                  main),
           "NCHW->NHWC");
        x[l] = nhwc_in[l];
      }
    }
    if (cfg.fused_neck_kernel && !prof_events) {
      ufpn::NeckLevel lv[4];
      for (int l = 0; l < 4; ++l) {
        lv[l].x = x[l];
        lv[l].lat_w = lat_wp[l];
        lv[l].lat_b = lat_b[l];
        lv[l].conv_w = out_wp[l];
        lv[l].conv_b = out_b[l];
        lv[l].merged = merged[l];
        lv[l].out = o[l];
        lv[l].Cin = cin[l];
        lv[l].H = H[l];
        lv[l].W = W[l];
        lv[l].lat_tiling = lat_tiling[l];
        lv[l].conv_tiling = tiling_for(l);
        lv[l].act = act();
        lv[l].act_alpha = cfg.activation_alpha;
      }
      ufpn::NeckPlan plan;
      check(ufpn::plan_neck(plan, dtype, batch, lv, o6, d_sched, d_status, 0,
                            trace_next ? d_trace : nullptr),
            "plan neck");
      if (cfg.test_stall_dependency_us > 0)
        check(ufpn::neck_plan_stall_dependency(
                  plan, 0, static_cast<unsigned long long>(cfg.test_stall_dependency_us) * 1000ull),
              "stall self-test");
      ok(ufpn::launch_neck(plan, main), "neck launch");
      if (nchw) {
        for (int l = 0; l < 4; ++l)
          ok(ufpn::launch_transpose(dtype, o[l], out[l], batch, cout, H[l] * W[l], false, main),
             "NHWC->NCHW");
        if (p6)
          ok(ufpn::launch_transpose(dtype, o6, p6, batch, cout,
                                    ((H[3] - 1) / 2 + 1) * ((W[3] - 1) / 2 + 1), false, main),
             "NHWC->NCHW");
      }
      return launches;
    }
    const bool one_stream = prof_events || cfg.single_stream;
    // Programmatic dependent launches for every kernel that follows a kernel of ours on its
    // stream (not under profiling events, which time kernels one by one).
    const bool pdl = !prof_events && cfg.programmatic_launch;
    // Launch options of the main-stream chain: programmatic launches, and (chain_priority) a
    // higher priority than the side streams' 3x3s, so that SMs freed while the chain's next
    // kernel waits for them go to it rather than to a side 3x3.
    ufpn::LaunchOpts chain;
    chain.pdl = pdl;
    chain.priority = cfg.chain_priority ? chain_priority_value : 0;
    ufpn::LaunchOpts chain_first = chain;  // first kernel of the forward: no kernel before it
    chain_first.pdl = false;
    // Main stream (the top-down data dependence):
    //   1. ONE grouped launch of the raw P5, P4, P3 laterals L5, L4, L3 (as GEMMs they do
    //      not depend on one another; only their top-down adds chain);
    //   2. the merges M4 = L4 + up(M5), M3 = L3 + up(M4) (M5 = L5): one bandwidth kernel
    //      for both when the maps upsample (merge_two_levels; L4 then sits in lat4_raw),
    //      else two in-place merges;
    //   3. the P2 lateral with the top-down add of M3 through its tensor-core k-block.
    // Side streams, one per level: the P5, P4 and P3 3x3s, each as soon as its merged map
    // exists, so the small P5 / P4 grids run beside the chain instead of one after the
    // other; the P2 3x3 follows the P2 lateral on the main stream.
    ufpn::NeckLevel lv[4];
    for (int l = 0; l < 4; ++l) {
      lv[l].x = x[l];
      lv[l].lat_w = lat_wp[l];
      lv[l].lat_b = lat_b[l];
      lv[l].conv_w = out_wp[l];
      lv[l].conv_b = out_b[l];
      lv[l].merged = merged[l];
      lv[l].out = o[l];
      lv[l].Cin = cin[l];
      lv[l].H = H[l];
      lv[l].W = W[l];
      lv[l].lat_tiling = lat_tiling[l];
      lv[l].conv_tiling = tiling_for(l);
      lv[l].act = act();
      lv[l].act_alpha = cfg.activation_alpha;
    }
    auto conv_level = [&](int l) {
      const cudaStream_t st = conv_stream(l, main, one_stream);
      if (st != main) {
        check(cudaEventRecord(ev_lat[l], main), "event");
        check(cudaStreamWaitEvent(st, ev_lat[l], 0), "event");
      }
      TcPlan conv;
      void* const p6_out = l == 3 ? o6 : nullptr;
      check(ufpn::plan_tc_conv3x3(conv, dtype, merged[l], out_wp[l], out_b[l], o[l], p6_out,
                                  batch, H[l], W[l],
                                  conv_tiling_for(l, tiling_for(l), p6_out != nullptr, batch),
                                  d_status, conv_ctas[l], act_scales(), conv_claim(l)),
            "plan conv3x3");
      // (on the main stream the 3x3 follows a kernel: the P2 lateral, or the previous
      // level's merge / 3x3 when every kernel runs on one stream)
      ok(ufpn::launch_tc(conv, st, st == main ? chain : ufpn::LaunchOpts()), "conv3x3 launch");
    };
    // With lat4_raw: L4 goes there and ONE launch merges M4 and M3 (merge_two_levels).
    const bool two_level = lat4_raw != nullptr && cfg.merge_two_levels;
    if (two_level) lv[2].merged = lat4_raw;
    // grouped_topdown: the grouped launch writes M5, M4, M3 itself (no merge kernels).
    const int td = cfg.grouped_topdown && !two_level ? 1 : 0;
    for (int l = 1; l < 4; ++l) {
      lv[l].split_part = split_part[l];
      lv[l].split_sem = split_sem ? split_sem + split_sem_off[l] : nullptr;
    }
    auto ks = [&](int l) { return split_part[l] ? split_alloc[l] : 1; };
    // channel halves: raw laterals (no top-down add in the launch) without split-K only
    auto ns = [&](int l) { return ks(l) == 1 && (l == 3 || !td) ? cfg.lateral_nsplit[l] : 1; };
    const ufpn::NeckJobSpec grouped[3] = {
        {0, 3, 0, ks(3), ns(3)}, {0, 2, td, ks(2), ns(2)}, {0, 1, td, ks(1), ns(1)}};
    // grouped_laterals_pair: the same raw laterals on CTA pairs (channel halves per level as
    // configured; no top-down add or split-K in the launch; a geometry too large for its
    // static plan falls back to the single-CTA launch).
    bool pair_done = false;
    if (cfg.grouped_laterals_pair && !td && ks(1) * ks(2) * ks(3) == 1) {
      ufpn::LateralGroupPlan lplan;
      const int which[3] = {3, 2, 1};
      const int halves[3] = {ns(3), ns(2), ns(1)};
      const cudaError_t pe = ufpn::plan_lateral_group_pair(lplan, dtype, batch, lv, which, 3,
                                                           d_status, 0, halves);
      if (pe == cudaSuccess) {
        ok(ufpn::launch_lateral_group_pair(lplan, main, nchw ? chain : chain_first),
           "grouped laterals (pairs) launch");
        pair_done = true;
      } else if (pe != cudaErrorNotSupported) {
        check(pe, "plan grouped laterals (pairs)");
      }
    }
    if (!pair_done) {
      ufpn::NeckPlan gplan;
      check(ufpn::plan_neck_jobs(gplan, dtype, batch, lv, nullptr, grouped, 3, d_sched, d_status,
                                 0, trace_next ? d_trace : nullptr),
            "plan grouped laterals");
      ok(ufpn::launch_neck(gplan, main, nchw ? chain : chain_first), "grouped laterals launch");
    }
    if (prof_events) prof_record(1, main);
    conv_level(3);
    if (prof_events) prof_record(2, main);
    if (td) {
      // M4 and M3 are complete: no merge stages (their profile slots stay empty).
      if (prof_events) prof_record(3, main);
      conv_level(2);
      if (prof_events) {
        prof_record(4, main);
        prof_record(5, main);
      }
      conv_level(1);
      if (prof_events) prof_record(6, main);
    } else if (two_level) {
      ok(ufpn::launch_merge_two_levels(dtype, merged[3], lat4_raw, merged[2], merged[1],
                                       merged[1], batch, H[3], W[3], H[2], W[2], H[1], W[1],
                                       main, nullptr, nullptr, nullptr, chain),
         "merge P4 and P3");
      if (prof_events) prof_record(3, main);
      conv_level(2);
      if (prof_events) {
        prof_record(4, main);
        prof_record(5, main);  // (no separate P3 merge)
      }
      conv_level(1);
      if (prof_events) prof_record(6, main);
    } else {
      for (int l = 2; l >= 1; --l) {
        ok(ufpn::launch_upsample_add(dtype, merged[l + 1], merged[l], merged[l], batch, cout,
                                     H[l + 1], W[l + 1], H[l], W[l], 0, Layout::NHWC, main,
                                     nullptr, nullptr, chain, merge_units),
           "merge");
        if (prof_events) prof_record(3 + 2 * (2 - l), main);
        conv_level(l);
        if (prof_events) prof_record(4 + 2 * (2 - l), main);
      }
    }
    // The P2 lateral of images [n0, n0 + nb) (all its maps are NHWC with whole images
    // contiguous, so an image group is a pointer offset).
    auto launch_lat2 = [&](int n0, int nb, const ufpn::LaunchOpts& lo) {
      if (p2_lateral_dynamic && n0 == 0 && nb == batch) {
        // One lateral job (P2, top-down add of M3 from a staged coarse box, fp32 taps) on the
        // neck kernel: CTAs claim tiles from a counter, so CTAs that start late (their SMs
        // held by a 3x3 of another level) take fewer tiles.  Own schedule counters.
        const ufpn::NeckJobSpec job[1] = {{0, 0, 1}};
        ufpn::NeckPlan p2plan;
        check(ufpn::plan_neck_jobs(p2plan, dtype, batch, lv, nullptr, job, 1, d_sched + 16,
                                   d_status, p2_lateral_ctas),
              "plan P2 lateral");
        ok(ufpn::launch_neck(p2plan, main, lo), "P2 lateral launch");
        return;
      }
      const size_t px0 = static_cast<size_t>(n0) * H[0] * W[0];
      const size_t px1 = static_cast<size_t>(n0) * H[1] * W[1];
      const size_t esz = ufpn::dtype_size(dtype);
      const void* xin = static_cast<const char*>(x[0]) + px0 * cin[0] * esz;
      const void* m3 = static_cast<const char*>(merged[1]) + px1 * cout * esz;
      void* m2 = static_cast<char*>(merged[0]) + px0 * cout * esz;
      TcPlan lat2;
      // p2_pair: CTA pairs with resident weight halves and fp32 top-down taps (when the level
      // qualifies: Cin <= 256, taps within a 64-pixel box); else one CTA per tile with the
      // top-down add as a tensor-core k-block.
      const cudaError_t pe =
          p2_pair ? ufpn::plan_tc_lateral_pair(lat2, dtype, xin, lat_wp[0], lat_b[0], m3, m2, nb,
                                               cin[0], H[0], W[0], H[1], W[1], lv[0].lat_tiling,
                                               d_status, p2_lateral_ctas)
                  : cudaErrorNotSupported;
      if (pe != cudaSuccess) {
        if (pe != cudaErrorNotSupported) check(pe, "plan lateral pair");
        check(ufpn::plan_tc_lateral(lat2, dtype, xin, lat_wp[0], lat_b[0], m3, m2, nb, cin[0],
                                    H[0], W[0], H[1], W[1], lv[0].lat_tiling, d_status,
                                    p2_lateral_ctas),
              "plan lateral");
        ufpn::tc_attach_wb_table(lat2, wb_table);
        if (cfg.lateral_wide_epilogue) ufpn::tc_use_wide_epilogue(lat2);
      }
      ok(ufpn::launch_tc(lat2, main, lo), "lateral launch");
    };
    const int parts = one_stream ? 1 : std::min({cfg.p2_parts, batch, Impl::kMaxP2Parts});
    if (parts <= 1) {
      launch_lat2(0, batch, chain);
      if (prof_events) prof_record(7, main);
      conv_level(0);
      if (prof_events) prof_record(8, main);
    } else {
      // Image groups: group g's lateral on the main stream, its 3x3 on p2_side after an
      // event, so the 3x3 of group g overlaps the lateral of group g + 1.
      for (int g = 0; g < parts; ++g) {
        const int n0 = batch * g / parts, n1 = batch * (g + 1) / parts;
        launch_lat2(n0, n1 - n0, chain);
        check(cudaEventRecord(ev_p2[g], main), "event");
        check(cudaStreamWaitEvent(p2_side, ev_p2[g], 0), "event");
        const size_t px0 = static_cast<size_t>(n0) * H[0] * W[0];
        const size_t esz = ufpn::dtype_size(dtype);
        TcPlan conv;
        check(ufpn::plan_tc_conv3x3(conv, dtype, static_cast<char*>(merged[0]) + px0 * cout * esz,
                                    out_wp[0], out_b[0], static_cast<char*>(o[0]) + px0 * cout * esz,
                                    nullptr, n1 - n0, H[0], W[0],
                                    conv_tiling_for(0, tiling_for(0), false, n1 - n0), d_status, 0,
                                    act_scales()),
              "plan conv3x3");
        ok(ufpn::launch_tc(conv, p2_side), "conv3x3 launch");
      }
      check(cudaEventRecord(ev_p2_join, p2_side), "event");
      check(cudaStreamWaitEvent(main, ev_p2_join, 0), "event");
    }
    if (!one_stream) join_conv_streams(main);
    if (nchw) {
      for (int l = 0; l < 4; ++l)
        ok(ufpn::launch_transpose(dtype, o[l], out[l], batch, cout, H[l] * W[l], false, main),
           "NHWC->NCHW");
      if (p6)
        ok(ufpn::launch_transpose(dtype, o6, p6, batch, cout,
                                  ((H[3] - 1) / 2 + 1) * ((W[3] - 1) / 2 + 1), false, main),
           "NHWC->NCHW");
    }
    return launches;
  }

  // Stream of level l's 3x3 in the split schedules: P5 on `side`, P4 / P3 on the two
  // lat_side streams (each after that stream's earlier work, if any), P2 on main.
  cudaStream_t conv_stream(int l, cudaStream_t main, bool one_stream) const {
    if (one_stream || l == 0) return main;
    return l == 3 ? side : lat_side[2 - l];
  }
  void join_conv_streams(cudaStream_t main) {
    check(cudaEventRecord(ev_join, side), "event");
    check(cudaStreamWaitEvent(main, ev_join, 0), "event");
    for (int i = 0; i < 2; ++i) {
      check(cudaEventRecord(ev_join_lat[i], lat_side[i]), "event");
      check(cudaStreamWaitEvent(main, ev_join_lat[i], 0), "event");
    }
  }

  // e4m3 inputs (NHWC), bf16 M_l and outputs.  Same dependence structure as the 16-bit
  // split schedule; each M_l additionally gets its per-image absmax from the kernel that
  // writes it (P5 / P2 lateral epilogue, P4 / P3 merge) and is quantised to e4m3 per image
  // on its 3x3's stream right before the 3x3 (per image, so an image's result does not
  // depend on the rest of its batch, e.g. on how a batch is sharded over GPUs):
  //   main:        zero amax | lat5 (amax5) | merge4 + merge3 (amax4, amax3, M3s) | lat2 + up(M3s) (amax2) | q2 3x3_2
  //   side:                                  q5 3x3_5 (+P6)
  //   lat_side[0]:             lat4                                                q4 3x3_4
  //   lat_side[1]:             lat3                                                q3 3x3_3
  // (the two merges are one launch when the maps upsample -- merge_two_levels, L4 from
  // lat4_raw -- else two in-place merges with q4 3x3_4 between them)
  int enqueue_e4m3(const void* const* in, void* const* out, void* p6, cudaStream_t main,
                   bool prof_events) {
    int launches = 0;
    auto ok = [&](cudaError_t e, const char* what) {
      check(e, what);
      ++launches;
    };
    const bool one_stream = prof_events || cfg.single_stream;
    // Programmatic dependent launches measured 2-5% slower on this schedule at the 640x640
    // batch-16 workload (its quantisation kernels release their dependents at their start,
    // so the next 3x3's CTAs wait on SMs the other streams could use), and still 1% slower
    // with the quantisation releasing them at its end: off.
    const bool pdl = false;
    auto opts = [](bool p) {
      ufpn::LaunchOpts o;
      o.pdl = p;
      return o;
    };
    const bool two_level = lat4_raw != nullptr && cfg.merge_two_levels;
    if (prof_events) prof_record(0, main);
    check(cudaMemsetAsync(fp8_amax, 0, 4 * static_cast<size_t>(batch) * sizeof(unsigned), main),
          "memset");
    if (!one_stream) {
      check(cudaEventRecord(ev_fork, main), "event");
      for (int i = 0; i < 2; ++i) check(cudaStreamWaitEvent(lat_side[i], ev_fork, 0), "event");
    }
    // out_mode: 0 store bf16 M_l (and its absmax into amax_out, if given), 1 publish only the
    // absmax, 2 store M_l quantised to e4m3 (qmerged[l]) with the absmax of pass 1.
    auto lateral = [&](int l, const void* coarse, unsigned* amax_out, cudaStream_t st,
                       bool after_kernel, int out_mode = 0) {
      ufpn::TcScales sc;
      sc.ascale = in_scale[l];
      sc.wscale = lat_ws[l];
      sc.amax_out = out_mode == 2 ? nullptr : amax_out;
      sc.coarse_prescaled = coarse != nullptr;  // coarse = m3_scaled
      sc.out_mode = out_mode;
      if (out_mode == 2) {
        sc.qamax = fp8_amax + l * batch;
        sc.qscale_out = fp8_scale + l * batch;
      }
      TcPlan p;
      // (with lat4_raw, L4 goes there: the two-level merge writes M4)
      void* lout = out_mode == 2 ? qmerged[l] : (l == 2 && two_level) ? lat4_raw : merged[l];
      check(ufpn::plan_tc_lateral(p, DType::E4M3, in[l], lat_wp[l], lat_b[l], coarse, lout,
                                  batch, cin[l], H[l], W[l], coarse ? H[l + 1] : 0,
                                  coarse ? W[l + 1] : 0, lat_tiling[l],
                                  d_status, 0, sc),
            "plan e4m3 lateral");
      if (l == 0) ufpn::tc_attach_wb_table(p, wb_table);
      ok(ufpn::launch_tc(p, st, opts(pdl && after_kernel)), "e4m3 lateral launch");
    };
    // quantise = false: qmerged[l] and its scales were written by the kernel producing M_l.
    auto conv_level = [&](int l, bool quantise = true) {
      const cudaStream_t conv_st = conv_stream(l, main, one_stream);
      if (conv_st != main) {
        check(cudaEventRecord(ev_lat[l], main), "event");
        check(cudaStreamWaitEvent(conv_st, ev_lat[l], 0), "event");
      }
      const long long n = static_cast<long long>(batch) * H[l] * W[l] * cout;
      Conv3x3Tiling t = tiling_for(l);
      if (!t.halo) t = ufpn::halo_pair_tiling();  // e4m3 runs halo tiles only
      t = conv_tiling_for(l, t, l == 3 && p6 != nullptr, batch);
      // The CTA-pair 3x3 can quantise M_l itself (per image, in shared memory; no quantise
      // pass, no e4m3 copy of M_l; fp8_quantise_in_conv), but its bf16 staging costs two of
      // the eight weight stages of this weight-feed-bound kernel: measured 240 us against
      // 181 + 43 us for quantise-then-convolve at the P2 map of the 640x640 batch-16
      // workload.  Off by default.
      const bool in_kernel = cfg.fp8_quantise_in_conv && t.pair;
      // (on the main stream the quantisation follows the P2 lateral kernel; on a side stream
      // it follows an event wait)
      if (quantise && !in_kernel)
        ok(ufpn::launch_quantize_e4m3(DType::BF16, merged[l], n, batch, fp8_amax + l * batch,
                                      qmerged[l], fp8_scale + l * batch, conv_st,
                                      opts(pdl && conv_st == main)),
           "quantise merged map");
      ufpn::TcScales sc = act_scales();
      sc.ascale = fp8_scale + l * batch;
      sc.ascale_per_image = true;
      sc.wscale = out_ws[l];
      if (in_kernel) sc.in_amax = fp8_amax + l * batch;
      TcPlan conv;
      check(ufpn::plan_tc_conv3x3(conv, DType::E4M3, in_kernel ? merged[l] : qmerged[l],
                                  out_wp[l], out_b[l], out[l], l == 3 ? p6 : nullptr, batch,
                                  H[l], W[l], t, d_status, conv_ctas[l], sc, conv_claim(l)),
            "plan e4m3 conv3x3");
      ok(ufpn::launch_tc(conv, conv_st,
                         opts(pdl && (conv_st == main || (quantise && !in_kernel)))),
         "e4m3 conv3x3 launch");
    };
    // The three raw laterals are independent GEMMs: P5 on the main stream, P4 and P3 on
    // their own streams so the small P5 grid shares the machine with the larger ones.
    lateral(3, nullptr, fp8_amax + 3 * batch, main, false);  // after the memset
    for (int i = 0; i < 2; ++i) {
      const cudaStream_t st = one_stream ? main : lat_side[i];
      lateral(2 - i, nullptr, nullptr, st, one_stream);
      if (!one_stream) check(cudaEventRecord(ev_lat_done[i], st), "event");
    }
    if (prof_events) prof_record(1, main);
    conv_level(3);
    if (prof_events) prof_record(2, main);
    // M3 also gets its copy pre-divided by the P2 lateral's per-channel scale, which the P2
    // lateral adds through its tensor-core top-down k-block.
    ufpn::MergeScaledCopy m3s;
    m3s.out = m3_scaled;
    m3s.scale_a = in_scale[0];
    m3s.scale_w = lat_ws[0];
    if (two_level) {
      if (!one_stream)
        for (int i = 0; i < 2; ++i) check(cudaStreamWaitEvent(main, ev_lat_done[i], 0), "event");
      ok(ufpn::launch_merge_two_levels(DType::BF16, merged[3], lat4_raw, merged[2], merged[1],
                                       merged[1], batch, H[3], W[3], H[2], W[2], H[1], W[1],
                                       main, fp8_amax + 2 * batch, fp8_amax + batch, &m3s,
                                       opts(pdl)),
         "merge P4 and P3");
      if (prof_events) prof_record(3, main);
      conv_level(2);
      if (prof_events) {
        prof_record(4, main);
        prof_record(5, main);  // (no separate P3 merge)
      }
      conv_level(1);
      if (prof_events) prof_record(6, main);
    } else {
      for (int l = 2; l >= 1; --l) {
        if (!one_stream) check(cudaStreamWaitEvent(main, ev_lat_done[2 - l], 0), "event");
        ok(ufpn::launch_upsample_add(DType::BF16, merged[l + 1], merged[l], merged[l], batch,
                                     cout, H[l + 1], W[l + 1], H[l], W[l], 0, Layout::NHWC, main,
                                     fp8_amax + l * batch, l == 1 ? &m3s : nullptr, opts(pdl),
                                     merge_units),
           "merge");
        if (prof_events) prof_record(3 + 2 * (2 - l), main);
        conv_level(l);
        if (prof_events) prof_record(4 + 2 * (2 - l), main);
      }
    }
    if (cfg.fp8_two_pass_p2) {
      // P2: absmax pass, then the quantised store -- M2 never exists in bf16 in HBM
      lateral(0, m3_scaled, fp8_amax, main, true, 1);
      lateral(0, m3_scaled, nullptr, main, true, 2);
    } else {
      lateral(0, m3_scaled, fp8_amax, main, true);
    }
    if (prof_events) prof_record(7, main);
    conv_level(0, !cfg.fp8_two_pass_p2);
    if (prof_events) prof_record(8, main);
    if (!one_stream) join_conv_streams(main);
    return launches;
  }

  double flops() const {
    double f = 0;
    for (int l = 0; l < 4; ++l) {
      const double px = static_cast<double>(batch) * H[l] * W[l];
      f += 2.0 * px * cout * cin[l] + 2.0 * px * cout * cout * 9;
    }
    return f;
  }
  double compulsory_bytes() const {
    const double esz = ufpn::dtype_size(dtype);              // inputs and weights
    const double osz = dtype == DType::E4M3 ? 2.0 : esz;     // outputs (bf16 for e4m3)
    double b = 0;
    for (int l = 0; l < 4; ++l) {
      const double px = static_cast<double>(batch) * H[l] * W[l];
      b += px * cin[l] * esz + px * cout * osz;              // read C_l, write P_l
      b += (static_cast<double>(cout) * cin[l] + 9.0 * cout * cout) * esz;  // weights
    }
    return b;
  }
};

UnifiedFPNCore::UnifiedFPNCore(size_t workspace_size, int device) : impl_(new Impl) {
  if (device < 0) CUDA_CHECK(cudaGetDevice(&device));
  impl_->device = device;
  impl_->workspace_cap = workspace_size;
  DeviceGuard g(device);
  CUDA_CHECK(cudaStreamCreateWithFlags(&impl_->side, cudaStreamNonBlocking));
  CUDA_CHECK(cudaStreamCreateWithFlags(&impl_->p2_side, cudaStreamNonBlocking));
  for (auto& e : impl_->ev_p2) CUDA_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CUDA_CHECK(cudaEventCreateWithFlags(&impl_->ev_p2_join, cudaEventDisableTiming));
  {
    int least = 0, greatest = 0;
    CUDA_CHECK(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    impl_->chain_priority_value = greatest;
  }
  CUDA_CHECK(cudaStreamCreateWithFlags(&impl_->capture, cudaStreamNonBlocking));
  CUDA_CHECK(cudaStreamCreateWithFlags(&impl_->setup, cudaStreamNonBlocking));
  for (int i = 0; i < 2; ++i) {
    CUDA_CHECK(cudaStreamCreateWithFlags(&impl_->lat_side[i], cudaStreamNonBlocking));
    CUDA_CHECK(cudaEventCreateWithFlags(&impl_->ev_lat_done[i], cudaEventDisableTiming));
  }
  CUDA_CHECK(cudaEventCreateWithFlags(&impl_->ev_fork, cudaEventDisableTiming));
  CUDA_CHECK(cudaEventCreateWithFlags(&impl_->ev_join, cudaEventDisableTiming));
  for (auto& e : impl_->ev_join_lat) CUDA_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : impl_->ev_lat) CUDA_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : impl_->prof) CUDA_CHECK(cudaEventCreate(&e));
  CUDA_CHECK(cudaMalloc(&impl_->d_status, 1024));
  CUDA_CHECK(cudaMemset(impl_->d_status, 0, 1024));
  impl_->d_sched = impl_->d_status + 64;
  impl_->d_trace = reinterpret_cast<unsigned long long*>(impl_->d_status + 128);
}

UnifiedFPNCore::~UnifiedFPNCore() = default;

void UnifiedFPNCore::configure_levels(const std::vector<FPNDimensions>& dims, int output_channels,
                                      FPNDataType dtype, FPNLayout layout) {
  Impl& m = *impl_;
  if (dims.size() != 4 && dims.size() != 5)
    FPN_THROW("configure_levels expects the dimensions of C2..C5 (or C2..C6)");
  if (output_channels != 256)
    FPN_THROW("only output_channels = 256 is supported (the tensor-core tile is 256 wide)");
  const DType dt = to_dtype(dtype);
  const Layout lay = layout == FPNLayout::NHWC ? Layout::NHWC : Layout::NCHW;
  if (dt == DType::F32 && lay != Layout::NCHW)
    FPN_THROW("the fp32 path takes NCHW (contiguous) tensors");
  if (dt == DType::E4M3 && lay != Layout::NHWC)
    FPN_THROW("FP8_E4M3 inputs must be NHWC (channels_last)");
  const int N = dims[0].batch_size;
  if (N <= 0) FPN_THROW("the batch must hold at least one image");
  for (int l = 0; l < 4; ++l) {
    if (dims[l].batch_size != N) FPN_THROW("all levels must share the batch size");
    if (dims[l].channels <= 0 || dims[l].height <= 0 || dims[l].width <= 0)
      FPN_THROW("level dimensions must be positive");
    if (dt != DType::F32 && (dims[l].channels * ufpn::dtype_size(dt)) % 16 != 0)
      FPN_THROW("tensor-core inputs need Cin x element size % 16 == 0 (16-byte TMA row stride)");
    if (l < 3 && (dims[l + 1].height > dims[l].height || dims[l + 1].width > dims[l].width))
      FPN_THROW("levels must be ordered fine (C2) to coarse (C5)");
  }
  DeviceGuard g(m.device);
  bool same = m.configured && m.batch == N && m.dtype == dt && m.layout == lay;
  for (int l = 0; l < 4 && same; ++l)
    same = m.cin[l] == dims[l].channels && m.H[l] == dims[l].height && m.W[l] == dims[l].width;
  if (same) return;
  m.release_graphs();
  m.free_workspace();
  m.batch = N;
  m.dtype = dt;
  m.layout = lay;
  m.cout = output_channels;
  for (int l = 0; l < 4; ++l) {
    m.cin[l] = dims[l].channels;
    m.H[l] = dims[l].height;
    m.W[l] = dims[l].width;
    // Single-CTA halo tiles on every level: their CTAs enter as other kernels free SMs, and a
    // single CTA takes any SM that frees while a CTA pair needs both SMs of a TPC.  Measured
    // against pairs on the maps with >= 4 tiles per SM (paired A/Bs): the P2 3x3 3-4.5 %
    // faster end to end (R50 800x1216 x 2 / x 4, 1024^2 x 8, Swin 1333x800 x 8), the P3 3x3 of
    // the x 8 workloads another 2-3 %; alone, the two forms time the same.  (e4m3: pairs.)
    const long long tiles = static_cast<long long>(N) * ((m.H[l] + 15) / 16) * ((m.W[l] + 7) / 8);
    m.tiling[l] = tiling_from_code(dt == DType::E4M3 && l > 0 && tiles >= 4LL * ufpn::sm_count()
                                       ? kDefaultTilingCode
                                       : 0);
    m.tiling_tuned[l] = false;
    auto it = m.tuning_db.find(m.tuning_key(l));
    if (it != m.tuning_db.end()) {
      m.tiling[l] = tiling_from_code(it->second.first);
      m.tiling_tuned[l] = true;
    }
    // lateral tiles: the standalone lateral tuner's choice for this shape, else the tiling
    // with the fewest padded pixels
    if (!ufpn::lateral_tiling_for(dt, N, m.cin[l], m.H[l], m.W[l], &m.lat_tiling[l]))
      m.lat_tiling[l] = ufpn::default_tiling(m.H[l], m.W[l]);
  }
  m.p2_pair = false;
  m.merge_units = 0;
  // The P2 lateral on every SM.  (With the P2 3x3 on CTA pairs, a short P2 lateral -- 4..10
  // tiles per SM -- ran best on 128 of 148 SMs, so that the P3 / P4 3x3s could run beside
  // it; with the P2 3x3 on single CTAs, whose tiles fill any SM the lateral frees, all SMs
  // are 0.6-1.2 % faster.  The option and the autotuner keep the cap.)
  {
    const int sms = ufpn::sm_count();
    m.p2_lateral_ctas = 0;
    // e4m3: the P3 3x3 (on CTA pairs, beside the P2 lateral's tail) on 96 of 148 SMs, so
    // that the quantisation pass over M2, which the P2 3x3 waits for, gets SMs as soon as
    // the P2 lateral ends (R50 640x640 x 16: -3.5..-5 %; its blocks did not start beside
    // the pair CTAs and waited ~40 us for them).
    for (int l = 0; l < 4; ++l) m.conv_ctas[l] = 0;
    if (dt == DType::E4M3) m.conv_ctas[1] = sms * 96 / 148;
  }
  m.p2_lateral_dynamic = false;
  m.apply_tuning_db2();         // a whole-neck tuning of this geometry, if any
  m.apply_explicit_options();   // then what the caller chose by name
  const size_t esz = ufpn::dtype_size(dt);
  const size_t msz = dt == DType::E4M3 ? 2 : esz;  // merged maps: bf16 for e4m3 inputs
  size_t total = 0;
  for (int l = 0; l < 4; ++l) {
    const size_t px = static_cast<size_t>(N) * m.H[l] * m.W[l];
    m.check(cudaMalloc(&m.merged[l], px * m.cout * msz), "workspace");
    total += px * m.cout * msz;
    if (dt == DType::E4M3) {
      m.check(cudaMalloc(&m.qmerged[l], px * m.cout), "workspace");
      total += px * m.cout;
    }
    if (m.tensor_core_path() && lay == Layout::NCHW) {
      m.check(cudaMalloc(&m.nhwc_in[l], px * m.cin[l] * esz), "workspace");
      m.check(cudaMalloc(&m.nhwc_out[l], px * m.cout * esz), "workspace");
      total += px * (m.cin[l] + m.cout) * esz;
    }
  }
  if (m.tensor_core_path() && m.cfg.merge_two_levels && m.cout == 256 && m.H[3] <= m.H[2] &&
      m.W[3] <= m.W[2] && m.H[2] <= m.H[1] && m.W[2] <= m.W[1]) {
    const size_t px4 = static_cast<size_t>(N) * m.H[2] * m.W[2];
    m.check(cudaMalloc(&m.lat4_raw, px4 * m.cout * msz), "workspace");
    total += px4 * m.cout * msz;
  }

  if (dt == DType::E4M3) {
    const size_t words = 4 * static_cast<size_t>(N);
    m.check(cudaMalloc(&m.fp8_amax, 2 * words * sizeof(float)), "workspace");
    m.fp8_scale = reinterpret_cast<float*>(m.fp8_amax + words);
    total += 2 * words * sizeof(float);
    const size_t px3 = static_cast<size_t>(N) * m.H[1] * m.W[1];
    m.check(cudaMalloc(&m.m3_scaled, px3 * m.cout * 2), "workspace");
    total += px3 * m.cout * 2;
  }
  if (m.tensor_core_path() && lay == Layout::NCHW) {
    const size_t px6 = static_cast<size_t>(N) * ((m.H[3] - 1) / 2 + 1) * ((m.W[3] - 1) / 2 + 1);
    m.check(cudaMalloc(&m.nhwc_out[4], px6 * m.cout * esz), "workspace");
    total += px6 * m.cout * esz;
  }
  m.workspace_bytes = total;
  m.configured = true;
  m.build_wb_table();
  if (m.weights_allocated) {
    m.packed_dtype = DType::F32;  // force repack in the new dtype
    m.ensure_weight_packing();
  }
}

void UnifiedFPNCore::allocate_weights(const std::vector<int>& channels, int output_channels) {
  Impl& m = *impl_;
  if (output_channels != 256) FPN_THROW("only output_channels = 256 is supported");
  std::vector<int> c = channels;
  if (c.size() == 5) c.erase(c.begin());  // reference form {C1 (unused), C2..C5}
  if (c.size() != 4) FPN_THROW("allocate_weights expects the channels of C2..C5");
  DeviceGuard g(m.device);
  m.release_graphs();
  m.free_weights();
  m.cout = output_channels;
  size_t bytes = 0;
  for (int l = 0; l < 4; ++l) {
    if (c[l] <= 0) FPN_THROW("channel counts must be positive");
    m.w_cin[l] = c[l];
    const size_t lw = static_cast<size_t>(m.cout) * c[l];
    const size_t ow = static_cast<size_t>(m.cout) * m.cout * 9;
    m.check(cudaMalloc(&m.lat_w32[l], lw * 4), "weights");
    m.check(cudaMalloc(&m.lat_b[l], m.cout * 4), "weights");
    m.check(cudaMalloc(&m.out_w32[l], ow * 4), "weights");
    m.check(cudaMalloc(&m.out_b[l], m.cout * 4), "weights");
    bytes += (lw + ow + 2 * m.cout) * 4;
    if (m.configured && m.tensor_core_path()) bytes += (lw + ow) * ufpn::dtype_size(m.dtype);
  }
  m.weight_bytes = bytes;
  m.weights_allocated = true;
  m.packed_dtype = DType::F32;
  m.ensure_weight_packing();
}

void UnifiedFPNCore::set_weights(int level, const float* lw, const float* lb, const float* ow,
                                 const float* ob) {
  Impl& m = *impl_;
  if (!m.weights_allocated || level < 0 || level >= 4)
    FPN_THROW("Invalid level or weights not allocated");
  if (!lw || !lb || !ow || !ob) FPN_THROW("null weight pointer");
  DeviceGuard g(m.device);
  const size_t lwn = static_cast<size_t>(m.cout) * m.w_cin[level];
  const size_t own = static_cast<size_t>(m.cout) * m.cout * 9;
  m.check(cudaMemcpyAsync(m.lat_w32[level], lw, lwn * 4, cudaMemcpyDefault, m.setup), "copy");
  m.check(cudaMemcpyAsync(m.lat_b[level], lb, m.cout * 4, cudaMemcpyDefault, m.setup), "copy");
  m.check(cudaMemcpyAsync(m.out_w32[level], ow, own * 4, cudaMemcpyDefault, m.setup), "copy");
  m.check(cudaMemcpyAsync(m.out_b[level], ob, m.cout * 4, cudaMemcpyDefault, m.setup), "copy");
  m.check(cudaStreamSynchronize(m.setup), "copy");
  m.weights_set[level] = true;
  m.release_graphs();
  if (m.configured && m.tensor_core_path()) {
    m.ensure_weight_packing();
    m.pack_level(level);
  }
}

void UnifiedFPNCore::forward_raw(const void* const* in, void* const* out, void* p6,
                                 cudaStream_t stream) {
  forward_raw_scaled(in, nullptr, out, p6, stream);
}

void UnifiedFPNCore::forward_raw_scaled(const void* const* in, const float* const* scales,
                                        void* const* out, void* p6, cudaStream_t stream) {
  Impl& m = *impl_;
  if (!m.configured) FPN_THROW("configure_levels() has not been called");
  for (int l = 0; l < 4; ++l) {
    if (!m.weights_set[l]) FPN_THROW("Weights not initialized");
    if (m.w_cin[l] != m.cin[l]) FPN_THROW("weights were allocated for different channel counts");
    if (!in[l] || !out[l]) FPN_THROW("null input/output pointer");
  }
  if (m.dtype == DType::E4M3) {
    if (!scales) FPN_THROW("FP8_E4M3 inputs need their per-tensor scales");
    if (!m.cfg.use_tensor_cores) FPN_THROW("FP8_E4M3 inputs run on the tensor cores only");
    for (int l = 0; l < 4; ++l) {
      if (!scales[l]) FPN_THROW("null input scale pointer");
      m.in_scale[l] = scales[l];
    }
  } else {
    if (scales) FPN_THROW("input scales apply to FP8_E4M3 inputs only");
    for (int l = 0; l < 4; ++l) m.in_scale[l] = nullptr;
  }
  DeviceGuard g(m.device);
  m.ensure_weight_packing();
  m.ensure_plan_buffers();
  if (m.profiling) {
    // The serialised schedule with an event between stages, captured and replayed as one
    // graph: the host's planning (tensor-map encoding) happens at capture, so the stage
    // times are device time only.  The graph runs twice and the events are read after the
    // second run: a graph's first launch uploads it, which showed up as ~20 us in the first
    // stage.
    cudaGraph_t graph = nullptr;
    m.check(cudaStreamBeginCapture(m.capture, cudaStreamCaptureModeThreadLocal), "capture");
    int n = 0;
    try {
      n = m.enqueue(in, out, p6, m.capture, true);
    } catch (...) {
      cudaStreamEndCapture(m.capture, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    m.check(cudaStreamEndCapture(m.capture, &graph), "capture");
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    m.check(ie, "cudaGraphInstantiate");
    cudaError_t le = cudaGraphLaunch(exec, stream);
    if (le == cudaSuccess) le = cudaGraphLaunch(exec, stream);
    if (le == cudaSuccess) cudaEventRecord(m.prof[9], stream);
    const cudaError_t se = le == cudaSuccess ? cudaEventSynchronize(m.prof[9]) : le;
    cudaGraphExecDestroy(exec);
    m.check(se, "profiled forward");
    float total = 0.f;
    for (int k = 0; k < 8; ++k) {
      float t = 0.f;
      m.check(cudaEventElapsedTime(&t, m.prof[k], m.prof[k + 1]), "stage time");
      m.metrics.kernel_times_ms[k] = t;
    }
    m.check(cudaEventElapsedTime(&total, m.prof[0], m.prof[9]), "forward time");
    m.metrics.forward_time_ms = total;
    m.metrics.memory_bandwidth_gb_s =
        total > 0 ? static_cast<float>(m.compulsory_bytes() / (total * 1e-3) / 1e9) : 0.f;
    double pk[3];
    ufpn::get_device_peaks(pk);
    const double peak = !m.tensor_core_path() ? pk[1] : (m.dtype == DType::E4M3 ? 2.0 * pk[0] : pk[0]);
    m.metrics.compute_utilization =
        total > 0 ? static_cast<float>(m.flops() / (total * 1e-3) / peak) : 0.f;
    m.metrics.num_kernel_launches = n;
    m.metrics.peak_memory_usage_bytes = m.workspace_bytes + m.weight_bytes;
    m.profiling = false;
    return;
  }
  if (m.trace_next) {
    // One directly launched forward with the neck kernel's timeline recorded.
    m.check(cudaMemsetAsync(m.d_trace, 0, 8 * sizeof(unsigned long long), stream), "memset");
    m.check(cudaMemsetAsync(m.d_trace, 0xFF, sizeof(unsigned long long), stream), "memset");
    m.metrics.num_kernel_launches = m.enqueue(in, out, p6, stream, false);
    m.check(cudaMemcpyAsync(m.last_trace, m.d_trace, sizeof(m.last_trace),
                            cudaMemcpyDeviceToHost, stream),
            "trace copy");
    m.check(cudaStreamSynchronize(stream), "trace sync");
    m.trace_next = false;
    return;
  }
  if (m.cfg.enable_graph_capture) {
    for (auto& e : m.graphs) {
      if (e.p6 != p6) continue;
      bool hit = true;
      for (int l = 0; l < 4 && hit; ++l)
        hit = e.in[l] == in[l] && e.out[l] == out[l] && e.scale[l] == m.in_scale[l];
      if (hit) {
        m.check(cudaGraphLaunch(e.exec, stream), "cudaGraphLaunch");
        m.metrics.num_kernel_launches = e.launches;
        ++m.stat_replays;
        return;
      }
    }
    // A pointer set is captured on its second use; the first runs as direct launches (a
    // caller that allocates new outputs every call pays launch latency, not a capture and
    // instantiation per call, and does not evict the graphs of sets that do repeat).
    bool seen = false;
    for (size_t i = 0; i < m.seen_once.size() && !seen; ++i) {
      const auto& k = m.seen_once[i];
      bool hit = k.p6 == p6;
      for (int l = 0; l < 4 && hit; ++l)
        hit = k.in[l] == in[l] && k.out[l] == out[l] && k.scale[l] == m.in_scale[l];
      if (hit) {
        seen = true;
        m.seen_once.erase(m.seen_once.begin() + static_cast<long>(i));
      }
    }
    if (!seen) {
      Impl::SeenKey k;
      for (int l = 0; l < 4; ++l) {
        k.in[l] = in[l];
        k.out[l] = out[l];
        k.scale[l] = m.in_scale[l];
      }
      k.p6 = p6;
      if (m.seen_once.size() >= 16) m.seen_once.erase(m.seen_once.begin());
      m.seen_once.push_back(k);
      m.metrics.num_kernel_launches = m.enqueue(in, out, p6, stream, false);
      ++m.stat_direct;
      return;
    }
    // Capture on the private stream (capturing the legacy default stream is not
    // allowed), ordered after the caller's prior work by the graph launch itself.
    cudaGraph_t graph = nullptr;
    m.check(cudaStreamBeginCapture(m.capture, cudaStreamCaptureModeThreadLocal), "capture");
    int n = 0;
    try {
      n = m.enqueue(in, out, p6, m.capture, false);
    } catch (...) {
      cudaStreamEndCapture(m.capture, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    m.check(cudaStreamEndCapture(m.capture, &graph), "capture");
    cudaGraphExec_t exec = nullptr;
    // Per-node priorities (the main-stream chain's launch priority) hold only when asked for.
    const cudaError_t ie =
        cudaGraphInstantiate(&exec, graph, cudaGraphInstantiateFlagUseNodePriority);
    cudaGraphDestroy(graph);
    m.check(ie, "cudaGraphInstantiate");
    if (m.graphs.size() >= 8) {
      cudaGraphExecDestroy(m.graphs.front().exec);
      m.graphs.erase(m.graphs.begin());
    }
    Impl::GraphEntry e;
    for (int l = 0; l < 4; ++l) {
      e.in[l] = in[l];
      e.out[l] = out[l];
      e.scale[l] = m.in_scale[l];
    }
    e.p6 = p6;
    e.exec = exec;
    e.launches = n;
    m.graphs.push_back(e);
    ++m.stat_captures;
    m.check(cudaGraphLaunch(exec, stream), "cudaGraphLaunch");
    m.metrics.num_kernel_launches = n;
    return;
  }
  m.metrics.num_kernel_launches = m.enqueue(in, out, p6, stream, false);
}

template <typename T>
void UnifiedFPNCore::forward(const std::vector<FPNTensor<T>>& features,
                             std::vector<FPNTensor<T>>& outputs, cudaStream_t stream) {
  if (features.size() != 4 && features.size() != 5)
    FPN_THROW("forward expects C2..C5 (or C2..C6) feature tensors");
  if (outputs.size() != 4 && outputs.size() != 5)
    FPN_THROW("forward expects P2..P5 (or P2..P6) output tensors");
  const void* in[4];
  void* out[4];
  for (int l = 0; l < 4; ++l) {
    in[l] = features[l].data;
    out[l] = outputs[l].data;
  }
  forward_raw(in, out, outputs.size() == 5 ? outputs[4].data : nullptr, stream);
}

template void UnifiedFPNCore::forward<float>(const std::vector<FPNTensor<float>>&,
                                             std::vector<FPNTensor<float>>&, cudaStream_t);
template void UnifiedFPNCore::forward<void>(const std::vector<FPNTensor<void>>&,
                                            std::vector<FPNTensor<void>>&, cudaStream_t);

const FPNPerformanceMetrics& UnifiedFPNCore::get_performance_metrics() const {
  return impl_->metrics;
}

void UnifiedFPNCore::set_kernel_config(const FPNKernelConfig& config) {
  if (static_cast<int>(config.activation) < 0 || static_cast<int>(config.activation) > 3)
    FPN_THROW("activation must be NONE, RELU, LEAKY_RELU or SWISH");
  if (config.tile_size != 0 &&
      (config.tile_size < 1 || config.tile_size > 128 || 128 % config.tile_size != 0))
    FPN_THROW("tile_size must divide 128 (8, 16, 32, 64, 128) or be 0 for automatic");
  impl_->release_graphs();
  impl_->cfg = config;
}

FPNKernelConfig UnifiedFPNCore::get_kernel_config() const { return impl_->cfg; }

size_t UnifiedFPNCore::get_memory_usage() const {
  return impl_->workspace_bytes + impl_->weight_bytes;
}

void UnifiedFPNCore::set_profiling(bool enable) { impl_->profiling = enable; }

void UnifiedFPNCore::graph_stats(long long* out4) const {
  out4[0] = impl_->stat_captures;
  out4[1] = impl_->stat_replays;
  out4[2] = impl_->stat_direct;
  out4[3] = static_cast<long long>(impl_->graphs.size());
}

void UnifiedFPNCore::trace_next_forward() { impl_->trace_next = true; }

void UnifiedFPNCore::get_neck_trace(unsigned long long* out8) const {
  std::memcpy(out8, impl_->last_trace, sizeof(impl_->last_trace));
}

int UnifiedFPNCore::device_status(bool reset) {
  DeviceGuard g(impl_->device);
  int v = 0;
  CUDA_CHECK(cudaDeviceSynchronize());
  CUDA_CHECK(cudaMemcpy(&v, impl_->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) CUDA_CHECK(cudaMemset(impl_->d_status, 0, sizeof(int)));
  // After a pipeline abort, make sure the neck kernel's schedule counters (and the split-K
  // arrival counters) start at zero.
  if (reset && v != 0) {
    CUDA_CHECK(cudaMemset(impl_->d_sched, 0, 64 * sizeof(int)));
    if (impl_->split_sem) {
      size_t n = 0;
      for (int l = 1; l < 4; ++l)
        n += static_cast<size_t>(ufpn::neck_lateral_tiles(impl_->batch, impl_->H[l], impl_->W[l],
                                                          impl_->split_tiling[l]));
      CUDA_CHECK(cudaMemset(impl_->split_sem, 0, n * sizeof(int)));
    }
  }
  return v;
}

// ------------------------------------------------------------------ named options
namespace {
struct EngineOption {
  const char* name;
  std::function<bool(int)> valid;
  std::function<void(UnifiedFPNCore::Impl&, int)> set;
  std::function<int(const UnifiedFPNCore::Impl&)> get;
};
bool in01(int v) { return v == 0 || v == 1; }
bool lat_w_ok(int v) { return v == 8 || v == 16 || v == 32 || v == 64 || v == 128; }
bool conv_code_ok(int v) { return v == -1 || v == 0 || lat_w_ok(v); }
Conv3x3Tiling lat_from_w(int w) {
  Conv3x3Tiling t;
  t.tile_w = w;
  t.tile_h = 128 / w;
  return t;
}
template <bool FPNKernelConfig::*F>
EngineOption bool_option(const char* name) {
  return {name, in01, [](UnifiedFPNCore::Impl& m, int v) { m.cfg.*F = v != 0; },
          [](const UnifiedFPNCore::Impl& m) { return (m.cfg.*F) ? 1 : 0; }};
}
const std::vector<EngineOption>& engine_options() {
  static const std::vector<EngineOption> opts = [] {
    std::vector<EngineOption> o;
    o.push_back(bool_option<&FPNKernelConfig::grouped_topdown>("grouped_topdown"));
    o.push_back(bool_option<&FPNKernelConfig::programmatic_launch>("programmatic_launch"));
    o.push_back(bool_option<&FPNKernelConfig::chain_priority>("chain_priority"));
    o.push_back(bool_option<&FPNKernelConfig::merge_two_levels>("merge_two_levels"));
    o.push_back(bool_option<&FPNKernelConfig::single_stream>("single_stream"));
    o.push_back(bool_option<&FPNKernelConfig::fused_neck_kernel>("fused_neck_kernel"));
    o.push_back(bool_option<&FPNKernelConfig::fp8_two_pass_p2>("fp8_two_pass_p2"));
    o.push_back(bool_option<&FPNKernelConfig::lateral_wide_epilogue>("lateral_wide_epilogue"));
    o.push_back(bool_option<&FPNKernelConfig::conv3x3_tail_halves>("conv3x3_tail_halves"));
    o.push_back(bool_option<&FPNKernelConfig::conv3x3_transpose>("conv3x3_transpose"));
    o.push_back(bool_option<&FPNKernelConfig::conv3x3_mixed>("conv3x3_mixed"));
    o.push_back(bool_option<&FPNKernelConfig::conv3x3_dynamic>("conv3x3_dynamic"));
    o.push_back(bool_option<&FPNKernelConfig::grouped_laterals_pair>("grouped_laterals_pair"));
    o.push_back(bool_option<&FPNKernelConfig::fp8_quantise_in_conv>("fp8_quantise_in_conv"));
    o.push_back({"p2_parts", [](int v) { return v >= 0 && v <= 8; },
                 [](UnifiedFPNCore::Impl& m, int v) { m.cfg.p2_parts = v; },
                 [](const UnifiedFPNCore::Impl& m) { return m.cfg.p2_parts; }});
    for (int l = 1; l < 4; ++l) {
      static const char* names[4] = {"", "ksplit_p3", "ksplit_p4", "ksplit_p5"};
      o.push_back({names[l], [](int v) { return v == 1 || v == 2 || v == 4; },
                   [l](UnifiedFPNCore::Impl& m, int v) { m.cfg.lateral_ksplit[l] = v; },
                   [l](const UnifiedFPNCore::Impl& m) { return m.cfg.lateral_ksplit[l]; }});
      static const char* halves[4] = {"", "nsplit_p3", "nsplit_p4", "nsplit_p5"};
      o.push_back({halves[l], [](int v) { return v == 1 || v == 2; },
                   [l](UnifiedFPNCore::Impl& m, int v) { m.cfg.lateral_nsplit[l] = v; },
                   [l](const UnifiedFPNCore::Impl& m) { return m.cfg.lateral_nsplit[l]; }});
    }
    for (int l = 0; l < 4; ++l) {
      static const char* lat[4] = {"lateral_tile_p2", "lateral_tile_p3", "lateral_tile_p4",
                                   "lateral_tile_p5"};
      static const char* conv[4] = {"conv3x3_p2", "conv3x3_p3", "conv3x3_p4", "conv3x3_p5"};
      o.push_back({lat[l], lat_w_ok,
                   [l](UnifiedFPNCore::Impl& m, int v) { m.lat_tiling[l] = lat_from_w(v); },
                   [l](const UnifiedFPNCore::Impl& m) { return m.lat_tiling[l].tile_w; }});
      o.push_back({conv[l], conv_code_ok,
                   [l](UnifiedFPNCore::Impl& m, int v) {
                     m.tiling[l] = tiling_from_code(v);
                     m.tiling_tuned[l] = true;
                   },
                   [l](const UnifiedFPNCore::Impl& m) { return tiling_code(m.tiling[l]); }});
    }
    o.push_back({"p2_lateral_pair", in01,
                 [](UnifiedFPNCore::Impl& m, int v) { m.p2_pair = v != 0; },
                 [](const UnifiedFPNCore::Impl& m) { return m.p2_pair ? 1 : 0; }});
    o.push_back({"p2_lateral_dynamic", in01,
                 [](UnifiedFPNCore::Impl& m, int v) { m.p2_lateral_dynamic = v != 0; },
                 [](const UnifiedFPNCore::Impl& m) { return m.p2_lateral_dynamic ? 1 : 0; }});
    o.push_back({"p2_lateral_ctas", [](int v) { return v >= 0 && v <= 4096; },
                 [](UnifiedFPNCore::Impl& m, int v) { m.p2_lateral_ctas = v; },
                 [](const UnifiedFPNCore::Impl& m) { return m.p2_lateral_ctas; }});
    for (int l = 0; l < 4; ++l) {
      static const char* names[4] = {"conv3x3_ctas_p2", "conv3x3_ctas_p3", "conv3x3_ctas_p4",
                                     "conv3x3_ctas_p5"};
      o.push_back({names[l], [](int v) { return v >= 0 && v <= 4096; },
                   [l](UnifiedFPNCore::Impl& m, int v) { m.conv_ctas[l] = v; },
                   [l](const UnifiedFPNCore::Impl& m) { return m.conv_ctas[l]; }});
    }
    o.push_back({"merge_units", [](int v) { return v >= -1 && v <= 256; },
                 [](UnifiedFPNCore::Impl& m, int v) { m.merge_units = v; },
                 [](const UnifiedFPNCore::Impl& m) { return m.merge_units; }});
    o.push_back({"test_stall_dependency_us", [](int v) { return v >= 0 && v <= 1000000; },
                 [](UnifiedFPNCore::Impl& m, int v) { m.cfg.test_stall_dependency_us = v; },
                 [](const UnifiedFPNCore::Impl& m) { return m.cfg.test_stall_dependency_us; }});
    return o;
  }();
  return opts;
}
const EngineOption* find_option(const std::string& name) {
  for (const auto& o : engine_options())
    if (name == o.name) return &o;
  return nullptr;
}
}  // namespace

void UnifiedFPNCore::Impl::apply_tuning_db2() {
  auto it = tuning_db2.find(geometry_key());
  if (it == tuning_db2.end()) return;
  for (const auto& kv : it->second.first) {
    const EngineOption* o = find_option(kv.first);
    if (o && o->valid(kv.second)) o->set(*this, kv.second);
  }
}

void UnifiedFPNCore::set_option(const std::string& name, int value) {
  const EngineOption* o = find_option(name);
  if (!o) FPN_THROW("unknown option " + name);
  if (!o->valid(value)) FPN_THROW("bad value for " + name + ": " + std::to_string(value));
  DeviceGuard g(impl_->device);
  impl_->release_graphs();
  o->set(*impl_, value);
  impl_->explicit_options[name] = value;
}

void UnifiedFPNCore::Impl::apply_explicit_options() {
  for (const auto& kv : explicit_options)
    if (const EngineOption* o = find_option(kv.first)) o->set(*this, kv.second);
}

int UnifiedFPNCore::get_option(const std::string& name) const {
  const EngineOption* o = find_option(name);
  if (!o) FPN_THROW("unknown option " + name);
  return o->get(*impl_);
}

// ------------------------------------------------------------------ autotuner
std::string UnifiedFPNCore::autotune(const void* const* in, void* const* out, void* p6,
                                     cudaStream_t stream, int iterations,
                                     const float* const* scales) {
  Impl& m = *impl_;
  if (!m.configured) FPN_THROW("configure_levels() has not been called");
  std::ostringstream rep;
  if (!m.tensor_core_path()) {
    rep << "fp32 path: nothing to tune\n";
    return rep.str();
  }
  if (m.dtype == DType::E4M3 && !scales) FPN_THROW("FP8_E4M3 autotuning needs the input scales");
  if (iterations < 1) iterations = 1;
  DeviceGuard g(m.device);
  const bool fp8 = m.dtype == DType::E4M3;
  const bool saved_graph = m.cfg.enable_graph_capture;
  m.cfg.enable_graph_capture = true;
  cudaEvent_t e0 = m.prof[0], e1 = m.prof[1];
  // One sample of the current settings: the whole forward, captured (second use of the
  // pointer set) and replayed `iterations` times; ms per forward.
  auto measure = [&]() -> float {
    m.release_graphs();
    for (int i = 0; i < 2; ++i) forward_raw_scaled(in, scales, out, p6, stream);
    CUDA_CHECK(cudaEventRecord(e0, stream));
    for (int i = 0; i < iterations; ++i) forward_raw_scaled(in, scales, out, p6, stream);
    CUDA_CHECK(cudaEventRecord(e1, stream));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    if (device_status(true) != 0) FPN_THROW("device pipeline timeout during autotuning");
    return ms / static_cast<float>(iterations);
  };
  auto median = [](std::vector<float> v) {
    std::sort(v.begin(), v.end());
    return v.empty() ? -1.f : v[v.size() / 2];
  };
  // Knobs and their candidates, in tuning order.
  struct Knob {
    std::string name;
    std::vector<int> values;
  };
  std::vector<Knob> knobs;
  for (int l = 0; l < 4; ++l) {
    Knob k{"conv3x3_p" + std::to_string(l + 2), {}};
    for (int v : fp8 ? std::vector<int>{-1, 0} : std::vector<int>{-1, 0, 8, 16, 32, 64, 128})
      if (v <= 0 || v <= 2 * m.W[l] || v == 8) k.values.push_back(v);
    knobs.push_back(k);
  }
  for (int l = 0; l < 4; ++l) {
    Knob k{"lateral_tile_p" + std::to_string(l + 2), {}};
    for (int v : {8, 16, 32, 64, 128})
      if (v <= 2 * m.W[l] || v == 8) k.values.push_back(v);
    knobs.push_back(k);
  }
  if (!fp8) {
    if (m.cin[0] <= 256) knobs.push_back({"p2_lateral_pair", {0, 1}});
    knobs.push_back({"grouped_laterals_pair", {0, 1}});
    knobs.push_back({"grouped_topdown", {0, 1}});
    knobs.push_back({"ksplit_p5", {1, 2, 4}});
    knobs.push_back({"ksplit_p4", {1, 2, 4}});
    knobs.push_back({"ksplit_p3", {1, 2}});
    knobs.push_back({"nsplit_p5", {1, 2}});
    knobs.push_back({"nsplit_p4", {1, 2}});
    knobs.push_back({"nsplit_p3", {1, 2}});
    knobs.push_back({"programmatic_launch", {1, 0}});
    knobs.push_back({"lateral_wide_epilogue", {0, 1}});
    {
      const int sms = ufpn::sm_count();
      knobs.push_back({"p2_lateral_ctas", {0, sms * 112 / 148, sms * 128 / 148}});
    }
    if (m.batch >= 2) {
      Knob k{"p2_parts", {0, 2}};
      if (m.batch >= 3) k.values.push_back(std::min(m.batch, 4));
      knobs.push_back(k);
    }
  } else {
    knobs.push_back({"fp8_two_pass_p2", {0, 1}});
    knobs.push_back({"fp8_quantise_in_conv", {0, 1}});
  }
  {
    const int sms = ufpn::sm_count();
    Knob k{"conv3x3_ctas_p3", {m.conv_ctas[1]}};
    for (int v : {0, sms * 80 / 148, sms * 96 / 148, sms * 112 / 148})
      if (std::find(k.values.begin(), k.values.end(), v) == k.values.end()) k.values.push_back(v);
    knobs.push_back(k);
  }
  knobs.push_back({"conv3x3_transpose", {1, 0}});
  knobs.push_back({"conv3x3_mixed", {1, 0}});
  knobs.push_back({"conv3x3_dynamic", {1, 0}});
  knobs.push_back({"merge_units", {0, -1, 2, 4, 8, 16}});
  knobs.push_back({"merge_two_levels", {0, 1}});
  // Each candidate is compared with the incumbent in back-to-back pairs (the GPU's clock,
  // which drifts over seconds under a power cap, is the same within a pair); it replaces the
  // incumbent if the median of its time ratios shows a gain of at least kMinGain.
  constexpr int kPairs = 3;
  constexpr float kMinGain = 0.02f;
  float best_all = -1.f;
  for (const auto& k : knobs) {
    const EngineOption* o = find_option(k.name);
    if (!o) continue;
    int inc = o->get(m);
    rep << k.name << " (" << inc << "):";
    for (int v : k.values) {
      if (v == inc) continue;
      std::vector<float> ratios;
      float v_ms = -1.f;
      try {
        for (int r = 0; r < kPairs; ++r) {
          o->set(m, inc);
          m.ensure_plan_buffers();
          const float a = measure();
          o->set(m, v);
          m.ensure_plan_buffers();
          const float b = measure();
          ratios.push_back(b / a);
          v_ms = b;
          if (best_all < 0) best_all = a;
        }
      } catch (const FPNException&) {
        ratios.clear();  // a candidate this geometry cannot run (e.g. a plan limit)
        device_status(true);
      }
      const float q = median(ratios);
      rep << " " << v << (q < 0 ? std::string("=n/a") : "=" + std::to_string(q).substr(0, 5) + "x");
      if (q > 0 && q < 1.f - kMinGain) {
        inc = v;
        best_all = v_ms;
      }
    }
    o->set(m, inc);
    m.ensure_plan_buffers();
    rep << " -> " << inc << "\n";
  }
  if (best_all < 0) best_all = measure();
  // Record every knob of this geometry (save_tuning persists them; configuring the same
  // geometry again applies them).
  std::map<std::string, int> chosen;
  for (const auto& k : knobs) {
    const EngineOption* o = find_option(k.name);
    if (o) chosen[k.name] = o->get(m);
    m.explicit_options.erase(k.name);  // the tuned choice replaces an explicit one
  }
  m.tuning_db2[m.geometry_key()] = {chosen, best_all};
  for (int l = 0; l < 4; ++l) m.tuning_db[m.tuning_key(l)] = {tiling_code(m.tiling[l]), best_all};
  m.cfg.enable_graph_capture = saved_graph;
  m.release_graphs();
  rep << "tuned: " << best_all * 1e3 << " us per forward (" << m.geometry_key() << ")\n";
  return rep.str();
}

bool UnifiedFPNCore::save_tuning(const std::string& path) const {
  std::ofstream f(path);
  if (!f) return false;
  f << "ufpn-tuning 2\n";
  for (auto& kv : impl_->tuning_db2) {
    f << "neck " << kv.first << " " << kv.second.second;
    for (auto& o : kv.second.first) f << " " << o.first << "=" << o.second;
    f << "\n";
  }
  for (auto& kv : impl_->tuning_db)
    f << "conv3x3 " << kv.first << " " << kv.second.first << " " << kv.second.second << "\n";
  return static_cast<bool>(f);
}

bool UnifiedFPNCore::load_tuning(const std::string& path) {
  std::ifstream f(path);
  if (!f) return false;
  std::string magic;
  int ver = 0;
  f >> magic >> ver;
  if (magic != "ufpn-tuning" || (ver != 1 && ver != 2)) return false;
  Impl& m = *impl_;
  std::string line;
  std::getline(f, line);
  while (std::getline(f, line)) {
    std::istringstream ls(line);
    if (ver == 1) {  // key tile_w ms
      std::string key;
      int tw;
      float ms;
      if ((ls >> key >> tw >> ms) && (tw == -1 || tw == 0 || lat_w_ok(tw))) m.tuning_db[key] = {tw, ms};
      continue;
    }
    std::string kind, key;
    if (!(ls >> kind >> key)) continue;
    if (kind == "conv3x3") {
      int tw;
      float ms;
      if ((ls >> tw >> ms) && conv_code_ok(tw)) m.tuning_db[key] = {tw, ms};
    } else if (kind == "neck") {
      float ms;
      if (!(ls >> ms)) continue;
      std::map<std::string, int> knobs;
      std::string kv;
      while (ls >> kv) {
        const size_t eq = kv.find('=');
        if (eq == std::string::npos) continue;
        const std::string name = kv.substr(0, eq);
        const EngineOption* o = find_option(name);
        const int v = std::atoi(kv.c_str() + eq + 1);
        if (o && o->valid(v)) knobs[name] = v;
      }
      m.tuning_db2[key] = {knobs, ms};
    }
  }
  if (m.configured) {
    for (int l = 0; l < 4; ++l) {
      auto it = m.tuning_db.find(m.tuning_key(l));
      if (it != m.tuning_db.end()) {
        m.tiling[l] = tiling_from_code(it->second.first);
        m.tiling_tuned[l] = true;
      }
    }
    m.apply_tuning_db2();
    m.release_graphs();
  }
  return true;
}
