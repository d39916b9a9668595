// The whole tensor-core FPN neck in ONE persistent kernel launch.
//
// The neck is 8 implicit-GEMM jobs over 128-pixel x 256-channel tiles:
//   lat5, lat4, conv5(+P6), lat3, conv4, lat2, conv3, conv2
// (lat_l = 1x1 lateral + bias [+ bilinear(M_{l+1}) when l < 5], conv_l = 3x3 pad-1 + bias).
// Reference schedule: UnifiedFPNCore::forward, lib/core/fpn_engine.cu:191-245
// (lateral loop, then top-down loop P5 -> P2); semantics as in tc_gemm.cuh.
//
// Tiles are numbered job by job in the order above and handed out by a global
// atomic counter (dynamic scheduling).  Data dependencies are enforced on the
// device with per-level completion counters:
//   * a conv_l tile's producer waits until every lat_l tile has been stored
//     before it loads M_l (its 3x3 halo crosses tile borders);
//   * a lat_l tile's epilogue waits until every lat_{l+1} tile has been stored
//     before it reads M_{l+1} for the bilinear taps.
// Because a tile only ever waits for tiles with smaller numbers, and tiles are
// taken in increasing order by CTAs that are already running, every wait is
// for work that a resident CTA has taken: the schedule cannot deadlock, even
// if not all CTAs are resident.  Every wait is still bounded (ptx.cuh).
//
// Split-K lateral tiles (job.ksplit > 1): a tile with a long K loop (the P5 lateral's
// 2048 input channels are 32 k-blocks; one 128-pixel tile would hold its SM for its whole
// weight stream) is cut into ksplit units over consecutive k-block ranges, numbered
// consecutively so that idle CTAs take them side by side.  Every unit writes its fp32
// partial accumulator to the job's workspace and counts itself on the tile's semaphore; the
// unit that arrives last sums the partials pairwise, p0 + p1 or (p0 + p1) + (p2 + p3) (its
// own part comes from TMEM, bitwise equal to what it wrote), and runs the tile's real
// epilogue.  Each add is commutative, so the bits do not depend on which unit arrives last:
// results are deterministic.  The last unit resets the semaphore for the next launch.
//
// Channel-half lateral tiles (job.nsplit == 2): a tile is cut into two units over its output
// channels (N = 128 each: a 128-row weight box, an N = 128 MMA, half the epilogue), numbered
// consecutively so that two CTAs stream the tile's pixels side by side (the second read hits
// L2).  Each unit streams half the weight bytes of a whole tile and issues half its MMA
// work, so a deep-K tile (the P5 lateral) holds an SM about half as long, with no partial
// sums to reduce.  Every unit stores and publishes its own half.
//
// Cross-CTA visibility: an epilogue waits for its own TMA stores to complete
// (cp.async.bulk.wait_group 0), fences the async proxy, synchronises the
// epilogue warps and publishes with a release add; consumers acquire the
// counter and fence the async proxy before issuing TMA loads.
//
// Roles per CTA (one CTA per SM):
//   warp 0 lane 0 : tile fetcher + TMA producer
//   warp 1        : TMEM allocator; lane 0 issues tcgen05.mma
//   warps 2..9    : epilogue (TMEM -> bias / bilinear -> smem -> TMA store);
//                   warp 2 lane 0 also loads the staged coarse box
// The fetched tile id is passed to the MMA and epilogue roles through a small
// shared-memory ring guarded by mbarriers.
#pragma once

#include "activation.cuh"
#include "tc_gemm.cuh"

namespace ufpn {

constexpr int kNeckMaxJobs = 8;
constexpr int kNeckRing = 4;
constexpr int kNeckStages = 3;

struct NeckJob {
  CUtensorMap map_a;       // activations (NHWC, 4-D box (64, tile_w, tile_h, 1))
  CUtensorMap map_b;       // weights [256][K]
  CUtensorMap map_out;     // output (NHWC, box (64, min(tile_w,32), 32/.., 1))
  CUtensorMap map_coarse;  // lateral: M_{l+1} (NHWC, box (64, cbox_w, cbox_h, 1))
  int mode;                // 0 lateral, 1 conv3x3
  int level;               // 0..3 = P2..P5
  int tile_start;          // first global tile number
  int num_tiles;
  int num_kb;
  int cin_blocks;
  int N_img, H, W;
  int tile_w, tile_h, tiles_x, tiles_y;
  const float* bias;
  const void* coarse;      // lateral with top-down add
  int Hc, Wc;
  float scale_y, scale_x;
  int cbox_w, cbox_h;
  void* p6;
  int H6, W6;
  int dep_level;           // level whose laterals must be complete (-1: none)
  int dep_count;           // number of tiles of that lateral job
  int publish;             // lateral: a later job of this launch waits on this level
  int act;                 // conv3x3: output activation after the bias (0 = none)
  float act_alpha;
  int ksplit;              // lateral: units per tile over K (1 = whole tiles)
  int nsplit;              // lateral: units per tile over the output channels (1 or 2)
  int kb_per;              // k-blocks per unit (the last unit of a tile may have fewer)
  float* part;             // ksplit > 1: fp32 partials, [unit][256 columns][128 rows]
  int* sem;                // ksplit > 1: per-tile arrival counters (zero between launches)
};

struct NeckParams {
  NeckJob jobs[kNeckMaxJobs];
  int num_jobs;
  int total_tiles;
  int lat_tiles[4];  // lateral tiles per level (completion targets)
  int* sched;   // [0] tile counter, [1 + l] completed lateral tiles of level l, [7] exit counter
  int* status;  // device status word
  // Limit of the level-dependency waits in ns (0: kWaitTimeoutNs).  Shortened only by the
  // wait-timeout self-test (neck_plan_stall_dependency).
  unsigned long long dep_wait_ns;
  // Optional timeline (globaltimer ns): [0] first CTA start (min), [1 + l] time level l's
  // laterals completed, [5] last CTA end (max), [6] first conv2 tile MMA start (min).
  unsigned long long* trace;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_release_gpu_add(int* p, int v) {
  int old;
  asm volatile("atom.release.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ void fence_proxy_async_all() {
  asm volatile("fence.proxy.async;" ::: "memory");
}
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kTcEpiWarps * 32) : "memory");
}
// Named barrier over the epilogue warps that also ANDs a predicate: every
// epilogue thread gets the same answer, so exits taken on it are uniform and no
// warp is ever left waiting at a later bar.sync for one that left.
__device__ __forceinline__ bool epi_vote_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(kTcEpiWarps * 32)
      : "memory");
  return r != 0;
}

// Bounded wait until *counter >= target (acquire).  Returns false on timeout/abort.
__device__ __forceinline__ bool wait_counter(const int* counter, int target,
                                             volatile int* abort_flag, int* status, int code,
                                             unsigned long long limit_ns = kWaitTimeoutNs) {
  if (ld_acquire_gpu(counter) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      __nanosleep(64);
      if (ld_acquire_gpu(counter) >= target) return true;
    }
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

__device__ __forceinline__ int neck_find_job(const NeckParams& p, int t) {
  int j = 0;
#pragma unroll 1
  for (int k = 1; k < p.num_jobs; ++k)
    if (t >= p.jobs[k].tile_start) j = k;
  return j;
}

// Unit `local` of a job -> its pixel tile and its part: of the K loop (split-K jobs) or of
// the output channels (channel-half jobs); a job splits one way at most.
__device__ __forceinline__ int neck_unit_tile(const NeckJob& jb, int local, int& part) {
  const int per = jb.ksplit * jb.nsplit;
  if (per <= 1) {
    part = 0;
    return local;
  }
  const int pt = local / per;
  part = local - pt * per;
  return pt;
}
// (a channel-half unit's part names its channels: it runs the whole K loop)
__device__ __forceinline__ void neck_unit_kb(const NeckJob& jb, int part, int& kb0, int& kb1) {
  if (jb.ksplit <= 1) {
    kb0 = 0;
    kb1 = jb.num_kb;
    return;
  }
  kb0 = part * jb.kb_per;
  kb1 = min(jb.num_kb, kb0 + jb.kb_per);
}
__device__ __forceinline__ int atom_acq_rel_gpu_add(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ void neck_tile_origin(const NeckJob& jb, int local, int& n, int& x0,
                                                 int& y0) {
  const int tx = local % jb.tiles_x;
  const int t2 = local / jb.tiles_x;
  const int ty = t2 % jb.tiles_y;
  n = t2 / jb.tiles_y;
  x0 = tx * jb.tile_w;
  y0 = ty * jb.tile_h;
}

constexpr int kNeckCoarseBlk = kTcCoarseMaxPix * 128;
// Shared-memory plan of fpn_neck_kernel: kStages operand stages, the epilogue staging and
// (kCoarse) the 32 KB coarse box of the lateral top-down taps.  A launch with no staged
// coarse box (the grouped raw laterals) trades that box for a fourth stage: per-tile
// timestamps showed its 32- and 16-k-block lateral tiles waiting on operand latency with 3.
template <int kStages, bool kCoarse>
struct NeckCfg {
  static constexpr int kOffB = kStages * kTcAStage;
  static constexpr int kOffStaging = kOffB + kStages * kTcBStage;
  static constexpr int kOffCoarse = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kOffBars = kOffCoarse + (kCoarse ? 4 * kNeckCoarseBlk : 0);
  static constexpr int kSmemBytes = kOffBars + 512 + 1024;
  static_assert(kSmemBytes <= 232448, "neck smem");
};

constexpr int kDevTimeoutDependency = 0x105;

template <typename T, int kStages = kNeckStages, bool kCoarse = true>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_neck_kernel(const __grid_constant__ NeckParams P) {
  using Cfg = NeckCfg<kStages, kCoarse>;
  constexpr int S = kStages;
  constexpr int R = kNeckRing;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + Cfg::kOffB;
  uint8_t* smem_stage = smem + Cfg::kOffStaging;
  uint8_t* smem_coarse = smem + Cfg::kOffCoarse;  // (kCoarse only)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* accf_bar = bars + 2 * S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint64_t* cfull_bar = done_bar + 1;
  uint64_t* rfull_bar = cfull_bar + 1;
  uint64_t* rempty_bar = rfull_bar + R;
  int* ring = reinterpret_cast<int*>(rempty_bar + R);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + R);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_last = abort_flag + 1;  // epilogue leader -> epilogue: last unit of a tile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* sched = P.sched;

  if (threadIdx.x == 0) {
    if (P.trace) atomicMin(&P.trace[0], globaltimer_ns());
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], kTcEpiWarps * 32);
    }
    mbar_init(done_bar, 1);
    mbar_init(cfull_bar, 1);
    for (int r = 0; r < R; ++r) {
      mbar_init(&rfull_bar[r], 1);
      mbar_init(&rempty_bar[r], 1 + kTcEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // (programmatic launch) the previous kernel's results are visible

  if (warp == 0) {
    // ------------------------------------------------------------ fetcher + TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      int issued = 0;
      bool ok = true;
      int ready_level_mask = 0;  // dependency levels already observed complete
      // The next tile number is claimed while the current tile's last k-block is issued:
      // the atomic's round trip overlaps the MMAs still queued for this tile, and a CTA
      // held by a long tile (a P5 lateral has 32 k-blocks) does not sit on a second tile
      // that an idle CTA could have taken (claimed one whole tile ahead, such a tile
      // started only when the long one ended and set the end of the launch).
      int t_next = atomicAdd(&sched[0], 1);
      while (ok) {
        const int t = t_next;
        t_next = P.total_tiles;
        if (!mbar_wait(&rempty_bar[rslot], rphase ^ 1u, abort_flag, P.status,
                       kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        ring[rslot] = t < P.total_tiles ? t : -1;
        mbar_arrive(&rfull_bar[rslot]);
        if (++rslot == R) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (t >= P.total_tiles) break;
        const int j = neck_find_job(P, t);
        const NeckJob& jb = P.jobs[j];
        int n, x0, y0, part, kb0, kb1;
        neck_tile_origin(jb, neck_unit_tile(jb, t - jb.tile_start, part), n, x0, y0);
        neck_unit_kb(jb, part, kb0, kb1);
        if (jb.mode == 1 && jb.dep_level >= 0 && !(ready_level_mask & (1 << jb.dep_level))) {
          if (!wait_counter(&sched[1 + jb.dep_level], jb.dep_count, abort_flag, P.status,
                            kDevTimeoutDependency,
                            P.dep_wait_ns ? P.dep_wait_ns : kWaitTimeoutNs)) {
            ok = false;
            break;
          }
          fence_proxy_async_all();
          ready_level_mask |= 1 << jb.dep_level;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, P.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kTcAStage + kTcBStage / jb.nsplit);
          int dy = 0, dx = 0, cb = kb;
          if (jb.mode == 1) {
            const int tap = kb / jb.cin_blocks;
            cb = kb - tap * jb.cin_blocks;
            dy = tap / 3 - 1;
            dx = tap % 3 - 1;
          }
          tma_load_4d(smem_a + stage * kTcAStage, &jb.map_a, &full_bar[stage], cb * kTcBlockK,
                      x0 + dx, y0 + dy, n, jb.mode == 0 ? kPolicyEvictFirst : kPolicyEvictLast);
          // (channel halves: a 128-row box of the unit's output channels)
          tma_load_2d(smem_b + stage * kTcBStage, &jb.map_b, &full_bar[stage], kb * kTcBlockK,
                      jb.nsplit > 1 ? part * (kTcBlockN / 2) : 0, kPolicyEvictLast);
          if (kb == kb1 - 1) t_next = atomicAdd(&sched[0], 1);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      griddep_launch_dependents();  // no tile left for this CTA
      if (!ok) {
        // Unblock the consumers: publish an end marker if a ring slot is free.
        if (mbar_test(smem_u32(&rempty_bar[rslot]), rphase ^ 1u)) {
          ring[rslot] = -1;
          mbar_arrive(&rfull_bar[rslot]);
        }
      }
      for (int i = 0; i < S && i < issued; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait_drain(&full_bar[stage], phase);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_full =
          make_idesc(kTcBlockM, kTcBlockN, Pack<T>::kFmt, Pack<T>::kFmt);
      constexpr uint32_t idesc_half =
          make_idesc(kTcBlockM, kTcBlockN / 2, Pack<T>::kFmt, Pack<T>::kFmt);
      int stage = 0;
      uint32_t phase = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      while (ok) {
        if (!mbar_wait(&rfull_bar[rslot], rphase, abort_flag, P.status, kDevTimeoutMma)) break;
        const int t = ring[rslot];
        mbar_arrive(&rempty_bar[rslot]);
        if (++rslot == R) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (t < 0) break;
        const NeckJob& jm = P.jobs[neck_find_job(P, t)];
        int mpart, kb0, kb1;
        neck_unit_tile(jm, t - jm.tile_start, mpart);
        neck_unit_kb(jm, mpart, kb0, kb1);
        const int num_kb = kb1 - kb0;
        const uint32_t idesc = jm.nsplit > 1 ? idesc_half : idesc_full;
        if (P.trace && jm.mode == 1 && jm.level == 0 && t == jm.tile_start)
          P.trace[6] = globaltimer_ns();
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, P.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, P.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(smem_a + stage * kTcAStage));
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kTcBStage));
#pragma unroll
          for (int k = 0; k < kTcBlockK / 16; ++k)
            tc_mma_f16(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      tc_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int chalf = ew >> 2;
    const int row = quarter * 32 + lane;
    const bool leader = (ew == 0) && (lane == 0);  // issues the coarse box loads
    const uint32_t stage_addr = smem_u32(smem_stage + ew * kTcStagingPerWarp);
    const uint32_t coarse_addr = smem_u32(smem_coarse);
    int rslot = 0;
    uint32_t rphase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t cphase = 0;
    int coarse_requested = -1;  // leader: tile whose coarse box is in flight / resident
    int ready_level_mask = 0;   // leader: dependency levels observed complete
    bool ok = true;

    // Leader: make sure the coarser level's laterals (the top-down input of lateral job jb)
    // are complete (acquire).
    auto wait_dep = [&](const NeckJob& jb) -> bool {
      if (!(ready_level_mask & (1 << (jb.level + 1)))) {
        if (!wait_counter(&sched[1 + jb.level + 1], jb.dep_count, abort_flag, P.status,
                          kDevTimeoutDependency))
          return false;
        fence_proxy_async_all();
        ready_level_mask |= 1 << (jb.level + 1);
      }
      return true;
    };
    // Leader: wait_dep, then load the coarse box of lateral tile `t` of job `jb`.
    auto request_coarse = [&](const NeckJob& jb, int t) -> bool {
      if (!wait_dep(jb)) return false;
      if (kCoarse && jb.cbox_w > 0) {
        int n, x0, y0;
        neck_tile_origin(jb, t - jb.tile_start, n, x0, y0);
        const int cy = static_cast<int>(tc_src(y0, jb.scale_y, jb.Hc));
        const int cx = static_cast<int>(tc_src(x0, jb.scale_x, jb.Wc));
        mbar_arrive_expect_tx(cfull_bar, static_cast<uint32_t>(jb.cbox_w * jb.cbox_h * 128 * 4));
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem_coarse + b * kNeckCoarseBlk, &jb.map_coarse, cfull_bar, b * 64, cx,
                      cy, n, kPolicyEvictLast);
      }
      coarse_requested = t;
      return true;
    };

    while (true) {
      const bool got =
          mbar_wait(&rfull_bar[rslot], rphase, abort_flag, P.status, kDevTimeoutEpilogue);
      const int t = got ? ring[rslot] : -1;
      __syncwarp();
      if (lane == 0 && got) mbar_arrive(&rempty_bar[rslot]);
      if (++rslot == R) {
        rslot = 0;
        rphase ^= 1u;
      }
      if (!epi_vote_all(got && ok) || t < 0) break;  // uniform: same ring slot for all
      const NeckJob& jb = P.jobs[neck_find_job(P, t)];
      const bool lateral = jb.mode == 0;
      const bool has_coarse = lateral && jb.coarse != nullptr;
      const bool staged = kCoarse && has_coarse && jb.cbox_w > 0;
      const bool split = lateral && jb.ksplit > 1;  // (split jobs never stage a coarse box)
      int part = 0;
      const int ptile = neck_unit_tile(jb, t - jb.tile_start, part);
      if (has_coarse && !split && leader && coarse_requested != t) ok = request_coarse(jb, t);
      bool wok = mbar_wait(&accf_bar[acc], acc_phase, abort_flag, P.status, kDevTimeoutEpilogue);
      if (staged && wok && ok)
        wok = mbar_wait(cfull_bar, cphase, abort_flag, P.status, kDevTimeoutEpilogue);
      // Uniform exit; the barrier also orders the leader's acquire of the coarse
      // level before every thread's global-memory taps (unstaged path).
      if (!epi_vote_all(wok && ok)) break;
      tc_fence_after();

      // Split-K unit: write the fp32 partial ([unit][column][row]: a warp stores 128
      // contiguous bytes per column), count the arrival; only the tile's last unit goes on.
      bool final_unit = true;
      if (split) {
        float* mine = jb.part + static_cast<size_t>(t - jb.tile_start) * (kTcBlockN * kTcBlockM);
        const uint32_t tacc = tmem_base + static_cast<uint32_t>(acc * kTcBlockN + chalf * 128) +
                              (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {  // this warp's 128 columns, 32 at a time
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(tacc + h * 32, r);
          tmem_wait_ld();
          float* dst = mine + static_cast<size_t>(chalf * 128 + h * 32) * kTcBlockM + row;
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(dst + static_cast<size_t>(i) * kTcBlockM, __uint_as_float(r[i]));
        }
        __threadfence();
        epi_bar_sync();
        if (leader) {
          const int before = atom_acq_rel_gpu_add(&jb.sem[ptile], 1);
          const int last = before == jb.ksplit - 1;
          if (last) jb.sem[ptile] = 0;  // every unit of the tile has arrived: reset for the next launch
          *split_last = last;
        }
        epi_bar_sync();
        final_unit = *split_last != 0;  // uniform
        if (final_unit) {
          fence_acq_rel_gpu();  // the other units' partials (published before their arrival)
          // Pairwise sum p0 + p1 (ksplit 2) or (p0 + p1) + (p2 + p3) (ksplit 4): every add
          // is commutative, so starting from its own part (in TMEM, bitwise what it wrote)
          // any unit computes the same bits.  Written back into the accumulator so the
          // epilogue below runs unchanged.
          const float* base = jb.part +
                              static_cast<size_t>(ptile) * jb.ksplit * (kTcBlockN * kTcBlockM) +
                              static_cast<size_t>(chalf * 128) * kTcBlockM + row;
          const int partner = part ^ 1;
          const int other0 = (part ^ 2) & ~1;  // ksplit 4: the other pair
#pragma unroll 1
          for (int h = 0; h < 4; ++h) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(tacc + h * 32, r);
            tmem_wait_ld();
            const float* ph = base + static_cast<size_t>(h * 32) * kTcBlockM;
            const float* pp = ph + static_cast<size_t>(partner) * (kTcBlockN * kTcBlockM);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              r[i] = __float_as_uint(__uint_as_float(r[i]) +
                                     __ldcg(pp + static_cast<size_t>(i) * kTcBlockM));
            if (jb.ksplit == 4) {
              const float* p0 = ph + static_cast<size_t>(other0) * (kTcBlockN * kTcBlockM);
              const float* p1 = p0 + static_cast<size_t>(kTcBlockN) * kTcBlockM;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                r[i] = __float_as_uint(__uint_as_float(r[i]) +
                                       (__ldcg(p0 + static_cast<size_t>(i) * kTcBlockM) +
                                        __ldcg(p1 + static_cast<size_t>(i) * kTcBlockM)));
            }
            tmem_st32(tacc + h * 32, r);
          }
          tmem_wait_st();
          if (has_coarse && leader) ok = wait_dep(jb);
          if (!epi_vote_all(ok)) break;
        } else {
          tc_fence_before();
          mbar_arrive(&acce_bar[acc]);  // this unit's accumulator is fully read
        }
      }
      if (final_unit) {
      int n, x0, y0;
      neck_tile_origin(jb, ptile, n, x0, y0);
      const int tw = jb.tile_w;
      const int py = y0 + row / tw;
      const int px = x0 + row % tw;
      const bool valid = (py < jb.H) && (px < jb.W);

      float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
      int r00 = 0, r01 = 0, r10 = 0, r11 = 0;
      bool corners_staged = false;
      const uint8_t* g00 = nullptr;
      const uint8_t* g01 = nullptr;
      const uint8_t* g10 = nullptr;
      const uint8_t* g11 = nullptr;
      if (has_coarse) {
        const float sy = tc_src(min(py, jb.H - 1), jb.scale_y, jb.Hc);
        const float sx = tc_src(min(px, jb.W - 1), jb.scale_x, jb.Wc);
        const int ya = static_cast<int>(sy);
        const int xa = static_cast<int>(sx);
        const int yb = min(ya + 1, jb.Hc - 1);
        const int xb = min(xa + 1, jb.Wc - 1);
        const float wy = sy - static_cast<float>(ya);
        const float wx = sx - static_cast<float>(xa);
        w00 = (1.f - wy) * (1.f - wx);
        w01 = (1.f - wy) * wx;
        w10 = wy * (1.f - wx);
        w11 = wy * wx;
        if (staged) {
          const int cy0 = static_cast<int>(tc_src(y0, jb.scale_y, jb.Hc));
          const int cx0 = static_cast<int>(tc_src(x0, jb.scale_x, jb.Wc));
          corners_staged = (ya - cy0) >= 0 && (yb - cy0) < jb.cbox_h && (xa - cx0) >= 0 &&
                           (xb - cx0) < jb.cbox_w;
          r00 = (ya - cy0) * jb.cbox_w + (xa - cx0);
          r01 = (ya - cy0) * jb.cbox_w + (xb - cx0);
          r10 = (yb - cy0) * jb.cbox_w + (xa - cx0);
          r11 = (yb - cy0) * jb.cbox_w + (xb - cx0);
        }
        if (!corners_staged) {
          const size_t rowb = static_cast<size_t>(kTcBlockN) * sizeof(T);
          const uint8_t* cbase = static_cast<const uint8_t*>(jb.coarse) +
                                 static_cast<size_t>(n) * jb.Hc * jb.Wc * rowb;
          g00 = cbase + (static_cast<size_t>(ya) * jb.Wc + xa) * rowb;
          g01 = cbase + (static_cast<size_t>(ya) * jb.Wc + xb) * rowb;
          g10 = cbase + (static_cast<size_t>(yb) * jb.Wc + xa) * rowb;
          g11 = cbase + (static_cast<size_t>(yb) * jb.Wc + xb) * rowb;
        }
      }
      const bool emit_p6 =
          (!lateral) && (jb.p6 != nullptr) && valid && ((py & 1) == 0) && ((px & 1) == 0);
      uint8_t* p6_row = nullptr;
      if (emit_p6) {
        const size_t p6pix = (static_cast<size_t>(n) * jb.H6 + (py >> 1)) * jb.W6 + (px >> 1);
        p6_row = static_cast<uint8_t*>(jb.p6) + p6pix * kTcBlockN * sizeof(T);
      }
      const int wrow0 = quarter * 32;
      const int ox = x0 + (wrow0 % tw);
      const int oy = y0 + wrow0 / tw;

      // This warp's accumulator columns: 128 of a whole tile (two 64-column steps), 64 of a
      // channel-half unit (whose N = 128 accumulator starts at the buffer's column 0 and
      // holds output channels part * 128 ..).
      const int nsteps = 2 / jb.nsplit;
      const int ocol = jb.nsplit > 1 ? part * (kTcBlockN / 2) : 0;
#pragma unroll 1
      for (int step = 0; step < nsteps; ++step) {
        const int tcol = chalf * 64 * nsteps + step * 64;
        const int col0 = ocol + tcol;  // output channel of the step's first column
        uint32_t r[64];
        __syncwarp();
        const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * kTcBlockN + tcol) +
                               (static_cast<uint32_t>(quarter * 32) << 16);
        tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_wait_ld();
        if (step == nsteps - 1) {
          tc_fence_before();
          mbar_arrive(&acce_bar[acc]);
        }
        float v[64];
        const float4* b4 = reinterpret_cast<const float4*>(jb.bias + col0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 bb = __ldg(b4 + i);
          v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + bb.x;
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
        }
        if (has_coarse) {
          const int blk = col0 >> 6;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 a, b, c, d;
            if (corners_staged) {
              const uint32_t base = coarse_addr + blk * kNeckCoarseBlk;
              a = ld_shared_v4(base + r00 * 128 + ((j ^ (r00 & 7)) << 4));
              b = ld_shared_v4(base + r01 * 128 + ((j ^ (r01 & 7)) << 4));
              c = ld_shared_v4(base + r10 * 128 + ((j ^ (r10 & 7)) << 4));
              d = ld_shared_v4(base + r11 * 128 + ((j ^ (r11 & 7)) << 4));
            } else {
              // Written by other CTAs during this launch: L2-coherent loads (ld.global.cg),
              // never the non-coherent / L1-cached read-only path.
              const size_t off = static_cast<size_t>(col0) * sizeof(T);
              a = __ldcg(reinterpret_cast<const uint4*>(g00 + off) + j);
              b = __ldcg(reinterpret_cast<const uint4*>(g01 + off) + j);
              c = __ldcg(reinterpret_cast<const uint4*>(g10 + off) + j);
              d = __ldcg(reinterpret_cast<const uint4*>(g11 + off) + j);
            }
            const uint32_t au[4] = {a.x, a.y, a.z, a.w};
            const uint32_t bu[4] = {b.x, b.y, b.z, b.w};
            const uint32_t cu[4] = {c.x, c.y, c.z, c.w};
            const uint32_t du[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 fa = Pack<T>::unpack(au[e]);
              const float2 fb = Pack<T>::unpack(bu[e]);
              const float2 fc = Pack<T>::unpack(cu[e]);
              const float2 fd = Pack<T>::unpack(du[e]);
              v[8 * j + 2 * e + 0] += w00 * fa.x + w01 * fb.x + w10 * fc.x + w11 * fd.x;
              v[8 * j + 2 * e + 1] += w00 * fa.y + w01 * fb.y + w10 * fc.y + w11 * fd.y;
            }
          }
        }
        epilogue_act(v, jb.act, jb.act_alpha);
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 o;
          o.x = Pack<T>::pack(v[8 * j + 0], v[8 * j + 1]);
          o.y = Pack<T>::pack(v[8 * j + 2], v[8 * j + 3]);
          o.z = Pack<T>::pack(v[8 * j + 4], v[8 * j + 5]);
          o.w = Pack<T>::pack(v[8 * j + 6], v[8 * j + 7]);
          st_shared_v4(stage_addr + lane * 128 + ((j ^ (lane & 7)) << 4), o);
          if (emit_p6)
            reinterpret_cast<uint4*>(p6_row + static_cast<size_t>(col0) * sizeof(T))[j] = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_4d(&jb.map_out, smem_stage + ew * kTcStagingPerWarp, col0, ox, oy, n);
          bulk_commit_group();
        }
      }
      if (staged) cphase ^= 1u;
      if (lateral && jb.publish) {
        // Publish the tile: own stores complete -> all epilogue warps -> one release add.
        if (lane == 0) {
          bulk_wait_group<0>();
          fence_proxy_async_all();
          __threadfence();
        }
        __syncwarp();
        epi_bar_sync();  // also: every warp is done reading this tile's coarse box
        if (leader) {
          const int before = atom_release_gpu_add(&sched[1 + jb.level], 1);
          if (P.trace && before + 1 == P.lat_tiles[jb.level])
            P.trace[1 + jb.level] = globaltimer_ns();
        }
      } else if (staged) {
        epi_bar_sync();  // every warp is done reading this tile's coarse box
      }
      if (P.trace && lateral && !jb.publish && leader)
        atomicMax(&P.trace[1 + jb.level], globaltimer_ns());  // stores issued, not complete
      }  // final_unit
      // The coarse buffer is free (lateral tiles passed the barrier above; other
      // tiles do not read it): prefetch the next tile's coarse box if that tile is
      // a lateral with a top-down add.
      if (leader && ok) {
        if (mbar_wait(&rfull_bar[rslot], rphase, abort_flag, P.status, kDevTimeoutEpilogue)) {
          const int tn = ring[rslot];
          if (tn >= 0) {
            const NeckJob& jn = P.jobs[neck_find_job(P, tn)];
            if (jn.mode == 0 && jn.coarse != nullptr && jn.ksplit <= 1)
              ok = request_coarse(jn, tn);
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
  if (threadIdx.x == 0) {
    if (P.trace) atomicMax(&P.trace[5], globaltimer_ns());
    // The last CTA to leave resets the schedule counters for the next launch.
    __threadfence();
    if (atomicAdd(&sched[7], 1) == static_cast<int>(gridDim.x) - 1) {
      for (int i = 0; i < 8; ++i) sched[i] = 0;
      __threadfence();
    }
  }
}

}  // namespace ufpn
