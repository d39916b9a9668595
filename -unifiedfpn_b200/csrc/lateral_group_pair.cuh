// Raw 1x1 laterals of several levels (the split schedule's P5, P4 and P3) in ONE launch on
// CTA PAIRS, weights streamed.
//
// The grouped single-CTA launch (fpn_neck_kernel with three lateral jobs) streams, per
// k-block, a 16 KB activation box and a full 32 KB weight box through each SM, and its
// k-block time is set by how many bytes an SM has in flight (the TMA round trip under load,
// about 2 us, over 4 stages).  Here the two CTAs of a (2,1,1) cluster run one tcgen05.mma
// stream of M = 256 (the leader's tile in rows 0..127, the next tile of the same level in
// rows 128..255, the peer's) and each CTA stages its own tile's activations and HALF of
// every weight k-block (output channels 128*rank..+127): 32 KB per k-block per SM instead of
// 48, so 6 stages fit where 4 did.  The deepest tiles, P5's 32 k-blocks, set the launch's
// length; on pairs each SM's share of them is both smaller and faster to feed.
//
// Channel halves (a job's nsplit = 2): each of its pair units runs as two items of N = 128
// (M = 256, each CTA staging 64 rows of every weight k-block through map_bh), so a deep
// unit (P5's 32 k-blocks) holds its pair about half as long; same bits as whole units.
//
// Schedule: static, computed on the host (plan_lateral_group_pair): the pair units (two
// consecutive tiles of one level) are dealt longest first to the least-loaded pair, so the
// 32-k-block P5 units start first and the short P3 units fill in behind them.  Each pair
// walks its own list; both CTAs of a pair read the same list, so nothing is exchanged at run
// time.  Same arithmetic as the single-CTA lateral (fp32 accumulation over the same K order,
// + bias, one rounding): the outputs are bitwise those of the grouped neck launch.
//
// Synchronisation (all waits bounded, as everywhere in this library):
//   full[s]            leader's; both CTAs' loads of stage s complete on it
//   empty[s], accf[a]  per CTA; the leader's MMA thread signals both with one commit
//   acce[a]            leader's; 16 warp arrivals (8 epilogue warps per CTA)
// Cluster barriers after initialisation and before TMEM is released, as in conv_pair.cuh.
#pragma once

#include "conv_pair.cuh"

namespace ufpn {

constexpr int kLgMaxJobs = 3;
constexpr int kLgMaxPairs = 128;
constexpr int kLgMaxItems = 2048;
constexpr int kLgStages = 6;

struct LgJob {
  CUtensorMap map_a;    // C_l NHWC, box (64 channels, tile_w, tile_h, 1)
  CUtensorMap map_b;    // weights [256][Cin], box (64, 128 rows): one CTA's half
  CUtensorMap map_out;  // L_l NHWC, box (64, min(tile_w, 32), 32 / that, 1)
  CUtensorMap map_bh;   // nsplit 2: weights, box (64, 64 rows): one CTA's half of a half
  const float* bias;    // [256]
  int num_tiles, num_kb, nsplit;
  int N_img, H, W;
  int tile_w, tile_h, tiles_x, tiles_y;
};

struct LgParams {
  LgJob jobs[kLgMaxJobs];
  int num_jobs;
  int num_pairs;
  int* status;
  // pair p's items: items[off[p] .. off[p + 1]), each (job << 14) | (part << 12) | unit:
  // unit u = tiles 2u and 2u + 1 of that job (a missing second tile is computed on
  // zero-filled input, never stored); part 0 = all 256 output channels, 1 / 2 = channels
  // 0..127 / 128..255 (N = 128)
  unsigned short off[kLgMaxPairs + 1];
  unsigned short items[kLgMaxItems];
};

struct LgCfg {
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kLgStages * kTcAStage;
  static constexpr int kOffStaging = kOffB + kLgStages * kPairBStage;
  static constexpr int kOffBars = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kSmemBytes = kOffBars + 256 + 1024;
};
static_assert(LgCfg::kSmemBytes <= 232448, "lateral group pair smem");

__device__ __forceinline__ int lg_job(unsigned it) { return static_cast<int>(it >> 14); }
__device__ __forceinline__ int lg_part(unsigned it) { return static_cast<int>((it >> 12) & 3u); }
__device__ __forceinline__ int lg_unit(unsigned it) { return static_cast<int>(it & 0xFFFu); }

__device__ __forceinline__ void lg_tile_origin(const LgJob& jb, int tile, int& n, int& x0,
                                               int& y0) {
  const int tx = tile % jb.tiles_x;
  const int t2 = tile / jb.tiles_x;
  const int ty = t2 % jb.tiles_y;
  n = t2 / jb.tiles_y;
  x0 = tx * jb.tile_w;
  y0 = ty * jb.tile_h;
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_lateral_group_pair_kernel(const __grid_constant__ LgParams P) {
  static_assert(!TcElem<T>::kFp8, "16-bit inputs");
  constexpr int S = kLgStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  // Both CTAs compute the same aligned offset (same dynamic shared memory layout).
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem + LgCfg::kOffA;
  uint8_t* smem_b = smem + LgCfg::kOffB;
  uint8_t* smem_stage = smem + LgCfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LgCfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* accf_bar = bars + 2 * S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int i0 = pair < P.num_pairs ? P.off[pair] : 0;
  const int i1 = pair < P.num_pairs ? P.off[pair + 1] : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 2 * kTcEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    for (int j = 0; j < P.num_jobs; ++j) {
      prefetch_tmap(&P.jobs[j].map_a);
      prefetch_tmap(&P.jobs[j].map_b);
      prefetch_tmap(&P.jobs[j].map_out);
      if (P.jobs[j].nsplit > 1) prefetch_tmap(&P.jobs[j].map_bh);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTcTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in BOTH CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // (programmatic launch) the previous kernel's results are visible

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (each CTA)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full_bar), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = i0; ok && i < i1; ++i) {
        const LgJob& jb = P.jobs[lg_job(P.items[i])];
        const int part = lg_part(P.items[i]);
        // weight rows this CTA stages per k-block: 128 of 256, or 64 of a half's 128
        const int brow = part == 0 ? static_cast<int>(rank) * (kTcBlockN / 2)
                                   : (part - 1) * (kTcBlockN / 2) +
                                         static_cast<int>(rank) * (kTcBlockN / 4);
        const CUtensorMap* mb = part == 0 ? &jb.map_b : &jb.map_bh;
        const uint32_t bytes = 2u * (kTcAStage + (part == 0 ? kPairBStage : kPairBStage / 2));
        int n, x0, y0;
        lg_tile_origin(jb, 2 * lg_unit(P.items[i]) + static_cast<int>(rank), n, x0, y0);
        for (int kb = 0; kb < jb.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, P.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], bytes);
          tma_load_4d_pair(smem_a + stage * kTcAStage, &jb.map_a, full0 + stage * 8u,
                           kb * kTcBlockK, x0, y0, n, kPolicyEvictFirst);
          tma_load_2d_pair(smem_b + stage * kPairBStage, mb, full0 + stage * 8u,
                           kb * kTcBlockK, brow, kPolicyEvictLast);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      griddep_launch_dependents();  // this CTA's last loads are issued
      // Copies in flight complete on barriers that may be the leader's; after an abort, give
      // them time to land before this CTA's shared memory can go away.
      if (!ok) pair_settle_ns(1000000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc_full =
          make_idesc(2 * kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt);
      constexpr uint32_t idesc_half =
          make_idesc(2 * kTcBlockM, kTcBlockN / 2, TcElem<T>::kFmt, TcElem<T>::kFmt);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int i = i0; ok && i < i1; ++i) {
        const int nkb = P.jobs[lg_job(P.items[i])].num_kb;
        const uint32_t idesc = lg_part(P.items[i]) == 0 ? idesc_full : idesc_half;
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, P.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, P.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(smem_a + stage * kTcAStage));
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kPairBStage));
#pragma unroll
          for (int k = 0; k < kMmaPerKb; ++k)
            tc_mma_pair<T>(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                           (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair_both(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_both(&accf_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued must finish before either CTA releases its TMEM.
      tc_commit_pair_local(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (each CTA)
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter..+31 (hardware: warp id % 4)
    const int chalf = ew >> 2;     // output channels chalf*128 .. +127
    const uint32_t stage_addr = smem_u32(smem_stage + ew * kTcStagingPerWarp);
    const uint32_t leader_acce = mapa_shared(smem_u32(acce_bar), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = i0; i < i1; ++i) {
      const LgJob& jb = P.jobs[lg_job(P.items[i])];
      const int part = lg_part(P.items[i]);
      const int tile = 2 * lg_unit(P.items[i]) + static_cast<int>(rank);
      const bool real = tile < jb.num_tiles;
      const bool ok =
          mbar_wait(&accf_bar[acc], acc_phase, abort_flag, P.status, kDevTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      int n, x0, y0;
      lg_tile_origin(jb, tile, n, x0, y0);
      const int tw = jb.tile_w;
      const int wrow0 = quarter * 32;
      const int ox = x0 + (wrow0 % tw);
      const int oy = y0 + wrow0 / tw;
      // a half item's N = 128 accumulator: columns 0..127 of the buffer, 64 per warp
      const int nsteps = part == 0 ? 2 : 1;
      const int tcol0 = part == 0 ? chalf * 128 : chalf * 64;
      const int ocol0 = part == 0 ? tcol0 : (part - 1) * 128 + tcol0;
#pragma unroll 1
      for (int step = 0; step < nsteps; ++step) {
        const int col0 = ocol0 + step * 64;  // output channel of the step's first column
        const uint32_t taddr = tmem_base +
                               static_cast<uint32_t>(acc * kTcBlockN + tcol0 + step * 64) +
                               (static_cast<uint32_t>(quarter * 32) << 16);
        // both 32-column halves of the step with one wait
        uint32_t r[64];
        __syncwarp();
        tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        if (lane == 0) bulk_wait_group_read<0>();  // the staging buffer's last store read it
        tmem_wait_ld();
        if (step == nsteps - 1) {
          // every accumulator column of this warp is in registers: free the TMEM buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_acce + static_cast<uint32_t>(acc) * 8u);
        }
        __syncwarp();
        const float4* b4 = reinterpret_cast<const float4*>(jb.bias + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16-byte chunk j of the 128-byte staging row
          const float4 ba = __ldg(b4 + 2 * j);
          const float4 bb = __ldg(b4 + 2 * j + 1);
          uint4 o;
          o.x = Pack<T>::pack(__uint_as_float(r[8 * j + 0]) + ba.x,
                              __uint_as_float(r[8 * j + 1]) + ba.y);
          o.y = Pack<T>::pack(__uint_as_float(r[8 * j + 2]) + ba.z,
                              __uint_as_float(r[8 * j + 3]) + ba.w);
          o.z = Pack<T>::pack(__uint_as_float(r[8 * j + 4]) + bb.x,
                              __uint_as_float(r[8 * j + 5]) + bb.y);
          o.w = Pack<T>::pack(__uint_as_float(r[8 * j + 6]) + bb.z,
                              __uint_as_float(r[8 * j + 7]) + bb.w);
          st_shared_v4(stage_addr + lane * 128 + ((j ^ (lane & 7)) << 4), o);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // every use commits a group (empty for the virtual tile past the end)
          if (real)
            tma_store_4d(&jb.map_out, smem_stage + ew * kTcStagingPerWarp, col0, ox, oy, n);
          bulk_commit_group();
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
  cluster_sync_all();  // the leader's MMAs are drained; no CTA touches the other any more
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTcTmemCols);
  }
}

}  // namespace ufpn
