// 3x3 conv with halo reuse on CTA PAIRS (tcgen05 cta_group::2).
//
// Same math, tiles and epilogue as fpn_conv3x3_halo_kernel (tc_gemm.cuh), but the two CTAs
// of a (2,1,1) cluster run ONE tcgen05.mma stream of M = 256 rows: the leader's 8x16 tile
// (rows 0..127) and the next tile (rows 128..255, the peer's).  Each CTA stages its own
// tile's halo (A) and HALF of every weight k-block (B: output channels 128*rank..+127), so
// the weight stream each SM pulls from L2 per tile halves; the leader issues the MMAs,
// which read both CTAs' shared memory and write each CTA's 128 accumulator lanes in its
// own TMEM.
//
// Tail items (args.pair_tail > 0): when the last round of pair units would leave pairs idle,
// each of the last pair_tail units runs as two items over the output channels (M = 256,
// N = 128; each CTA stages 64 rows of every weight k-block through map_bh, a 64-row box),
// so the last round takes about half as long.  Each output element accumulates over the
// same K order either way: the results are bitwise those of whole units.
//
// Synchronisation (all waits bounded, as everywhere in this library):
//   full[s], hfull[h]  leader's barriers; the leader's producer arms them with BOTH CTAs'
//                      byte counts, both producers' TMA loads complete on them
//   empty[s], hempty[h] per CTA; the leader's MMA thread releases a stage in both CTAs
//                      with one tcgen05.commit to the same offset in both
//   accf[a]            per CTA, same commit; the epilogue of each CTA waits on its own
//   acce[a]            leader's; 16 warp arrivals (8 epilogue warps per CTA)
// A cluster barrier after initialisation and another before TMEM is released keep either
// CTA from touching the other's shared memory or TMEM outside their lifetimes.
//
// kCvt (e4m3 only): the input is the bf16 merged map and its per-image absmax; each CTA's
// producer brings the bf16 halo (two 64-channel boxes) into a raw buffer (rfull / rempty,
// local), and 4 converter warps quantise it into the e4m3 halo buffer exactly as the
// standalone quantiser does (e4m3(x * 448 / amax[n]), nearest even, saturated), then arrive
// on the leader's hfull (8 arrivals: 4 warps x 2 CTAs).  No separate quantise pass and no
// e4m3 copy of the map in HBM.
#pragma once

#include "tc_gemm.cuh"

namespace ufpn {

constexpr int kPairBStage = (kTcBlockN / 2) * 128;  // half of a weight k-block: 16 KB
constexpr int kPairCvtWarps = 4;
template <bool kCvt>
struct PairCfgT {
  static constexpr int kStages = kCvt ? 6 : 8;
  static constexpr int kThreads = kTcThreads + (kCvt ? 32 * kPairCvtWarps : 0);
  static constexpr int kOffHalo = kStages * kPairBStage;
  static constexpr int kOffRaw = kOffHalo + kHaloBufs * kHaloBytes;  // kCvt: 2 bf16 boxes
  static constexpr int kOffStaging = kOffRaw + (kCvt ? 2 * kHaloBytes : 0);
  static constexpr int kOffBars = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kSmemBytes = kOffBars + 512 + 1024;
};
using PairCfg = PairCfgT<false>;
static_assert(PairCfgT<false>::kSmemBytes <= 232448 && PairCfgT<true>::kSmemBytes <= 232448,
              "pair smem");

template <typename T>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (TcElem<T>::kFp8)
    tc_mma_f8_pair(d_tmem, adesc, bdesc, idesc, accumulate);
  else
    tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, accumulate);
}

// Bounded idle wait (teardown after an abort: lets copies already in flight land).
__device__ __forceinline__ void pair_settle_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}

template <typename T, bool kCvt = false, bool kClaims = false>
__global__ void __launch_bounds__(PairCfgT<kCvt>::kThreads, 1)
    fpn_conv3x3_halo_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                                 const __grid_constant__ CUtensorMap map_b,
                                 const __grid_constant__ CUtensorMap map_out,
                                 const __grid_constant__ CUtensorMap map_bh,
                                 const __grid_constant__ CUtensorMap map_a2,
                                 const __grid_constant__ CUtensorMap map_out2,
                                 const TcGemmArgs args) {
  static_assert(!kCvt || TcElem<T>::kFp8, "the converter quantises to e4m3");
  using Cfg = PairCfgT<kCvt>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  // Both CTAs compute the same aligned offset (same dynamic shared memory layout).
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_b = smem;
  uint8_t* smem_halo = smem + Cfg::kOffHalo;
  uint8_t* smem_rawbuf = smem + Cfg::kOffRaw;
  uint8_t* smem_stage = smem + Cfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* hfull_bar = bars + 2 * S;
  uint64_t* hempty_bar = hfull_bar + kHaloBufs;
  uint64_t* accf_bar = hempty_bar + kHaloBufs;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint64_t* rfull_bar = done_bar + 1;   // kCvt
  uint64_t* rempty_bar = rfull_bar + 1;  // kCvt
  uint64_t* cfull_bar = rempty_bar + 1;  // claim ring [kClaimRecs]
  uint64_t* cempty_bar = cfull_bar + kClaimRecs;  // claim ring, the leader's [kClaimRecs]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cempty_bar + kClaimRecs);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* claim_rec = abort_flag + 1;  // [kClaimRecs]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cin_blocks = args.cin_blocks;
  const int units = (args.num_tiles + 1) / 2;
  const int items = units + args.pair_tail;  // work items (pair_item_unit)
  const int u0 = static_cast<int>(blockIdx.x >> 1);
  const int ustep = static_cast<int>(gridDim.x >> 1);
  // Dynamic claims: every role but the claimer reads the items from the ring; per CTA the
  // readers are the epilogue warps, the converter warps and one thread (the MMA issuer in
  // the leader, the producer in the peer).
  constexpr bool dyn = kClaims;  // (the launcher: kClaims == (args.claim != nullptr))
  constexpr int kClaimReaders = 2 * (kTcEpiWarps + 1 + (kCvt ? kPairCvtWarps : 0));
  ClaimRing ring{claim_rec, cfull_bar, mapa_shared(smem_u32(cempty_bar), 0), 0, 0u};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int h = 0; h < kHaloBufs; ++h) {
      mbar_init(&hfull_bar[h], kCvt ? 2 * kPairCvtWarps : 1);
      mbar_init(&hempty_bar[h], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 2 * kTcEpiWarps);
    }
    mbar_init(done_bar, 1);
    mbar_init(rfull_bar, 1);
    mbar_init(rempty_bar, kPairCvtWarps);
    for (int r = 0; r < kClaimRecs; ++r) {
      mbar_init(&cfull_bar[r], 1);
      mbar_init(&cempty_bar[r], kClaimReaders);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    prefetch_tmap(&map_out);
    if (args.pair_tail > 0) prefetch_tmap(&map_bh);
    if (args.strip_first > 0) {
      prefetch_tmap(&map_a2);
      prefetch_tmap(&map_out2);
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
      int stage = 0, hb = 0;
      uint32_t phase = 0, hphase = 0;
      bool ok = true;
      const uint32_t full0 = mapa_shared(smem_u32(full_bar), 0);
      const uint32_t hfull0 = mapa_shared(smem_u32(hfull_bar), 0);
      uint32_t rphase = 0;
      // Dynamic claims (leader): the next item is claimed as the current item's last channel
      // block starts, so that the atomic's round trip overlaps that block's nine weight loads,
      // and published once the current item's loads are all issued.
      int cslot = 0;
      uint32_t cphase = 0;
      int pending = 0;
      auto claim_begin = [&]() -> bool {
        if (!mbar_wait_acq_cluster(&cempty_bar[cslot], cphase ^ 1u, abort_flag, args.status,
                                   kDevTimeoutProducer))
          return false;
        pending = atomicAdd(args.claim, 1);
        return true;
      };
      auto claim_end = [&](int& item) {
        item = pending < items ? pending : items;
        claim_publish(claim_rec, cfull_bar, cslot, item);
        if (++cslot == kClaimRecs) {
          cslot = 0;
          cphase ^= 1u;
        }
      };
      int it = u0;
      if (dyn) {
        if (leader) {
          ok = claim_begin();
          if (ok) claim_end(it);
        } else {
          ok = ring.next(it, abort_flag, args.status, kDevTimeoutProducer);
        }
      }
      for (; ok && it < items;) {
        int half;
        const int u = pair_item_unit(args, units, it, half);
        // weight rows this CTA stages per k-block: 128 of 256, or 64 of a half's 128
        const int brow = half < 0 ? static_cast<int>(rank) * (kTcBlockN / 2)
                                  : half * (kTcBlockN / 2) + static_cast<int>(rank) * (kTcBlockN / 4);
        const CUtensorMap* mb = half < 0 ? &map_b : &map_bh;
        const uint32_t bbytes = half < 0 ? 2 * kPairBStage : kPairBStage;  // both CTAs
        const HaloTile ht = halo_tile(args, 2 * u + static_cast<int>(rank));
        const int n = ht.n, x0 = ht.x0, y0 = ht.y0;
        const CUtensorMap* ma = ht.strip ? &map_a2 : &map_a;
        for (int cb = 0; ok && cb < cin_blocks; ++cb) {
          if (dyn && leader && cb == cin_blocks - 1 && !claim_begin()) {
            ok = false;
            break;
          }
          if constexpr (kCvt) {
            // bf16 halo (channels cb*128 .. +127 as two 64-channel boxes) for the converter
            if (!mbar_wait(rempty_bar, rphase ^ 1u, abort_flag, args.status,
                           kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(rfull_bar, 2 * kHaloRows * 128);
            for (int j = 0; j < 2; ++j)
              tma_load_4d(smem_rawbuf + j * kHaloBytes, ma, rfull_bar, cb * 128 + j * 64,
                          x0 - 1, y0 - 1, n, kPolicyEvictLast);
            rphase ^= 1u;
          } else {
            if (!mbar_wait(&hempty_bar[hb], hphase ^ 1u, abort_flag, args.status,
                           kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&hfull_bar[hb], 2 * kHaloRows * 128);
            tma_load_4d_pair(smem_halo + hb * kHaloBytes, ma, hfull0 + hb * 8u,
                             cb * kKbElems<T>, x0 - 1, y0 - 1, n, kPolicyEvictLast);
            if (++hb == kHaloBufs) {
              hb = 0;
              hphase ^= 1u;
            }
          }
          for (int tap = 0; tap < 9; ++tap) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                           kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], bbytes);
            tma_load_2d_pair(smem_b + stage * kPairBStage, mb, full0 + stage * 8u,
                             (tap * cin_blocks + cb) * kKbElems<T>, brow, kPolicyEvictLast);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!dyn)
          it += ustep;
        else if (ok && leader)
          claim_end(it);
        else if (ok)
          ok = ring.next(it, abort_flag, args.status, kDevTimeoutProducer);
      }
      griddep_launch_dependents();  // this CTA's last loads are issued
      // Copies in flight complete on the leader's barriers; after an abort, give them time
      // to land before this CTA's shared memory can go away.
      if (!ok) pair_settle_ns(1000000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc_full =
          make_idesc(2 * kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt);
      constexpr uint32_t idesc_half =
          make_idesc(2 * kTcBlockM, kTcBlockN / 2, TcElem<T>::kFmt, TcElem<T>::kFmt);
      int stage = 0, hb = 0, acc = 0;
      uint32_t phase = 0, hphase = 0, acc_phase = 0;
      bool ok = true;
      for (int it = u0;; it += ustep) {
        if (dyn && !ring.next(it, abort_flag, args.status, kDevTimeoutMma)) break;
        if (!ok || it >= items) break;
        int half;
        const int u = pair_item_unit(args, units, it, half);
        const uint32_t idesc = half < 0 ? idesc_full : idesc_half;
        // (both tiles of a unit are of one view: one tap offset for both CTAs' halos)
        const int tr = halo_tile(args, 2 * u).tr;
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        for (int cb = 0; ok && cb < cin_blocks; ++cb) {
          if (!mbar_wait(&hfull_bar[hb], hphase, abort_flag, args.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t halo_addr = smem_u32(smem_halo + hb * kHaloBytes);
          for (int tap = 0; tap < 9; ++tap) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t adesc = sdesc_kmajor_sw128_stride(
                halo_addr + static_cast<uint32_t>(halo_tap_offset(tap, tr) * 128),
                (kHaloTileW + 2) * 128);
            const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kPairBStage));
#pragma unroll
            for (int k = 0; k < kMmaPerKb; ++k)
              tc_mma_pair<T>(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                             (cb > 0 || tap > 0 || k > 0) ? 1u : 0u);
            tc_commit_pair_both(&empty_bar[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit_pair_both(&hempty_bar[hb]);
          if (++hb == kHaloBufs) {
            hb = 0;
            hphase ^= 1u;
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
  } else if (warp < 2 + kTcEpiWarps) {
    tc_epilogue<1, T, true>(args, &map_out, tmem_base, accf_bar, acce_bar, smem_stage,
                            abort_flag, warp, lane, false,
                            mapa_shared(smem_u32(acce_bar), 0), nullptr,
                            kClaims ? &ring : nullptr, &map_out2);
  } else if constexpr (kCvt) {
    // ------------------------------------------------------------ converter (each CTA)
    const int ct = threadIdx.x - 32 * (2 + kTcEpiWarps);  // 0 .. 32 * kPairCvtWarps - 1
    const uint32_t hfull0 = mapa_shared(smem_u32(hfull_bar), 0);
    const uint32_t raw_addr0 = smem_u32(smem_rawbuf);
    int hb = 0;
    uint32_t hphase = 0, rphase = 0;
    bool ok = true;
    for (int it = u0;; it += ustep) {
      if (dyn && !ring.next_warp(it, lane, abort_flag, args.status, kDevTimeoutProducer)) break;
      if (!ok || it >= items) break;
      int half;
      const int tile = 2 * pair_item_unit(args, units, it, half) + static_cast<int>(rank);
      const int n = halo_tile(args, tile).n;
      // virtual tile (past the end): its halo is all padding, any finite scale will do
      const unsigned am = tile < args.num_tiles ? __ldg(args.in_amax + n) : 0u;
      const float inv = e4m3_inv_of(am);
      for (int cb = 0; ok && cb < cin_blocks; ++cb) {
        bool w = mbar_wait(rfull_bar, rphase, abort_flag, args.status, kDevTimeoutProducer);
        if (w) w = mbar_wait(&hempty_bar[hb], hphase ^ 1u, abort_flag, args.status,
                             kDevTimeoutProducer);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        const uint32_t dst0 = smem_u32(smem_halo + hb * kHaloBytes);
        // item = (halo row r, 16-channel group g): 32 bf16 bytes -> 16 e4m3 bytes
        for (int it = ct; it < kHaloRows * 8; it += 32 * kPairCvtWarps) {
          const int r = it >> 3, g = it & 7;
          const uint32_t src = raw_addr0 + (g >> 2) * kHaloBytes + r * 128;
          const int c0 = (g & 3) * 2;
          const uint4 lo = ld_shared_v4(src + (((c0) ^ (r & 7)) << 4));
          const uint4 hi = ld_shared_v4(src + (((c0 + 1) ^ (r & 7)) << 4));
          const float2 f0 = Pack<__nv_bfloat16>::unpack(lo.x), f1 = Pack<__nv_bfloat16>::unpack(lo.y);
          const float2 f2 = Pack<__nv_bfloat16>::unpack(lo.z), f3 = Pack<__nv_bfloat16>::unpack(lo.w);
          const float2 f4 = Pack<__nv_bfloat16>::unpack(hi.x), f5 = Pack<__nv_bfloat16>::unpack(hi.y);
          const float2 f6 = Pack<__nv_bfloat16>::unpack(hi.z), f7 = Pack<__nv_bfloat16>::unpack(hi.w);
          uint4 q;
          q.x = tc_e4m3x4(f0.x, f0.y, f1.x, f1.y, inv);
          q.y = tc_e4m3x4(f2.x, f2.y, f3.x, f3.y, inv);
          q.z = tc_e4m3x4(f4.x, f4.y, f5.x, f5.y, inv);
          q.w = tc_e4m3x4(f6.x, f6.y, f7.x, f7.y, inv);
          st_shared_v4(dst0 + r * 128 + ((g ^ (r & 7)) << 4), q);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(rempty_bar);                       // raw buffer consumed
          mbar_arrive_cluster(hfull0 + hb * 8u);         // e4m3 halo ready (leader's barrier)
        }
        rphase ^= 1u;
        if (++hb == kHaloBufs) {
          hb = 0;
          hphase ^= 1u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs are drained; no CTA touches the other any more
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTcTmemCols);
  }
  if (dyn && threadIdx.x == 0) {
    // The last CTA to leave (every claim of the launch is made by then) resets the counters
    // for the next launch.
    __threadfence();
    if (atomicAdd(args.claim + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      args.claim[0] = 0;
      args.claim[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace ufpn
