// 1x1 lateral (+ bias + bilinear top-down add) on CTA PAIRS with resident weights.
//
// The single-CTA lateral (fpn_tc_gemm_kernel, mode 0) streams a full 32 KB weight k-block
// with every 16 KB activation k-block, so per tile most of its shared-memory fill is weights
// that every tile reloads.  Here the two CTAs of a (2,1,1) cluster run ONE tcgen05.mma
// stream of M = 256 rows (the leader's 128-pixel tile in rows 0..127, the next tile in rows
// 128..255, the peer's), and each CTA keeps HALF of the weights -- output channels
// 128*rank..+127, every k-block -- resident in shared memory for the whole launch.  Per tile
// a CTA then moves only its activations (16 KB per k-block) and its tile's coarse box.
//
// The top-down add is done in the epilogue: each CTA stages its own tile's coarse box of
// M_{l+1} (TMA, 4 boxes of 64 channels, double-buffered) and every epilogue thread adds the
// four bilinear taps of its pixel from shared memory (fp32: acc + bias + sum of taps, one
// rounding), as the grouped neck kernel does.  Semantics: lib/kernels/compute/
// fpn_compute_kernels.cu:127-230 (1x1 conv + bias) and the top-down upsample + add of
// lib/core/fpn_engine.cu:274-313.
//
// Synchronisation (all waits bounded):
//   bfull              leader's; both CTAs' resident weight loads complete on it (once)
//   full[s]            leader's; both CTAs' activation k-blocks of stage s complete on it
//   empty[s], accf[a]  per CTA; the leader's MMA thread signals both with one commit
//   acce[a]            leader's; 16 warp arrivals (8 epilogue warps per CTA)
//   cfull[c], cempty[c] per CTA (its own coarse box; 8 epilogue-warp arrivals free it)
// Cluster barriers after initialisation and before TMEM is released, as in conv_pair.cuh.
#pragma once

#include "conv_pair.cuh"

namespace ufpn {

constexpr int kLpMaxKb = 4;  // resident weight k-blocks (Cin <= 256 for 16-bit inputs)
constexpr int kLpStages = 4;
constexpr int kLpCoarseBufBytes = kTcCoarseMaxPix * 128 * 4;  // 64 px x 256 ch x 2 bytes
struct LpCfg {
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kLpMaxKb * kPairBStage;
  static constexpr int kOffCoarse = kOffA + kLpStages * kTcAStage;
  static constexpr int kOffStaging = kOffCoarse + 2 * kLpCoarseBufBytes;
  static constexpr int kOffBars = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kSmemBytes = kOffBars + 256 + 1024;
};
static_assert(LpCfg::kSmemBytes <= 232448, "lateral pair smem");

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_lateral_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b,
                            const __grid_constant__ CUtensorMap map_out,
                            const __grid_constant__ CUtensorMap map_coarse,
                            const TcGemmArgs args) {
  static_assert(!TcElem<T>::kFp8, "16-bit inputs");
  constexpr int S = kLpStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_b = smem + LpCfg::kOffB;
  uint8_t* smem_a = smem + LpCfg::kOffA;
  uint8_t* smem_coarse = smem + LpCfg::kOffCoarse;
  uint8_t* smem_stage = smem + LpCfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LpCfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* bfull_bar = bars + 2 * S;
  uint64_t* cfull_bar = bfull_bar + 1;
  uint64_t* cempty_bar = cfull_bar + 2;
  uint64_t* accf_bar = cempty_bar + 2;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int nkb = args.num_kb;  // <= kLpMaxKb (host)
  const int units = (args.num_tiles + 1) / 2;
  const int u0 = static_cast<int>(blockIdx.x >> 1);
  const int ustep = static_cast<int>(gridDim.x >> 1);
  const bool has_coarse = args.coarse != nullptr && args.cbox_w > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(bfull_bar, 1);
    for (int c = 0; c < 2; ++c) {
      mbar_init(&cfull_bar[c], 1);
      mbar_init(&cempty_bar[c], kTcEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 2 * kTcEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    prefetch_tmap(&map_out);
    if (has_coarse) prefetch_tmap(&map_coarse);
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
      const uint32_t bfull0 = mapa_shared(smem_u32(bfull_bar), 0);
      const int brow = static_cast<int>(rank) * (kTcBlockN / 2);
      // resident weights: this CTA's 128 output channels, every k-block
      if (leader) mbar_arrive_expect_tx(bfull_bar, 2u * nkb * kPairBStage);
      for (int kb = 0; kb < nkb; ++kb)
        tma_load_2d_pair(smem_b + kb * kPairBStage, &map_b, bfull0, kb * kTcBlockK, brow,
                         kPolicyEvictLast);
      const uint32_t box_bytes = static_cast<uint32_t>(args.cbox_w * args.cbox_h * 128 * 4);
      int stage = 0, cb = 0;
      uint32_t phase = 0, cphase = 0;
      bool ok = true;
      for (int u = u0; ok && u < units; u += ustep) {
        int n, x0, y0;
        tc_tile_origin(args, 2 * u + static_cast<int>(rank), n, x0, y0);
        if (has_coarse) {
          if (!mbar_wait(&cempty_bar[cb], cphase ^ 1u, abort_flag, args.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const int cy = static_cast<int>(tc_src(y0, args.scale_y, args.Hc));
          const int cx = static_cast<int>(tc_src(x0, args.scale_x, args.Wc));
          mbar_arrive_expect_tx(&cfull_bar[cb], box_bytes);
          for (int b = 0; b < 4; ++b)
            tma_load_4d(smem_coarse + cb * kLpCoarseBufBytes + b * (kTcCoarseMaxPix * 128),
                        &map_coarse, &cfull_bar[cb], b * 64, cx, cy, n, kPolicyEvictLast);
          if (++cb == 2) {
            cb = 0;
            cphase ^= 1u;
          }
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2u * kTcAStage);
          tma_load_4d_pair(smem_a + stage * kTcAStage, &map_a, full0 + stage * 8u,
                           kb * kTcBlockK, x0, y0, n, kPolicyEvictFirst);
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
      constexpr uint32_t idesc =
          make_idesc(2 * kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = mbar_wait(bfull_bar, 0, abort_flag, args.status, kDevTimeoutMma);
      for (int u = u0; ok && u < units; u += ustep) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(smem_a + stage * kTcAStage));
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + kb * kPairBStage));
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
    const int row = quarter * 32 + lane;
    const int tw = args.tile_w;
    const uint32_t stage_addr = smem_u32(smem_stage + ew * kTcStagingPerWarp);
    const uint32_t leader_acce = mapa_shared(smem_u32(acce_bar), 0);
    const uint32_t coarse_addr = smem_u32(smem_coarse);
    constexpr int kCoarseBlk = kTcCoarseMaxPix * 128;
    int acc = 0, cb = 0;
    uint32_t acc_phase = 0, cphase = 0;
    for (int u = u0; u < units; u += ustep) {
      const int tile = 2 * u + static_cast<int>(rank);
      const bool real = tile < args.num_tiles;
      bool ok = mbar_wait(&accf_bar[acc], acc_phase, abort_flag, args.status,
                          kDevTimeoutEpilogue);
      if (ok && has_coarse)
        ok = mbar_wait(&cfull_bar[cb], cphase, abort_flag, args.status, kDevTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();

      int n, x0, y0;
      tc_tile_origin(args, tile, n, x0, y0);
      const int py = y0 + row / tw;
      const int px = x0 + row % tw;
      // bilinear taps of this thread's pixel, as offsets into the staged coarse box (or, if
      // the box cannot hold them, global addresses)
      float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
      int r00 = 0, r01 = 0, r10 = 0, r11 = 0;
      bool staged = false;
      const uint8_t* g00 = nullptr;
      const uint8_t* g01 = nullptr;
      const uint8_t* g10 = nullptr;
      const uint8_t* g11 = nullptr;
      if (has_coarse) {
        const TcTaps tp =
            tc_taps(py, px, args.H, args.W, args.Hc, args.Wc, args.scale_y, args.scale_x);
        w00 = tp.w00;
        w01 = tp.w01;
        w10 = tp.w10;
        w11 = tp.w11;
        const int cy0 = static_cast<int>(tc_src(y0, args.scale_y, args.Hc));
        const int cx0 = static_cast<int>(tc_src(x0, args.scale_x, args.Wc));
        staged = (tp.ya - cy0) >= 0 && (tp.yb - cy0) < args.cbox_h && (tp.xa - cx0) >= 0 &&
                 (tp.xb - cx0) < args.cbox_w;
        r00 = (tp.ya - cy0) * args.cbox_w + (tp.xa - cx0);
        r01 = (tp.ya - cy0) * args.cbox_w + (tp.xb - cx0);
        r10 = (tp.yb - cy0) * args.cbox_w + (tp.xa - cx0);
        r11 = (tp.yb - cy0) * args.cbox_w + (tp.xb - cx0);
        if (!staged) {
          const size_t rowb = static_cast<size_t>(kTcBlockN) * sizeof(T);
          const uint8_t* cbase = static_cast<const uint8_t*>(args.coarse) +
                                 static_cast<size_t>(real ? n : 0) * args.Hc * args.Wc * rowb;
          g00 = cbase + (static_cast<size_t>(tp.ya) * args.Wc + tp.xa) * rowb;
          g01 = cbase + (static_cast<size_t>(tp.ya) * args.Wc + tp.xb) * rowb;
          g10 = cbase + (static_cast<size_t>(tp.yb) * args.Wc + tp.xa) * rowb;
          g11 = cbase + (static_cast<size_t>(tp.yb) * args.Wc + tp.xb) * rowb;
        }
      }
      const int wrow0 = quarter * 32;
      const int ox = x0 + (wrow0 % tw);
      const int oy = y0 + wrow0 / tw;
      const uint32_t cbuf = coarse_addr + static_cast<uint32_t>(cb * kLpCoarseBufBytes);

#pragma unroll 1
      for (int step = 0; step < 2; ++step) {
        const int col0 = chalf * 128 + step * 64;
        const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * kTcBlockN + col0) +
                               (static_cast<uint32_t>(quarter * 32) << 16);
        if (lane == 0) bulk_wait_group_read<0>();  // the staging buffer's last store read it
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          const int c0 = col0 + half * 32;
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(taddr + half * 32, r);
          tmem_wait_ld();
          if (step == 1 && half == 1) {
            // every accumulator column of this warp is in registers: free the TMEM buffer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_acce + static_cast<uint32_t>(acc) * 8u);
          }
          float v[32];
          const float4* b4 = reinterpret_cast<const float4*>(args.bias + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(b4 + i);
            v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + bb.x;
            v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
            v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
            v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
          }
          if (has_coarse) {
            const int blk = col0 >> 6;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int j = half * 4 + jj;  // 16-byte chunk of the 64-channel block
              uint4 a, b, c, d;
              if (staged) {
                const uint32_t base = cbuf + static_cast<uint32_t>(blk * kCoarseBlk);
                a = ld_shared_v4(base + r00 * 128 + ((j ^ (r00 & 7)) << 4));
                b = ld_shared_v4(base + r01 * 128 + ((j ^ (r01 & 7)) << 4));
                c = ld_shared_v4(base + r10 * 128 + ((j ^ (r10 & 7)) << 4));
                d = ld_shared_v4(base + r11 * 128 + ((j ^ (r11 & 7)) << 4));
              } else {
                const size_t off = static_cast<size_t>(col0) * sizeof(T);
                a = __ldg(reinterpret_cast<const uint4*>(g00 + off) + j);
                b = __ldg(reinterpret_cast<const uint4*>(g01 + off) + j);
                c = __ldg(reinterpret_cast<const uint4*>(g10 + off) + j);
                d = __ldg(reinterpret_cast<const uint4*>(g11 + off) + j);
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
                v[8 * jj + 2 * e + 0] += w00 * fa.x + w01 * fb.x + w10 * fc.x + w11 * fd.x;
                v[8 * jj + 2 * e + 1] += w00 * fa.y + w01 * fb.y + w10 * fc.y + w11 * fd.y;
              }
            }
          }
          __syncwarp();
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int j = half * 4 + jj;
            uint4 o;
            o.x = Pack<T>::pack(v[8 * jj + 0], v[8 * jj + 1]);
            o.y = Pack<T>::pack(v[8 * jj + 2], v[8 * jj + 3]);
            o.z = Pack<T>::pack(v[8 * jj + 4], v[8 * jj + 5]);
            o.w = Pack<T>::pack(v[8 * jj + 6], v[8 * jj + 7]);
            st_shared_v4(stage_addr + lane * 128 + ((j ^ (lane & 7)) << 4), o);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // every use commits a group (empty for the virtual tile past the end)
          if (real) tma_store_4d(&map_out, smem_stage + ew * kTcStagingPerWarp, col0, ox, oy, n);
          bulk_commit_group();
        }
      }
      if (has_coarse) {
        __syncwarp();  // every lane is done with the coarse box
        if (lane == 0) mbar_arrive(&cempty_bar[cb]);
        if (++cb == 2) {
          cb = 0;
          cphase ^= 1u;
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
