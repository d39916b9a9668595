// tcgen05 / TMEM / TMA implicit-GEMM engine shared by the two tensor-core FPN kernels.
//
//   Lateral (mode 0):  M_l[p, o] = sum_c C_l[p, c] * Wlat[o, c] + b[o]
//                                  + bilinear(M_{l+1})[p, o]      (optional)
//     Reference semantics: lib/kernels/compute/fpn_compute_kernels.cu:127-230
//     (1x1 conv, out = sum_c in * W[o,c] + bias[o]) followed by the top-down
//     upsample + add of lib/core/fpn_engine.cu:274-313 (bilinear, half-pixel,
//     scale = in/out), fused into the same accumulator.
//
//   Conv3x3 (mode 1): P_l[p, o] = sum_{tap, c} M_l[p + tap, c] * W3[o, tap, c] + b[o]
//     K = 9 * 256.  The top level also emits P6 = max_pool2d(P5, k=1, s=2) = P5[::2, ::2].
//
// Both modes tile the output as tile_h x tile_w = 128 pixels of one image by all
// 256 output channels.  A (activations, NHWC) arrives through a 4-D TMA box
// (64 ch, tile_w, tile_h, 1) whose origin is shifted by the tap; TMA zero-fills
// coordinates outside the image, which is exactly the 3x3 conv's pad = 1 (and the
// ragged right/bottom tiles of both modes).  B (weights, [256][K] K-major) arrives
// as a 2-D box (64, 256).  Operands use the 128-byte swizzle.
//
// The top-down add is itself a small GEMM on the same accumulator: over one tile,
// bilinear(M_{l+1}) = Wb (128 px x k coarse px, 4 non-zeros per row) . Mbox (k coarse
// px x 256 ch).  Mbox is the tile's coarse box (at most 64 pixels), fetched by TMA
// into a B stage where, channel-contiguous, it is an MN-major B operand; Wb is written
// into the A stage by the producer warp.  One extra k-block of 4 MMAs replaces all of
// the epilogue's bilinear arithmetic.  (If the box cannot hold a tile's taps, the
// epilogue reads the taps from global memory instead.)
//
// The fp32 accumulator lives in TMEM (two 256-column buffers, so the epilogue of
// tile i overlaps the main loop of tile i+1).  The epilogue reads TMEM, adds the
// bias, converts, writes a 128-byte swizzled staging tile and stores it with a TMA
// tensor store (which also clips ragged tiles).
//
// Inputs are bf16, fp16 or e4m3 (kind::f8f6f4, 128 channels per 128-byte row, bf16
// output scaled per tensor x per output channel); the accumulator is fp32 throughout.
//
// One CTA per SM (persistent, static round-robin over tiles):
//   warp 0      : TMA producer (lane 0 issues; the whole warp builds Wb)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one lane)
//   warps 2..9  : epilogue; warp w may access TMEM lanes 32*(w%4)..+31, and
//                 handles 128 of the 256 output channels ((w-2)/4 selects which)
#pragma once

#include "activation.cuh"
#include "ptx.cuh"

namespace ufpn {

constexpr int kTcBlockM = 128;
constexpr int kTcBlockN = 256;
constexpr int kTcBlockK = 64;  // 16-bit elements in one 128-byte swizzled row
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 64 + kTcEpiWarps * 32;
constexpr int kTcAStage = kTcBlockM * 128;
constexpr int kTcBStage = kTcBlockN * 128;
constexpr int kTcTmemCols = 2 * kTcBlockN;
constexpr int kTcStagingPerWarp = 32 * 128;  // 32 rows x 64 channels (bf16/fp16)
constexpr int kTcCoarseMaxPix = 64;          // coarse-box pixels = one MMA k-block
constexpr int kTcStages = 4;


// Operand element traits.  A k-block is one 128-byte swizzled row of channels:
// 64 channels of a 16-bit type, 128 of e4m3.  Either way a k-block is 4 MMAs of
// 32 bytes along K (K = 16 for kind::f16, 32 for kind::f8f6f4), so the shared-memory
// layout, descriptors and TMA byte counts are the same for every input type.
// e4m3 inputs produce bf16 outputs: acc * (activation scale * per-channel weight
// scale) + bias.
template <typename T>
struct TcElem;
template <>
struct TcElem<__nv_bfloat16> {
  using Out = __nv_bfloat16;
  static constexpr bool kFp8 = false;
  static constexpr uint32_t kFmt = 1;  // kind::f16 BF16
};
template <>
struct TcElem<__half> {
  using Out = __half;
  static constexpr bool kFp8 = false;
  static constexpr uint32_t kFmt = 0;  // kind::f16 F16
};
template <>
struct TcElem<__nv_fp8_e4m3> {
  using Out = __nv_bfloat16;
  static constexpr bool kFp8 = true;
  static constexpr uint32_t kFmt = 0;  // kind::f8f6f4 E4M3
};
template <typename T>
constexpr int kKbElems = 128 / static_cast<int>(sizeof(T));  // channels per k-block
constexpr int kMmaPerKb = 4;                                   // 32-byte K steps per k-block

// Shared-memory and warp plan of fpn_tc_gemm_kernel: kStages operand stages, kEpiWarps
// epilogue warps with kStageBufs staging buffers each.  The e4m3 lateral (mode 0) has a
// 2-k-block loop per tile, so its time per tile is the epilogue's latency chain (TMEM ->
// registers -> scale -> bf16 -> staging -> TMA store) rather than the MMAs: it runs 16
// epilogue warps, each owning 64 of the 256 output channels, and pays for their staging
// with one operand stage.  kWideEpi selects the same plan for a 16-bit lateral (an option:
// per-tile timestamps of the P2 lateral, K = 256, showed its 8-warp epilogue at 3.3 us per
// tile against a 2.9 us main loop).
template <int kMode, typename T, bool kWideEpi = kMode == 0 && TcElem<T>::kFp8>
struct TcCfgT {
  static constexpr bool kWide = kMode == 0 && kWideEpi;
  static constexpr int kEpiWarps = kWide ? 16 : kTcEpiWarps;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kStages = kWide ? 3 : kTcStages;
  static constexpr int kStageBufs = 1;
  static constexpr int kOffB = kStages * kTcAStage;
  static constexpr int kOffStaging = kOffB + kStages * kTcBStage;
  static constexpr int kOffBars = kOffStaging + kStageBufs * kEpiWarps * kTcStagingPerWarp;
  // the tile's 256 fp32 biases, staged once per CTA (16-bit lateral without channel slices)
  static constexpr int kOffBias = kOffBars + 256;
  static constexpr int kSmemBytes = kOffBias + 1024 + 1024 /*alignment slack*/;
};
static_assert(TcCfgT<0, __nv_fp8_e4m3>::kSmemBytes <= 232448 &&
                  TcCfgT<0, __nv_bfloat16>::kSmemBytes <= 232448 &&
                  TcCfgT<1, __nv_bfloat16>::kSmemBytes <= 232448,
              "tc smem");

template <typename T>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (TcElem<T>::kFp8)
    tc_mma_f8(d_tmem, adesc, bdesc, idesc, accumulate);
  else
    tc_mma_f16(d_tmem, adesc, bdesc, idesc, accumulate);
}

struct TcGemmArgs {
  int num_tiles;
  int num_kb;      // taps * cin_blocks (main loop only)
  int cin_blocks;  // ceil(Cin / channels per k-block)
  int N_img, H, W;
  int tile_w, tile_h, tiles_x, tiles_y;
  const float* bias;  // [256] fp32
  // lateral: coarser merged map M_{l+1}, NHWC [N][Hc][Wc][256]
  const void* coarse;  // null = no top-down add
  int Hc, Wc;
  float scale_y, scale_x;  // Hc / H, Wc / W
  int cbox_w, cbox_h;      // coarse box of the MMA path (0 = taps from global memory)
  // conv3x3 top level: P6 NHWC [N][H6][W6][256], or null
  void* p6;
  int H6, W6;
  int* status;  // device status word (0 = ok)
  // e4m3 inputs only: out = acc * (ascale[n * ascale_stride] * wscale[o]) + bias[o]
  const float* ascale;  // activation scale(s), device: one (stride 0) or one per image (1)
  int ascale_stride;
  const float* wscale;  // per-output-channel weight scales [256]
  // optional: amax_out[n] = atomicMax of |out| (fp32 bits) over image n's stored elements
  // (the absmax a following per-image e4m3 quantisation of this output needs)
  unsigned* amax_out;
  // 0: store the 16-bit output; 1: store nothing (only amax_out); 2: store the output
  // quantised to e4m3 per image with the absmax in qamax[n] (the 16-bit value rounded
  // first, then e4m3(x * 448 / amax)), writing the dequantisation scales to qscale_out[n]
  int out_mode;
  const unsigned* qamax;
  float* qscale_out;
  // lateral top-down k-block: precomputed Wb table (tc_wb_table_kernel), or null to build
  // Wb per tile in the producer warp
  const uint8_t* wb_table;
  // e4m3 3x3 that quantises its bf16 input in shared memory: per-image absmax of the input
  // (fp32 bits); the activation scale is then amax[n] / 448 (ascale unused)
  const unsigned* in_amax;
  // 16-bit output: store only columns [0, out_cols) (0 = all 256), for an output view whose
  // channel slice is narrower than a tile (no TMA store then starts beyond the tensor)
  int out_cols;
  // 16-bit lateral without a top-down add: output channel slices of 256 in one launch (0 or
  // 1 = one).  Slice s uses weight rows [256 s, 256 s + 256), bias[256 s ..] and writes
  // channels [256 s, 256 s + 256) of the output (columns below out_cols); the tile index runs
  // over slices x images x tile rows x tile columns.
  int slices;
  // output activation after the bias (FPNActivation numbering; 0 = none) and its alpha
  int act;
  float act_alpha;
  // 3x3 on CTA pairs: the last pair_tail pair units each run as two work items over the
  // output channels (N = 128: channels 0..127, then 128..255), so that a last round with
  // fewer units than pairs takes half as long (0 = every unit whole)
  int pair_tail;
  // halo 3x3 on the map's transposed view (H, W and the tensor maps swapped by the host):
  // tap (ky, kx) of the weights shifts the halo by (kx, ky) in the view
  int transposed;
  // 3x3 on CTA pairs: dynamic item claims.  claim[0] = next work item, claim[1] = CTAs done;
  // both zero at launch, reset by the last CTA to leave.  Pairs that reach an SM late (other
  // streams' CTAs still hold it) then take fewer items instead of ending the launch late.
  // null: static round robin over the pairs.
  int* claim;
  // halo 3x3 with a mixed tiling (strip_first > 0): tiles [0, strip_first) on the map's own
  // view (tiles_x x tiles_y per image, the tile rows covering the first 16 tiles_y rows of
  // the map), tiles from strip_first on the transposed view, through the second pair of
  // tensor maps: the strip of rows [strip_y0, H) (at most 8), strip_tx tiles of 16 columns
  // per image.  strip_first is even for CTA pairs (a pair's two tiles share one tap offset).
  int strip_first;
  int strip_y0, strip_tx;
};

// Work items of a CTA pair claimed at run time: the leader's producer claims each item from
// the global counter and publishes it to a ring of kClaimRecs records in BOTH CTAs; every
// other role of either CTA takes the items in order from its own CTA's ring and, once it has
// read a record, arrives on the leader's empty barrier of that record (release at cluster
// scope), so that the claimer reuses a slot only after all of them have read it.
constexpr int kClaimRecs = 4;
struct ClaimRing {
  volatile int* rec;  // this CTA's records [kClaimRecs]
  uint64_t* full;     // this CTA's full barriers [kClaimRecs] (one arrival: the claimer)
  uint32_t empty0;    // shared::cluster address of the leader's empty barriers
  int slot;
  uint32_t phase;
  __device__ __forceinline__ void advance() {
    if (++slot == kClaimRecs) {
      slot = 0;
      phase ^= 1u;
    }
  }
  // One thread: the next item (false after an abort or a timeout).
  __device__ __forceinline__ bool next(int& item, volatile int* abort_flag, int* status,
                                       int code) {
    if (!mbar_wait_acq_cluster(&full[slot], phase, abort_flag, status, code)) return false;
    item = rec[slot];
    mbar_arrive_cluster(empty0 + static_cast<uint32_t>(slot) * 8u);
    advance();
    return true;
  }
  // A whole warp: every lane reads the record before lane 0 releases it.
  __device__ __forceinline__ bool next_warp(int& item, int lane, volatile int* abort_flag,
                                            int* status, int code) {
    const bool ok = mbar_wait_acq_cluster(&full[slot], phase, abort_flag, status, code);
    if (!__all_sync(0xffffffffu, ok)) return false;
    item = rec[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(empty0 + static_cast<uint32_t>(slot) * 8u);
    advance();
    return true;
  }
};
// The claimer (the leader's producer thread): record `item` in slot `slot` of both CTAs'
// rings, then arrive on both full barriers (release at cluster scope orders the stores).
__device__ __forceinline__ void claim_publish(volatile int* rec, uint64_t* full, int slot,
                                              int item) {
  const uint32_t r = smem_u32(const_cast<int*>(rec) + slot);
  st_cluster_u32(mapa_shared(r, 1), static_cast<uint32_t>(item));
  rec[slot] = item;
  const uint32_t f = smem_u32(&full[slot]);
  mbar_arrive_cluster(mapa_shared(f, 1));
  mbar_arrive_cluster(mapa_shared(f, 0));
}

// Halo 3x3 tiles: 8 wide x 16 high in the view the kernel runs on.
constexpr int kHaloTileW = 8;
constexpr int kHaloTileH = 16;
constexpr int kHaloRows = (kHaloTileW + 2) * (kHaloTileH + 2);  // 180
// Halo row offset of weight tap `tap` (ky * 3 + kx).  On the transposed view of a map (rows
// and columns swapped) the same tap shifts the halo by (kx, ky).
__device__ __forceinline__ int halo_tap_offset(int tap, int transposed) {
  const int ky = tap / 3, kx = tap - 3 * (tap / 3);
  return transposed ? kx * (kHaloTileW + 2) + ky : ky * (kHaloTileW + 2) + kx;
}
// One halo tile: its image, origin in the coordinates of the view it runs on (x0 along the
// view's rows, y0 down its columns), whether its taps are mirrored (transposed view), and
// whether it is a strip tile of a mixed tiling (second pair of tensor maps).
struct HaloTile {
  int n, x0, y0;
  int tr;
  bool strip;
};
__device__ __forceinline__ HaloTile halo_tile(const TcGemmArgs& a, int tile) {
  HaloTile t;
  if (a.strip_first > 0 && tile >= a.strip_first) {
    const int s = tile - a.strip_first;
    t.n = s / a.strip_tx;
    t.x0 = a.strip_y0;                        // rows [strip_y0, strip_y0 + 8)
    t.y0 = (s - t.n * a.strip_tx) * kHaloTileH;  // columns [16 i, 16 i + 16)
    t.tr = 1;
    t.strip = true;
    return t;
  }
  const int tx = tile % a.tiles_x;
  const int t2 = tile / a.tiles_x;
  const int ty = t2 % a.tiles_y;
  t.n = t2 / a.tiles_y;
  t.x0 = tx * a.tile_w;
  t.y0 = ty * a.tile_h;
  t.tr = a.transposed;
  t.strip = false;
  return t;
}

// Work items of a CTA-pair 3x3: units [0, units - pair_tail) whole (half = -1), then two
// channel-half items per tail unit.  Returns the item's pair unit.
__device__ __forceinline__ int pair_item_unit(const TcGemmArgs& a, int units, int item,
                                              int& half) {
  const int first = units - a.pair_tail;
  if (item < first) {
    half = -1;
    return item;
  }
  half = (item - first) & 1;
  return first + ((item - first) >> 1);
}

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t u) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(v);
  }
  __device__ static __forceinline__ uint16_t bits(float a) {
    __nv_bfloat16 v = __float2bfloat16_rn(a);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};
template <>
struct Pack<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t u) {
    __half2 v = *reinterpret_cast<__half2*>(&u);
    return __half22float2(v);
  }
  __device__ static __forceinline__ uint16_t bits(float a) {
    __half v = __float2half_rn(a);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};

__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(x), "r"(y) : "memory");
}
// Four floats scaled by `inv` to four e4m3 bytes (nearest even, saturated), low byte first.
__device__ __forceinline__ uint32_t tc_e4m3x4(float a, float b, float c, float d, float inv) {
  const uint32_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(a * inv, b * inv), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(c * inv, d * inv), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

// The quantiser's inverse and dequantisation scale from an absmax (fp32 bits):
// amax > 0: 448 / amax and amax / 448 (single correctly rounded divisions); else 1.
__device__ __forceinline__ float e4m3_inv_of(unsigned amax_bits) {
  const float a = __uint_as_float(amax_bits);
  return a > 0.f ? __fdiv_rn(448.f, a) : 1.f;
}
__device__ __forceinline__ float e4m3_scale_of(unsigned amax_bits) {
  const float a = __uint_as_float(amax_bits);
  return a > 0.f ? __fdiv_rn(a, 448.f) : 1.f;
}

__device__ __forceinline__ void tc_tile_origin(const TcGemmArgs& a, int tile, int& n, int& x0,
                                               int& y0, int& slice) {
  const int tx = tile % a.tiles_x;
  const int t2 = tile / a.tiles_x;
  const int ty = t2 % a.tiles_y;
  n = t2 / a.tiles_y;
  slice = 0;
  if (a.slices > 1) {
    slice = n / a.N_img;
    n -= slice * a.N_img;
  }
  x0 = tx * a.tile_w;
  y0 = ty * a.tile_h;
}
__device__ __forceinline__ void tc_tile_origin(const TcGemmArgs& a, int tile, int& n, int& x0,
                                               int& y0) {  // kernels without channel slices
  const int tx = tile % a.tiles_x;
  const int t2 = tile / a.tiles_x;
  const int ty = t2 % a.tiles_y;
  n = t2 / a.tiles_y;
  x0 = tx * a.tile_w;
  y0 = ty * a.tile_h;
}

// Bilinear source index along one axis (half-pixel, clamped).  Every step is an
// explicitly rounded fp32 operation so the host can replay it bit for bit when it
// sizes the coarse box.
__device__ __forceinline__ float tc_src(int o, float scale, int in) {
  const float s = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(o), 0.5f), scale), 0.5f);
  return fminf(fmaxf(s, 0.f), static_cast<float>(in - 1));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Geometry of one bilinear tap set (shared by the Wb builder and the epilogue fallback).
struct TcTaps {
  int ya, yb, xa, xb;
  float w00, w01, w10, w11;
};
__device__ __forceinline__ TcTaps tc_taps(int py, int px, int H, int W, int Hc, int Wc,
                                          float scale_y, float scale_x) {
  const float sy = tc_src(min(py, H - 1), scale_y, Hc);
  const float sx = tc_src(min(px, W - 1), scale_x, Wc);
  TcTaps t;
  t.ya = static_cast<int>(sy);
  t.xa = static_cast<int>(sx);
  t.yb = min(t.ya + 1, Hc - 1);
  t.xb = min(t.xa + 1, Wc - 1);
  const float wy = sy - static_cast<float>(t.ya);
  const float wx = sx - static_cast<float>(t.xa);
  t.w00 = (1.f - wy) * (1.f - wx);
  t.w01 = (1.f - wy) * wx;
  t.w10 = wy * (1.f - wx);
  t.w11 = wy * wx;
  return t;
}

// Bilinear operands of one tile's top-down k-block, written by a whole warp with generic
// stores (the caller fences the async proxy afterwards):
//   tc_build_wb:    Wb, 128 rows (tile pixels) x 64 k (box pixels), K-major 128-byte
//                   swizzle relative to a 1024-byte-aligned base (so the same bytes, stored
//                   in global memory, form a table a bulk copy can bring back unchanged);
//   tc_zero_btail:  zeroes the box rows k >= cbox_w * cbox_h of the nb MN-major 64-channel
//                   blocks of the B stage (TMA fills rows below that), so no stale bits
//                   meet a zero weight.
__device__ __forceinline__ void tc_zero_btail(uint8_t* b_stage, int lane, int kbox, int nb) {
  const uint32_t b_addr = smem_u32(b_stage);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  const int per = (kTcCoarseMaxPix - kbox) * 8;  // 16-byte chunks per block
  for (int i = lane; i < nb * per; i += 32) {
    const int blk = i / per;
    const int rem = i - blk * per;
    const int row = kbox + (rem >> 3);
    st_shared_v4(b_addr + blk * (kTcCoarseMaxPix * 128) + row * 128 + (rem & 7) * 16, z);
  }
}

template <typename T>
__device__ __forceinline__ void tc_build_wb(uint8_t* a_stage, int lane, int x0, int y0,
                                            int tile_w, int H, int W, int Hc, int Wc,
                                            float scale_y, float scale_x, int cbox_w,
                                            int cbox_h) {
  const uint32_t a_addr = smem_u32(a_stage);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int i = lane; i < kTcAStage / 16; i += 32) st_shared_v4(a_addr + i * 16, z);
  __syncwarp();
  const int kbox = cbox_w * cbox_h;
  const int cy0 = static_cast<int>(tc_src(y0, scale_y, Hc));
  const int cx0 = static_cast<int>(tc_src(x0, scale_x, Wc));
#pragma unroll 1
  for (int r = lane; r < kTcBlockM; r += 32) {
    const TcTaps t = tc_taps(y0 + r / tile_w, x0 + r % tile_w, H, W, Hc, Wc, scale_y, scale_x);
    int k[4] = {(t.ya - cy0) * cbox_w + (t.xa - cx0), (t.ya - cy0) * cbox_w + (t.xb - cx0),
                (t.yb - cy0) * cbox_w + (t.xa - cx0), (t.yb - cy0) * cbox_w + (t.xb - cx0)};
    float w[4] = {t.w00, t.w01, t.w10, t.w11};
    // Corners that coincide (clamped at the map border) add their weights.
#pragma unroll
    for (int i = 1; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < i; ++j)
        if (k[i] == k[j] && w[j] != 0.f) {
          w[j] += w[i];
          w[i] = 0.f;
        }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (w[i] == 0.f || k[i] < 0 || k[i] >= kbox) continue;
      const uint32_t byte = static_cast<uint32_t>(k[i]) * 2u;
      const uint32_t off = r * 128 + ((((byte >> 4) ^ (r & 7)) & 7) << 4) + (byte & 15);
      st_shared_u16(a_addr + off, Pack<T>::bits(w[i]));
    }
  }
}

template <typename T>
__device__ __forceinline__ void tc_build_bilinear(uint8_t* a_stage, uint8_t* b_stage, int lane,
                                                  int x0, int y0, int tile_w, int H, int W,
                                                  int Hc, int Wc, float scale_y, float scale_x,
                                                  int cbox_w, int cbox_h) {
  tc_zero_btail(b_stage, lane, cbox_w * cbox_h, 4);
  tc_build_wb<T>(a_stage, lane, x0, y0, tile_w, H, W, Hc, Wc, scale_y, scale_x, cbox_w, cbox_h);
}

// Precomputed Wb table: entry ty * tiles_x + tx holds the 16 KB Wb of tile (tx, ty) (the
// same for every image).  One 32-thread block per entry.
template <typename T>
__global__ void __launch_bounds__(32) tc_wb_table_kernel(const TcGemmArgs a, uint8_t* table) {
  extern __shared__ uint8_t wb_raw[];
  uint8_t* buf = wb_raw + ((1024u - (smem_u32(wb_raw) & 1023u)) & 1023u);
  const int e = blockIdx.x;
  const int tx = e % a.tiles_x, ty = e / a.tiles_x;
  tc_build_wb<T>(buf, threadIdx.x, tx * a.tile_w, ty * a.tile_h, a.tile_w, a.H, a.W, a.Hc, a.Wc,
                 a.scale_y, a.scale_x, a.cbox_w, a.cbox_h);
  __syncwarp();
  const uint4* src = reinterpret_cast<const uint4*>(buf);
  uint4* dst = reinterpret_cast<uint4*>(table + static_cast<size_t>(e) * kTcAStage);
  for (int i = threadIdx.x; i < kTcAStage / 16; i += 32) dst[i] = src[i];
}

// Epilogue role (warps 2 .. 2 + kEpiW - 1) of the tensor-core kernels: per tile, TMEM -> registers,
// + bias (+ global-memory bilinear taps on the lateral fallback path), convert,
// 128-byte-swizzled staging tile, TMA tensor store; P6 rows for the top 3x3.
// kPair: the CTA is one half of a cta_group::2 pair; pair unit u covers tiles 2u (rank 0)
// and 2u + 1 (rank 1; past the last tile it is a virtual, all-padding tile that is
// computed but never stored), and each warp releases its accumulator on the pair
// leader's barrier (shared::cluster address leader_acce).
// bias_s (optional): the 256 biases staged in shared memory (read there instead of from
// global memory every tile; the epilogue's latency chain is its per-tile cost).
template <int kMode, typename T, bool kPair = false, int kStageBufs = 1,
          int kEpiW = kTcEpiWarps>
__device__ __forceinline__ void tc_epilogue(const TcGemmArgs& args, const CUtensorMap* map_out,
                                            uint32_t tmem_base, uint64_t* accf_bar,
                                            uint64_t* acce_bar, uint8_t* smem_stage,
                                            volatile int* abort_flag, int warp, int lane,
                                            bool bil_mma, uint32_t leader_acce = 0,
                                            const float* bias_s = nullptr,
                                            ClaimRing* ring = nullptr,
                                            const CUtensorMap* map_out2 = nullptr) {
  using O = typename TcElem<T>::Out;
  constexpr bool kFp8 = TcElem<T>::kFp8;
  // kEpiW / 4 warps share each TMEM lane quarter; each owns kChans output channels,
  // processed in 64-channel steps.
  constexpr int kChans = kTcBlockN / (kEpiW / 4);
  constexpr int kSteps = kChans / 64;
  static_assert(kEpiW % 4 == 0 && kChans % 64 == 0, "epilogue warp split");
  const int ew = warp - 2;
  const int quarter = warp & 3;  // TMEM lanes 32*quarter..+31 (hardware: warp id % 4)
  const int chalf = ew >> 2;     // output channels chalf*kChans .. +kChans-1
  const int row = quarter * 32 + lane;
  const int tw = args.tile_w;
  // Staging buffers of this warp: kStageBufs x (32 rows x 128 bytes), used round robin.
  uint8_t* const my_stage = smem_stage + ew * kStageBufs * kTcStagingPerWarp;
  int sbuf = 0;
  const bool taps_global = (kMode == 0) && args.coarse != nullptr && !bil_mma;
  int acc = 0;
  uint32_t acc_phase = 0;
  const int rank = kPair ? static_cast<int>(cluster_ctarank()) : 0;
  const int units = kPair ? (args.num_tiles + 1) / 2 : args.num_tiles;
  // (3x3: the last pair_tail units -- pair units, or tiles on single CTAs -- run as two
  // channel-half items each; 0 for the laterals)
  const int items = units + args.pair_tail;
  const int ustep = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // (kPair with a claim ring: the items in the order the leader claimed them)
  for (int it = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);;
       it += ustep) {
    if (kPair && ring != nullptr &&
        !ring->next_warp(it, lane, abort_flag, args.status, kDevTimeoutEpilogue))
      break;
    if (it >= items) break;
    int half = -1;  // channel-half item of a CTA-pair 3x3 (its accumulator has N = 128)
    const int u = pair_item_unit(args, units, it, half);
    const int tile = kPair ? 2 * u + rank : u;
    const bool real = tile < args.num_tiles;
    const bool ok =
        mbar_wait(&accf_bar[acc], acc_phase, abort_flag, args.status, kDevTimeoutEpilogue);
    if (!__all_sync(0xffffffffu, ok)) break;
    tc_fence_after();

    int n, x0, y0, slice = 0;
    // the tile's view: a strip tile of a mixed 3x3 tiling runs on the transposed view (its
    // rows along the map's columns) and stores through the second output map
    const CUtensorMap* mo = map_out;
    int vH = args.H, vW = args.W;
    if constexpr (kMode == 0 && !kPair) {
      tc_tile_origin(args, tile, n, x0, y0, slice);
    } else if constexpr (kMode == 1) {
      const HaloTile ht = halo_tile(args, tile);
      n = ht.n;
      x0 = ht.x0;
      y0 = ht.y0;
      if (ht.strip) {
        mo = map_out2;
        vH = args.W;
        vW = args.H;
      }
    } else {
      tc_tile_origin(args, tile, n, x0, y0);
    }
    const int scol = slice * kTcBlockN;  // channel offset of this tile's output slice
    const int py = y0 + row / tw;
    const int px = x0 + row % tw;
    const bool valid = real && (py < vH) && (px < vW);
    const float ascale = !(kFp8 && real) ? 1.f
                         : args.in_amax != nullptr ? e4m3_scale_of(__ldg(args.in_amax + n))
                                                   : __ldg(args.ascale + n * args.ascale_stride);
    uint32_t amax_bits = 0;  // max |stored value| of this thread in this tile (fp32 bits)
    const int omode = args.out_mode;
    float qinv = 1.f;
    if (omode == 2 && real) {
      const float qa = __uint_as_float(__ldg(args.qamax + n));
      qinv = qa > 0.f ? __fdiv_rn(448.f, qa) : 1.f;
      if (ew == 0 && lane == 0) args.qscale_out[n] = qa > 0.f ? __fdiv_rn(qa, 448.f) : 1.f;
    }

    // Fallback only: bilinear taps of the coarser merged map from global memory.
    TcTaps tp{};
    const uint8_t* g00 = nullptr;
    const uint8_t* g01 = nullptr;
    const uint8_t* g10 = nullptr;
    const uint8_t* g11 = nullptr;
    if (taps_global) {
      tp = tc_taps(py, px, args.H, args.W, args.Hc, args.Wc, args.scale_y, args.scale_x);
      const size_t rowb = static_cast<size_t>(kTcBlockN) * sizeof(O);
      const uint8_t* cbase = static_cast<const uint8_t*>(args.coarse) +
                             static_cast<size_t>(n) * args.Hc * args.Wc * rowb;
      g00 = cbase + (static_cast<size_t>(tp.ya) * args.Wc + tp.xa) * rowb;
      g01 = cbase + (static_cast<size_t>(tp.ya) * args.Wc + tp.xb) * rowb;
      g10 = cbase + (static_cast<size_t>(tp.yb) * args.Wc + tp.xa) * rowb;
      g11 = cbase + (static_cast<size_t>(tp.yb) * args.Wc + tp.xb) * rowb;
    }
    const bool emit_p6 =
        (kMode == 1) && (args.p6 != nullptr) && valid && ((py & 1) == 0) && ((px & 1) == 0);
    uint8_t* p6_row = nullptr;
    if (emit_p6) {
      const size_t p6pix =
          (static_cast<size_t>(n) * args.H6 + (py >> 1)) * args.W6 + (px >> 1);
      p6_row = static_cast<uint8_t*>(args.p6) + p6pix * kTcBlockN * sizeof(O);
    }
    // Output box of this warp's 32 rows.
    const int wrow0 = quarter * 32;
    const int ox = x0 + (wrow0 % tw);
    const int oy = y0 + wrow0 / tw;

    // A channel-half item: kChans / 2 accumulator columns per warp, output channels from
    // half * 128 (kSteps is even wherever items are halved: 8 epilogue warps).
    const int nsteps = half < 0 ? kSteps : kSteps / 2;
    const int tcol0 = half < 0 ? chalf * kChans : chalf * (kChans / 2);
    const int ocol0 = half < 0 ? tcol0 : half * (kTcBlockN / 2) + tcol0;
#pragma unroll 1
    for (int step = 0; step < nsteps; ++step) {
      const int col0 = ocol0 + step * 64;  // output channel of the step's first column
      const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * kTcBlockN + tcol0 + step * 64) +
                             (static_cast<uint32_t>(quarter * 32) << 16);
      // With 8 epilogue warps (registers to spare), both 32-column halves of the step are
      // loaded from TMEM with one wait: the loads overlap each other and the staging-buffer
      // wait below (per-tile timestamps of the lateral showed its epilogue bound by serial
      // TMEM round trips).  16 warps (at most 112 registers each) load a half at a time.
      constexpr bool kBoth = kEpiW <= 8;
      uint32_t rr[kBoth ? 64 : 32];
      auto release_acc = [&] {
        // All of this tile's accumulator columns for this warp are in registers:
        // hand the TMEM buffer back to the MMA warp before the memory work.
        tc_fence_before();
        if constexpr (kPair) {
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_acce + static_cast<uint32_t>(acc) * 8u);
        } else {
          mbar_arrive(&acce_bar[acc]);
        }
      };
      if constexpr (kBoth) {
        __syncwarp();
        tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
        tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[32]));
      }
      // The TMA store that last read this staging buffer must be done with it (the e4m3
      // row of a tile is assembled from both steps, so it is only waited for at step 0).
      if (omode == 0 || (omode == 2 && step == 0)) {
        if (lane == 0) bulk_wait_group_read<kStageBufs - 1>();
      }
      const uint32_t stage_addr = smem_u32(my_stage + sbuf * kTcStagingPerWarp);
      if constexpr (kBoth) {
        tmem_wait_ld();
        if (step == nsteps - 1) release_acc();
      }
      // Two 32-column halves per 64-channel step.
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int c0 = col0 + hh * 32;
        const uint32_t* r = kBoth ? rr + hh * 32 : rr;
        if constexpr (!kBoth) {
          __syncwarp();
          tmem_ld32(taddr + hh * 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
          tmem_wait_ld();
          if (step == nsteps - 1 && hh == 1) release_acc();
        }
        float v[32];
        const float4* b4 = reinterpret_cast<const float4*>(args.bias + scol + c0);
        if constexpr (kFp8) {
          const float4* s4 = reinterpret_cast<const float4*>(args.wscale + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(b4 + i);
            const float4 ss = __ldg(s4 + i);
            v[4 * i + 0] = fmaf(__uint_as_float(r[4 * i + 0]), ascale * ss.x, bb.x);
            v[4 * i + 1] = fmaf(__uint_as_float(r[4 * i + 1]), ascale * ss.y, bb.y);
            v[4 * i + 2] = fmaf(__uint_as_float(r[4 * i + 2]), ascale * ss.z, bb.z);
            v[4 * i + 3] = fmaf(__uint_as_float(r[4 * i + 3]), ascale * ss.w, bb.w);
          }
        } else {
          const float4* bs4 = bias_s ? reinterpret_cast<const float4*>(bias_s + c0) : nullptr;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = bs4 ? bs4[i] : __ldg(b4 + i);
            v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + bb.x;
            v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
            v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
            v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
          }
        }
        if (taps_global) {
          const size_t off = static_cast<size_t>(c0) * sizeof(O);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(g00 + off) + j);
            const uint4 b = __ldg(reinterpret_cast<const uint4*>(g01 + off) + j);
            const uint4 c = __ldg(reinterpret_cast<const uint4*>(g10 + off) + j);
            const uint4 d = __ldg(reinterpret_cast<const uint4*>(g11 + off) + j);
            const uint32_t au[4] = {a.x, a.y, a.z, a.w};
            const uint32_t bu[4] = {b.x, b.y, b.z, b.w};
            const uint32_t cu[4] = {c.x, c.y, c.z, c.w};
            const uint32_t du[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 fa = Pack<O>::unpack(au[e]);
              const float2 fb = Pack<O>::unpack(bu[e]);
              const float2 fc = Pack<O>::unpack(cu[e]);
              const float2 fd = Pack<O>::unpack(du[e]);
              v[8 * j + 2 * e + 0] += tp.w00 * fa.x + tp.w01 * fb.x + tp.w10 * fc.x + tp.w11 * fd.x;
              v[8 * j + 2 * e + 1] += tp.w00 * fa.y + tp.w01 * fb.y + tp.w10 * fc.y + tp.w11 * fd.y;
            }
          }
        }
        if constexpr (kMode == 1) epilogue_act(v, args.act, args.act_alpha);
        __syncwarp();
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = hh * 4 + jj;  // 16-byte chunk of the 128-byte staging row
          uint4 o;
          o.x = Pack<O>::pack(v[8 * jj + 0], v[8 * jj + 1]);
          o.y = Pack<O>::pack(v[8 * jj + 2], v[8 * jj + 3]);
          o.z = Pack<O>::pack(v[8 * jj + 4], v[8 * jj + 5]);
          o.w = Pack<O>::pack(v[8 * jj + 6], v[8 * jj + 7]);
          if (args.amax_out != nullptr && valid) {
            // max |x| of the rounded 16-bit values: clear the sign bits, then compare as
            // unsigned (order-preserving for non-negative floats of one format).
            const uint32_t w4[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = Pack<O>::unpack(w4[e] & 0x7FFF7FFFu);
              amax_bits = max(amax_bits, max(__float_as_uint(f.x), __float_as_uint(f.y)));
            }
          }
          if (omode == 0) {
            st_shared_v4(stage_addr + lane * 128 + ((j ^ (lane & 7)) << 4), o);
            if (emit_p6)
              reinterpret_cast<uint4*>(p6_row + static_cast<size_t>(col0) * sizeof(O))[j] = o;
          } else if (kSteps == 1 && omode == 2) {
            // 8 channels -> 8 e4m3 bytes, half of 16-byte chunk j / 2 of the warp's 64-byte
            // row; the 64-byte swizzle puts chunk c of row r at c ^ ((r >> 1) & 3)
            const float2 f0 = Pack<O>::unpack(o.x), f1 = Pack<O>::unpack(o.y);
            const float2 f2 = Pack<O>::unpack(o.z), f3 = Pack<O>::unpack(o.w);
            const uint32_t q0 = tc_e4m3x4(f0.x, f0.y, f1.x, f1.y, qinv);
            const uint32_t q1 = tc_e4m3x4(f2.x, f2.y, f3.x, f3.y, qinv);
            const int chunk = (j >> 1) ^ ((lane >> 1) & 3);
            st_shared_v2(stage_addr + lane * 64 + (chunk << 4) + (j & 1) * 8, q0, q1);
          } else if (kSteps == 2 && omode == 2) {
            // 8 channels -> 8 e4m3 bytes, half of 16-byte chunk (step * 4 + j / 2) of the row
            const float2 f0 = Pack<O>::unpack(o.x), f1 = Pack<O>::unpack(o.y);
            const float2 f2 = Pack<O>::unpack(o.z), f3 = Pack<O>::unpack(o.w);
            const uint32_t q0 = tc_e4m3x4(f0.x, f0.y, f1.x, f1.y, qinv);
            const uint32_t q1 = tc_e4m3x4(f2.x, f2.y, f3.x, f3.y, qinv);
            const int chunk = step * 4 + (j >> 1);
            st_shared_v2(stage_addr + lane * 128 + ((chunk ^ (lane & 7)) << 4) + (j & 1) * 8,
                         q0, q1);
          }
        }
      }
      if (omode == 0 || (omode == 2 && step == kSteps - 1)) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // e4m3: the warp's 128 channels (128 bytes per pixel) in one store.  Every buffer
          // use commits a group (empty for virtual tiles) so group counts stay in step.
          if (real && (omode != 0 || args.out_cols == 0 || scol + col0 < args.out_cols))
            tma_store_4d(mo, my_stage + sbuf * kTcStagingPerWarp,
                         omode == 0 ? scol + col0 : chalf * kChans, ox, oy, n);
          bulk_commit_group();
        }
        if (++sbuf == kStageBufs) sbuf = 0;
      }
    }
    if (args.amax_out != nullptr) {
      // One atomic per warp and tile at most, skipped once the image's maximum is larger.
      amax_bits = __reduce_max_sync(0xffffffffu, amax_bits);
      if (lane == 0 && real &&
          amax_bits > *reinterpret_cast<volatile unsigned*>(args.amax_out + n))
        atomicMax(args.amax_out + n, amax_bits);
    }
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1u;
    }
  }
  if (lane == 0) bulk_wait_group<0>();
  __syncwarp();
}

template <int kMode, typename T, bool kWideEpi = kMode == 0 && TcElem<T>::kFp8>
__global__ void __launch_bounds__(TcCfgT<kMode, T, kWideEpi>::kThreads, 1)
    fpn_tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_out,
                       const __grid_constant__ CUtensorMap map_coarse, const TcGemmArgs args) {
  using Cfg = TcCfgT<kMode, T, kWideEpi>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + Cfg::kOffB;
  uint8_t* smem_stage = smem + Cfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* accf_bar = bars + 2 * S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* bias_s = reinterpret_cast<float*>(smem + Cfg::kOffBias);
  // (16-bit laterals with one 256-channel output slice read their biases from shared memory)
  const bool stage_bias = kMode == 0 && !TcElem<T>::kFp8 && args.slices <= 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Top-down add through the tensor core (coarse box fits one k-block).
  // (e4m3 inputs: the planner enables it only for a coarse map pre-divided by the
  // epilogue's per-channel scale, so the scaled accumulator holds the right top-down term.)
  const bool bil_mma = (kMode == 0) && args.coarse != nullptr && args.cbox_w > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], Cfg::kEpiWarps * 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    prefetch_tmap(&map_out);
    if (bil_mma) prefetch_tmap(&map_coarse);
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
    // ------------------------------------------------------------ TMA producer (whole warp)
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    const uint32_t coarse_bytes = static_cast<uint32_t>(args.cbox_w * args.cbox_h * 128 * 4);
    for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
      int n, x0, y0, slice = 0;
      if constexpr (kMode == 0)
        tc_tile_origin(args, tile, n, x0, y0, slice);
      else
        tc_tile_origin(args, tile, n, x0, y0);
      const int nkb = args.num_kb + (bil_mma ? 1 : 0);
      for (int kb = 0; kb < nkb; ++kb) {
        ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                       kDevTimeoutProducer);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        if (kb < args.num_kb) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&full_bar[stage], kTcAStage + kTcBStage);
            int dy = 0, dx = 0, cb = kb;
            if constexpr (kMode == 1) {
              const int tap = kb / args.cin_blocks;
              cb = kb - tap * args.cin_blocks;
              dy = tap / 3 - 1;
              dx = tap % 3 - 1;
            }
            tma_load_4d(smem_a + stage * kTcAStage, &map_a, &full_bar[stage], cb * kKbElems<T>,
                        x0 + dx, y0 + dy, n,
                        kMode == 0 ? kPolicyEvictFirst : kPolicyEvictLast);
            tma_load_2d(smem_b + stage * kTcBStage, &map_b, &full_bar[stage], kb * kKbElems<T>,
                        slice * kTcBlockN, kPolicyEvictLast);
          }
        } else {
          // Bilinear k-block: Wb into the A stage (a bulk copy of the tile's precomputed
          // table entry, else generic stores by the whole warp), the coarse box into the
          // B stage (TMA), then one arrival with the async bytes.
          if (args.wb_table != nullptr)
            tc_zero_btail(smem_b + stage * kTcBStage, lane, args.cbox_w * args.cbox_h, 4);
          else
            tc_build_bilinear<typename TcElem<T>::Out>(
                smem_a + stage * kTcAStage, smem_b + stage * kTcBStage, lane, x0, y0,
                args.tile_w, args.H, args.W, args.Hc, args.Wc, args.scale_y, args.scale_x,
                args.cbox_w, args.cbox_h);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int cy = static_cast<int>(tc_src(y0, args.scale_y, args.Hc));
            const int cx = static_cast<int>(tc_src(x0, args.scale_x, args.Wc));
            if (args.wb_table != nullptr) {
              mbar_arrive_expect_tx(&full_bar[stage], coarse_bytes + kTcAStage);
              const int e = (tile % args.tiles_x) + ((tile / args.tiles_x) % args.tiles_y) *
                                                       args.tiles_x;
              bulk_load(smem_a + stage * kTcAStage,
                        args.wb_table + static_cast<size_t>(e) * kTcAStage, kTcAStage,
                        &full_bar[stage]);
            } else {
              mbar_arrive_expect_tx(&full_bar[stage], coarse_bytes);
            }
            for (int b = 0; b < 4; ++b)
              tma_load_4d(smem_b + stage * kTcBStage + b * (kTcCoarseMaxPix * 128), &map_coarse,
                          &full_bar[stage], b * 64, cx, cy, n, kPolicyEvictLast);
          }
        }
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    griddep_launch_dependents();  // this CTA's last loads are issued
    // Teardown: every copy issued must land before the CTA exits (matters only when
    // another role aborted early).
    if (lane == 0) {
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
      constexpr uint32_t idesc =
          make_idesc(kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt);
      // bilinear k-block: Wb and the coarse box are the 16-bit output type
      constexpr uint32_t kOutFmt = TcElem<typename TcElem<T>::Out>::kFmt;
      constexpr uint32_t idesc_bmn = make_idesc(kTcBlockM, kTcBlockN, kOutFmt, kOutFmt, 1u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int nkb = args.num_kb + (bil_mma ? 1 : 0);
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
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
          if (kb < args.num_kb) {
            const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kTcBStage));
#pragma unroll
            for (int k = 0; k < kMmaPerKb; ++k) {
              // +32 bytes along K per MMA step (encoded >> 4).
              tc_mma<T>(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
            }
          } else {
            // Bilinear k-block: B (coarse box) is MN-major, 64-channel chunks 8 KB apart;
            // +16 box rows (2048 bytes, encoded >> 4) per MMA step.
            const uint64_t bdesc =
                sdesc_mnmajor_sw128(smem_u32(smem_b + stage * kTcBStage), kTcCoarseMaxPix * 128);
#pragma unroll
            for (int k = 0; k < kMmaPerKb; ++k)
              tc_mma_f16(d_tmem, adesc + 2u * k, bdesc + 128u * k, idesc_bmn, 1u);
          }
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
      // Wait for every MMA issued by this thread before TMEM can be released.
      tc_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    if (stage_bias) {
      // (after griddep_wait: the biases may come from the kernel before this one)
      for (int i = threadIdx.x - 64; i < kTcBlockN; i += Cfg::kEpiWarps * 32)
        bias_s[i] = __ldg(args.bias + i);
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::kEpiWarps * 32) : "memory");
    }
    tc_epilogue<kMode, T, false, Cfg::kStageBufs, Cfg::kEpiWarps>(
        args, &map_out, tmem_base, accf_bar, acce_bar, smem_stage, abort_flag, warp, lane,
        bil_mma, 0, stage_bias ? bias_s : nullptr);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

// ---------------------------------------------------------------------------------
// 3x3 conv with halo reuse.  Tiles are 8 wide x 16 high.  For each 64-channel block
// the (16+2) x (8+2) halo of the tile is fetched ONCE by TMA (zero-filled outside the
// image = pad 1) and all nine taps read it in place: the A operand of tap (dy, dx)
// starts at halo row dy*10 + dx, and because a tile row is exactly one 8-row swizzle
// atom, successive atoms are a constant 10 rows (1280 bytes) apart -- a plain
// K-major descriptor with that stride.  Per tile this moves 4 x 23 KB of activations
// instead of 36 x 16 KB; only the weights stream per tap.
constexpr int kHaloBytes = ((kHaloRows * 128 + 1023) / 1024) * 1024;
constexpr int kHaloStages = 4;  // weight stages
constexpr int kHaloBufs = 2;    // halo buffers
struct HaloCfg {
  static constexpr int kOffHalo = kHaloStages * kTcBStage;
  static constexpr int kOffStaging = kOffHalo + kHaloBufs * kHaloBytes;
  static constexpr int kOffBars = kOffStaging + kTcEpiWarps * kTcStagingPerWarp;
  static constexpr int kSmemBytes = kOffBars + 256 + 1024;
};
static_assert(HaloCfg::kSmemBytes <= 232448, "halo smem");

// K-major 128B-swizzle descriptor whose 8-row atoms are `atom_stride` bytes apart and
// whose start need not be 1024-byte aligned.  The base-offset field stays 0: the
// hardware applies the swizzle to the computed address bits, exactly as TMA did when
// it wrote the halo (verified against the CPU oracle; encoding the start's phase in
// the base-offset field gives wrong results).
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128_stride(uint32_t saddr,
                                                              uint32_t atom_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>((atom_stride >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    fpn_conv3x3_halo_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b,
                            const __grid_constant__ CUtensorMap map_out,
                            const __grid_constant__ CUtensorMap map_a2,
                            const __grid_constant__ CUtensorMap map_out2,
                            const __grid_constant__ CUtensorMap map_bh, const TcGemmArgs args) {
  constexpr int S = kHaloStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smem_b = smem;
  uint8_t* smem_halo = smem + HaloCfg::kOffHalo;
  uint8_t* smem_stage = smem + HaloCfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + HaloCfg::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + S;
  uint64_t* hfull_bar = bars + 2 * S;
  uint64_t* hempty_bar = hfull_bar + kHaloBufs;
  uint64_t* accf_bar = hempty_bar + kHaloBufs;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* done_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cin_blocks = args.cin_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int h = 0; h < kHaloBufs; ++h) {
      mbar_init(&hfull_bar[h], 1);
      mbar_init(&hempty_bar[h], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], kTcEpiWarps * 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    prefetch_tmap(&map_out);
    if (args.strip_first > 0) {
      prefetch_tmap(&map_a2);
      prefetch_tmap(&map_out2);
    }
    if (args.pair_tail > 0) prefetch_tmap(&map_bh);
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0, hb = 0, issued = 0, hissued = 0;
      uint32_t phase = 0, hphase = 0;
      bool ok = true;
      // items: tiles, the last pair_tail of them as two channel halves each (N = 128 items
      // load 128 weight rows through map_bh)
      const int items = args.num_tiles + args.pair_tail;
      for (int it = blockIdx.x; ok && it < items; it += gridDim.x) {
        int half;
        const int tile = pair_item_unit(args, args.num_tiles, it, half);
        const HaloTile ht = halo_tile(args, tile);
        const int n = ht.n, x0 = ht.x0, y0 = ht.y0;
        const CUtensorMap* ma = ht.strip ? &map_a2 : &map_a;
        const CUtensorMap* mb = half < 0 ? &map_b : &map_bh;
        const uint32_t bbytes = half < 0 ? kTcBStage : kTcBStage / 2;
        const int brow = half < 0 ? 0 : half * (kTcBlockN / 2);
        for (int cb = 0; ok && cb < cin_blocks; ++cb) {
          if (!mbar_wait(&hempty_bar[hb], hphase ^ 1u, abort_flag, args.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&hfull_bar[hb], kHaloRows * 128);
          tma_load_4d(smem_halo + hb * kHaloBytes, ma, &hfull_bar[hb], cb * kKbElems<T>, x0 - 1,
                      y0 - 1, n, kPolicyEvictLast);
          ++hissued;
          if (++hb == kHaloBufs) {
            hb = 0;
            hphase ^= 1u;
          }
          for (int tap = 0; tap < 9; ++tap) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status,
                           kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full_bar[stage], bbytes);
            tma_load_2d(smem_b + stage * kTcBStage, mb, &full_bar[stage],
                        (tap * cin_blocks + cb) * kKbElems<T>, brow, kPolicyEvictLast);
            ++issued;
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      griddep_launch_dependents();  // this CTA's last loads are issued
      for (int i = 0; i < S && i < issued; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait_drain(&full_bar[stage], phase);
      }
      for (int i = 0; i < kHaloBufs && i < hissued; ++i) {
        if (--hb < 0) {
          hb = kHaloBufs - 1;
          hphase ^= 1u;
        }
        mbar_wait_drain(&hfull_bar[hb], hphase);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_full =
          make_idesc(kTcBlockM, kTcBlockN, TcElem<T>::kFmt, TcElem<T>::kFmt);
      constexpr uint32_t idesc_half =
          make_idesc(kTcBlockM, kTcBlockN / 2, TcElem<T>::kFmt, TcElem<T>::kFmt);
      int stage = 0, hb = 0, acc = 0;
      uint32_t phase = 0, hphase = 0, acc_phase = 0;
      bool ok = true;
      const int items = args.num_tiles + args.pair_tail;
      for (int it = blockIdx.x; ok && it < items; it += gridDim.x) {
        int half;
        const int tile = pair_item_unit(args, args.num_tiles, it, half);
        const uint32_t idesc = half < 0 ? idesc_full : idesc_half;
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcBlockN);
        const int tr = halo_tile(args, tile).tr;
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
            const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(smem_b + stage * kTcBStage));
#pragma unroll
            for (int k = 0; k < kMmaPerKb; ++k)
              tc_mma<T>(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc,
                         (cb > 0 || tap > 0 || k > 0) ? 1u : 0u);
            tc_commit(&empty_bar[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit(&hempty_bar[hb]);
          if (++hb == kHaloBufs) {
            hb = 0;
            hphase ^= 1u;
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
    tc_epilogue<1, T>(args, &map_out, tmem_base, accf_bar, acce_bar, smem_stage, abort_flag, warp,
                      lane, false, 0, nullptr, nullptr, &map_out2);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

}  // namespace ufpn
