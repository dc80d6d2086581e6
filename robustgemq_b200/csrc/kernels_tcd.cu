// Decode-batch grouped dequant GEMM on tcgen05 with the dequantised weights in
// tensor memory (sm_100a).
//
// Same product as k_moe_tc (D[n, t] = sum_k deq(W_e)[k, n] * act[row_t, k], fp32 in
// TMEM; the reference's x @ deq(W), dequant_group_gemm.py:109-138) for token tiles
// of 16 or 32 rows (decode batches, where each expert sees a handful of tokens and
// the kernel must stream packed weights at HBM speed) and of 64 rows (prefill).
// Differences from k_moe_tc:
//   * the dequant warps write the A tile (128 features x 128 k per stage and
//     matrix) straight into tensor memory with tcgen05.st, and the MMA reads A from
//     there: the tile never round-trips through shared memory;
//   * K advances in stages of 128 and the activations arrive in the slot order of
//     kperm.cuh (written so by dispatch / the gate-up epilogue), so every column of
//     the A tile is one shift + one mask of a packed word, then the exact
//     fma.rn.f16 dequant (utils.py:206-210);
//   * scale / zero rows are fetched 16 groups at a time into their own ring, and
//     the per-stage copies are issued by two producer warps (one issuing lane
//     sustains roughly one bulk tensor copy per 100+ cycles); packed words, scales
//     and zeros are read with an L2 evict-first policy (read once per launch);
//   * the down projection (route-weight mode) pairs two 128-feature tiles of the
//     same expert in one work item, as the two "matrices" of the gate/up item.
//
// Warps (768 threads, one CTA per SM; work items round-robin, see ItemWalk):
//   0      producer: activation sub-tile 0 (k0..k0+63) and packed words of matrix 0
//   1      TMEM allocation; MMA issue and commits from an elected lane
//   2      producer: activation sub-tile 1 (k0+64..k0+127) and words of matrix 1
//   3      producer: scale / zero chunks
//   4-7    epilogue: tcgen05.ld -> rounding -> global stores (lane quarter = warp % 4)
//   8-23   dequant: two groups of 8 warps taking alternate stages of the CTA's whole
//          stage sequence (group (w-8)/8 the even / odd ones); in a group, warp w
//          owns features 32*(w%4) .. +31 (its TMEM lane quarter) of matrix
//          ((w-8)/4)%2, all 128 k
// Every wait is bounded (gemq_common.cuh); on expiry all roles drain and return.
#include <cudaTypedefs.h>

#include <utility>

#include "gemq_common.cuh"
#include "gemq_internal.h"
#include "kperm.cuh"
#include "tc_work.cuh"

namespace gemq {

namespace {

using tcw::Meta;
using tcw::Work;

// Two groups of eight dequant warps take alternate stages; in a group, one warp per
// (matrix, TMEM lane quarter) dequantises all 128 k of its matrix. While one group
// waits for and reads a stage, the other group's warps on the same sub-partition
// compute, so the integer and fp16 pipes stay busy.
constexpr int kDqWarp0 = 8;
constexpr int kDqGroup = 8;  // warps per group
constexpr int kNumDqWarps = 2 * kDqGroup;
constexpr int kThreadsD = 32 * (kDqWarp0 + kNumDqWarps);
constexpr int kSK = kperm::kStageK;  // 128
constexpr int kScRows = 16;          // scale rows (groups) per chunk
constexpr int kMaxWordRows = 16;
constexpr uint32_t kIdleSleepNs = 256;  // pause between polls of waiters off the critical path
// Pause between polls of the dequant warps and the MMA issuer: a spinning warp takes
// issue slots and integer-pipe cycles from the dequant warps of its sub-partition.
constexpr uint32_t kBusySleepNs = 64;
// Items per CTA whose segment is looked up once at kernel start (later ones search).
constexpr int kMaxCtaItems = 256;

__constant__ kperm::Perm3 c_perm3 = kperm::make_perm3();

__host__ __device__ constexpr int cmin_d(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int round_up_d(int v, int m) { return (v + m - 1) / m * m; }

template <int NT, GemmMode MODE, bool SUB>
struct CfgD {
  static constexpr bool kSub = SUB;  // subnormal-operand dequant (see dq_col_sub)
  // Two matrices per work item: w1 and w3 for SwiGLU; for the down projection two
  // adjacent 128-feature tiles of w2, so both modes have the same per-stage shape.
  static constexpr int kMats = 2;
  static constexpr bool kPairTiles = (MODE == GemmMode::kRouteWeight);
  static constexpr int kActSub = NT * 128;  // one 64-wide SW128 sub-tile
  static constexpr int kActBytes = 2 * kActSub;
  static constexpr int kWordBytes = kMaxWordRows * 128 * 4;
  static constexpr int kStageBytes = round_up_d(kActBytes + kMats * kWordBytes, 1024);
  static constexpr int kScBytes = kScRows * 128 * 2;
  static constexpr int kChunkBytes = kMats * 2 * kScBytes;
  // route-weight epilogue: each of the 4 epilogue warps stages 16 rows of its 64
  // output columns (32 per feature tile) before writing them as 16-byte pieces
  static constexpr int kOutBytes = (MODE == GemmMode::kRouteWeight) ? 4 * 16 * 64 * 2 : 0;
  static constexpr int kItemBytes = kMaxCtaItems * 4;  // segment of each of the CTA's items
  static constexpr int kBudget = 225 * 1024 - tcw::kMetaBytes - 2 * kChunkBytes - 2048 - kOutBytes - kItemBytes;
  static constexpr int kStages = cmin_d(8, kBudget / kStageBytes);
  static constexpr int kChunkOff = kStages * kStageBytes;
  static constexpr int kOutOff = kChunkOff + 2 * kChunkBytes;
  static constexpr int kItemOff = kOutOff + kOutBytes;
  static constexpr int kBarOff = kItemOff + kItemBytes;
  // TMEM: accumulator buffers (two when they fit beside the A ring, so one item's
  // epilogue overlaps the next item's MMAs), then the A ring.
  static constexpr int kAccCols = kMats * NT;  // one accumulator buffer
  static constexpr int kACols = kMats * 64;    // one A stage: 128 fp16 k per matrix
  static constexpr int kAccBufs = (2 * kAccCols + 2 * kACols <= 512) ? 2 : 1;
  static constexpr int kACol0 = kAccBufs * kAccCols;  // first A column
  static constexpr int kAStages = cmin_d(3, (512 - kACol0) / kACols);
  static constexpr int kNumBars = 2 * kStages + 4 + 2 * kAStages + 5;
  static constexpr int kMetaOff = round_up_d(kBarOff + kNumBars * 8 + 16, 16);
  static constexpr int kSmemBytes = kMetaOff + tcw::kMetaBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kIdesc = idesc_f16_f32(128, NT);
  static_assert(kStages >= 3, "shared memory budget too small");
  static_assert(kAStages >= 2, "tensor memory budget too small");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget exceeded");
  static_assert(kACol0 + kAStages * kACols <= 512, "tensor memory budget exceeded");
};

struct KArgsD {
  const int32_t* nbits;
  const int32_t* wq_strides0;
  const int32_t* zs_strides0;
  const int32_t* wq_strides1;
  const int32_t* zs_strides1;
  const Seg* segs;
  const int32_t* tile_prefix;
  int num_segs;
  int N;
  int K;
  int group_size;
  int n_tiles;
  void* out;
  int64_t out_ld;
  const __half* row_weight;
  const int32_t* perm_out_nbits;  // kSwiGLU: store h in the slot order of these bit-widths
  // Chained gate/up -> down launch of one forward: per token tile, the number of
  // gate/up epilogue warps that have stored their h columns. kSwiGLU adds to it and
  // lets the down launch start early; kRouteWeight waits for chain_target before
  // loading a tile's h rows (and skips the grid-completion wait).
  int32_t* chain_done;
  int chain_target;
};

// Packed-word maps per matrix and box height (4, 8, 14, 16 rows for b = 1, 2, 3, 4).
struct WordMapsD {
  CUtensorMap m[2][4];
};
__host__ __device__ constexpr int box_index(int nb) { return nb - 1; }

// ---------------------------------------------------------------- work order
// CTA c's work items: round-robin over the whole waves (items c, c + G, ...), then
// one item of the last, partial wave in reverse CTA order. Dispatch orders the
// segments by dequant cost, heaviest bit-width first, so the last wave holds the
// cheapest items and they go to the CTAs whose earlier items were the cheapest.
struct ItemWalk {
  int j, n, full;
  __device__ __forceinline__ explicit ItemWalk(int total) : j(0) {
    const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
    full = total / G * G;
    n = total / G + ((G - 1 - c) < total - full ? 1 : 0);
  }
  // the CTA's item number i
  __device__ __forceinline__ int w_of(int i) const {
    const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
    return (i * G < full) ? i * G + c : full + (G - 1 - c);
  }
  __device__ __forceinline__ bool next(int& w) {
    if (j >= n) return false;
    w = w_of(j);
    ++j;
    return true;
  }
};

// ---------------------------------------------------------------- dequant
struct ScaleSet {
  __half2 s0, s1, s01, z0, z1, z01;
  __half2 t0, t1, t01;  // subnormal form: the scales of the second offset class
};

// Column C (codes of slots 2C, 2C+1) of a stage as the fma.rn.f16 dequant pair.
// Pairs are (j, j + eps/2) of one word for b in {1, 2, 4} (both codes at offset b*j
// of their 16-bit halves; offsets past the fp16 mantissa read the word shifted right
// by 8) and (j, j + 5) for 3-bit (codes j at bit 3j, j + 5 at bit 15 + 3j; the word
// shifted left by 1 or right by 8 brings each pair inside the mantissas).
template <int NB, int PH, bool G2, int C>
__device__ __forceinline__ uint32_t dq_col(const uint32_t (&w)[kMaxWordRows], const ScaleSet& sc) {
  if constexpr (NB == 3) {
    constexpr kperm::Pair3 pr = kperm::pair3(PH, C);
    constexpr bool ga = G2 && pr.qa >= 64, gb = G2 && pr.qb >= 64;
    const __half2 s2 = ga ? sc.s1 : (gb ? sc.s01 : sc.s0);
    const __half2 z2 = ga ? sc.z1 : (gb ? sc.z01 : sc.z0);
    if constexpr (pr.kind == 0) {
      const uint32_t x = w[pr.wa];
      if constexpr (pr.sa == 0) return dq_pair_at<3, 1, 0>(x << 1, s2, z2);
      if constexpr (pr.sa == 1) return dq_pair_at<3, 3, 2>(x, s2, z2);
      if constexpr (pr.sa == 2) return dq_pair_at<3, 6, 5>(x, s2, z2);
      if constexpr (pr.sa == 3) return dq_pair_at<3, 1, 0>(x >> 8, s2, z2);
      return dq_pair_at<3, 4, 3>(x >> 8, s2, z2);
    } else {
      const uint32_t x = ((w[pr.wa] >> (3 * pr.sa)) & 7u) | (((w[pr.wb] >> (3 * pr.sb)) & 7u) << 16);
      return dq_pair_at<3, 0, 0>(x, s2, z2);
    }
  } else {
    constexpr int eps = 32 / NB;
    constexpr int qa = kperm::perm_pow2(NB, 2 * C);
    constexpr int wi = qa / eps, j = qa % eps;
    constexpr int o = NB * j;
    constexpr int sh = (o + NB <= 10) ? 0 : 8;
    const uint32_t x = sh ? (w[wi] >> 8) : w[wi];
    constexpr bool g1 = G2 && qa >= 64;
    return dq_pair_at<NB, o - sh, o - sh>(x, g1 ? sc.s1 : sc.s0, g1 ? sc.z1 : sc.z0);
  }
}

// The same column in the subnormal-operand form. The pair is moved (one shift per
// word and shift amount, shared by the pairs that use it) to mantissa offsets where
// the fp16 halves, with a zero exponent field, read exactly q * 2^(o - 24); the scales
// carry the inverse power of two in their exponent, s * 2^(24 - o) (exact: a power of
// two added to the exponent of a normal number that stays finite). One mask and one
// fma.rn.f16x2 then give fp16(q * s + z) with its single rounding: the value
// utils.py:206-210 rounds, so the weights are bit-identical to the magic-number form,
// with one fp16 instruction per pair instead of two. Offsets: b = 2 at 6 and 8,
// b = 1 at 8 and 9, b = 4 at 6, b = 3 at (6, 5) per half for (j, j + 5) pairs and
// (6, 6) for the pairs that straddle words. The launcher takes this form only when
// every scale of the projection is a normal number with s * 2^(24 - o) finite
// (scale_exponents_ok).
template <int NB, int PH, bool G2, int C>
__device__ __forceinline__ uint32_t dq_col_sub(const uint32_t (&w)[kMaxWordRows], const ScaleSet& sc) {
  if constexpr (NB == 3) {
    constexpr kperm::Pair3 pr = kperm::pair3(PH, C);
    constexpr bool ga = G2 && pr.qa >= 64, gb = G2 && pr.qb >= 64;
    if constexpr (pr.kind == 0) {
      const __half2 s2 = ga ? sc.s1 : (gb ? sc.s01 : sc.s0);
      const __half2 z2 = ga ? sc.z1 : (gb ? sc.z01 : sc.z0);
      constexpr int sh = 6 - 3 * pr.sa;  // code sa: bit 3 sa -> 6; code sa + 5: bit 15 + 3 sa -> 21
      const uint32_t x = sh >= 0 ? (w[pr.wa] << sh) : (w[pr.wa] >> (-sh));
      constexpr uint32_t mask = (7u << 6) | (7u << 21);
      return h2_as_u32(__hfma2(u32_as_h2(x & mask), s2, z2));
    } else {
      const __half2 s2 = ga ? sc.t1 : (gb ? sc.t01 : sc.t0);
      const __half2 z2 = ga ? sc.z1 : (gb ? sc.z01 : sc.z0);
      const uint32_t lo = ((w[pr.wa] >> (3 * pr.sa)) & 7u) << 6;
      const uint32_t hi = ((w[pr.wb] >> (3 * pr.sb)) & 7u) << 22;
      return h2_as_u32(__hfma2(u32_as_h2(lo | hi), s2, z2));
    }
  } else {
    constexpr int eps = 32 / NB;
    constexpr int qa = kperm::perm_pow2(NB, 2 * C);
    constexpr int wi = qa / eps, j = qa % eps;
    constexpr bool alt = (NB != 4) && (j & 1);  // second offset class (b = 1, 2)
    constexpr int o = NB == 4 ? 6 : (NB == 2 ? 6 : 8) + (alt ? (NB == 2 ? 2 : 1) : 0);
    constexpr int sh = o - NB * j;
    const uint32_t x = sh >= 0 ? (w[wi] << sh) : (w[wi] >> (-sh));
    constexpr uint32_t cm = (1u << NB) - 1u;
    constexpr uint32_t mask = (cm << o) | (cm << (o + 16));
    constexpr bool g1 = G2 && qa >= 64;
    const __half2 s2 = g1 ? (alt ? sc.t1 : sc.s1) : (alt ? sc.t0 : sc.s0);
    return h2_as_u32(__hfma2(u32_as_h2(x & mask), s2, g1 ? sc.z1 : sc.z0));
  }
}

template <bool SUB, int NB, int PH, bool G2, int C0, int NC, int... Cs>
__device__ __forceinline__ void dq_cols(const uint32_t (&w)[kMaxWordRows], const ScaleSet& sc, uint32_t (&o)[NC],
                                        std::integer_sequence<int, Cs...>) {
  if constexpr (SUB) ((o[Cs] = dq_col_sub<NB, PH, G2, C0 + Cs>(w, sc)), ...);
  else ((o[Cs] = dq_col<NB, PH, G2, C0 + Cs>(w, sc)), ...);
}

// Dequantises columns [C0, C0 + NC) of a stage and stores them to TMEM at `taddr`.
// Stored 16 columns at a time, so that only 16 results are live at once.
template <bool SUB, int NB, int PH, bool G2, int C0, int NC>
__device__ __forceinline__ void dq_store(const uint32_t (&w)[kMaxWordRows], const ScaleSet& sc, uint32_t taddr) {
  static_assert(NC % 16 == 0, "columns are stored 16 at a time");
  uint32_t o[16];
  dq_cols<SUB, NB, PH, G2, C0, 16>(w, sc, o, std::make_integer_sequence<int, 16>{});
  tmem_st16(taddr, o);
  if constexpr (NC > 16) dq_store<SUB, NB, PH, G2, C0 + 16, NC - 16>(w, sc, taddr + 16u);
}

// fp16 bits of h with k added to the exponent field (h * 2^k for a normal h whose
// result stays finite), as the low / high halves of a pair
__device__ __forceinline__ __half2 exp_pair(__half lo, int klo, __half hi, int khi) {
  const uint32_t a = static_cast<uint32_t>(__half_as_ushort(lo)) + (static_cast<uint32_t>(klo) << 10);
  const uint32_t b = static_cast<uint32_t>(__half_as_ushort(hi)) + (static_cast<uint32_t>(khi) << 10);
  return u32_as_h2((a & 0xffffu) | (b << 16));
}

// Scale / zero registers of a stage for either dequant form.
template <bool SUB, int NB>
__device__ __forceinline__ ScaleSet make_scales(__half sa, __half za, __half sb, __half zb) {
  ScaleSet sc;
  sc.z0 = __halves2half2(za, za);
  sc.z1 = __halves2half2(zb, zb);
  sc.z01 = __halves2half2(za, zb);
  if constexpr (!SUB) {
    sc.s0 = __halves2half2(sa, sa);
    sc.s1 = __halves2half2(sb, sb);
    sc.s01 = __halves2half2(sa, sb);
  } else if constexpr (NB == 3) {
    sc.s0 = exp_pair(sa, 18, sa, 19);
    sc.s1 = exp_pair(sb, 18, sb, 19);
    sc.s01 = exp_pair(sa, 18, sb, 19);
    sc.t0 = exp_pair(sa, 18, sa, 18);
    sc.t1 = exp_pair(sb, 18, sb, 18);
    sc.t01 = exp_pair(sa, 18, sb, 18);
  } else {
    constexpr int k0 = NB == 1 ? 16 : 18;               // offset 8 (b = 1) / 6 (b = 2, 4)
    constexpr int k1 = NB == 1 ? 15 : (NB == 2 ? 16 : 18);  // offset 9 / 8
    sc.s0 = exp_pair(sa, k0, sa, k0);
    sc.s1 = exp_pair(sb, k0, sb, k0);
    sc.t0 = exp_pair(sa, k1, sa, k1);
    sc.t1 = exp_pair(sb, k1, sb, k1);
  }
  return sc;
}

// Ring positions and barriers a dequant warp walks through; advanced in place.
struct DqRings {
  int s, as, c;
  uint32_t ph, aph, cph;
};

// Shared addresses of the kernel's mbarriers, in array order: full[kStages],
// empty[kStages], sfull[2], sempty[2], afull[kAStages], aempty[kAStages].
template <class C>
struct BarsD {
  static __device__ __forceinline__ uint32_t full(uint32_t b, int s) { return b + 8u * s; }
  static __device__ __forceinline__ uint32_t empty(uint32_t b, int s) { return b + 8u * (C::kStages + s); }
  static __device__ __forceinline__ uint32_t sfull(uint32_t b, int c) { return b + 8u * (2 * C::kStages + c); }
  static __device__ __forceinline__ uint32_t sempty(uint32_t b, int c) { return b + 8u * (2 * C::kStages + 2 + c); }
  static __device__ __forceinline__ uint32_t afull(uint32_t b, int a) { return b + 8u * (2 * C::kStages + 4 + a); }
  static __device__ __forceinline__ uint32_t aempty(uint32_t b, int a) {
    return b + 8u * (2 * C::kStages + 4 + C::kAStages + a);
  }
};

// Everything a dequant warp needs for one work item besides its rings.
struct DqEnv {
  uint8_t* stages;         // stage ring base (shared memory)
  const uint8_t* chunks;   // scale / zero chunk ring base
  uint32_t bars;           // shared address of the barrier array (layout: BarsD)
  uint32_t a_col0;         // TMEM address of this warp's lane quarter, A ring column 0
  uint32_t n;              // feature row inside the tile (= TMEM lane)
  int lane, mat, grp, KT, log2g;
};

// Packed words and scale / zero of one stage and feature row, held in registers.
struct DqStage {
  uint32_t w[kMaxWordRows];
  __half sa, za, sb, zb;
};

// Moves a dequant warp's scale-chunk ring to chunk `target` (the chunk of 16 scale
// groups its next stage reads): the chunk held is released, and so is every chunk
// passed over without being read (an item's last chunk may hold only stages of the
// other group), so each slot the producer fills gets all warps' releases. A chunk
// passed over is waited for before its release, so that the release cannot count
// toward the slot's previous round. With `wait`, waits for the target chunk too.
// `ch` is the chunk held (-1: none).
template <class C>
__device__ __forceinline__ bool dq_chunk_to(int target, bool wait, int& ch, DqRings& r, const DqEnv& e) {
  using Bar = BarsD<C>;
  if (ch == target) return true;
  auto release = [&]() {
    __syncwarp();
    if (e.lane == 0) mbar_arrive(Bar::sempty(e.bars, r.c));
    if (++r.c == 2) { r.c = 0; r.cph ^= 1u; }
  };
  if (ch >= 0) release();
  for (int c2 = ch + 1; c2 < target; ++c2) {
    if (!warp_wait(Bar::sfull(e.bars, r.c), r.cph, kDevTimeoutTmaFull, kBusySleepNs)) return false;
    release();
  }
  ch = target;
  return !wait || warp_wait(Bar::sfull(e.bars, r.c), r.cph, kDevTimeoutTmaFull, kBusySleepNs);
}
__device__ __forceinline__ int chunk_of(int kt, int log2g) { return ((kt * kSK) >> log2g) / kScRows; }

// Reads stage kt (ring slot r.s) of a dequant warp's feature row into `d` and
// releases the slot; `tok` is the result of an earlier try_wait on its full barrier.
template <class C, int NB, bool G2>
__device__ __forceinline__ bool dq_fetch(int kt, DqStage& d, bool tok, int ch, const DqRings& r, const DqEnv& e) {
  constexpr int kRows = kperm::stage_word_rows(NB);
  using Bar = BarsD<C>;
  if (!warp_wait_tok(Bar::full(e.bars, r.s), r.ph, tok, kDevTimeoutTmaFull, kBusySleepNs)) return false;
  const uint32_t* wcol =
      reinterpret_cast<const uint32_t*>(e.stages + r.s * C::kStageBytes + C::kActBytes + e.mat * C::kWordBytes) + e.n;
#pragma unroll
  for (int i = 0; i < kMaxWordRows; ++i) d.w[i] = (i < kRows) ? wcol[i * 128] : 0u;
  const __half* sp = reinterpret_cast<const __half*>(e.chunks + r.c * C::kChunkBytes + (2 * e.mat) * C::kScBytes) + e.n;
  const __half* zp = sp + C::kScBytes / 2;
  const int r0 = (((kt * kSK) >> e.log2g) - ch * kScRows) * 128;
  d.sa = sp[r0];
  d.za = zp[r0];
  d.sb = d.sa;
  d.zb = d.za;
  if constexpr (G2) {
    d.sb = sp[r0 + 128];
    d.zb = zp[r0 + 128];
  }
  __syncwarp();
  if (e.lane == 0) mbar_arrive(Bar::empty(e.bars, r.s));
  return true;
}

// One work item of one dequant warp, specialised by bit-width, group layout and the
// warp's columns [C0, C0 + NC) of its matrix. The two groups take alternate stages
// of the CTA's whole sequence of stages (all its items back to back), so this warp's
// stages in the item are kt0, kt0 + 2, ... with kt0 = (grp + stages before the item)
// % 2. For each: read the packed words and scale / zero of its feature row, release
// the stage, dequantise into TMEM and hand the A stage to the MMA. The first poll of
// its next stage's A slot is issued while the TMEM stores are in flight. Ring
// positions (two per own stage) stay on this warp's next own stage across items.
//
// The A slot waits are parity tests, unambiguous only while the slot's reads lag the
// position waited for by at most one round: the MMA must have read position
// P - 2 * kAStages. It reads positions in order, and once this warp's wait for
// position Q has passed it has read every position up to Q - kAStages. This warp
// waits (and polls) positions two apart, in this item or the next, so kAStages >= 2
// is enough. (Restarting each item at kt = grp would make group 1 jump three
// positions after an item with an odd stage count.)
// Returns false if a wait expired.
template <class C, int NB, bool G2, int C0, int NC>
__device__ __forceinline__ bool dq_item(int kt0, DqRings& r, const DqEnv& e) {
  using Bar = BarsD<C>;
  int ch = -1;
  // 3-bit phase index of stage kt: P = (128 kt) % 10 = 0, 8, 6, 4, 2 -> P / 2
  int ph3 = ((kSK * kt0) % 10) / 2;
  bool tok_a = false;
  // the group's stages only (every chunk of 16 scale groups either holds stages of
  // both groups or is passed over and released by dq_chunk_to)
  for (int kt = kt0; kt < e.KT; kt += 2) {
    if (!dq_chunk_to<C>(chunk_of(kt, e.log2g), true, ch, r, e)) return false;
    {
      const bool tok_f = mbar_try_wait(Bar::full(e.bars, r.s), r.ph);
      // item's first own stage: poll its A slot before the fetch. With two slots that
      // slot's last use is this warp's previous stage, still being read by the MMA, and
      // the try_wait would hold the fetch back: the fetch goes first then.
      if (C::kAStages > 2 && kt == kt0) tok_a = mbar_try_wait(Bar::aempty(e.bars, r.as), r.aph ^ 1u);
      DqStage cur;
      if (!dq_fetch<C, NB, G2>(kt, cur, tok_f, ch, r, e)) return false;
      if (!warp_wait_tok(Bar::aempty(e.bars, r.as), r.aph ^ 1u, tok_a, kDevTimeoutAEmpty, kBusySleepNs))
        return false;
      tc_fence_after();
      constexpr bool kSub = C::kSub;
      const ScaleSet sc = make_scales<kSub, NB>(cur.sa, cur.za, cur.sb, cur.zb);
      const uint32_t taddr = e.a_col0 + static_cast<uint32_t>(r.as * C::kACols + e.mat * 64 + C0);
      if constexpr (NB == 3) {
        switch (ph3) {
          case 0: dq_store<kSub, 3, 0, G2, C0, NC>(cur.w, sc, taddr); break;
          case 1: dq_store<kSub, 3, 1, G2, C0, NC>(cur.w, sc, taddr); break;
          case 2: dq_store<kSub, 3, 2, G2, C0, NC>(cur.w, sc, taddr); break;
          case 3: dq_store<kSub, 3, 3, G2, C0, NC>(cur.w, sc, taddr); break;
          default: dq_store<kSub, 3, 4, G2, C0, NC>(cur.w, sc, taddr); break;
        }
      } else {
        dq_store<kSub, NB, 0, G2, C0, NC>(cur.w, sc, taddr);
      }
      // first poll of the A slot of this warp's next stage (two positions on), in
      // flight with the stores; unambiguous as the waits are (see dq_item). With two
      // A slots that is the slot just written, which the MMA cannot release before
      // this warp hands it over: no poll then (try_wait may block until a time limit).
      if constexpr (C::kAStages > 2) {
        int as2 = r.as + 2;
        uint32_t aph2 = r.aph;
        if (as2 >= C::kAStages) { as2 -= C::kAStages; aph2 ^= 1u; }
        tok_a = mbar_try_wait(Bar::aempty(e.bars, as2), aph2 ^ 1u);
      } else {
        tok_a = false;
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (e.lane == 0) mbar_arrive(Bar::afull(e.bars, r.as));
    }
    // two ring positions on
    r.s += 2;
    if (r.s >= C::kStages) { r.s -= C::kStages; r.ph ^= 1u; }
    r.as += 2;
    if (r.as >= C::kAStages) { r.as -= C::kAStages; r.aph ^= 1u; }
    if constexpr (NB == 3) ph3 = (ph3 + 3) % 5;
  }
  // release the item's remaining scale chunks, through its last
  dq_chunk_to<C>(chunk_of(e.KT - 1, e.log2g) + 1, false, ch, r, e);
  return true;
}

template <class C, bool G2, int C0, int NC>
__device__ __forceinline__ bool dq_item_nb(int nb, int kt0, DqRings& r, const DqEnv& e) {
  switch (nb) {
    case 1: return dq_item<C, 1, G2, C0, NC>(kt0, r, e);
    case 2: return dq_item<C, 2, G2, C0, NC>(kt0, r, e);
    case 3: return dq_item<C, 3, G2, C0, NC>(kt0, r, e);
    default: return dq_item<C, 4, G2, C0, NC>(kt0, r, e);
  }
}

template <class C, int C0, int NC>
__device__ __forceinline__ bool dq_item_any(bool g2, int nb, int kt0, DqRings& r, const DqEnv& e) {
  return g2 ? dq_item_nb<C, true, C0, NC>(nb, kt0, r, e) : dq_item_nb<C, false, C0, NC>(nb, kt0, r, e);
}

// Destination column of source column f of the next projection's input.
__device__ __forceinline__ int perm_dst(int nb, int f) {
  const int st = f >> 7, q = f & 127;
  if (nb == 3) return (st << 7) + c_perm3.inv[kperm::phase3(st)][q];
  return (st << 7) + kperm::inv_pow2(nb, q);
}

// ---------------------------------------------------------------- epilogue math
// F.silu in fp32 from the hardware exponential and reciprocal: within a few fp32 ulps
// of x / (1 + exp(-x)); the caller rounds it to fp16, as torch does, so the two differ
// only where the exact value sits within those ulps of an fp16 rounding midpoint
// (one fp16 ulp there; the exponential's error grows with |x|, to about 14 ulps at
// |x| = 10). The exponent is clamped at 80 so the divisor stays below 2^126, where
// the fast quotient is defined; silu(x) for x < -80 has magnitude below 2^-100 and
// rounds to -0 in fp16 either way.
__device__ __forceinline__ float silu_fast_d(float x) { return __fdividef(x, 1.f + __expf(fminf(-x, 80.f))); }

// ---------------------------------------------------------------- the kernel
template <int NT, GemmMode MODE, bool SUB>
__global__ void __launch_bounds__(kThreadsD, 1)
    k_moe_tcd(const KArgsD p, const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ WordMapsD tm_words,
              const __grid_constant__ CUtensorMap tm_s0, const __grid_constant__ CUtensorMap tm_z0,
              const __grid_constant__ CUtensorMap tm_s1, const __grid_constant__ CUtensorMap tm_z1) {
  using C = CfgD<NT, MODE, SUB>;
  constexpr int kMats = C::kMats;
  constexpr int kStages = C::kStages;
  constexpr int kAStages = C::kAStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned, derived from the shared array by pointer arithmetic so that the
  // compiler keeps reads through it as shared-memory loads
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* full = bars;                   // [kStages] activations + words landed
  uint64_t* empty = full + kStages;        // [kStages] stage consumed
  uint64_t* sfull = empty + kStages;       // [2] scale chunk landed
  uint64_t* sempty = sfull + 2;            // [2] scale chunk consumed
  uint64_t* afull = sempty + 2;            // [kAStages] A stage written to TMEM
  uint64_t* aempty = afull + kAStages;     // [kAStages] A stage read by the MMAs
  uint64_t* acc_full = aempty + kAStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 2);       // both producers arm the stage
      mbar_init(&empty[s], 1 + kDqGroup);  // MMA commit + the stage's dequant group
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&sfull[c], 1);
      mbar_init(&sempty[c], kNumDqWarps);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&afull[s], kDqGroup);
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  // everything above is private to this CTA; from here on it reads the segment
  // table, activations and weights, and writes outputs other kernels use. A chained
  // down launch reads the segment table and routing weights the dispatch wrote before
  // the gate/up launch got past its own wait, and waits per tile for h instead.
  const bool chained_down = MODE == GemmMode::kRouteWeight && p.chain_done != nullptr;
  if (!chained_down) grid_dep_wait();
  Meta& meta = *reinterpret_cast<Meta*>(smem + C::kMetaOff);
  tcw::stage_meta(meta, p, false);
  __syncthreads();
  const int total = meta.tp[p.num_segs] * p.n_tiles;
  // segment of each of the CTA's first kMaxCtaItems items, searched once here instead
  // of by every role at every item
  int* item_seg = reinterpret_cast<int*>(smem + C::kItemOff);
  {
    const ItemWalk iw(total);
    for (int i = threadIdx.x; i < iw.n && i < kMaxCtaItems; i += blockDim.x)
      item_seg[i] = tcw::seg_of_tile(meta, p.num_segs, iw.w_of(i) / p.n_tiles);
  }
  __syncthreads();
  auto work_of = [&](int i, int w) {
    return i < kMaxCtaItems ? tcw::work_in_seg<NT>(meta, item_seg[i], p.n_tiles, w)
                            : tcw::decode_work<NT>(meta, p.num_segs, p.n_tiles, w);
  };
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KT = p.K / kSK;
  const int g = p.group_size;
  const int groups = p.K / g;
  const int nchunks = (groups + kScRows - 1) / kScRows;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ stage producers
    {
      const bool first = (warp == 0);
      const int mat = first ? 0 : 1;
      const uint64_t stream_policy = l2_evict_first_policy();
      if (elect_one()) {
        if (first) {
          tma_prefetch_desc(&tm_act);
          for (int i = 0; i < 4; ++i) tma_prefetch_desc(&tm_words.m[0][i]);
        } else if (kMats == 2) {
          for (int i = 0; i < 4; ++i) tma_prefetch_desc(&tm_words.m[1][i]);
        }
      }
      __syncwarp();
      int s = 0;
      uint32_t ph = 0;
      int armed = 0;
      bool ok = true;
      ItemWalk items(total);
      int w;
      while (ok && items.next(w)) {
        const Work wk = work_of(items.j - 1, w);
        const int nb = min(max(wk.nb, 1), 4);
        const int rows = kperm::stage_word_rows(nb);
        const bool words = first || kMats == 2;
        const uint32_t tx = C::kActSub + (words ? rows * 512 : 0);
        const CUtensorMap* wmap = &tm_words.m[mat][box_index(nb)];
        const int wrow = first ? wk.wrow0 : wk.wrow1;
        const int ncol = C::kPairTiles ? 2 * wk.n0 + mat * 128 : wk.n0;
        if (chained_down) {  // the tile's h rows: every gate/up item of the tile stored
          bool done = true;
          if (elect_one()) done = tile_done_wait(p.chain_done + w / p.n_tiles, p.chain_target);
          if (__any_sync(0xffffffffu, !done)) {
            ok = false;
            break;
          }
        }
        for (int kt = 0; kt < KT; ++kt) {
          if (!warp_wait(&empty[s], ph ^ 1u, kDevTimeoutTmaEmpty, kIdleSleepNs)) { ok = false; break; }
          uint8_t* st = smem + s * C::kStageBytes;
          if (elect_one()) {
            mbar_arrive_expect_tx(&full[s], tx);
            tma_load_2d(st + mat * C::kActSub, &tm_act, &full[s], kt * kSK + mat * 64, wk.act_row);
            if (words)
              tma_load_2d_hint(st + C::kActBytes + mat * C::kWordBytes, wmap, &full[s], ncol,
                               wrow + kperm::stage_word_row(nb, kt), stream_policy);
          }
          __syncwarp();
          ++armed;
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      for (int st = 0; st < kStages && st < armed; ++st) {
        const int times = (armed - 1 - st) / kStages + 1;
        mbar_wait_drain(&full[st], static_cast<uint32_t>((times - 1) & 1));
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ scale / zero chunks
    {
      const uint64_t stream_policy = l2_evict_first_policy();
      if (elect_one()) {
        tma_prefetch_desc(&tm_s0);
        tma_prefetch_desc(&tm_z0);
        if (kMats == 2) {
          tma_prefetch_desc(&tm_s1);
          tma_prefetch_desc(&tm_z1);
        }
      }
      __syncwarp();
      int c = 0;
      uint32_t cph = 0;
      int armed = 0;
      bool ok = true;
      ItemWalk items(total);
      int w;
      while (ok && items.next(w)) {
        const Work wk = work_of(items.j - 1, w);
        for (int ch = 0; ch < nchunks; ++ch) {
          if (!warp_wait(&sempty[c], cph ^ 1u, kDevTimeoutTmaEmpty, kIdleSleepNs)) { ok = false; break; }
          uint8_t* cb = smem + C::kChunkOff + c * C::kChunkBytes;
          if (elect_one()) {
            mbar_arrive_expect_tx(&sfull[c], C::kChunkBytes);
            const int n0 = C::kPairTiles ? 2 * wk.n0 : wk.n0;
            tma_load_2d_hint(cb, &tm_s0, &sfull[c], n0, wk.srow0 + ch * kScRows, stream_policy);
            tma_load_2d_hint(cb + C::kScBytes, &tm_z0, &sfull[c], n0, wk.srow0 + ch * kScRows, stream_policy);
            if constexpr (kMats == 2) {
              const int n1 = C::kPairTiles ? 2 * wk.n0 + 128 : wk.n0;
              tma_load_2d_hint(cb + 2 * C::kScBytes, &tm_s1, &sfull[c], n1, wk.srow1 + ch * kScRows, stream_policy);
              tma_load_2d_hint(cb + 3 * C::kScBytes, &tm_z1, &sfull[c], n1, wk.srow1 + ch * kScRows, stream_policy);
            }
          }
          __syncwarp();
          ++armed;
          if (++c == 2) { c = 0; cph ^= 1u; }
        }
      }
      for (int st = 0; st < 2 && st < armed; ++st) {
        const int times = (armed - 1 - st) / 2 + 1;
        mbar_wait_drain(&sfull[st], static_cast<uint32_t>((times - 1) & 1));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop; one elected lane (always the same, lane 0 of a
    // converged warp) issues every MMA and commit, so each commit tracks them all.
    {
      int s = 0, as = 0;
      uint32_t aph = 0;
      int it = 0;
      bool ok = true;
      ItemWalk items(total);
      int w;
      const bool chain_up = MODE == GemmMode::kSwiGLU && p.chain_done != nullptr;
      if (chain_up && items.n == 0) grid_dep_launch();
      for (; ok && items.next(w); ++it) {
        if (chain_up && items.j == items.n) grid_dep_launch();  // this CTA's last item
        const int buf = it % C::kAccBufs;
        const uint32_t d_base = tmem + static_cast<uint32_t>(buf * C::kAccCols);
        if (!warp_wait(&acc_empty[buf], ((it / C::kAccBufs) & 1) ^ 1u, kDevTimeoutAccEmpty, kBusySleepNs)) break;
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt) {
          // The stage's A slot only: each dequant warp of the group waited for the
          // stage's full barrier (activations and words landed) before it arrived on
          // afull, so afull completing orders the stage's copies before these MMAs
          // (release / acquire through the two barriers).
          if (!warp_wait(smem_u32(&afull[as]), aph, kDevTimeoutAFull, kBusySleepNs)) { ok = false; break; }
          tc_fence_after();
          const uint32_t act = smem_u32(smem + s * C::kStageBytes);
          const uint64_t b0 = sdesc_sw128(act);
          const uint32_t a0 = tmem + static_cast<uint32_t>(C::kACol0 + as * C::kACols);
          if (elect_one()) {
            // per matrix, the 8 K=16 steps of the stage: +32 B per step inside a
            // 128-byte row, the second 64-k sub-tile kActSub bytes on
#pragma unroll
            for (int m = 0; m < kMats; ++m)
              umma_f16_ts_k128<C::kActSub / 16>(d_base + static_cast<uint32_t>(m * NT),
                                                a0 + static_cast<uint32_t>(m * 64), b0, C::kIdesc, kt != 0 ? 1u : 0u);
            umma_commit(&empty[s]);
            umma_commit(&aempty[as]);
          }
          __syncwarp();
          if (++s == kStages) s = 0;
          if (++as == kAStages) { as = 0; aph ^= 1u; }
        }
        if (!ok) break;
        if (elect_one()) umma_commit(&acc_full[buf]);
        __syncwarp();
      }
      if (elect_one()) umma_commit(drain);
      __syncwarp();
      mbar_wait_drain(drain, 0);
    }
  } else if (warp < kDqWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int it = 0;
    ItemWalk items(total);
    int w;
    for (; items.next(w); ++it) {
      const int buf = it % C::kAccBufs;
      const uint32_t lane_base =
          tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * C::kAccCols);
      const Work wk = work_of(items.j - 1, w);
      // routing weights of the item's rows, before the wait: lane j holds rows 2j and
      // 2j + 1 as an fp16 pair (loads issued together here, not one per row behind
      // the output stores, which the compiler may not move them past)
      uint32_t wpair = 0;
      if constexpr (MODE == GemmMode::kRouteWeight) {
        const int r = 2 * lane;
        const __half wa = r < wk.rows ? p.row_weight[wk.out_row + r] : __ushort_as_half(0);
        const __half wb = r + 1 < wk.rows ? p.row_weight[wk.out_row + r + 1] : __ushort_as_half(0);
        wpair = h2_as_u32(__halves2half2(wa, wb));
      }
      if (!warp_wait(&acc_full[buf], (it / C::kAccBufs) & 1, kDevTimeoutAccFull, kIdleSleepNs)) break;
      tc_fence_after();
      __half* out = static_cast<__half*>(p.out);
      // 16 token columns at a time; the accumulator buffer goes back to the MMA issuer
      // as soon as the item's last columns are in registers. Two tokens per step, as
      // fp16 pairs: fp16(a) * fp16(b) rounded once to fp16 is the fp32 product
      // rounded to fp16 (the product of two fp16 numbers is exact in fp32).
      const int nck = (min(wk.rows, NT) + 15) >> 4;  // warp-uniform
      if (nck == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      const int f = (MODE == GemmMode::kSwiGLU ? wk.n0 : 2 * wk.n0) + 32 * q + lane;
      int col = f;
      // this warp's staging rows (route-weight mode): [16][64] fp16
      __half* stg = reinterpret_cast<__half*>(smem + C::kOutOff) + q * (16 * 64);
      if constexpr (MODE == GemmMode::kSwiGLU)
        if (p.perm_out_nbits != nullptr) col = perm_dst(min(max(__ldg(p.perm_out_nbits + wk.e), 1), 4), f);
#pragma unroll
      for (int ck = 0; ck < NT / 16; ++ck) {
        if (ck >= nck) break;
        const int c0 = 16 * ck;
        uint32_t r0[16], r1[16];
        tmem_ld16(lane_base + c0, r0);
        tmem_ld16(lane_base + NT + c0, r1);
        tmem_ld_wait();
        if (ck == nck - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const int64_t row = wk.out_row + c0 + i;
          const bool v0 = c0 + i < wk.rows, v1 = c0 + i + 1 < wk.rows;
          const __half2 a0 = __floats2half2_rn(__uint_as_float(r0[i]), __uint_as_float(r0[i + 1]));
          const __half2 a1 = __floats2half2_rn(__uint_as_float(r1[i]), __uint_as_float(r1[i + 1]));
          if constexpr (MODE == GemmMode::kSwiGLU) {
            // x1, x3 stored fp16; F.silu(x1) -> fp16; * x3 -> fp16 (moe_block.py:774-775)
            const float2 x1 = __half22float2(a0);
            const __half2 h = __hmul2(__floats2half2_rn(silu_fast_d(x1.x), silu_fast_d(x1.y)), a1);
            if (v0) out[row * p.out_ld + col] = __low2half(h);
            if (v1) out[(row + 1) * p.out_ld + col] = __high2half(h);
          } else {
            // two feature tiles: y = fp16(acc), y * w -> fp16 (moe_block.py:778, 811),
            // staged as row i: [tile 0: 32 features | tile 1: 32 features]
            const __half2 wv = u32_as_h2(__shfl_sync(0xffffffffu, wpair, (c0 + i) >> 1));
            const __half2 y0 = __hmul2(a0, wv), y1 = __hmul2(a1, wv);
            stg[i * 64 + lane] = __low2half(y0);
            stg[i * 64 + 32 + lane] = __low2half(y1);
            stg[(i + 1) * 64 + lane] = __high2half(y0);
            stg[(i + 1) * 64 + 32 + lane] = __high2half(y1);
          }
        }
        if constexpr (MODE == GemmMode::kRouteWeight) {
          // the chunk's rows: 2 x 64-byte pieces each (one per feature tile), written
          // as 16-byte stores, 8 rows per warp instruction
          __syncwarp();
          const uint4* s4 = reinterpret_cast<const uint4*>(stg);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int idx = lane + 32 * u, r = idx >> 3, pc = idx & 7;
            if (c0 + r < wk.rows)
              *reinterpret_cast<uint4*>(out + (wk.out_row + c0 + r) * p.out_ld + col - lane + (pc >> 2) * 128 +
                                        (pc & 3) * 8) = s4[idx];
          }
          __syncwarp();
        }
      }
      // this warp's h columns of the item are stored: one count on the token tile
      if constexpr (MODE == GemmMode::kSwiGLU)
        if (p.chain_done != nullptr) tile_done_signal(p.chain_done + w / p.n_tiles);
    }
  } else {
    // ------------------------------------------------------------ dequant
    const int dw = warp - kDqWarp0;  // 0..15
    const int q = warp & 3;           // TMEM lane quarter = features 32q .. 32q+31
    DqEnv env;
    env.stages = smem;
    env.chunks = smem + C::kChunkOff;
    env.bars = smem_u32(bars);
    env.a_col0 = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(C::kACol0);
    env.n = static_cast<uint32_t>(32 * q + lane);
    env.lane = lane;
    env.mat = (dw >> 2) & 1;
    env.grp = dw >> 3;
    env.KT = KT;
    env.log2g = 31 - __clz(g);
    const bool g2 = (g == 64);
    // group 1 starts at the CTA's second stage
    DqRings rings{env.grp, env.grp, 0, 0u, 0u, 0u};
    ItemWalk items(total);
    int w;
    for (int it = 0; items.next(w); ++it) {
      const Work wk = work_of(items.j - 1, w);
      if ((wk.nb < 1 || wk.nb > 4) && dw == 0 && lane == 0) set_device_error(kDevBadBits);
      const int nb = min(max(wk.nb, 1), 4);
      const int kt0 = (env.grp + it * KT) & 1;  // first own stage of the item
      if (!dq_item_any<C, 0, 64>(g2, nb, kt0, rings, env)) break;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn_d() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  }
  return fn;
}

bool make_map_d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn_d();
  if (fn == nullptr || base == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_word_maps_d(CUtensorMap (&maps)[4], const ProjDev& w) {
  for (int nb = 1; nb <= 4; ++nb) {
    if (!make_map_d(&maps[box_index(nb)], w.wq, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, w.n, w.wq_rows, 128,
                    kperm::stage_word_rows(nb), CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  return true;
}

template <int NT, GemmMode MODE, bool SUB>
cudaError_t launch_d(const GemmArgs& a, cudaStream_t stream) {
  using C = CfgD<NT, MODE, SUB>;
  CUtensorMap m_act, m_s0, m_z0, m_s1, m_z1;
  WordMapsD words;
  const int K = a.w0.k;
  if (!make_map_d(&m_act, a.act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, static_cast<uint64_t>(a.act_rows), 64, NT,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const uint64_t srows = static_cast<uint64_t>(a.w0.num_experts) * (a.w0.k / a.w0.group_size);
  if (!make_word_maps_d(words.m[0], a.w0) ||
      !make_map_d(&m_s0, a.w0.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w0.n, srows, 128, kScRows,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_d(&m_z0, a.w0.zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w0.n, srows, 128, kScRows,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if constexpr (!C::kPairTiles) {
    const uint64_t srows1 = static_cast<uint64_t>(a.w1.num_experts) * (a.w1.k / a.w1.group_size);
    if (!make_word_maps_d(words.m[1], a.w1) ||
        !make_map_d(&m_s1, a.w1.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w1.n, srows1, 128, kScRows,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_d(&m_z1, a.w1.zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w1.n, srows1, 128, kScRows,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    for (int i = 0; i < 4; ++i) words.m[1][i] = words.m[0][i];
    m_s1 = m_s0;
    m_z1 = m_z0;
  }
  KArgsD p;
  p.nbits = a.w0.nbits;
  p.wq_strides0 = a.w0.wq_strides;
  p.zs_strides0 = a.w0.zs_strides;
  p.wq_strides1 = C::kPairTiles ? a.w0.wq_strides : a.w1.wq_strides;
  p.zs_strides1 = C::kPairTiles ? a.w0.zs_strides : a.w1.zs_strides;
  p.segs = a.segs;
  p.tile_prefix = a.tile_prefix;
  p.num_segs = a.num_segs;
  p.N = a.w0.n;
  p.K = K;
  p.group_size = a.w0.group_size;
  p.n_tiles = a.w0.n / (C::kPairTiles ? 256 : 128);
  p.out = a.out;
  p.out_ld = a.out_ld;
  p.row_weight = reinterpret_cast<const __half*>(a.row_weight);
  p.perm_out_nbits = a.perm_out_nbits;
  p.chain_done = a.chain_done;
  p.chain_target = a.chain_target;
  auto kern = k_moe_tcd<NT, MODE, SUB>;
  // set once per instantiation and device (outside any graph capture)
  static std::atomic<size_t> smem_done[kMaxDevices];
  if (cudaError_t err = raise_smem_limit(kern, static_cast<size_t>(C::kSmemBytes), smem_done); err != cudaSuccess)
    return err;
  return launch_dep(kern, dim3(a.num_sms), dim3(kThreadsD), C::kSmemBytes, stream, p, m_act, words, m_s0, m_z0, m_s1,
                    m_z1);
}

}  // namespace

bool tcd_gemm_supported(const GemmArgs& a) {
  if (encode_fn_d() == nullptr) return false;
  // 16 / 32-token tiles (decode batches) and 64-token tiles (prefill). A 128-token
  // tile leaves TMEM room for one accumulator buffer only (the epilogue then stalls
  // the MMAs); on a Qwen3-shaped prefill layer 64-token tiles measured 10% faster than
  // the shared-memory-A kernel's 128-token tiles, the down projection 35%.
  if (a.nt != kNtSmall && a.nt != kNtTiny && a.nt != kNtMid) return false;
  if (a.mode != GemmMode::kSwiGLU && a.mode != GemmMode::kRouteWeight) return false;
  if (a.w0.k <= 0 || a.w0.k % kSK != 0 || a.w0.n % 128 != 0) return false;
  const int g = a.w0.group_size;
  if ((g & (g - 1)) != 0 || (g != 64 && g % 128 != 0)) return false;  // 64 or a power of two >= 128
  if (a.num_segs <= 0 || a.num_segs > tcw::kMaxSegs) return false;
  if (a.mode == GemmMode::kSwiGLU && (a.w1.n != a.w0.n || a.w1.k != a.w0.k || a.w1.group_size != a.w0.group_size))
    return false;
  if (a.mode == GemmMode::kRouteWeight) {
    if (a.w0.n % 256 != 0) return false;  // tiles pair up
    // the epilogue writes 16-byte pieces of its output rows
    if ((reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 || a.out_ld % 8 != 0) return false;
  }
  return (reinterpret_cast<uintptr_t>(a.act) & 15u) == 0;
}

template <int NT>
cudaError_t launch_nt_d(const GemmArgs& a, bool sub, cudaStream_t stream) {
  if (a.mode == GemmMode::kSwiGLU)
    return sub ? launch_d<NT, GemmMode::kSwiGLU, true>(a, stream) : launch_d<NT, GemmMode::kSwiGLU, false>(a, stream);
  return sub ? launch_d<NT, GemmMode::kRouteWeight, true>(a, stream)
             : launch_d<NT, GemmMode::kRouteWeight, false>(a, stream);
}

cudaError_t launch_tcd_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (!tcd_gemm_supported(a)) return cudaErrorNotSupported;
  // the subnormal dequant form when every scale of the projection(s) allows it
  const bool sub = a.w0.sub_ok != 0 && (a.mode != GemmMode::kSwiGLU || a.w1.sub_ok != 0);
  if (a.nt == kNtTiny) return launch_nt_d<kNtTiny>(a, sub, stream);
  if (a.nt == kNtMid) return launch_nt_d<kNtMid>(a, sub, stream);
  return launch_nt_d<kNtSmall>(a, sub, stream);
}

// Source column of destination column k of an activation row stored in the decode
// GEMM's slot order for bit-width nb (host copy of the table, for tests).
int kperm_source_column(int nb, int k) {
  const int st = k / kSK, s = k % kSK;
  if (nb == 3) {
    constexpr kperm::Perm3 t = kperm::make_perm3();
    return st * kSK + t.fwd[kperm::phase3(st)][s];
  }
  return st * kSK + kperm::perm_pow2(nb, s);
}

}  // namespace gemq
