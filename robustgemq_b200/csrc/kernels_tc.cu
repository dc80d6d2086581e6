// Persistent grouped dequant GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Computes, for every work item (segment s -> expert e, a tile of up to NT activation
// rows, a tile of 128 output features n0..n0+127):
//     D[n, t] = sum_k deq(W_e)[k, n] * act[row_t, k]          (fp32 in TMEM)
// i.e. the reference's x @ deq(W) (dequant_group_gemm.py:109-138) with the weight
// tile as the UMMA A operand (M = 128 features) and the tokens as B (N = NT), so
// the same kernel serves prefill (NT = 128) and small decode batches (NT = 32).
//
// Warp roles (448 threads, one CTA per SM, grid-stride over work items):
//   warp 0      TMA producer: activation tile (128B swizzle), packed int32 words
//               (2/4/8 word rows x 128 features, by bit-width) and fp16 scale/zero
//               rows; no multicast
//   warp 1      TMEM allocation + single-thread tcgen05.mma issue + commits
//   warps 2-5   epilogue: tcgen05.ld -> mode-specific rounding -> global stores
//   warps 6-13  dequant: packed words -> fp16 via fma.rn.f16 (bit-exact with
//               utils.py:206-210) written as the 128B-swizzled K-major A tile
// Accumulators are double-buffered in TMEM so the epilogue of one item overlaps the
// MMAs of the next. Dense modes (router gate) load A by TMA and skip the dequant
// warps. Every wait is bounded (gemq_common.cuh); on expiry all roles drain and
// return.
#include <cudaTypedefs.h>

#include "gemq_common.cuh"
#include "gemq_internal.h"
#include "tc_work.cuh"

namespace gemq {

namespace {

constexpr int kBK = 64;        // K per stage: one 128-byte swizzle row of fp16
constexpr int kBM = 128;       // features per tile (UMMA M)
constexpr int kWordRows = 8;   // word-row slots per stage (covers 64 k for b in {1,2,3,4})
constexpr int kThreads = 448;  // 14 warps
constexpr int kDqWarp0 = 6;
constexpr int kNumDqThreads = 256;
using tcw::kMaxSegs;
using tcw::kMetaBytes;
using tcw::Meta;
using tcw::Work;
constexpr int kSmemBudget = 225 * 1024 - kMetaBytes;

__host__ __device__ constexpr int round_up(int v, int m) { return (v + m - 1) / m * m; }
__host__ __device__ constexpr int tmem_cols_for(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }

// Word rows a 64-wide K tile needs: 64 / (32 / b) for b in {1, 2, 4}; 3-bit tiles
// straddle words (ten codes per word) and need up to 8.
__host__ __device__ constexpr int word_rows_for(int nb) { return nb == 1 ? 2 : nb == 2 ? 4 : 8; }

template <int NT, GemmMode MODE>
struct Cfg {
  static constexpr bool kDense = (MODE == GemmMode::kDenseF16 || MODE == GemmMode::kDenseF32);
  static constexpr int kMats = (MODE == GemmMode::kSwiGLU) ? 2 : 1;
  static constexpr int kActBytes = NT * 128;
  static constexpr int kWqBytes = kWordRows * kBM * 4;
  static constexpr int kSzBytes = kBM * 2;
  static constexpr int kATile = kBM * 128;
  static constexpr int kWqOff = kActBytes;                              // dequant: packed words
  static constexpr int kSzOff = kActBytes + kMats * kWqBytes;           // dequant: scales, zeros
  static constexpr int kStageRaw = kDense ? kActBytes + kATile : kActBytes + kMats * (kWqBytes + 2 * kSzBytes);
  static constexpr int kStageBytes = round_up(kStageRaw, 1024);
  // dequantised-A ring depth: a buffer returns only when the MMAs that read it
  // commit, so the ring must cover that round trip (deeper for short K tiles of
  // few tokens, where the round trip dominates)
  static constexpr int kAStages = kDense ? 1 : (NT <= 32 ? (kMats == 2 ? 4 : 6) : (kMats == 2 ? 3 : 4));
  static constexpr int kARingBytes = kDense ? 0 : kAStages * kMats * kATile;
  static constexpr int kStages = cmin(8, (kSmemBudget - kARingBytes - 2048) / kStageBytes);
  static constexpr int kARingOff = kStages * kStageBytes;
  static constexpr int kBarOff = kARingOff + kARingBytes;
  static constexpr int kNumBars = 2 * kStages + 2 * kAStages + 5;
  static constexpr int kMetaOff = round_up(kBarOff + kNumBars * 8 + 16, 16);
  static constexpr int kSmemBytes = kMetaOff + kMetaBytes + 1024;  // + alignment slack
  static constexpr int kAccCols = kMats * NT;                             // one accumulator buffer
  static constexpr int kTmemCols = tmem_cols_for(2 * kAccCols);
  static constexpr uint32_t kIdesc = idesc_f16_f32(kBM, NT);
  static_assert(kStages >= 2, "shared memory budget too small");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget exceeded");
  // bytes one stage delivers for a given bit-width (dense: fixed)
  __host__ __device__ static constexpr uint32_t tx_bytes(int nb) {
    return kDense ? kActBytes + kATile : kActBytes + kMats * (word_rows_for(nb) * kBM * 4 + 2 * kSzBytes);
  }
};

struct KArgs {
  const int32_t* nbits;
  const int32_t* wq_strides0;
  const int32_t* zs_strides0;
  const int32_t* wq_strides1;
  const int32_t* zs_strides1;
  const Seg* segs;
  const int32_t* tile_prefix;
  int num_segs;
  int N;           // weight features (rows of A); output columns limit
  int K;
  int group_size;
  int n_tiles;
  void* out;
  int64_t out_ld;
  const __half* row_weight;
};

// Packed-word maps, one per box height (2, 4, 8 word rows) and matrix.
struct WordMaps {
  CUtensorMap m[2][3];
};

// ---------------------------------------------------------------- dequant of one row
// Thread owns feature row `n` of the 128 x 64 A tile; writes 16-byte chunks
// [c0, c1) (k = 8c .. 8c+7) of that row. `w` holds the loaded word rows of this
// feature column; for 3-bit the tile starts at code slot `phase` of word 0.
template <int NB>
__device__ __forceinline__ void dq_row_pow2(const uint32_t (&w)[kWordRows], __half2 s2, __half2 z2, uint8_t* row_base,
                                            uint32_t n, int c0, int c1) {
  constexpr int kChunksPerWord = (32 / NB) / 8;
#pragma unroll
  for (int wi = 0; wi < 8 / kChunksPerWord; ++wi) {
    const int cw = wi * kChunksPerWord;
    if (cw >= c0 && cw < c1) {
      dq_word_pow2<NB>(w[wi], s2, z2, [&](int c, uint4 v) {
        *reinterpret_cast<uint4*>(row_base + sw128_offset(n, cw + c)) = v;
      });
    }
  }
}

template <int P>
__device__ __forceinline__ void dq_row_3bit(const uint32_t (&w)[kWordRows], __half2 s2, __half2 z2, uint8_t* row_base,
                                            uint32_t n, int c0, int c1) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c >= c0 && c < c1) {
      uint32_t o[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = 8 * c + 2 * m;
        const int a = (P + j) / 10, sa = (P + j) % 10;
        const int b = (P + j + 1) / 10, sb = (P + j + 1) % 10;
        o[m] = dq_pair(magic3(w[a], sa, w[b], sb), s2, z2);
      }
      *reinterpret_cast<uint4*>(row_base + sw128_offset(n, c)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__device__ __forceinline__ void dq_row(int nb, int phase, const uint32_t (&w)[kWordRows], __half2 s2, __half2 z2,
                                       uint8_t* row_base, uint32_t n, int c0, int c1) {
  switch (nb) {
    case 4: dq_row_pow2<4>(w, s2, z2, row_base, n, c0, c1); break;
    case 2: dq_row_pow2<2>(w, s2, z2, row_base, n, c0, c1); break;
    case 1: dq_row_pow2<1>(w, s2, z2, row_base, n, c0, c1); break;
    case 3:
      switch (phase) {
        case 0: dq_row_3bit<0>(w, s2, z2, row_base, n, c0, c1); break;
        case 2: dq_row_3bit<2>(w, s2, z2, row_base, n, c0, c1); break;
        case 4: dq_row_3bit<4>(w, s2, z2, row_base, n, c0, c1); break;
        case 6: dq_row_3bit<6>(w, s2, z2, row_base, n, c0, c1); break;
        default: dq_row_3bit<8>(w, s2, z2, row_base, n, c0, c1); break;
      }
      break;
    default: break;
  }
}

// ---------------------------------------------------------------- epilogue math
__device__ __forceinline__ float silu_ref(float x) { return x / (1.f + expf(-x)); }

template <GemmMode MODE>
__device__ __forceinline__ void store_one(const KArgs& p, int64_t row, int col, float a0, float a1) {
  if constexpr (MODE == GemmMode::kSwiGLU) {
    // x1, x3 stored fp16; F.silu(x1) -> fp16; * x3 -> fp16 (moe_block.py:774-775)
    const float x1 = __half2float(__float2half_rn(a0));
    const float x3 = __half2float(__float2half_rn(a1));
    const float sl = __half2float(__float2half_rn(silu_ref(x1)));
    static_cast<__half*>(p.out)[row * p.out_ld + col] = __float2half_rn(sl * x3);
  } else if constexpr (MODE == GemmMode::kRouteWeight) {
    const float y = __half2float(__float2half_rn(a0));
    const float wv = __half2float(p.row_weight[row]);
    static_cast<__half*>(p.out)[row * p.out_ld + col] = __float2half_rn(y * wv);
  } else if constexpr (MODE == GemmMode::kDenseF32) {
    static_cast<float*>(p.out)[row * p.out_ld + col] = a0;
  } else {
    static_cast<__half*>(p.out)[row * p.out_ld + col] = __float2half_rn(a0);
  }
}

// ---------------------------------------------------------------- the kernel
template <int NT, GemmMode MODE>
__global__ void __launch_bounds__(kThreads, 1)
    k_moe_tc(const KArgs p, const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ WordMaps tm_words,
             const __grid_constant__ CUtensorMap tm_s0, const __grid_constant__ CUtensorMap tm_z0,
             const __grid_constant__ CUtensorMap tm_s1, const __grid_constant__ CUtensorMap tm_z1) {
  using C = Cfg<NT, MODE>;
  constexpr bool kDense = C::kDense;
  constexpr int kMats = C::kMats;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* afull = bars + 2 * kStages;
  constexpr int kAStages = C::kAStages;
  uint64_t* aempty = afull + kAStages;
  uint64_t* acc_full = aempty + kAStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDense ? 1 : (kNumDqThreads / 32) + 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&afull[s], kNumDqThreads / 32);  // one arrival per dequant warp
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_act);
    tma_prefetch_desc(&tm_words.m[0][2]);
    if (!kDense) {
      tma_prefetch_desc(&tm_s0);
      tma_prefetch_desc(&tm_z0);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  // everything above is private to this CTA; from here on it reads the segment
  // table, activations and weights, and writes outputs other kernels use
  grid_dep_wait();
  Meta& meta = *reinterpret_cast<Meta*>(smem + C::kMetaOff);
  tcw::stage_meta(meta, p, kDense);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = meta.tp[p.num_segs] * p.n_tiles;
  const int KT = p.K / kBK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp runs the loop; an elected lane issues (operands stay warp-uniform).
    {
      int s = 0;
      uint32_t ph = 0;
      int armed = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        const Work wk = tcw::decode_work<NT>(meta, p.num_segs, p.n_tiles, w);
        const int nb = kDense ? 4 : min(max(wk.nb, 1), 4);
        const int eps = 32 / nb;
        const int box = nb == 1 ? 0 : nb == 2 ? 1 : 2;  // word-row map index
        const uint32_t tx = C::tx_bytes(nb);
        for (int kt = 0; kt < KT; ++kt) {
          if (!warp_wait(&empty[s], ph ^ 1u, kDevTimeoutTmaEmpty, 128)) { ok = false; break; }
          uint8_t* st = smem + s * C::kStageBytes;
          const int k0 = kt * kBK;
          if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d(st, &tm_act, &full[s], k0, wk.act_row);
          if constexpr (kDense) {
            tma_load_2d(st + C::kActBytes, &tm_words.m[0][2], &full[s], k0, wk.n0);
          } else {
            const int wr = k0 / eps;
            const int sr = k0 / p.group_size;
            tma_load_2d(st + C::kWqOff, &tm_words.m[0][box], &full[s], wk.n0, wk.wrow0 + wr);
            tma_load_2d(st + C::kSzOff, &tm_s0, &full[s], wk.n0, wk.srow0 + sr);
            tma_load_2d(st + C::kSzOff + C::kSzBytes, &tm_z0, &full[s], wk.n0, wk.srow0 + sr);
            if constexpr (kMats == 2) {
              tma_load_2d(st + C::kWqOff + C::kWqBytes, &tm_words.m[1][box], &full[s], wk.n0, wk.wrow1 + wr);
              tma_load_2d(st + C::kSzOff + 2 * C::kSzBytes, &tm_s1, &full[s], wk.n0, wk.srow1 + sr);
              tma_load_2d(st + C::kSzOff + 3 * C::kSzBytes, &tm_z1, &full[s], wk.n0, wk.srow1 + sr);
            }
          }
          }
          __syncwarp();
          ++armed;
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      // drain: wait for the last armed phase of every stage (loads still in flight)
      for (int st = 0; st < kStages && st < armed; ++st) {
        const int times = (armed - 1 - st) / kStages + 1;
        mbar_wait_drain(&full[st], static_cast<uint32_t>((times - 1) & 1));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop; one elected lane (lane 0 of the converged warp,
    // always the same one) issues every MMA and commit, so each commit tracks them all.
    {
      int s = 0, as = 0;
      uint32_t ph = 0, aph = 0;
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t d_base = tmem + static_cast<uint32_t>(buf * C::kAccCols);
        if (!warp_wait(&acc_empty[buf], ((it >> 1) & 1) ^ 1u, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt) {
          if (!warp_wait(&full[s], ph, kDevTimeoutTmaFull)) { ok = false; break; }
          if constexpr (!kDense) {
            if (!warp_wait(&afull[as], aph, kDevTimeoutAFull)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t act_addr = smem_u32(smem + s * C::kStageBytes);
          if (elect_one()) {
#pragma unroll
          for (int m = 0; m < kMats; ++m) {
            const uint32_t a_addr = kDense ? act_addr + C::kActBytes
                                           : smem_u32(smem + C::kARingOff + (as * kMats + m) * C::kATile);
            // the 4 K=16 steps of the stage from one asm block (+32 B per step)
            umma_f16_k64(d_base + static_cast<uint32_t>(m * NT), sdesc_sw128(a_addr), sdesc_sw128(act_addr),
                         C::kIdesc, kt != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          if constexpr (!kDense) umma_commit(&aempty[as]);
          }
          __syncwarp();
          if (++s == kStages) { s = 0; ph ^= 1u; }
          if constexpr (!kDense) {
            if (++as == kAStages) { as = 0; aph ^= 1u; }
          }
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
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * C::kAccCols);
      const Work wk = tcw::decode_work<NT>(meta, p.num_segs, p.n_tiles, w);
      if (!mbar_wait(&acc_full[buf], (it >> 1) & 1, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const int col = wk.n0 + 32 * q + lane;
      for (int c0 = 0; c0 < NT; c0 += 16) {
        if (c0 >= wk.rows) break;
        uint32_t r0[16], r1[16];
        tmem_ld16(lane_base + c0, r0);
        if constexpr (kMats == 2) tmem_ld16(lane_base + NT + c0, r1);
        tmem_ld_wait();
        if (col < p.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (c0 + i < wk.rows) {
              const float a0 = __uint_as_float(r0[i]);
              const float a1 = kMats == 2 ? __uint_as_float(r1[i]) : 0.f;
              store_one<MODE>(p, static_cast<int64_t>(wk.out_row + c0 + i), col, a0, a1);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else if constexpr (!kDense) {
    // ------------------------------------------------------------ dequant
    const int dt = threadIdx.x - kDqWarp0 * 32;
    const int wg = dt >> 7;
    const uint32_t n = static_cast<uint32_t>(dt & 127);
    const int mat = (kMats == 2) ? wg : 0;
    const int c0 = (kMats == 2) ? 0 : 4 * wg;
    const int c1 = (kMats == 2) ? 8 : 4 * wg + 4;
    int s = 0, as = 0;
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
      const Work wk = tcw::decode_work<NT>(meta, p.num_segs, p.n_tiles, w);
      const int nb = wk.nb;
      if (nb < 1 || nb > 4) {
        if (dt == 0) set_device_error(kDevBadBits);
      }
      const int rows_needed = word_rows_for(nb);
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[s], ph, kDevTimeoutTmaFull)) { ok = false; break; }
        if (!mbar_wait(&aempty[as], aph ^ 1u, kDevTimeoutAEmpty)) { ok = false; break; }
        const uint8_t* st = smem + s * C::kStageBytes;
        const uint32_t* wcol = reinterpret_cast<const uint32_t*>(st + C::kWqOff + mat * C::kWqBytes) + n;
        uint32_t wv[kWordRows];
#pragma unroll
        for (int r = 0; r < kWordRows; ++r) wv[r] = (r < rows_needed) ? wcol[r * kBM] : 0u;
        const __half sh = reinterpret_cast<const __half*>(st + C::kSzOff + (2 * mat) * C::kSzBytes)[n];
        const __half zh = reinterpret_cast<const __half*>(st + C::kSzOff + (2 * mat + 1) * C::kSzBytes)[n];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        const int phase = (nb == 3) ? (kt * kBK) % 10 : 0;
        uint8_t* a_tile = smem + C::kARingOff + (as * kMats + mat) * C::kATile;
        dq_row(nb, phase, wv, __halves2half2(sh, sh), __halves2half2(zh, zh), a_tile, n, c0, c1);
        // every writer makes its A-tile stores visible to the tensor core's async
        // proxy, the warp converges, and one lane releases the warp's part
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[as]);
        if (++s == kStages) { s = 0; ph ^= 1u; }
        if (++as == kAStages) { as = 0; aph ^= 1u; }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  // looked up once per process (a function-local static is initialised once, even
  // when several host threads create layers at the same time)
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner, uint64_t outer,
              uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_word_maps(CUtensorMap (&maps)[3], const ProjDev& w) {
  const uint32_t heights[3] = {2, 4, 8};
  for (int i = 0; i < 3; ++i) {
    if (!make_map(&maps[i], w.wq, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, w.n, w.wq_rows, kBM, heights[i],
                  CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  return true;
}

template <int NT, GemmMode MODE>
cudaError_t launch_t(const GemmArgs& a, cudaStream_t stream) {
  using C = Cfg<NT, MODE>;
  CUtensorMap m_act, m_s0, m_z0, m_s1, m_z1;
  WordMaps words;
  const int K = a.w0.k;
  if (!make_map(&m_act, a.act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, static_cast<uint64_t>(a.act_rows), 64, NT,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if constexpr (C::kDense) {
    if (!make_map(&words.m[0][2], a.dense_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, a.w0.n, 64, kBM,
                  CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
    for (int i = 0; i < 3; ++i) words.m[0][i] = words.m[1][i] = words.m[0][2];
    m_s0 = m_z0 = m_s1 = m_z1 = m_act;
  } else {
    const uint64_t srows = static_cast<uint64_t>(a.w0.num_experts) * (a.w0.k / a.w0.group_size);
    if (!make_word_maps(words.m[0], a.w0) ||
        !make_map(&m_s0, a.w0.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w0.n, srows, kBM, 1,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&m_z0, a.w0.zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w0.n, srows, kBM, 1,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
    if constexpr (C::kMats == 2) {
      const uint64_t srows1 = static_cast<uint64_t>(a.w1.num_experts) * (a.w1.k / a.w1.group_size);
      if (!make_word_maps(words.m[1], a.w1) ||
          !make_map(&m_s1, a.w1.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w1.n, srows1, kBM, 1,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
          !make_map(&m_z1, a.w1.zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.w1.n, srows1, kBM, 1,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    } else {
      for (int i = 0; i < 3; ++i) words.m[1][i] = words.m[0][i];
      m_s1 = m_s0;
      m_z1 = m_z0;
    }
  }
  KArgs p;
  p.nbits = a.w0.nbits;
  p.wq_strides0 = a.w0.wq_strides;
  p.zs_strides0 = a.w0.zs_strides;
  p.wq_strides1 = C::kMats == 2 ? a.w1.wq_strides : a.w0.wq_strides;
  p.zs_strides1 = C::kMats == 2 ? a.w1.zs_strides : a.w0.zs_strides;
  p.segs = a.segs;
  p.tile_prefix = a.tile_prefix;
  p.num_segs = a.num_segs;
  p.N = a.w0.n;
  p.K = K;
  p.group_size = C::kDense ? 64 : a.w0.group_size;
  p.n_tiles = (a.w0.n + kBM - 1) / kBM;
  p.out = a.out;
  p.out_ld = a.out_ld;
  p.row_weight = reinterpret_cast<const __half*>(a.row_weight);
  auto kern = k_moe_tc<NT, MODE>;
  // set once per instantiation and device (outside any graph capture)
  static std::atomic<size_t> smem_done[kMaxDevices];
  if (cudaError_t err = raise_smem_limit(kern, static_cast<size_t>(C::kSmemBytes), smem_done); err != cudaSuccess)
    return err;
  return launch_dep(kern, dim3(a.num_sms), dim3(kThreads), C::kSmemBytes, stream, p, m_act, words, m_s0, m_z0, m_s1,
                    m_z1);
}

template <int NT>
cudaError_t launch_nt(const GemmArgs& a, cudaStream_t stream) {
  switch (a.mode) {
    case GemmMode::kSwiGLU: return launch_t<NT, GemmMode::kSwiGLU>(a, stream);
    case GemmMode::kRouteWeight: return launch_t<NT, GemmMode::kRouteWeight>(a, stream);
    case GemmMode::kStoreF16: return launch_t<NT, GemmMode::kStoreF16>(a, stream);
    case GemmMode::kDenseF16: return launch_t<NT, GemmMode::kDenseF16>(a, stream);
    case GemmMode::kDenseF32: return launch_t<NT, GemmMode::kDenseF32>(a, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

bool tc_gemm_supported(const GemmArgs& a) {
  if (encode_fn() == nullptr) return false;
  if (a.nt != kNtSmall && a.nt != kNtLarge) return false;
  if (a.w0.k % kBK != 0 || a.w0.k <= 0) return false;
  if (a.num_segs <= 0 || a.num_segs > kMaxSegs) return false;
  const bool dense = (a.mode == GemmMode::kDenseF16 || a.mode == GemmMode::kDenseF32);
  if (dense) return (reinterpret_cast<uintptr_t>(a.dense_a) & 15u) == 0;
  if (a.w0.n % kBM != 0 || a.w0.group_size % kBK != 0) return false;
  if (a.mode == GemmMode::kSwiGLU && (a.w1.n != a.w0.n || a.w1.k != a.w0.k || a.w1.group_size != a.w0.group_size))
    return false;
  return (reinterpret_cast<uintptr_t>(a.act) & 15u) == 0;
}

cudaError_t launch_tc_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (!tc_gemm_supported(a)) return cudaErrorNotSupported;
  return a.nt == kNtSmall ? launch_nt<kNtSmall>(a, stream) : launch_nt<kNtLarge>(a, stream);
}

}  // namespace gemq
