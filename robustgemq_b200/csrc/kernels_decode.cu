// Decode GEMV family (CUDA cores, deterministic split-K), the one-token path of
// forward_one_token (moe_block.py:817-853) and the batch-1 dequant GEMV of
// dequant_gemv.py:118-156.
//
// part[mat][s][a][n] = split s of sum_k xin_a[k] * deq(W_{mat, idx[a]})[k, n] in fp32.
// A block covers 128 output features (4 per lane, one 16-byte load = the same word
// row of 4 features) of one (matrix, row a) and one K split; its word rows are cut
// into 8 contiguous runs, one per warp, reduced through shared memory in a fixed
// order, so every result is bit-reproducible (the reference's fp16 atomics are not,
// dequant_gemv.py:115).
//
// Inner loop: two codes per pair dequantised with one fma.rn.f16x2 (bit-exact with
// utils.py:206-210), in the single-instruction subnormal-operand form when the
// layer's scale check allows it, else the magic-number form; the inputs are staged
// in shared memory as fp32 (fp16 inputs convert exactly; the one-token path's SiLU*mul
// is fp32) and accumulate with fma.rn.f32x2 (exact products, one rounding each).
//
// Input modes (xin):
//   kGemvX        fp16 rows x[a * x_stride + k]
//   kGemvSwiGLU   fp32 silu(x1) * x3 from fp16 rows (fused_dequant_bmm.py:237-239)
//   kGemvPartF32  x1 = fp16(sum_s up[0][s][a][k]), x3 = fp16(sum_s up[1][s][a][k]),
//                 then fp32 silu(x1) * x3: reads the up-projection partials directly
//   kGemvPartF16  as kGemvPartF32 but h = fp16(fp16(silu(x1)) * x3) (the fp16
//                 ``F.silu(x1) * x3`` of the shared experts, moe_block.py:619)
#include <cuda_fp16.h>

#include "gemq_common.cuh"
#include "gemq_internal.h"

namespace gemq {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvCols = 128;
constexpr int kGemvCtasPerSm = 2;  // 128 registers per thread (fewer spill)

__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

// (d0, d1) += (a0, a1) * (b0, b1), each lane one rounding
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 A, B, C;\n\t"
      "mov.b64 A, {%2, %3};\n\t"
      "mov.b64 B, {%4, %5};\n\t"
      "mov.b64 C, {%0, %1};\n\t"
      "fma.rn.f32x2 C, A, B, C;\n\t"
      "mov.b64 {%0, %1}, C;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// x values of one word row, read from shared memory with 16-byte loads (pow2 widths:
// a row starts on a multiple of eps elements, so on a 16-byte boundary) or 8-byte
// loads (3-bit: ten fp32 values at 40-byte offsets). The staging interleaves each row
// by code pair: slot 2p holds code p, slot 2p + 1 code p + eps/2 (p + 5 at 3 bits),
// so the two inputs of a pair's fma.rn.f32x2 are one aligned register pair.
template <int NB, bool XF16>
struct XRow {
  static constexpr int kN = (NB == 3) ? 10 : 32 / NB;
  static constexpr int kBytes = kN * (XF16 ? 2 : 4);
  static constexpr int kVec = (NB == 3) ? 4 : 16;  // load width in bytes
  uint32_t v[kBytes / 4];
  __device__ __forceinline__ void load(const void* xr) {
    if constexpr (kVec == 16) {
#pragma unroll
      for (int i = 0; i < kBytes / 16; ++i) {
        const uint4 t = static_cast<const uint4*>(xr)[i];
        v[4 * i] = t.x;
        v[4 * i + 1] = t.y;
        v[4 * i + 2] = t.z;
        v[4 * i + 3] = t.w;
      }
    } else if constexpr (XF16) {
#pragma unroll
      for (int i = 0; i < kBytes / 4; ++i) v[i] = static_cast<const uint32_t*>(xr)[i];
    } else {
#pragma unroll
      for (int i = 0; i < kBytes / 8; ++i) {
        const uint2 t = static_cast<const uint2*>(xr)[i];
        v[2 * i] = t.x;
        v[2 * i + 1] = t.y;
      }
    }
  }
  __device__ __forceinline__ __half h(int j) const {
    return __ushort_as_half(static_cast<unsigned short>(v[j >> 1] >> (16 * (j & 1))));
  }
  __device__ __forceinline__ float f(int j) const { return __uint_as_float(v[j]); }
};

// Adds k_lo / k_hi to the exponent fields of the two halves of a pair (the scale
// times 2^k, exact for the normal scales the subnormal form is used with).
__device__ __forceinline__ __half2 exp_add2(__half2 v, int k_lo, int k_hi) {
  return u32_as_h2(h2_as_u32(v) + ((static_cast<uint32_t>(k_lo) << 10) | (static_cast<uint32_t>(k_hi) << 26)));
}

// Accumulates one word of one feature column. Pair p holds codes (p, p + eps/2):
// 16 bits apart, so one shift + mask per pair. SUB: the subnormal-operand form of
// the tensor-memory GEMM (kernels_tcd.cu, dq_col_sub): the pair moved to mantissa
// offset o (b = 4: 6; b = 2: 6 / 8 for even / odd p; b = 1: 8 / 9) reads as
// q * 2^(o - 24), the scale carries 2^(24 - o), one fma.rn.f16x2 gives the same
// single rounding of q * s + z'. Otherwise the magic-number form. Products with the
// fp32 inputs are exact, each sum rounded once (fma.rn.f32x2).
template <int NB, bool XF16, bool SUB>
__device__ __forceinline__ void word_pow2(uint32_t w, __half2 s2, __half2 z2, const XRow<NB, XF16>& x, float& acc0,
                                          float& acc1) {
  static_assert(!XF16, "inputs are staged as fp32");
  constexpr int kEps = 32 / NB, kHalf = kEps / 2;
  constexpr uint32_t kMask = ((1u << NB) - 1u) * 0x00010001u;
  __half2 sa2 = s2, sb2 = s2;
  if constexpr (SUB) {
    sa2 = exp_add2(s2, NB == 1 ? 16 : 18, NB == 1 ? 16 : 18);
    sb2 = exp_add2(s2, NB == 1 ? 15 : (NB == 2 ? 16 : 18), NB == 1 ? 15 : (NB == 2 ? 16 : 18));
  }
#pragma unroll
  for (int j = 0; j < kHalf; ++j) {
    __half2 wq;
    if constexpr (SUB) {
      const bool alt = (NB != 4) && (j & 1);
      const int o = (NB == 4 ? 6 : (NB == 2 ? 6 : 8)) + (alt ? (NB == 2 ? 2 : 1) : 0);
      const int sh = o - NB * j;
      const uint32_t v = sh >= 0 ? (w << sh) : (w >> (-sh));
      wq = __hfma2(u32_as_h2(v & (kMask << o)), alt ? sb2 : sa2, z2);
    } else {
      wq = u32_as_h2(dq_pair(((w >> (NB * j)) & kMask) | 0x64006400u, s2, z2));
    }
    const float2 wf = __half22float2(wq);
    ffma2(acc0, acc1, x.f(2 * j), x.f(2 * j + 1), wf.x, wf.y);
  }
}

// 3-bit: ten codes per word (bits 30-31 unused); pair p holds codes (p, p + 5).
// A word may straddle a scale-group boundary: codes j < b use (sa, za), codes
// j >= b the next group's (sb, zb) (b = 10 when the word lies in one group). SUB:
// code p moved to bit 6 (o = 6), code p + 5 to bit 21 (o = 5 of the high half).
template <bool XF16, bool SUB>
__device__ __forceinline__ void word_3bit(uint32_t w, __half sa, __half za, __half sb, __half zb, int b,
                                          const XRow<3, XF16>& x, float& acc0, float& acc1) {
  static_assert(!XF16, "inputs are staged as fp32");
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const __half2 s2 = __halves2half2(j >= b ? sb : sa, j + 5 >= b ? sb : sa);
    const __half2 z2 = __halves2half2(j >= b ? zb : za, j + 5 >= b ? zb : za);
    __half2 wq;
    if constexpr (SUB) {
      const int sh = 6 - 3 * j;  // code j: bit 3j -> 6; code j + 5: bit 3j + 15 -> 21
      const uint32_t v = sh >= 0 ? (w << sh) : (w >> (-sh));
      wq = __hfma2(u32_as_h2(v & ((7u << 6) | (7u << 21))), exp_add2(s2, 18, 19), z2);
    } else {
      const uint32_t t = w >> (3 * j);       // code j at bits 0..2
      const uint32_t u = w >> (3 * j + 15);  // code j + 5 at bits 0..2
      const uint32_t m = (t & 7u) | ((u & 7u) << 16) | 0x64006400u;
      wq = u32_as_h2(dq_pair(m, s2, z2));
    }
    const float2 wf = __half22float2(wq);
    ffma2(acc0, acc1, x.f(2 * j), x.f(2 * j + 1), wf.x, wf.y);
  }
}

// Scale/zero rows of the groups a block's K range touches, staged in shared memory
// ([group][128 features] fp16 each) so that a group change costs a shared load.
struct GroupStage {
  const __half* s;
  const __half* z;
  int g0;  // first staged group
};

constexpr int kBatch = 4;  // word rows of a warp whose loads are in flight together (8 spills registers)

// Loads word rows [rb, min(rb + kBatch, wr1)) of features n..n+3.
__device__ __forceinline__ void load_words(const int32_t* wbase, int N, int n, int rb, int wr1, uint4 (&wv)[kBatch]) {
#pragma unroll
  for (int i = 0; i < kBatch; ++i)
    wv[i] = (rb + i < wr1) ? __ldcs(reinterpret_cast<const uint4*>(wbase + static_cast<int64_t>(rb + i) * N + n))
                           : make_uint4(0, 0, 0, 0);  // read once: streamed, evicted first
}

// One word row of the four feature columns of a lane.
template <int NB, bool SUB>
__device__ __forceinline__ void row_pow2(const uint4& wv, const void* xr, const __half2 (&s_c)[4],
                                         const __half2 (&z_c)[4], float (&acc)[4][2]) {
  XRow<NB, false> x;
  x.load(xr);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) word_pow2<NB, false, SUB>(words[c], s_c[c], z_c[c], x, acc[c][0], acc[c][1]);
}

// Accumulates word rows of a warp, one row (its 16-byte word piece of the four
// feature columns) at a time, keeping the current group's scale and zero.
template <bool SUB>
struct RowAcc {
  int K, g, nb, lane, k0, eps, cur_g;
  const char* xbase;
  GroupStage gs;
  __half2 s_c[4], z_c[4];  // scale / zero of the current group, per column

  __device__ __forceinline__ RowAcc(int K_, int g_, int nb_, int lane_, int k0_, const void* s_x, const GroupStage& gs_)
      : K(K_), g(g_), nb(nb_), lane(lane_), k0(k0_), eps(32 / nb_), cur_g(-1),
        xbase(static_cast<const char*>(s_x)), gs(gs_) {}

  __device__ __forceinline__ void load_group(int gi, __half2 (&sd)[4], __half2 (&zd)[4]) const {
    const int off = (gi - gs.g0) * 128 + lane * 4;
    const uint2 sv = *reinterpret_cast<const uint2*>(gs.s + off);
    const uint2 zv = *reinterpret_cast<const uint2*>(gs.z + off);
    const __half* sp = reinterpret_cast<const __half*>(&sv);
    const __half* zp = reinterpret_cast<const __half*>(&zv);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      sd[c] = __halves2half2(sp[c], sp[c]);
      zd[c] = __halves2half2(zp[c], zp[c]);
    }
  }

  __device__ __forceinline__ void row(int r, const uint4& w, float (&acc)[4][2]) {
    constexpr int kXBytes = 4;  // fp32 inputs
    const int kr = r * eps;
    const int ga = kr / g;
    if (ga != cur_g) {
      cur_g = ga;
      load_group(ga, s_c, z_c);
    }
    const void* xr = xbase + static_cast<size_t>(kr - k0) * kXBytes;
    if (nb == 3) {
      XRow<3, false> x;
      x.load(xr);
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
      const int gb = min(kr + 9, K - 1) / g;
      if (gb == ga) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          word_3bit<false, SUB>(words[c], __low2half(s_c[c]), __low2half(z_c[c]), __low2half(s_c[c]), __low2half(z_c[c]), 10,
                          x, acc[c][0], acc[c][1]);
      } else {
        // codes at k >= gb * g use the next group's scale and zero
        __half2 s_n[4], z_n[4];
        load_group(gb, s_n, z_n);
        const int b = gb * g - kr;  // first code index in the next group (1..9)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          word_3bit<false, SUB>(words[c], __low2half(s_c[c]), __low2half(z_c[c]), __low2half(s_n[c]), __low2half(z_n[c]), b,
                          x, acc[c][0], acc[c][1]);
        cur_g = gb;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s_c[c] = s_n[c];
          z_c[c] = z_n[c];
        }
      }
      // codes past K in a ragged last word are zero-padded and their x staged as 0
    } else if (nb == 2) {
      row_pow2<2, SUB>(w, xr, s_c, z_c, acc);
    } else if (nb == 4) {
      row_pow2<4, SUB>(w, xr, s_c, z_c, acc);
    } else {
      row_pow2<1, SUB>(w, xr, s_c, z_c, acc);
    }
  }
};

// Accumulates word rows [wr0, wr1) of a warp from global memory; `wv` holds the
// first batch, loaded by the caller before it staged x and the scales. The next
// batch's loads are issued before the current one is used.
template <bool SUB>
__device__ __forceinline__ void gemv_rows(const int32_t* wbase, int N, int n, int wr0, int wr1, RowAcc<SUB>& ra,
                                          uint4 (&wv)[kBatch], float (&acc)[4][2]) {
  for (int rb = wr0; rb < wr1; rb += kBatch) {
    uint4 nx[kBatch];
    const bool more = rb + kBatch < wr1;
    if (more) load_words(wbase, N, n, rb + kBatch, wr1, nx);
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (rb + i >= wr1) break;
      ra.row(rb + i, wv[i], acc);
    }
    if (more) {
#pragma unroll
      for (int i = 0; i < kBatch; ++i) wv[i] = nx[i];
    }
  }
}

// Shared memory of one block: x of its K range (padded to whole words), then the
// staged scale and zero rows.
__host__ __device__ inline int gemv_x_elems(int k, int splits) { return (k + splits - 1) / splits + 128; }
__host__ __device__ inline int gemv_groups(int k, int splits, int g) { return gemv_x_elems(k, splits) / g + 2; }
// word rows of a split, bounded over bit-widths (4-bit has the most: k / 8)
__host__ __device__ inline int gemv_word_rows(int k, int splits) { return (k / 8 + 1 + splits - 1) / splits + 1; }
__host__ __device__ inline int gemv_words_off(int k, int splits, int g, bool xf16) {
  const int xbytes = ((xf16 ? 2 : 4) * gemv_x_elems(k, splits) + 15) & ~15;
  return xbytes + 2 * 2 * 128 * gemv_groups(k, splits, g);
}
// Words of a split staged whole in shared memory by bulk copies (one per 512-byte row
// piece of the block's 128 features), when they fit this budget.
constexpr int kGemvWordBudget = 96 * 1024;

template <bool SUB>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) k_gemv(ProjDev w0, ProjDev w1, const int32_t* __restrict__ idx,
                                                          int rows_a, GemvSrc src, float* __restrict__ part,
                                                          int splits, int bulk_words) {
  // chained one-token GEMVs: the up launch signals per row, the down launch waits per
  // row (the routing ids and weights it reads were complete before the up launch got
  // past its own wait)
  const bool chain_out = src.done != nullptr && src.mode == kGemvX;
  const bool chain_in = src.done != nullptr && src.mode == kGemvPartF32;
  if (!chain_in) grid_dep_wait();
  if (chain_out) grid_dep_launch();
  extern __shared__ __align__(16) unsigned char s_raw[];
  __shared__ float s_red[8][kGemvCols];
  __shared__ uint64_t s_wbar;
  const int slab = blockIdx.x, s = blockIdx.y;
  const int mat = blockIdx.z / rows_a, a = blockIdx.z - mat * rows_a;
  const ProjDev& w = (mat == 0) ? w0 : w1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a chained up CTA that stores nothing still counts itself done
  auto signal_row = [&]() {
    if (chain_out && threadIdx.x == 0) {
      __threadfence();
      atomicAdd(src.done + a, 1);
    }
  };
  const int e = (idx != nullptr) ? idx[a] : a;
  if (e < 0 || e >= w.num_experts) {
    if (threadIdx.x == 0) set_device_error(kDevBadExpert);
    signal_row();
    return;
  }
  const int nb = w.nbits[e];
  if (nb < 1 || nb > 4) {
    if (threadIdx.x == 0) set_device_error(kDevBadBits);
    signal_row();
    return;
  }
  const int eps = 32 / nb;
  const int K = w.k, N = w.n, g = w.group_size;
  const int rows = (K + eps - 1) / eps;
  const int r0 = static_cast<int>((static_cast<int64_t>(rows) * s) / splits);
  const int r1 = static_cast<int>((static_cast<int64_t>(rows) * (s + 1)) / splits);
  const int k0 = r0 * eps;
  const int kspan = (r1 - r0) * eps;  // padded to whole words; entries past K are 0
  // this warp's word rows; their first loads go out before x and the scales are
  // staged, so the three HBM round trips overlap
  const int n = slab * kGemvCols + lane * 4;
  const int per = (r1 - r0 + 7) / 8;
  const int wr0 = r0 + warp * per, wr1 = min(r1, wr0 + per);
  const int32_t* wbase = w.wq + static_cast<int64_t>(w.wq_strides[e]);
  uint4 wv[kBatch];
  // whole-split staging: every row piece of the block in flight at once (one HBM
  // round trip for all its words), else each warp's rows in batches of kBatch
  const bool bulk = bulk_words != 0 && (N % kGemvCols) == 0 && (reinterpret_cast<uintptr_t>(wbase) & 15u) == 0;
  int32_t* s_words = reinterpret_cast<int32_t*>(s_raw + gemv_words_off(K, splits, g, false));
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_init(&s_wbar, 1);
      fence_barrier_init();
    }
    __syncthreads();
    const int nr = r1 - r0;
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&s_wbar, static_cast<uint32_t>(nr) * kGemvCols * 4u);
    const uint64_t policy = l2_evict_first_policy();  // read once: streamed
    for (int r = threadIdx.x; r < nr; r += blockDim.x)
      bulk_load_hint(s_words + r * kGemvCols, wbase + static_cast<int64_t>(r0 + r) * N + slab * kGemvCols,
                     kGemvCols * 4u, &s_wbar, policy);
  } else if (n < N) {
    load_words(wbase, N, n, wr0, wr1, wv);
  }
  constexpr int kXB = 4;  // elements per thread per batch of a staging loop
  // the scale / zero rows of the groups [g0, g1] this block's K range touches
  const int xbytes = 4 * gemv_x_elems(K, splits);
  __half* s_s = reinterpret_cast<__half*>(s_raw + ((xbytes + 15) & ~15));
  const int ng_max = gemv_groups(K, splits, g);
  __half* s_z = s_s + ng_max * 128;
  const int g0 = k0 / g;
  const int g1 = (min(k0 + max(kspan, 1), K) - 1) / g;
  const int64_t zbase = static_cast<int64_t>(w.zs_strides[e]);
  const int ngr = g1 - g0 + 1;
  if ((N & 127) == 0 && ((reinterpret_cast<uintptr_t>(w.scales) | reinterpret_cast<uintptr_t>(w.zeros)) & 15) == 0) {
    // whole slabs: 16-byte loads of scales and zeros, a batch of them per thread
    const int n16 = ngr * 32;
    for (int base = 0; base < n16; base += kXB * kGemvThreads) {
      uint4 sv[kXB];
#pragma unroll
      for (int j = 0; j < kXB; ++j) {
        const int i = base + j * kGemvThreads + threadIdx.x;
        if (i < n16) {
          const int arr = i / (ngr * 16), jj = i - arr * ngr * 16;
          const int gl = jj >> 4, c8 = (jj & 15) * 8;
          const int64_t off = zbase + static_cast<int64_t>(g0 + gl) * N + slab * kGemvCols + c8;
          sv[j] = __ldcs(reinterpret_cast<const uint4*>((arr == 0 ? w.scales : w.zeros) + off));
        }
      }
#pragma unroll
      for (int j = 0; j < kXB; ++j) {
        const int i = base + j * kGemvThreads + threadIdx.x;
        if (i < n16) {
          const int arr = i / (ngr * 16), jj = i - arr * ngr * 16;
          const int gl = jj >> 4, c8 = (jj & 15) * 8;
          *reinterpret_cast<uint4*>((arr == 0 ? s_s : s_z) + gl * 128 + c8) = sv[j];
        }
      }
    }
  } else {
#pragma unroll 4
    for (int i = threadIdx.x; i < ngr * 128; i += blockDim.x) {
      const int gl = i >> 7, c = i & 127;
      const int nn = slab * kGemvCols + c;
      if (nn < N) {
        const int64_t off = zbase + static_cast<int64_t>(g0 + gl) * N + nn;
        s_s[i] = __ushort_as_half(__ldg(w.scales + off));
        s_z[i] = __ushort_as_half(__ldg(w.zeros + off));
      }
    }
  }
  // Stage x (after the scale / zero rows above, which do not depend on the up
  // projection). Every thread first issues all of its loads for a batch of elements
  // into registers and only then stores them, so a batch costs one memory round trip
  // instead of one per element. A chained down launch first waits for its row's up
  // partials (one thread polls; the barrier passes the acquire on) and reads them past
  // L1.
  if (chain_in) {
    if (threadIdx.x == 0) tile_done_wait(src.done + a, src.done_target);
    __syncthreads();
  }
  for (int base = 0; base < kspan; base += kXB * kGemvThreads) {
    float v[kXB];
    if (src.mode == kGemvX || src.mode == kGemvSwiGLU) {
      __half x1[kXB], x3[kXB];
#pragma unroll
      for (int j = 0; j < kXB; ++j) {
        const int kk = k0 + base + j * kGemvThreads + threadIdx.x;
        const bool in = (base + j * kGemvThreads + threadIdx.x < kspan) && kk < K;
        x1[j] = in ? src.x[a * src.x_stride + kk] : __float2half_rn(0.f);
        x3[j] = (in && src.mode == kGemvSwiGLU) ? src.x3[a * src.x_stride + kk] : __float2half_rn(0.f);
      }
#pragma unroll
      for (int j = 0; j < kXB; ++j)
        v[j] = (src.mode == kGemvX) ? __half2float(x1[j]) : silu_f32(__half2float(x1[j])) * __half2float(x3[j]);
    } else {
      const int64_t mstride = static_cast<int64_t>(src.part_splits) * src.part_rows * src.part_n;
      float g1[kXB], g3[kXB];
#pragma unroll
      for (int j = 0; j < kXB; ++j) g1[j] = g3[j] = 0.f;
      // split-major: the loads of all elements of one split issue together
      for (int q = 0; q < src.part_splits; ++q) {
#pragma unroll
        for (int j = 0; j < kXB; ++j) {
          const int kk = k0 + base + j * kGemvThreads + threadIdx.x;
          if (base + j * kGemvThreads + threadIdx.x < kspan && kk < K) {
            const int64_t off = (static_cast<int64_t>(q) * src.part_rows + a) * src.part_n + kk;
            g1[j] += __ldcg(src.part + off);
            g3[j] += __ldcg(src.part + mstride + off);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kXB; ++j) {
        const float x1 = __half2float(__float2half_rn(g1[j]));
        const float x3 = __half2float(__float2half_rn(g3[j]));
        v[j] = (src.mode == kGemvPartF32)
                   ? silu_f32(x1) * x3
                   : __half2float(__float2half_rn(__half2float(__float2half_rn(silu_f32(x1))) * x3));
      }
    }
#pragma unroll
    for (int j = 0; j < kXB; ++j) {
      const int i = base + j * kGemvThreads + threadIdx.x;
      if (i < kspan) {
        // code c of word row r at slot r * eps + (c < eps/2 ? 2c : 2(c - eps/2) + 1)
        const int r = i / eps, c = i - r * eps, h = eps >> 1;
        const int slot = r * eps + (c < h ? 2 * c : 2 * (c - h) + 1);
        reinterpret_cast<float*>(s_raw)[slot] = v[j];  // fp32 (fp16 inputs convert exactly)
      }
    }
  }
  __syncthreads();
  float acc[4][2] = {};
  const GroupStage gs{s_s, s_z, g0};
  RowAcc<SUB> ra(K, g, nb, lane, k0, s_raw, gs);
  if (bulk) {
    if (warp_wait(&s_wbar, 0u, kDevTimeoutTmaFull)) {
      for (int r = wr0; r < wr1; ++r)
        ra.row(r, *reinterpret_cast<const uint4*>(s_words + (r - r0) * kGemvCols + lane * 4), acc);
    }
  } else if (n < N) {
    gemv_rows<SUB>(wbase, N, n, wr0, wr1, ra, wv, acc);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) s_red[warp][lane * 4 + c] = acc[c][0] + acc[c][1];
  __syncthreads();
  if (threadIdx.x < kGemvCols) {
    const int nn = slab * kGemvCols + threadIdx.x;
    if (nn < N) {
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) v += s_red[i][threadIdx.x];
      part[((static_cast<int64_t>(mat) * splits + s) * rows_a + a) * N + nn] = v;
    }
  }
  if (chain_out) {
    __syncthreads();
    signal_row();
  }
}

__global__ void k_gemv_reduce(const float* __restrict__ part, int splits, int64_t count, __half* __restrict__ out) {
  grid_dep_wait();
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= count) return;
  float v = 0.f;
#pragma unroll 4
  for (int s = 0; s < splits; ++s) v += part[s * count + i];
  out[i] = __float2half_rn(v);
}

// out[n] = fp16(sum_a w[a] * x2[a][n]) with x2 = fp16(sum_s part[s][a][n]): the fp32
// einsum combine of forward_one_token (moe_block.py:849-850); then the shared
// experts' fp16 output (moe_block.py:620) and an optional residual, each in fp16.
__global__ void k_decode_combine(const float* __restrict__ part, int splits, int A, int n, const __half* __restrict__ w,
                                 const float* __restrict__ shared_part, int shared_splits,
                                 const __half* __restrict__ residual, __half* __restrict__ out) {
  grid_dep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  // split-major, so the partials of all rows a of one split load together; each
  // x2[a] is still summed in split order
  float x2[16];
#pragma unroll
  for (int a = 0; a < 16; ++a) x2[a] = 0.f;
  for (int s = 0; s < splits; ++s) {
#pragma unroll
    for (int a = 0; a < 16; ++a)
      if (a < A) x2[a] += part[(static_cast<int64_t>(s) * A + a) * n + i];
  }
  float acc = 0.f;
#pragma unroll
  for (int a = 0; a < 16; ++a)
    if (a < A) acc = fmaf(__half2float(w[a]), __half2float(__float2half_rn(x2[a])), acc);
  __half r = __float2half_rn(acc);
  if (shared_part != nullptr) {
    float v = 0.f;
    for (int s = 0; s < shared_splits; ++s) v += shared_part[static_cast<int64_t>(s) * n + i];
    r = __float2half_rn(__half2float(r) + __half2float(__float2half_rn(v)));
  }
  if (residual != nullptr) r = __float2half_rn(__half2float(r) + __half2float(residual[i]));
  out[i] = r;
}

template <bool SUB>
cudaError_t launch_gemv_t(const ProjDev& w0, const ProjDev* w1, const int32_t* idx, int rows_a, const GemvSrc& src,
                          float* part, int splits, cudaStream_t s) {
  const int nmat = (w1 != nullptr) ? 2 : 1;
  // x of a split (at most cdiv(rows, splits) word rows of <= 32 codes: < k/splits + 64)
  // plus the scale and zero rows of the groups it touches
  const int word_bytes = gemv_word_rows(w0.k, splits) * kGemvCols * 4;
  const int bulk = (w0.n % kGemvCols == 0 && word_bytes <= kGemvWordBudget) ? 1 : 0;
  const size_t smem = static_cast<size_t>(gemv_words_off(w0.k, splits, w0.group_size, false)) + (bulk ? word_bytes : 0);
  static std::atomic<size_t> smem_done[kMaxDevices];  // per device: the attribute is per device
  if (smem > 48 * 1024) {
    cudaError_t e = raise_smem_limit(k_gemv<SUB>, smem, smem_done);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((w0.n + kGemvCols - 1) / kGemvCols, splits, nmat * rows_a);
  return launch_dep(k_gemv<SUB>, grid, dim3(kGemvThreads), smem, s, w0, w1 != nullptr ? *w1 : w0, idx, rows_a, src,
                    part, splits, bulk);
}

}  // namespace

int gemv_default_splits(int k, int n, int rows_a, int num_sms, int nmat) {
  // the largest power-of-two split that keeps the grid within one wave of
  // kGemvCtasPerSm CTAs per SM (each CTA issues all its word loads early; a second
  // wave would pay the HBM latency again), with at least 256 k per split
  const int ctas = ((n + kGemvCols - 1) / kGemvCols) * rows_a * nmat;
  int s = 1;
  while (ctas * s * 2 <= kGemvCtasPerSm * num_sms && s < 16 && (k / (s * 2)) >= 256) s *= 2;
  return s;
}

cudaError_t launch_gemv(const ProjDev& w0, const ProjDev* w1, const int32_t* idx, int rows_a, const GemvSrc& src,
                        float* part, int splits, cudaStream_t s) {
  if (rows_a == 0) return cudaSuccess;
  // the fast inner loop needs whole words inside one scale group for b in {1, 2, 4}
  if (w0.group_size % 32 != 0 || (w1 != nullptr && w1->group_size % 32 != 0)) return cudaErrorNotSupported;
  // the single-instruction dequant when every scale of the projection(s) allows it
  const bool sub = w0.sub_ok != 0 && (w1 == nullptr || w1->sub_ok != 0);
  return sub ? launch_gemv_t<true>(w0, w1, idx, rows_a, src, part, splits, s)
             : launch_gemv_t<false>(w0, w1, idx, rows_a, src, part, splits, s);
}

cudaError_t launch_gemv_reduce(const float* part, int splits, int rows_a, int n, uint16_t* out, cudaStream_t s) {
  const int64_t count = static_cast<int64_t>(rows_a) * n;
  if (count == 0) return cudaSuccess;
  return launch_dep(k_gemv_reduce, dim3(static_cast<unsigned>((count + 255) / 256)), dim3(256), 0, s, part, splits,
                    count, reinterpret_cast<__half*>(out));
}

cudaError_t launch_decode_combine(const float* part, int splits, int A, int n, const uint16_t* w,
                                  const float* shared_part, int shared_splits, const uint16_t* residual, uint16_t* out,
                                  cudaStream_t s) {
  return launch_dep(k_decode_combine, dim3((n + 255) / 256), dim3(256), 0, s, part, splits, A, n,
                    reinterpret_cast<const __half*>(w), shared_part, shared_splits,
                    reinterpret_cast<const __half*>(residual), reinterpret_cast<__half*>(out));
}

}  // namespace gemq
