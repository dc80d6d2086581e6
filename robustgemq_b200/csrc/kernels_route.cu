// Routing, dispatch and combine of the quantized MoE block.
//
// Reference behaviour restated (paths relative to the RobustGEMQ root):
//   router     gemq/inference/moe_block.py:790-797 (fp16 logits), 549-556 (fp32 logits),
//              280-283 (Mixtral one-token: fp16 softmax / top-k / renorm); DeepSeek-V2's
//              group-limited greedy selection and routed_scaling_factor, which the
//              reference's fused block rejects (moe_block.py:18-66), as transformers'
//              DeepseekV2Moe.route_tokens_to_experts computes them
//   dispatch   gemq/inference/moe_block.py:804-810 (one_hot / nonzero / where / gather)
//   combine    gemq/inference/moe_block.py:799-812 (fp16 index_add_ in ascending expert order)
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>

#include "gemq_common.cuh"
#include "gemq_internal.h"
#include "kperm.cuh"

namespace gemq {

namespace {
__constant__ kperm::Perm3 c_perm3_route = kperm::make_perm3();
}  // namespace

namespace {

constexpr int kMaxExperts = 256;

// Routing options of the top-k step beyond the plain greedy selection.
struct TopkOpts {
  int norm;          // renormalise: w / (sum of the k weights)
  int fp16_softmax;  // Mixtral one-token router: probabilities and sums rounded to fp16
  int n_group;       // group-limited greedy: E experts in n_group equal groups (1 = off)
  int topk_group;    // groups kept per token
  float scale;       // factor on the weights when not renormalising (routed_scaling_factor)
};

// Top-k of one token's probabilities v (slot i of lane l = expert 32 i + l; NV slots
// in use) in k rounds of a warp argmax, in the order "larger probability first,
// lower expert id on ties", NaN ahead of every number (torch.topk's order). Each
// value has an unsigned key that orders the same way: the probability's bits + 1
// (non-negative floats order as their bits; a NaN counts as FLT_MAX, a zero of
// either sign as +0), 0 for a slot out of range or already taken. A round takes the
// warp maximum of the lanes' best keys, then the lowest expert id holding it (two
// redux.sync). The selected weights are summed in selection order, then lane r
// writes the rank-r expert and its weight: w / sum when renormalising, else w * scale.
//
// Group-limited greedy (n_group > 1): each group's score is the largest probability
// among its E / n_group consecutive experts; the topk_group best groups are kept
// (larger score first, lower group id on ties; lane g holds group g's key), and the
// probabilities of every other group's experts become 0.0 before the k rounds, as
// masked_fill(~mask, 0.0) does, so they stay selectable only behind every kept one.
template <int NV>
__device__ __forceinline__ void select_topk(float (&v)[kMaxExperts / 32], int E, int k, const TopkOpts& o,
                                            int32_t* __restrict__ idx_out, __half* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  uint32_t key[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t bits = __float_as_uint(v[i] != v[i] ? FLT_MAX : v[i]);
    key[i] = (i * 32 + lane >= E) ? 0u : (bits & 0x80000000u) ? 1u : bits + 1u;
  }
  if (o.n_group > 1) {
    const int gsize = E / o.n_group;
    int grp[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) grp[i] = (i * 32 + lane < E) ? (i * 32 + lane) / gsize : -1;
    uint32_t gkey = 0u;
    for (int g = 0; g < o.n_group; ++g) {
      uint32_t m = 0u;
#pragma unroll
      for (int i = 0; i < NV; ++i) m = (grp[i] == g && key[i] > m) ? key[i] : m;
      m = __reduce_max_sync(0xffffffffu, m);
      if (lane == g) gkey = m;
    }
    uint32_t keep = 0u;  // bit g: group g kept (warp-uniform)
    for (int r = 0; r < o.topk_group; ++r) {
      const uint32_t gmax = __reduce_max_sync(0xffffffffu, gkey);
      if (gmax == 0u) break;
      const uint32_t win = __reduce_min_sync(0xffffffffu, gkey == gmax ? static_cast<uint32_t>(lane) : 32u);
      keep |= 1u << win;
      if (lane == static_cast<int>(win)) gkey = 0u;
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (grp[i] >= 0 && !((keep >> grp[i]) & 1u)) {
        v[i] = 0.f;
        key[i] = 1u;  // +0.0
      }
    }
  }
  float wsum = 0.f, myw = 0.f;
  int mye = 0;
  for (int r = 0; r < k; ++r) {
    uint32_t best = 0u;
    int bi = 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (key[i] > best) {  // strict: the lowest slot (expert id) of the lane on ties
        best = key[i];
        bi = i;
      }
    }
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, best);
    if (wmax == 0u) break;  // fewer valid experts than k (warp-uniform)
    const uint32_t win = __reduce_min_sync(0xffffffffu, best == wmax ? static_cast<uint32_t>(bi * 32 + lane) : ~0u);
    float mine = v[0];
#pragma unroll
    for (int i = 1; i < NV; ++i) mine = (bi == i) ? v[i] : mine;
    const int src = static_cast<int>(win & 31u);
    const float val = __shfl_sync(0xffffffffu, mine, src);
    wsum += val;
    if (lane == r) {
      myw = val;
      mye = static_cast<int>(win);
    }
    if (lane == src) {
#pragma unroll
      for (int i = 0; i < NV; ++i) key[i] = (i == bi) ? 0u : key[i];
    }
  }
  if (lane < k) {
    if (o.fp16_softmax) wsum = __half2float(__float2half_rn(wsum));
    idx_out[lane] = mye;
    w_out[lane] = __float2half_rn(o.norm ? myw / wsum : myw * o.scale);
  }
}

// Softmax + top-k + optional renormalisation of one token's logits by one warp.
// Softmax in fp32 with expf; selection takes the larger probability first and the
// lower expert id on ties; NaN ranks above every number (torch.topk's order), so
// the selected ids are always valid. fp16_softmax rounds the probabilities, their
// sum and the quotients to fp16 as the fp16 tensors of moe_block.py:280-283 do.
template <typename GetLogit>
__device__ __forceinline__ void topk_warp(GetLogit get, int E, int k, const TopkOpts& o, int32_t* __restrict__ idx_out,
                                          __half* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  float v[kMaxExperts / 32];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i) {
    const int e = i * 32 + lane;
    const float l = (e < E) ? get(e) : -FLT_MAX;
    v[i] = l;
    mx = fmaxf(mx, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i) {
    const int e = i * 32 + lane;
    v[i] = (e < E) ? expf(v[i] - mx) : 0.f;
    sum += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i) {
    const int e = i * 32 + lane;
    float pr = (e < E) ? v[i] / sum : -1.f;
    if (o.fp16_softmax && e < E) pr = __half2float(__float2half_rn(pr));
    v[i] = pr;
  }
  const int nv = (E + 31) / 32;  // value slots per lane in use
  if (nv <= 1) select_topk<1>(v, E, k, o, idx_out, w_out);
  else if (nv <= 2) select_topk<2>(v, E, k, o, idx_out, w_out);
  else if (nv <= 4) select_topk<4>(v, E, k, o, idx_out, w_out);
  else select_topk<8>(v, E, k, o, idx_out, w_out);
}

// One warp per token, logits from global memory (the tensor-core router's output
// or given logits).
__global__ void k_topk(const void* __restrict__ logits, int logits_fp32, int64_t T, int E, int k, TopkOpts o,
                       int32_t* __restrict__ topk_idx, __half* __restrict__ topk_w, int32_t* __restrict__ zero_buf,
                       int zero_n) {
  grid_dep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < zero_n; i += gridDim.x * blockDim.x)
    zero_buf[i] = 0;  // the forward's chained-GEMV counters
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (t >= T) return;
  auto get = [&](int e) {
    return logits_fp32 ? static_cast<const float*>(logits)[t * E + e]
                       : __half2float(static_cast<const __half*>(logits)[t * E + e]);
  };
  topk_warp(get, E, k, o, topk_idx + t * k, topk_w + t * k);
}

// Gate logits for small batches, spread over many CTAs: CTA (i, j) computes experts
// 8i .. 8i+7 (one warp each) for tokens 8j .. 8j+7 (rows staged in shared memory),
// fp32 accumulation; the fp16 router rounds each logit to fp16 as F.linear's fp16
// output does (moe_block.py:790), the fp32 router keeps it (moe_block.py:549).
constexpr int kLogitExperts = 8;
constexpr int kLogitTokens = 8;

__global__ void __launch_bounds__(256) k_gate_logits(const __half* __restrict__ x, int64_t T, int D,
                                                     const __half* __restrict__ gate, int E, int fp32_logits,
                                                     void* __restrict__ logits) {
  grid_dep_wait();
  extern __shared__ uint4 s_rows4[];  // [kLogitTokens][D / 8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kLogitTokens;
  const int nt = (T - t0 < kLogitTokens) ? static_cast<int>(T - t0) : kLogitTokens;
  const int d8 = D / 8;
  // all of a thread's row loads in flight before any store (one round trip)
  for (int base = threadIdx.x; base < nt * d8; base += 8 * blockDim.x) {
    uint4 t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * blockDim.x;
      if (i < nt * d8) {
        const int r = i / d8, c = i - r * d8;
        t[j] = reinterpret_cast<const uint4*>(x + (t0 + r) * D)[c];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * blockDim.x;
      if (i < nt * d8) s_rows4[i] = t[j];
    }
  }
  __syncthreads();
  const int e = blockIdx.x * kLogitExperts + warp;
  if (e >= E) return;
  const uint4* gr = reinterpret_cast<const uint4*>(gate + static_cast<int64_t>(e) * D);
  float acc[kLogitTokens];
#pragma unroll
  for (int r = 0; r < kLogitTokens; ++r) acc[r] = 0.f;
#pragma unroll 8
  for (int c = lane; c < d8; c += 32) {
    const uint4 gv = __ldg(gr + c);
    const __half2* gh = reinterpret_cast<const __half2*>(&gv);
    float2 g2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) g2[j] = __half22float2(gh[j]);
#pragma unroll
    for (int r = 0; r < kLogitTokens; ++r) {
      if (r < nt) {
        const uint4 xv = s_rows4[r * d8 + c];
        const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = __half22float2(xh[j]);
          acc[r] = fmaf(a.x, g2[j].x, acc[r]);
          acc[r] = fmaf(a.y, g2[j].y, acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kLogitTokens; ++r) {
    float v = acc[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && r < nt) {
      const int64_t i = (t0 + r) * E + e;
      if (fp32_logits) static_cast<float*>(logits)[i] = v;
      else static_cast<__half*>(logits)[i] = __float2half_rn(v);
    }
  }
}

// Loads token row `src` (D fp16, D % 8 == 0) into the warp's staging buffer `sbuf`
// (D halves of shared memory), each lane's 16-byte chunks of a batch of 8 in flight
// together.
__device__ __forceinline__ void stage_row(const __half* __restrict__ src, __half* sbuf, int D, int lane) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* b4 = reinterpret_cast<uint4*>(sbuf);
  for (int base = lane; base < D / 8; base += 8 * 32) {
    uint4 t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (base + 32 * j < D / 8) t[j] = s4[base + 32 * j];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (base + 32 * j < D / 8) b4[base + 32 * j] = t[j];
  }
  __syncwarp();
}

// Writes the staged row to `dst` by one warp: as is (nb = 0), or in the decode
// GEMM's K slot order for bit-width nb (kperm.cuh; D % 128 == 0 then), gathered
// through the 3-bit slot table `fwd3` staged in shared memory (lanes index it
// divergently).
__device__ __forceinline__ void store_row(const __half* sbuf, __half* __restrict__ dst, int D, int nb, int lane,
                                          const uint8_t (*fwd3)[128]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  if (nb == 0) {
    const uint4* b4 = reinterpret_cast<const uint4*>(sbuf);
    for (int i = lane; i < D / 8; i += 32) d4[i] = b4[i];
    return;
  }
  const unsigned short* b16 = reinterpret_cast<const unsigned short*>(sbuf);
  // b in {1, 2, 4}: eps = 32 / b codes per word, slot 2j + h of a word block <-> code
  // j + h * eps / 2 (kperm::perm_pow2), with shifts and masks instead of divisions
  const int lg_eps = 5 - (nb >> 1);  // nb = 1, 2, 4 -> 5, 4, 3
  const int eps_mask = (1 << lg_eps) - 1, half = 1 << (lg_eps - 1);
  auto chunk = [&](int i) {
    const int k0 = 8 * i, st = k0 >> 7;
    const unsigned short* row = b16 + (st << 7);
    if (nb == 3) {
      const uint2 fw = *reinterpret_cast<const uint2*>(fwd3[kperm::phase3(st)] + (k0 & 127));
      uint32_t v[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t f = m < 2 ? fw.x : fw.y;
        const int sh = 16 * (m & 1);
        v[m] = static_cast<uint32_t>(row[(f >> sh) & 0xffu]) | (static_cast<uint32_t>(row[(f >> (sh + 8)) & 0xffu]) << 16);
      }
      return make_uint4(v[0], v[1], v[2], v[3]);
    }
    // slots 2m, 2m + 1 of the chunk hold codes j0 + m and j0 + m + eps / 2 of its word
    // block: two runs of four consecutive halves (8-byte aligned), interleaved
    const int sa = k0 & 127;
    const int a = (sa & ~eps_mask) + ((sa & eps_mask) >> 1);
    const uint2 lo = *reinterpret_cast<const uint2*>(row + a);
    const uint2 hi = *reinterpret_cast<const uint2*>(row + a + half);
    return make_uint4(__byte_perm(lo.x, hi.x, 0x5410), __byte_perm(lo.x, hi.x, 0x7632),
                      __byte_perm(lo.y, hi.y, 0x5410), __byte_perm(lo.y, hi.y, 0x7632));
  };
  // four chunks gathered, then their four stores issued together
  for (int base = lane; base < D / 8; base += 4 * 32) {
    uint4 o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (base + 32 * u < D / 8) o[u] = chunk(base + 32 * u);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (base + 32 * u < D / 8) d4[base + 32 * u] = o[u];
  }
}

// Copies token row `src` to `dst` by one warp: as is (nb = 0: directly, `sbuf` unused
// and may be empty) or in the K slot order of bit-width nb through the warp's staging
// buffer (store_row).
__device__ __forceinline__ void copy_row(const __half* __restrict__ src, __half* __restrict__ dst, int D, int nb,
                                         int lane, __half* sbuf, const uint8_t (*fwd3)[128]) {
  if (nb == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int base = lane; base < D / 8; base += 8 * 32) {
      uint4 t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (base + 32 * j < D / 8) t[j] = s4[base + 32 * j];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (base + 32 * j < D / 8) d4[base + 32 * j] = t[j];
    }
    return;
  }
  stage_row(src, sbuf, D, lane);
  store_row(sbuf, dst, D, nb, lane, fwd3);
  __syncwarp();
}

__device__ __forceinline__ void stage_fwd3(uint8_t (*fwd3)[128]) {
  for (int i = threadIdx.x; i < 5 * 128; i += blockDim.x) fwd3[i >> 7][i & 127] = c_perm3_route.fwd[i >> 7][i & 127];
}

// ------------------------------------------------------------------ dispatch (large batches)
// Rows per expert: a shared-memory histogram per CTA over a stretch of slots, then
// one global atomic per expert hit (E <= 1024).
constexpr int kCountSlotsPerCta = 2048;

__global__ void k_count(const int32_t* __restrict__ topk_idx, int64_t P, int E, int32_t* __restrict__ counts) {
  grid_dep_wait();
  __shared__ int s_cnt[1024];
  for (int i = threadIdx.x; i < E; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kCountSlotsPerCta;
  for (int64_t i = i0 + threadIdx.x; i < P && i < i0 + kCountSlotsPerCta; i += blockDim.x) {
    const int e = topk_idx[i];
    if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
    else set_device_error(kDevBadExpert);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (s_cnt[i] != 0) atomicAdd(&counts[i], s_cnt[i]);
}

// Single block: exclusive scans over experts (E <= 1024).
__global__ void k_scan_segs(const int32_t* __restrict__ counts, int E, int nt, Seg* __restrict__ segs,
                            int32_t* __restrict__ tile_prefix, int32_t* __restrict__ cursor,
                            int32_t* __restrict__ zero_buf, int zero_n) {
  grid_dep_wait();
  for (int i = threadIdx.x; i < zero_n; i += blockDim.x) zero_buf[i] = 0;  // per-forward tile counters
  __shared__ int s_rows[1024];
  __shared__ int s_tiles[1024];
  const int e = threadIdx.x;
  const int c = (e < E) ? counts[e] : 0;
  s_rows[e] = c;
  s_tiles[e] = (c + nt - 1) / nt;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int a = (e >= off) ? s_rows[e - off] : 0;
    const int b = (e >= off) ? s_tiles[e - off] : 0;
    __syncthreads();
    s_rows[e] += a;
    s_tiles[e] += b;
    __syncthreads();
  }
  if (e < E) {
    const int start = s_rows[e] - c;
    segs[e] = make_int4(e, start, start, c);
    tile_prefix[e] = s_tiles[e] - (c + nt - 1) / nt;
    cursor[e] = start;
    if (e == E - 1) tile_prefix[E] = s_tiles[e];
  }
}

// One warp per token: lanes j < k claim the rows of the token's slots (one atomic
// each, in parallel) and record them; the token's activation row is staged in the
// warp's shared buffer once and written to each claimed row, as is or in the K slot
// order of the expert's bit-width. Rows within a segment are in arrival order, which
// changes no result: each row is computed alone and the combine visits a token's
// experts in ascending id. A slot whose expert id is out of range (k_count recorded
// kDevBadExpert) gets no row and slot_pos -1, which the combine skips.
constexpr int kScatterWarps = 8;

__global__ void __launch_bounds__(32 * kScatterWarps, 4)
    k_scatter(const int32_t* __restrict__ topk_idx, const __half* __restrict__ topk_w, const __half* __restrict__ x,
              int64_t T, int k, int E, int D, int32_t* __restrict__ cursor, int32_t* __restrict__ slot_pos,
              __half* __restrict__ w_perm, __half* __restrict__ x_perm, const int32_t* __restrict__ perm_nbits) {
  grid_dep_wait();
  __shared__ __align__(16) uint8_t s_fwd3[5][128];
  if (perm_nbits != nullptr) {
    stage_fwd3(s_fwd3);
    __syncthreads();
  }
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  int pos = -1, nb = 0;
  if (lane < k) {
    const int64_t slot = t * k + lane;
    const int e = topk_idx[slot];
    if (e >= 0 && e < E) {
      pos = atomicAdd(&cursor[e], 1);
      w_perm[pos] = topk_w[slot];
      if (perm_nbits != nullptr) nb = min(max(__ldg(perm_nbits + e), 1), 4);
    }
    slot_pos[slot] = pos;
  }
  extern __shared__ __align__(16) __half s_stage_rows[];
  __half* sbuf = s_stage_rows + static_cast<size_t>(threadIdx.x >> 5) * D;
  const __half* src = x + t * D;
  if (perm_nbits != nullptr) stage_row(src, sbuf, D, lane);
  for (int j = 0; j < k; ++j) {
    const int pj = __shfl_sync(0xffffffffu, pos, j), nj = __shfl_sync(0xffffffffu, nb, j);
    if (pj < 0) continue;  // warp-uniform
    __half* dst = x_perm + static_cast<int64_t>(pj) * D;
    if (perm_nbits != nullptr) {
      store_row(sbuf, dst, D, nj, lane, s_fwd3);
    } else {
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      for (int i = lane; i < D / 8; i += 32) d4[i] = s4[i];
    }
  }
}

// ------------------------------------------------------------------ dispatch (small batches)
// One launch: every CTA recounts the (small) slot list in shared memory, scans it,
// and places its own 8 slots at deterministic positions (rank among earlier slots
// of the same expert); CTA 0 also publishes counts, segments and the tile prefix.
constexpr int kSmallDispatchMaxSlots = 4096;

__device__ __forceinline__ void warp_exclusive_scan_256(const int* in, int* out, int E, int lane) {
  // E <= 256: each lane owns 8 consecutive entries
  int vals[8];
  int local = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane * 8 + i;
    vals[i] = (e < E) ? in[e] : 0;
    local += vals[i];
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int run = incl - local;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane * 8 + i;
    if (e < E) out[e] = run;
    run += vals[i];
  }
  if (lane == 31) out[E] = incl;
}

__global__ void __launch_bounds__(256) k_dispatch_small(const int32_t* __restrict__ topk_idx,
                                                        const __half* __restrict__ topk_w, const __half* __restrict__ x,
                                                        int P, int k, int E, int D, int nt, int32_t* __restrict__ counts,
                                                        Seg* __restrict__ segs, int32_t* __restrict__ tile_prefix,
                                                        int32_t* __restrict__ slot_pos, __half* __restrict__ w_perm,
                                                        __half* __restrict__ x_perm,
                                                        const int32_t* __restrict__ perm_nbits,
                                                        const int32_t* __restrict__ order_nbits,
                                                        int32_t* __restrict__ zero_buf, int zero_n) {
  grid_dep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < zero_n; i += gridDim.x * blockDim.x)
    zero_buf[i] = 0;  // per-forward tile counters
  __shared__ int s_idx[kSmallDispatchMaxSlots];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_tiles[kMaxExperts];
  __shared__ int s_start[kMaxExperts + 1];
  __shared__ int s_tstart[kMaxExperts + 1];
  __shared__ __align__(16) uint8_t s_fwd3[5][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  if (perm_nbits != nullptr) stage_fwd3(s_fwd3);
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = topk_idx[i];
    s_idx[i] = e;
    if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
    else if (blockIdx.x == 0) set_device_error(kDevBadExpert);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_tiles[e] = (s_cnt[e] + nt - 1) / nt;
  __syncthreads();
  if (warp == 0) warp_exclusive_scan_256(s_cnt, s_start, E, lane);
  __syncthreads();
  if (blockIdx.x == 0) {
    // Segment order (rows keep their expert-order positions): expert id, or with
    // order_nbits the dequant cost of the expert's bit-width, 3-bit first, then 4, 2
    // and 1 bits, stable in expert id. The decode GEMM hands out work items in this
    // order, whole waves round-robin, so its last, partial wave holds the cheapest.
    __shared__ int s_wcnt[8][4];
    __shared__ int s_order[kMaxExperts];
    const int e = threadIdx.x;  // E <= 256 = blockDim.x
    const bool valid = e < E;
    int cls = 0;
    if (order_nbits != nullptr && valid) {
      const int nb = order_nbits[e];
      cls = (nb == 3) ? 0 : (nb == 4) ? 1 : (nb == 2) ? 2 : 3;
    }
    const unsigned lt = (1u << lane) - 1u;
    int within = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const unsigned b = __ballot_sync(0xffffffffu, valid && cls == c);
      if (lane == 0) s_wcnt[warp][c] = __popc(b);
      if (cls == c) within = __popc(b & lt);
    }
    __syncthreads();
    int pos = within;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int w = 0; w < 8; ++w) pos += (c < cls || (c == cls && w < warp)) ? s_wcnt[w][c] : 0;
    if (valid) {
      s_order[pos] = e;
      s_tstart[pos] = s_tiles[e];  // tiles in segment order, scanned below
    }
    __syncthreads();
    if (warp == 0) warp_exclusive_scan_256(s_tstart, s_tstart, E, lane);
    __syncthreads();
    if (valid) {
      const int eo = s_order[e];  // segment e
      counts[e] = s_cnt[e];
      segs[e] = make_int4(eo, s_start[eo], s_start[eo], s_cnt[eo]);
      tile_prefix[e] = s_tstart[e];
    }
    if (threadIdx.x == 0) tile_prefix[E] = s_tstart[E];
  }
  const int slot = blockIdx.x * 8 + warp;
  if (slot >= P) return;
  const int e = s_idx[slot];
  if (e < 0 || e >= E) {
    if (lane == 0) slot_pos[slot] = -1;
    return;
  }
  int rank = 0;
  for (int s = lane; s < slot; s += 32) rank += (s_idx[s] == e) ? 1 : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
  const int pos = s_start[e] + rank;
  if (lane == 0) {
    slot_pos[slot] = pos;
    w_perm[pos] = topk_w[slot];
  }
  const int nb = perm_nbits != nullptr ? min(max(__ldg(perm_nbits + e), 1), 4) : 0;
  extern __shared__ __align__(16) __half s_stage_rows[];
  copy_row(x + static_cast<int64_t>(slot / k) * D, x_perm + static_cast<int64_t>(pos) * D, D, nb, lane,
           s_stage_rows + static_cast<size_t>(warp) * D, s_fwd3);
}

// ------------------------------------------------------------------ combine
// out[t] = ((0 + y_{e1}) + y_{e2}) + ... over the token's experts in ascending id,
// every partial sum rounded to fp16: the fp16 index_add_ of forward_n_tokens
// (moe_block.py:799-812). fp32_sum: one fp32 sum, one rounding. `add` (DeepSeek
// shared experts) is added in fp16 afterwards (moe_block.py:575), then `residual`.
//
// One warp per (token, column part): 8 warps per CTA over tokens, blockIdx.y the
// part of the row (parts > 1 for small batches, so that enough warps share the
// loads). Lane j < k holds slot j; its rank in the order (expert id, then slot index)
// is counted with shuffles, and lane r ends up with the row of the rank-r slot. Each
// lane then sums 16-byte chunks of the rows in rank order, the loads of two chunks
// of every row in flight together.
constexpr int kCombineWarps = 8;
constexpr int kCombineSms = 148;  // sizing of the column split only

template <int KMAX>  // bound on k: 8 or 16 (registers for the rows in flight)
__global__ void __launch_bounds__(32 * kCombineWarps, KMAX == 8 ? 2 : 1)
    k_combine(const __half* __restrict__ y_perm, const int32_t* __restrict__ slot_pos,
              const int32_t* __restrict__ topk_idx, int64_t T, int k, int D, int fp32_sum,
              const __half* __restrict__ add, const __half* __restrict__ residual, __half* __restrict__ out) {
  grid_dep_wait();
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int e = lane < k ? topk_idx[t * k + lane] : 0x7fffffff;
  const int pos = lane < k ? slot_pos[t * k + lane] : -1;
  int rank = 0;
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e, j);
    rank += (ej < e || (ej == e && j < lane)) ? 1 : 0;
  }
  int row_r = -1;  // row of the rank-`lane` slot
  for (int j = 0; j < k; ++j) {
    const int rj = __shfl_sync(0xffffffffu, rank, j), pj = __shfl_sync(0xffffffffu, pos, j);
    if (lane == rj) row_r = pj;
  }
  int rows[KMAX];
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    const int p = __shfl_sync(0xffffffffu, row_r, r);
    rows[r] = (r < k) ? p : -1;  // -1: a slot with an invalid expert id
  }
  const int d8 = D / 8;
  const int per = (d8 + gridDim.y - 1) / gridDim.y;  // chunks of this part
  const int cbeg = blockIdx.y * per, cend = min(d8, cbeg + per);
  for (int c0 = cbeg + lane; c0 < cend; c0 += 64) {
    uint4 yv[2][KMAX];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + 32 * h;
#pragma unroll
      for (int r = 0; r < KMAX; ++r)
        if (rows[r] >= 0 && c < cend)
          yv[h][r] = reinterpret_cast<const uint4*>(y_perm + static_cast<int64_t>(rows[r]) * D)[c];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + 32 * h;
      if (c >= cend) break;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
      for (int r = 0; r < KMAX; ++r) {
        if (rows[r] < 0) continue;
        const __half* yh = reinterpret_cast<const __half*>(&yv[h][r]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float y = __half2float(yh[i]);
          acc[i] = fp32_sum ? acc[i] + y : __half2float(__float2half_rn(acc[i] + y));
        }
      }
      __half res[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) res[i] = __float2half_rn(acc[i]);
      const int64_t o = t * D + 8 * static_cast<int64_t>(c);
      if (add != nullptr) {
        const uint4 av = *reinterpret_cast<const uint4*>(add + o);
        const __half* ah = reinterpret_cast<const __half*>(&av);
#pragma unroll
        for (int i = 0; i < 8; ++i) res[i] = __float2half_rn(__half2float(res[i]) + __half2float(ah[i]));
      }
      if (residual != nullptr) {
        const uint4 rv = *reinterpret_cast<const uint4*>(residual + o);
        const __half* rh = reinterpret_cast<const __half*>(&rv);
#pragma unroll
        for (int i = 0; i < 8; ++i) res[i] = __float2half_rn(__half2float(res[i]) + __half2float(rh[i]));
      }
      *reinterpret_cast<uint4*>(out + o) = *reinterpret_cast<const uint4*>(res);
    }
  }
}

}  // namespace

cudaError_t launch_topk(const void* logits, bool logits_fp32, int64_t T, int E, int k, bool norm, bool fp16_softmax,
                        int n_group, int topk_group, float scale, int32_t* topk_idx, uint16_t* topk_w,
                        cudaStream_t stream, int32_t* zero_buf, int zero_n) {
  if (T == 0) return cudaSuccess;
  const TopkOpts o{norm ? 1 : 0, fp16_softmax ? 1 : 0, n_group, topk_group, scale};
  return launch_dep(k_topk, dim3(static_cast<unsigned>((T * 32 + 255) / 256)), dim3(256), 0, stream, logits,
                    logits_fp32 ? 1 : 0, T, E, k, o, topk_idx, reinterpret_cast<__half*>(topk_w), zero_buf, zero_n);
}

cudaError_t launch_gate_logits(const uint16_t* x, int64_t T, int D, const uint16_t* gate, int E, bool fp32_logits,
                               void* logits, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(kLogitTokens) * D * 2;
  static std::atomic<size_t> smem_done[kMaxDevices];  // per device: the attribute is per device
  if (smem > 48 * 1024) {
    cudaError_t e = raise_smem_limit(k_gate_logits, smem, smem_done);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid((E + kLogitExperts - 1) / kLogitExperts, static_cast<unsigned>((T + kLogitTokens - 1) / kLogitTokens));
  return launch_dep(k_gate_logits, grid, dim3(32 * kLogitExperts), smem, stream, reinterpret_cast<const __half*>(x), T,
                    D, reinterpret_cast<const __half*>(gate), E, fp32_logits ? 1 : 0, logits);
}


// ------------------------------------------------------------------ grouped segments
// Rows arrive grouped as [group 0: expert 0 rows, expert 1 rows, ... | group 1: ...]
// (expert parallelism: one group per source rank, each sorted by local expert).
// Segment g * E + e covers the rows of expert e in group g; one block scans the
// G * E counts (at most 1024) into row starts and token-tile starts.
__global__ void k_group_segs(const int32_t* __restrict__ counts, int n, int E, int nt, Seg* __restrict__ segs,
                             int32_t* __restrict__ tile_prefix) {
  grid_dep_wait();
  __shared__ int s_rows[1024];
  __shared__ int s_tiles[1024];
  const int i = threadIdx.x;
  int c = (i < n) ? counts[i] : 0;
  if (c < 0) {
    set_device_error(kDevBadExpert);
    c = 0;
  }
  s_rows[i] = c;
  s_tiles[i] = (c + nt - 1) / nt;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int a = (i >= off) ? s_rows[i - off] : 0;
    const int b = (i >= off) ? s_tiles[i - off] : 0;
    __syncthreads();
    s_rows[i] += a;
    s_tiles[i] += b;
    __syncthreads();
  }
  if (i < n) {
    const int start = s_rows[i] - c;
    segs[i] = make_int4(i % E, start, start, c);
    tile_prefix[i] = s_tiles[i] - (c + nt - 1) / nt;
    if (i == n - 1) tile_prefix[n] = s_tiles[i];
  }
}

cudaError_t launch_group_segs(const int32_t* counts, int n, int E, int nt, Seg* segs, int32_t* tile_prefix,
                              cudaStream_t stream) {
  if (n <= 0 || n > 1024 || E <= 0) return cudaErrorInvalidValue;
  return launch_dep(k_group_segs, dim3(1), dim3(1024), 0, stream, counts, n, E, nt, segs, tile_prefix);
}

bool small_dispatch_ok(int64_t P, int E) { return P <= kSmallDispatchMaxSlots && E <= kMaxExperts; }

cudaError_t launch_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t T, int k,
                            int E, int D, int nt, int32_t* counts, int32_t* cursor, Seg* segs, int32_t* tile_prefix,
                            int32_t* slot_pos, uint16_t* w_perm, uint16_t* x_perm, const int32_t* perm_nbits,
                            const int32_t* order_nbits, int32_t* zero_buf, int zero_n, cudaStream_t stream) {
  const int64_t P = T * k;
  if (perm_nbits != nullptr && D % kperm::kStageK != 0) return cudaErrorInvalidValue;
  // permuted copies stage each warp's row in shared memory (8 warps per block)
  const size_t row_smem = perm_nbits != nullptr ? static_cast<size_t>(8) * D * sizeof(__half) : 0;
  if (row_smem > 0) {
    // raised per device and per larger row size (outside graph capture)
    static std::atomic<size_t> small_done[kMaxDevices], scatter_done[kMaxDevices];
    cudaError_t e = raise_smem_limit(k_dispatch_small, row_smem, small_done);
    if (e == cudaSuccess) e = raise_smem_limit(k_scatter, row_smem, scatter_done);
    if (e != cudaSuccess) return e;
  }
  cudaError_t err;
  if (small_dispatch_ok(P, E)) {
    const unsigned grid = static_cast<unsigned>(P > 0 ? (P + 7) / 8 : 1);
    return launch_dep(k_dispatch_small, dim3(grid), dim3(256), row_smem, stream, topk_idx,
                      reinterpret_cast<const __half*>(topk_w), reinterpret_cast<const __half*>(x), static_cast<int>(P),
                      k, E, D, nt, counts, segs, tile_prefix, slot_pos, reinterpret_cast<__half*>(w_perm),
                      reinterpret_cast<__half*>(x_perm), perm_nbits, order_nbits, zero_buf, zero_n);
  }
  err = cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream);
  if (err != cudaSuccess) return err;
  err = launch_dep(k_count, dim3(static_cast<unsigned>((P + kCountSlotsPerCta - 1) / kCountSlotsPerCta)), dim3(256), 0,
                   stream, topk_idx, P, E, counts);
  if (err != cudaSuccess) return err;
  err = launch_dep(k_scan_segs, dim3(1), dim3(1024), 0, stream, counts, E, nt, segs, tile_prefix, cursor, zero_buf,
                   zero_n);
  if (err != cudaSuccess) return err;
  return launch_dep(k_scatter, dim3(static_cast<unsigned>((T + kScatterWarps - 1) / kScatterWarps)),
                    dim3(32 * kScatterWarps), row_smem, stream, topk_idx, reinterpret_cast<const __half*>(topk_w),
                    reinterpret_cast<const __half*>(x), T, k, E, D, cursor, slot_pos,
                    reinterpret_cast<__half*>(w_perm), reinterpret_cast<__half*>(x_perm), perm_nbits);
}

cudaError_t launch_combine(const uint16_t* y_perm, const int32_t* slot_pos, const int32_t* topk_idx, int64_t T, int k,
                           int D, bool fp32_sum, const uint16_t* add, const uint16_t* residual, uint16_t* out,
                           cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((T + kCombineWarps - 1) / kCombineWarps);
  // column parts of 32 chunks (256 halves) or more, until about 16 warps per SM
  const int64_t want = (static_cast<int64_t>(kCombineSms) * 16 + T - 1) / T;
  const unsigned parts = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, D / 256)));
  return launch_dep(k <= 8 ? k_combine<8> : k_combine<16>, dim3(grid, parts), dim3(32 * kCombineWarps), 0, stream,
                    reinterpret_cast<const __half*>(y_perm), slot_pos, topk_idx, T, k, D, fp32_sum ? 1 : 0,
                    reinterpret_cast<const __half*>(add), reinterpret_cast<const __half*>(residual),
                    reinterpret_cast<__half*>(out));
}

}  // namespace gemq
