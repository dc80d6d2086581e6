// Packing, dequant, routing, dispatch, combine and the decode GEMV family.
//
// Reference behaviour restated (paths relative to the RobustGEMQ root):
//   pack/unpack          gemq/triton_kernels/utils.py:33-189
//   dequant              gemq/triton_kernels/utils.py:192-212
//   router               gemq/inference/moe_block.py:790-797 (fp16), 549-556 (fp32), 280-283 (fp16 softmax)
//   dispatch / combine   gemq/inference/moe_block.py:804-812
//   decode GEMVs         gemq/triton_kernels/fused_dequant_bmm.py, dequant_gemv.py
#include <cuda_fp16.h>

#include <cfloat>

#include "gemq_common.cuh"
#include "gemq_internal.h"

namespace gemq {

__device__ uint32_t g_device_error = 0;

// ------------------------------------------------------------------ pack / unpack
// One thread per output word. Codes are OR-ed in without masking, as the reference
// does (utils.py:57-66): a code wider than nbits spills into its neighbour, and
// bits shifted past 32 are dropped.
__global__ void k_pack(const uint8_t* __restrict__ codes, int64_t rows, int64_t cols, int nbits, int eps,
                       int64_t pcols, int32_t* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= rows * pcols) return;
  const int64_t r = i / pcols, c = i - r * pcols;
  const uint8_t* src = codes + r * cols + c * eps;
  uint32_t w = 0;
  for (int j = 0; j < eps; ++j) {
    if (c * eps + j < cols) w |= static_cast<uint32_t>(src[j]) << (j * nbits);
  }
  out[i] = static_cast<int32_t>(w);
}

__global__ void k_unpack(const int32_t* __restrict__ packed, int64_t rows, int64_t pcols, int64_t ocols, int nbits,
                         int eps, uint8_t* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= rows * ocols) return;
  const int64_t r = i / ocols, c = i - r * ocols;
  const uint32_t w = static_cast<uint32_t>(packed[r * pcols + c / eps]);
  out[i] = static_cast<uint8_t>((w >> ((c % eps) * nbits)) & ((1u << nbits) - 1u));
}

cudaError_t launch_pack(const uint8_t* codes, int64_t rows, int64_t cols, int nbits, int32_t* out, cudaStream_t s) {
  const int eps = 32 / nbits;
  const int64_t pcols = (cols + eps - 1) / eps;
  const int64_t n = rows * pcols;
  if (n == 0) return cudaSuccess;
  k_pack<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(codes, rows, cols, nbits, eps, pcols, out);
  return cudaGetLastError();
}

cudaError_t launch_unpack(const int32_t* packed, int64_t rows, int64_t pcols, int64_t ocols, int nbits, uint8_t* out,
                          cudaStream_t s) {
  const int64_t n = rows * ocols;
  if (n == 0) return cudaSuccess;
  k_unpack<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(packed, rows, pcols, ocols, nbits, 32 / nbits, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ dequant one expert
__global__ void k_dequant_expert(ProjDev p, int e, __half* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t total = static_cast<int64_t>(p.k) * p.n;
  if (i >= total) return;
  const int k = static_cast<int>(i / p.n), n = static_cast<int>(i - static_cast<int64_t>(k) * p.n);
  const int nb = p.nbits[e];
  if (nb < 1 || nb > 4) {
    set_device_error(kDevBadBits);
    return;
  }
  const int eps = 32 / nb;
  const uint32_t w = static_cast<uint32_t>(p.wq[static_cast<int64_t>(p.wq_strides[e]) + static_cast<int64_t>(k / eps) * p.n + n]);
  const uint32_t q = (w >> ((k % eps) * nb)) & ((1u << nb) - 1u);
  const int64_t zi = static_cast<int64_t>(p.zs_strides[e]) + static_cast<int64_t>(k / p.group_size) * p.n + n;
  out[i] = dq_scalar(q, __ushort_as_half(p.scales[zi]), __ushort_as_half(p.zeros[zi]));
}

cudaError_t launch_dequant_expert(const ProjDev& p, int expert, uint16_t* out, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(p.k) * p.n;
  if (total == 0) return cudaSuccess;
  k_dequant_expert<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(p, expert, reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ router (CUDA cores)
// logits[t, e] = sum_d x[t, d] * gate[e, d], fp32 accumulation; one warp per (t, e).
// Used for small token counts; large ones go through the tensor-core dense GEMM.
__global__ void k_router_simt(const __half* __restrict__ x, int64_t T, const __half* __restrict__ gate, int E, int D,
                              int fp32_out, void* __restrict__ logits) {
  const int64_t wid = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= T * E) return;
  const int64_t t = wid / E;
  const int e = static_cast<int>(wid - t * E);
  const __half* xr = x + t * D;
  const __half* gr = gate + static_cast<int64_t>(e) * D;
  float acc = 0.f;
  for (int d = lane * 8; d < D; d += 256) {
    if (d + 8 <= D) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + d);
      const uint4 gv = *reinterpret_cast<const uint4*>(gr + d);
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
      const __half2* gh = reinterpret_cast<const __half2*>(&gv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = __half22float2(xh[j]);
        const float2 b = __half22float2(gh[j]);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    } else {
      for (int j = d; j < D; ++j) acc = fmaf(__half2float(xr[j]), __half2float(gr[j]), acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    if (fp32_out)
      static_cast<float*>(logits)[t * E + e] = acc;
    else
      static_cast<__half*>(logits)[t * E + e] = __float2half_rn(acc);
  }
}

cudaError_t launch_router_simt(const uint16_t* x, int64_t T, const uint16_t* gate, int E, int D, bool fp32_out,
                               void* logits, cudaStream_t stream) {
  const int64_t warps = T * E;
  if (warps == 0) return cudaSuccess;
  k_router_simt<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __half*>(x), T, reinterpret_cast<const __half*>(gate), E, D, fp32_out ? 1 : 0, logits);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ softmax + top-k
// One warp per token; E <= 256 (8 values per lane). Softmax in fp32 with expf, top-k
// by repeated warp arg-max (larger value first, lower expert id on ties),
// renormalisation in fp32, then the fp16 cast (moe_block.py:792-797).
// fp16_softmax: probabilities are rounded to fp16 first and the renormalisation is
// done on fp16 tensors (Mixtral's one-token router, moe_block.py:280-283).
constexpr int kMaxExperts = 256;

__global__ void k_topk(const void* __restrict__ logits, int logits_fp32, int64_t T, int E, int k, int norm,
                       int fp16_softmax, int32_t* __restrict__ topk_idx, __half* __restrict__ topk_w) {
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v[kMaxExperts / 32];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i) {
    const int e = i * 32 + lane;
    float l = -FLT_MAX;
    if (e < E) {
      l = logits_fp32 ? static_cast<const float*>(logits)[t * E + e]
                      : __half2float(static_cast<const __half*>(logits)[t * E + e]);
    }
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
    if (fp16_softmax && e < E) pr = __half2float(__float2half_rn(pr));
    v[i] = pr;
  }
  float wsel[16];
  int isel[16];
  float wsum = 0.f;
  // Selection key: NaN ranks above every number (torch.topk's order); taken
  // entries are -3, so the arg-max is always a valid, untaken expert id.
  auto key = [](float a) { return (a != a) ? FLT_MAX : a; };
  for (int j = 0; j < k; ++j) {
    float best = -FLT_MAX, bestv = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      const int e = i * 32 + lane;
      if (e < E && v[i] != -3.f && (key(v[i]) > best || (key(v[i]) == best && e < bi))) {
        best = key(v[i]);
        bestv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const float ov = __shfl_xor_sync(0xffffffffu, bestv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bestv = ov;
        bi = oi;
      }
    }
    best = bestv;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i)
      if (i * 32 + lane == bi) v[i] = -3.f;
    wsel[j] = best;
    isel[j] = bi;
    wsum += best;
  }
  if (lane == 0) {
    if (fp16_softmax) wsum = __half2float(__float2half_rn(wsum));
    for (int j = 0; j < k; ++j) {
      float w = wsel[j];
      if (norm) w = w / wsum;
      topk_idx[t * k + j] = isel[j];
      topk_w[t * k + j] = __float2half_rn(w);
    }
  }
}

cudaError_t launch_topk(const void* logits, bool logits_fp32, int64_t T, int E, int k, bool norm, bool fp16_softmax,
                        int32_t* topk_idx, uint16_t* topk_w, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  k_topk<<<static_cast<unsigned>((T * 32 + 255) / 256), 256, 0, stream>>>(
      logits, logits_fp32 ? 1 : 0, T, E, k, norm ? 1 : 0, fp16_softmax ? 1 : 0, topk_idx,
      reinterpret_cast<__half*>(topk_w));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ dispatch
// counts[e] = #slots routed to e; seg e covers rows [start_e, start_e + counts[e]) of
// the permuted activations; every (t, j) slot gets a row. Rows within a segment are
// in arrival order, which does not affect any result: each row is computed alone
// and the combine visits a token's experts in ascending id.
__global__ void k_count(const int32_t* __restrict__ topk_idx, int64_t P, int E, int32_t* __restrict__ counts) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= P) return;
  const int e = topk_idx[i];
  if (e < 0 || e >= E) {
    set_device_error(kDevBadExpert);
    return;
  }
  atomicAdd(&counts[e], 1);
}

// Single block: exclusive scans over experts (E <= 1024).
__global__ void k_scan_segs(const int32_t* __restrict__ counts, int E, int nt, Seg* __restrict__ segs,
                            int32_t* __restrict__ tile_prefix, int32_t* __restrict__ cursor) {
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

// One warp per slot: claim a row, record it, copy the token's activation row.
// A slot whose expert id is out of range (k_count already recorded kDevBadExpert)
// gets no row and slot_pos -1, which the combine skips.
__global__ void k_scatter(const int32_t* __restrict__ topk_idx, const __half* __restrict__ topk_w,
                          const __half* __restrict__ x, int64_t P, int k, int E, int D, int32_t* __restrict__ cursor,
                          int32_t* __restrict__ slot_pos, __half* __restrict__ w_perm, __half* __restrict__ x_perm) {
  const int64_t slot = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (slot >= P) return;
  const int e = topk_idx[slot];
  if (e < 0 || e >= E) {
    if (lane == 0) slot_pos[slot] = -1;
    return;
  }
  int pos = 0;
  if (lane == 0) {
    pos = atomicAdd(&cursor[e], 1);
    slot_pos[slot] = pos;
    w_perm[pos] = topk_w[slot];
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  const int64_t t = slot / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<int64_t>(pos) * D);
  for (int i = lane; i < D / 8; i += 32) dst[i] = src[i];
}

cudaError_t launch_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t T, int k,
                            int E, int D, int nt, int32_t* counts, int32_t* cursor, Seg* segs, int32_t* tile_prefix,
                            int32_t* slot_pos, uint16_t* w_perm, uint16_t* x_perm, cudaStream_t stream) {
  const int64_t P = T * k;
  cudaError_t err = cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream);
  if (err != cudaSuccess) return err;
  if (P > 0) {
    k_count<<<static_cast<unsigned>((P + 255) / 256), 256, 0, stream>>>(topk_idx, P, E, counts);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  k_scan_segs<<<1, 1024, 0, stream>>>(counts, E, nt, segs, tile_prefix, cursor);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if (P > 0) {
    k_scatter<<<static_cast<unsigned>((P * 32 + 255) / 256), 256, 0, stream>>>(
        topk_idx, reinterpret_cast<const __half*>(topk_w), reinterpret_cast<const __half*>(x), P, k, E, D, cursor,
        slot_pos, reinterpret_cast<__half*>(w_perm), reinterpret_cast<__half*>(x_perm));
    err = cudaGetLastError();
  }
  return err;
}

// One segment per index of dequant_group_gemm: all `m` rows of x, outputs stacked.
// An index outside [0, num_experts) gets an empty segment (and kDevBadExpert), so
// no kernel ever reads that expert's metadata.
__global__ void k_index_segs(const int32_t* __restrict__ indices, int A, int num_experts, int64_t m, int nt,
                             Seg* __restrict__ segs, int32_t* __restrict__ tile_prefix) {
  __shared__ int s_tiles[1024];
  const int a = threadIdx.x;
  int tiles = 0;
  if (a < A) {
    const int e = indices != nullptr ? indices[a] : a;
    const bool ok = e >= 0 && e < num_experts;
    if (!ok) set_device_error(kDevBadExpert);
    segs[a] = make_int4(ok ? e : 0, 0, static_cast<int>(a * m), ok ? static_cast<int>(m) : 0);
    tiles = ok ? static_cast<int>((m + nt - 1) / nt) : 0;
  }
  s_tiles[a] = tiles;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int v = (a >= off) ? s_tiles[a - off] : 0;
    __syncthreads();
    s_tiles[a] += v;
    __syncthreads();
  }
  if (a < A) tile_prefix[a] = s_tiles[a] - tiles;
  if (a == A - 1) tile_prefix[A] = s_tiles[a];
}

cudaError_t launch_build_index_segs(const int32_t* indices, int num_indices, int num_experts, int64_t m, int nt,
                                    Seg* segs, int32_t* tile_prefix, cudaStream_t stream) {
  if (num_indices <= 0 || num_indices > 1024) return cudaErrorInvalidValue;
  k_index_segs<<<1, 1024, 0, stream>>>(indices, num_indices, num_experts, m, nt, segs, tile_prefix);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ combine
// out[t] = ((0 + y_{e1}) + y_{e2}) + ... over the token's experts in ascending id,
// every partial sum rounded to fp16: the fp16 index_add_ of forward_n_tokens
// (moe_block.py:799-812). fp32_sum: one fp32 sum, one rounding. `add` (DeepSeek
// shared experts) is added in fp16 afterwards (moe_block.py:575).
__global__ void k_combine(const __half* __restrict__ y_perm, const int32_t* __restrict__ slot_pos,
                          const int32_t* __restrict__ topk_idx, int64_t T, int k, int D, int fp32_sum,
                          const __half* __restrict__ add, const __half* __restrict__ residual,
                          __half* __restrict__ out) {
  const int64_t t = blockIdx.x;
  int order[16];
  int eid[16];
  for (int j = 0; j < k; ++j) {
    order[j] = slot_pos[t * k + j];
    eid[j] = topk_idx[t * k + j];
  }
  for (int a = 1; a < k; ++a) {  // insertion sort by expert id
    int e = eid[a], o = order[a], b = a - 1;
    while (b >= 0 && eid[b] > e) {
      eid[b + 1] = eid[b];
      order[b + 1] = order[b];
      --b;
    }
    eid[b + 1] = e;
    order[b + 1] = o;
  }
  for (int d = threadIdx.x * 2; d < D; d += blockDim.x * 2) {
    float2 acc = make_float2(0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      if (order[j] < 0) continue;  // slot with an invalid expert id (recorded by k_count)
      const float2 y = __half22float2(*reinterpret_cast<const __half2*>(y_perm + static_cast<int64_t>(order[j]) * D + d));
      if (fp32_sum) {
        acc.x += y.x;
        acc.y += y.y;
      } else {
        acc.x = __half2float(__float2half_rn(acc.x + y.x));
        acc.y = __half2float(__float2half_rn(acc.y + y.y));
      }
    }
    __half2 r = __floats2half2_rn(acc.x, acc.y);
    if (add != nullptr) {
      const float2 a2 = __half22float2(*reinterpret_cast<const __half2*>(add + t * D + d));
      const float2 r2 = __half22float2(r);
      r = __floats2half2_rn(r2.x + a2.x, r2.y + a2.y);
    }
    if (residual != nullptr) {
      const float2 a2 = __half22float2(*reinterpret_cast<const __half2*>(residual + t * D + d));
      const float2 r2 = __half22float2(r);
      r = __floats2half2_rn(r2.x + a2.x, r2.y + a2.y);
    }
    *reinterpret_cast<__half2*>(out + t * D + d) = r;
  }
}

cudaError_t launch_combine(const uint16_t* y_perm, const int32_t* slot_pos, const int32_t* topk_idx, int64_t T, int k,
                           int D, bool fp32_sum, const uint16_t* add, const uint16_t* residual, uint16_t* out,
                           cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  k_combine<<<static_cast<unsigned>(T), 256, 0, stream>>>(
      reinterpret_cast<const __half*>(y_perm), slot_pos, topk_idx, T, k, D, fp32_sum ? 1 : 0,
      reinterpret_cast<const __half*>(add), reinterpret_cast<const __half*>(residual), reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

__global__ void k_swiglu_f16(const __half* __restrict__ a, const __half* __restrict__ b, int64_t n,
                             __half* __restrict__ h) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const float x = __half2float(a[i]);
  const __half s = __float2half_rn(x / (1.f + expf(-x)));
  h[i] = __float2half_rn(__half2float(s) * __half2float(b[i]));
}

cudaError_t launch_swiglu_f16(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* h, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_swiglu_f16<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const __half*>(a), reinterpret_cast<const __half*>(b), n, reinterpret_cast<__half*>(h));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ decode GEMV family
// part[s][a][n]: split s of sum_k xin_a[k] * deq(W_{idx[a]})[k, n] in fp32.
// Block = 8 warps over 128 output columns (4 per lane, 16-byte word loads); the
// split's word rows are cut into 8 contiguous runs, one per warp; warps reduce
// through shared memory in a fixed order, so the result is deterministic.
// xin: x_mode 0 -> fp16 x rows; 1 -> fp32 silu(x1)*x3 from fp16 x1/x3 (the fused
// decode down projection, fused_dequant_bmm.py:237-239).
constexpr int kGemvThreads = 256;
constexpr int kGemvCols = 128;

size_t gemv_partial_floats(int rows_a, int n, int k) {
  (void)k;
  return static_cast<size_t>(rows_a) * n;
}

int gemv_default_splits(int k, int n, int rows_a, int num_sms) {
  const int ctas = ((n + kGemvCols - 1) / kGemvCols) * rows_a;
  int s = 1;
  while (ctas * s < 2 * num_sms && s < 16 && (k / (s * 2)) >= 256) s *= 2;
  return s;
}

__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kGemvThreads) k_gemv_partials(ProjDev w, const int32_t* __restrict__ idx,
                                                                const __half* __restrict__ x, int64_t x_stride,
                                                                const __half* __restrict__ x3, float* __restrict__ part,
                                                                int rows_a, int splits) {
  extern __shared__ float s_x[];  // [k range of this split]
  __shared__ float s_red[8][kGemvCols];
  const int slab = blockIdx.x, s = blockIdx.y, a = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = (idx != nullptr) ? idx[a] : a;
  if (e < 0 || e >= w.num_experts) {
    if (threadIdx.x == 0) set_device_error(kDevBadExpert);
    return;
  }
  const int nb = w.nbits[e];
  if (nb < 1 || nb > 4) {
    if (threadIdx.x == 0) set_device_error(kDevBadBits);
    return;
  }
  const int eps = 32 / nb;
  const int K = w.k, N = w.n, g = w.group_size;
  const int rows = (K + eps - 1) / eps;
  const int r0 = static_cast<int>((static_cast<int64_t>(rows) * s) / splits);
  const int r1 = static_cast<int>((static_cast<int64_t>(rows) * (s + 1)) / splits);
  const int k0 = r0 * eps;
  const int k1 = min(r1 * eps, K);
  // stage the split's inputs
  const __half* xa = x + a * x_stride;
  for (int kk = k0 + threadIdx.x; kk < k1; kk += blockDim.x) {
    float v;
    if (x3 == nullptr) {
      v = __half2float(xa[kk]);
    } else {
      const float g1 = __half2float(xa[kk]);
      v = silu_f32(g1) * __half2float(x3[a * x_stride + kk]);
    }
    s_x[kk - k0] = v;
  }
  __syncthreads();
  const int n = slab * kGemvCols + lane * 4;
  const bool col_ok = n < N;  // N % 4 == 0 is required by the host
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int per = (r1 - r0 + 7) / 8;
  const int wr0 = r0 + warp * per, wr1 = min(r1, wr0 + per);
  const int32_t* wbase = w.wq + static_cast<int64_t>(w.wq_strides[e]);
  const int64_t zbase = static_cast<int64_t>(w.zs_strides[e]);
  const uint32_t mask = (1u << nb) - 1u;
  int cur_g = -1;
  __half sh[4], zh[4];
  if (col_ok) {
    for (int r = wr0; r < wr1; ++r) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wbase + static_cast<int64_t>(r) * N + n));
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      for (int j = 0; j < eps; ++j) {
        const int kk = r * eps + j;
        if (kk >= K) break;
        const int gi = kk / g;
        if (gi != cur_g) {
          cur_g = gi;
          const uint2 sv = __ldg(reinterpret_cast<const uint2*>(w.scales + zbase + static_cast<int64_t>(gi) * N + n));
          const uint2 zv = __ldg(reinterpret_cast<const uint2*>(w.zeros + zbase + static_cast<int64_t>(gi) * N + n));
          const __half* sp = reinterpret_cast<const __half*>(&sv);
          const __half* zp = reinterpret_cast<const __half*>(&zv);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            sh[c] = sp[c];
            zh[c] = zp[c];
          }
        }
        const float xv = s_x[kk - k0];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t q = (words[c] >> (j * nb)) & mask;
          acc[c] = fmaf(xv, __half2float(dq_scalar(q, sh[c], zh[c])), acc[c]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) s_red[warp][lane * 4 + c] = acc[c];
  __syncthreads();
  if (threadIdx.x < kGemvCols) {
    const int nn = slab * kGemvCols + threadIdx.x;
    if (nn < N) {
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) v += s_red[i][threadIdx.x];
      part[(static_cast<int64_t>(s) * rows_a + a) * N + nn] = v;
    }
  }
}

cudaError_t launch_gemv_partials(const ProjDev& w, const int32_t* idx, int rows_a, const uint16_t* x, int64_t x_stride,
                                 const uint16_t* x3_for_swiglu, float* part, int splits, cudaStream_t s) {
  if (rows_a == 0) return cudaSuccess;
  // a split covers at most cdiv(rows, splits) + 1 word rows of <= 32 codes each
  const int kmax = (w.k + splits - 1) / splits + 64;
  const size_t smem = sizeof(float) * static_cast<size_t>(kmax);
  dim3 grid((w.n + kGemvCols - 1) / kGemvCols, splits, rows_a);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_partials, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  k_gemv_partials<<<grid, kGemvThreads, smem, s>>>(w, idx, reinterpret_cast<const __half*>(x), x_stride,
                                                    reinterpret_cast<const __half*>(x3_for_swiglu), part, rows_a,
                                                    splits);
  return cudaGetLastError();
}

__global__ void k_gemv_reduce(const float* __restrict__ part, int splits, int64_t count, __half* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= count) return;
  float v = 0.f;
  for (int s = 0; s < splits; ++s) v += part[s * count + i];
  out[i] = __float2half_rn(v);
}

cudaError_t launch_gemv_reduce(const float* part, int splits, int rows_a, int n, uint16_t* out, cudaStream_t s) {
  const int64_t count = static_cast<int64_t>(rows_a) * n;
  if (count == 0) return cudaSuccess;
  k_gemv_reduce<<<static_cast<unsigned>((count + 255) / 256), 256, 0, s>>>(part, splits, count,
                                                                            reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

// out[n] = fp16(sum_a w[a] * x2[a][n]) with fp32 accumulation: the einsum combine
// of forward_one_token (moe_block.py:849-850); then `add` in fp16 (moe_block.py:620).
__global__ void k_decode_combine(const __half* __restrict__ x2, const __half* __restrict__ w, int A, int n,
                                 const __half* __restrict__ add, const __half* __restrict__ residual,
                                 __half* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int a = 0; a < A; ++a) acc = fmaf(__half2float(w[a]), __half2float(x2[static_cast<int64_t>(a) * n + i]), acc);
  __half r = __float2half_rn(acc);
  if (add != nullptr) r = __float2half_rn(__half2float(r) + __half2float(add[i]));
  if (residual != nullptr) r = __float2half_rn(__half2float(r) + __half2float(residual[i]));
  out[i] = r;
}

cudaError_t launch_decode_combine(const uint16_t* x2, const uint16_t* w, int A, int n, const uint16_t* add,
                                  const uint16_t* residual, uint16_t* out, cudaStream_t s) {
  k_decode_combine<<<(n + 255) / 256, 256, 0, s>>>(
      reinterpret_cast<const __half*>(x2), reinterpret_cast<const __half*>(w), A, n,
      reinterpret_cast<const __half*>(add), reinterpret_cast<const __half*>(residual), reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

}  // namespace gemq
