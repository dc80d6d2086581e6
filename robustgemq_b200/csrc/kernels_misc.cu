// Packing, single-expert dequant, index segments and the fp16 SwiGLU helper.
//
// Reference behaviour restated (paths relative to the RobustGEMQ root):
//   pack/unpack   gemq/triton_kernels/utils.py:33-189
//   dequant       gemq/triton_kernels/utils.py:192-212
#include <cuda_fp16.h>

#include <cmath>
#include <mutex>

#include "gemq_common.cuh"
#include "gemq_internal.h"

namespace gemq {

__device__ uint32_t g_device_error = 0;
__device__ uint32_t g_device_abort = 0;

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
  const uint32_t w =
      static_cast<uint32_t>(p.wq[static_cast<int64_t>(p.wq_strides[e]) + static_cast<int64_t>(k / eps) * p.n + n]);
  const uint32_t q = (w >> ((k % eps) * nb)) & ((1u << nb) - 1u);
  const int64_t zi = static_cast<int64_t>(p.zs_strides[e]) + static_cast<int64_t>(k / p.group_size) * p.n + n;
  out[i] = dq_scalar(q, __ushort_as_half(p.scales[zi]), __ushort_as_half(p.zeros[zi]));
}

cudaError_t launch_dequant_expert(const ProjDev& p, int expert, uint16_t* out, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(p.k) * p.n;
  if (total == 0) return cudaSuccess;
  k_dequant_expert<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(p, expert,
                                                                               reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ scale exponents
// Largest fp16 exponent field a scale may have for each bit-width so that s * 2^(24 - o)
// (o the smallest code offset the subnormal form uses) stays finite: b = 1 (o = 8):
// 14; b = 2, 4 (o = 6): 12; b = 3 (o = 5): 11. The field must also be at least 1
// (a normal number). One CTA per expert; any scale outside the range sets *bad.
__device__ unsigned g_scale_check;

__global__ void k_scale_exponents(const ProjDev p, unsigned* bad) {
  const int e = blockIdx.x;
  const int nb = p.nbits[e];
  const int lim = nb == 1 ? 14 : (nb == 2 || nb == 4) ? 12 : nb == 3 ? 11 : 0;
  const int64_t z0 = p.zs_strides[e];
  const int64_t n = static_cast<int64_t>(p.k / p.group_size) * p.n;
  const unsigned short* sc = reinterpret_cast<const unsigned short*>(p.scales);
  bool out = (lim == 0);
  for (int64_t i = threadIdx.x; i < n && !out; i += blockDim.x) {
    const int ex = (sc[z0 + i] >> 10) & 31;
    out = ex < 1 || ex > lim;
  }
  if (out) atomicOr(bad, 1u);
}

cudaError_t scale_exponents_ok(const ProjDev& p, int* ok) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  *ok = 0;
  if (p.num_experts <= 0 || p.group_size <= 0) return cudaSuccess;
  const unsigned zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_scale_check, &zero, sizeof(zero));
  if (e != cudaSuccess) return e;
  unsigned* flag = nullptr;
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&flag), g_scale_check);
  if (e != cudaSuccess) return e;
  k_scale_exponents<<<static_cast<unsigned>(p.num_experts), 256>>>(p, flag);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  unsigned bad = 1;
  e = cudaMemcpyFromSymbol(&bad, g_scale_check, sizeof(bad));  // synchronous
  if (e != cudaSuccess) return e;
  *ok = bad == 0 ? 1 : 0;
  return cudaSuccess;
}

// ------------------------------------------------------------------ index segments
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

// ------------------------------------------------------------------ fp16 SwiGLU
// h = fp16(fp16(silu(a)) * b): ``F.silu(x1) * x3`` on fp16 tensors (moe_block.py:619).
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

// ------------------------------------------------------------------ RMSNorm (model harness)
// y = fp16(w * fp16(x * rsqrt(mean(x^2) + eps))), x in fp32: the RMSNorm of the
// decoder layers around the MoE blocks (transformers' OlmoeRMSNorm, T5-style), one
// launch instead of the six element-wise and reduction kernels of the eager module.
// One CTA per row, 8 fp16 per thread and chunk (n % 8 == 0); the sum of squares is
// reduced in fp32 (warp shuffles, then the warps' sums in order).
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) k_rms_norm(const __half* __restrict__ x, const __half* __restrict__ w,
                                                          int n, float eps, __half* __restrict__ y) {
  const int64_t row = blockIdx.x;
  const uint4* x4 = reinterpret_cast<const uint4*>(x + row * n);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  uint4* y4 = reinterpret_cast<uint4*>(y + row * n);
  const int n8 = n / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n8; i += kNormThreads) {
    const uint4 v = x4[i];
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  __shared__ float s_part[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += s_part[i];
  const float inv = rsqrtf(tot / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n8; i += kNormThreads) {
    const uint4 v = x4[i], wv = w4[i];
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      oh[j] = __hmul2(wh[j], __floats2half2_rn(f.x * inv, f.y * inv));
    }
    y4[i] = o;
  }
}

cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, int64_t rows, int n, float eps, uint16_t* y,
                            cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  k_rms_norm<<<static_cast<unsigned>(rows), kNormThreads, 0, s>>>(
      reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(w), n, eps, reinterpret_cast<__half*>(y));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ Q/K norm + rotary (model harness)
// For one token row of a fused q|k|v projection (row stride ld): qn = RMSNorm(q) and
// kn = RMSNorm(k) with their own weights (as k_rms_norm), then the rotary embedding
// of transformers' apply_rotary_pos_emb on fp16 tensors: out = fp16(fp16(x * cos) +
// fp16(rotate_half(x) * sin)), rotate_half(x)[j] = -x[j + hd/2] for j < hd/2, else
// x[j - hd/2], per head of hd values; cos / sin fp16 [rows, hd]. The normalised rows
// are staged in shared memory (the rotation pairs values of different threads).
// With k_cache (one row only): k and v (the third block of qkv) also go to row
// *cache_len of the caches ([n / hd heads][max_len][hd] fp16), and *cache_len
// advances by one, as a static cache's update does; a position past max_len writes
// nothing and records kDevBadCachePos.
__global__ void __launch_bounds__(kNormThreads) k_qk_norm_rope(const __half* __restrict__ qkv, int64_t ld, int n, int hd,
                                                              const __half* __restrict__ wq, const __half* __restrict__ wk,
                                                              float eps, const __half* __restrict__ cos_t,
                                                              const __half* __restrict__ sin_t, __half* __restrict__ q_out,
                                                              __half* __restrict__ k_out, __half* __restrict__ k_cache,
                                                              __half* __restrict__ v_cache, int max_len,
                                                              int64_t* __restrict__ cache_len) {
  extern __shared__ __align__(16) __half s_qk[];  // [2][n]
  const int64_t row = blockIdx.x;
  const __half* src[2] = {qkv + row * ld, qkv + row * ld + n};
  const __half* wts[2] = {wq, wk};
  const int n8 = n / 8;
  float ss[2] = {0.f, 0.f};
  for (int m = 0; m < 2; ++m) {
    const uint4* x4 = reinterpret_cast<const uint4*>(src[m]);
    for (int i = threadIdx.x; i < n8; i += kNormThreads) {
      const uint4 v = x4[i];
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        ss[m] = fmaf(f.x, f.x, ss[m]);
        ss[m] = fmaf(f.y, f.y, ss[m]);
      }
    }
  }
  __shared__ float s_part[2][kNormThreads / 32];
#pragma unroll
  for (int m = 0; m < 2; ++m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
    if ((threadIdx.x & 31) == 0) s_part[m][threadIdx.x >> 5] = ss[m];
  }
  __syncthreads();
  for (int m = 0; m < 2; ++m) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += s_part[m][i];
    const float inv = rsqrtf(tot / static_cast<float>(n) + eps);
    const uint4* x4 = reinterpret_cast<const uint4*>(src[m]);
    const uint4* w4 = reinterpret_cast<const uint4*>(wts[m]);
    uint4* d4 = reinterpret_cast<uint4*>(s_qk + m * n);
    for (int i = threadIdx.x; i < n8; i += kNormThreads) {
      const uint4 v = x4[i], wv = w4[i];
      const __half2* h = reinterpret_cast<const __half2*>(&v);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        oh[j] = __hmul2(wh[j], __floats2half2_rn(f.x * inv, f.y * inv));
      }
      d4[i] = o;
    }
  }
  int64_t pos = -1;
  if (k_cache != nullptr) {
    pos = *cache_len;
    if (pos < 0 || pos >= max_len) {
      if (threadIdx.x == 0) set_device_error(kDevBadCachePos);
      pos = -1;
    }
  }
  __syncthreads();  // every thread has read the cache length before it advances
  if (k_cache != nullptr && threadIdx.x == 0) *cache_len += 1;
  const int half = hd / 2;
  const __half* c = cos_t + row * hd;
  const __half* sn = sin_t + row * hd;
  for (int m = 0; m < 2; ++m) {
    const __half* xs = s_qk + m * n;
    __half* out = (m == 0 ? q_out : k_out);
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
      const int j = i % hd;
      const __half x = xs[i];
      const __half rot = j < half ? __hneg(xs[i + half]) : xs[i - half];
      // the _rn forms keep each product and the sum rounded on its own, as the
      // three fp16 tensor ops are (no contraction into an fp16 fma)
      const __half r = __hadd_rn(__hmul_rn(x, c[j]), __hmul_rn(rot, sn[j]));
      if (out != nullptr) out[row * n + i] = r;
      if (m == 1 && pos >= 0) k_cache[(static_cast<int64_t>(i / hd) * max_len + pos) * hd + j] = r;
    }
  }
  if (pos >= 0) {
    const __half* v = qkv + row * ld + 2 * n;
    for (int i = threadIdx.x; i < n; i += kNormThreads)
      v_cache[(static_cast<int64_t>(i / hd) * max_len + pos) * hd + i % hd] = v[i];
  }
}

cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t ld, int64_t rows, int n, int hd, const uint16_t* wq,
                                const uint16_t* wk, float eps, const uint16_t* cos_t, const uint16_t* sin_t,
                                uint16_t* q_out, uint16_t* k_out, uint16_t* k_cache, uint16_t* v_cache, int max_len,
                                int64_t* cache_len, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const size_t smem = 2 * static_cast<size_t>(n) * sizeof(__half);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(k_qk_norm_rope, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  k_qk_norm_rope<<<static_cast<unsigned>(rows), kNormThreads, smem, s>>>(
      reinterpret_cast<const __half*>(qkv), ld, n, hd, reinterpret_cast<const __half*>(wq),
      reinterpret_cast<const __half*>(wk), eps, reinterpret_cast<const __half*>(cos_t),
      reinterpret_cast<const __half*>(sin_t), reinterpret_cast<__half*>(q_out), reinterpret_cast<__half*>(k_out),
      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), max_len, cache_len);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ one-token attention (model harness)
// softmax(scale * q K^T) V for one query token of one sequence against the first L =
// *cache_len positions of a static KV cache ([heads][max_len][hd] fp16): the causal
// mask of a one-token decode step, which hides exactly the positions not yet written.
// One CTA per head: each thread takes whole keys (its dot product from 16-byte loads
// of the key, q staged in shared memory as fp32), the scores stay in shared memory,
// the block reduces their maximum and the sum of exp(score - max), and thread d sums
// p_j * v_j[d] in fp32 (loads of eight positions in flight) before one rounding to
// fp16. head_dim % 8 == 0, at most kAttnMaxHd.
constexpr int kAttnThreads = 128;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* s_red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // s_red may still be read by the previous reduction
  if ((threadIdx.x & 31) == 0) s_red[warp] = v;
  __syncthreads();
  float r = s_red[0];
  for (int i = 1; i < kAttnThreads / 32; ++i) r = is_max ? fmaxf(r, s_red[i]) : r + s_red[i];
  return r;
}

constexpr int kAttnMaxHd = 256;

__global__ void __launch_bounds__(kAttnThreads) k_decode_attention(const __half* __restrict__ q,
                                                                  const __half* __restrict__ kc,
                                                                  const __half* __restrict__ vc, int max_len, int hd,
                                                                  const int64_t* __restrict__ cache_len, float scale,
                                                                  __half* __restrict__ out) {
  extern __shared__ float s_sc[];  // [max_len]
  __shared__ float s_red[kAttnThreads / 32];
  __shared__ float s_q[kAttnMaxHd];
  const int h = blockIdx.x;
  const int64_t len = *cache_len;
  const int L = static_cast<int>(len < 0 ? 0 : (len > max_len ? max_len : len));
  const __half* qh = q + static_cast<int64_t>(h) * hd;
  const __half* kh = kc + static_cast<int64_t>(h) * max_len * hd;
  const __half* vh = vc + static_cast<int64_t>(h) * max_len * hd;
  for (int c = threadIdx.x; c < hd; c += kAttnThreads) s_q[c] = __half2float(qh[c]);
  __syncthreads();
  const int hd8 = hd / 8;
  for (int j = threadIdx.x; j < L; j += kAttnThreads) {
    const uint4* k4 = reinterpret_cast<const uint4*>(kh + static_cast<int64_t>(j) * hd);
    float d = 0.f;
#pragma unroll 4
    for (int c = 0; c < hd8; ++c) {
      const uint4 kv = k4[c];
      const __half2* k2 = reinterpret_cast<const __half2*>(&kv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(k2[e]);
        d = fmaf(s_q[8 * c + 2 * e], f.x, d);
        d = fmaf(s_q[8 * c + 2 * e + 1], f.y, d);
      }
    }
    s_sc[j] = d * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = threadIdx.x; j < L; j += kAttnThreads) m = fmaxf(m, s_sc[j]);
  m = block_reduce(m, true, s_red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < L; j += kAttnThreads) {
    const float p = expf(s_sc[j] - m);
    s_sc[j] = p;
    sum += p;
  }
  sum = block_reduce(sum, false, s_red);  // its barriers also publish the p_j
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
    float acc = 0.f;
    int j = 0;
    for (; j + 8 <= L; j += 8) {
      __half v8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v8[u] = vh[static_cast<int64_t>(j + u) * hd + d];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = fmaf(s_sc[j + u], __half2float(v8[u]), acc);
    }
    for (; j < L; ++j) acc = fmaf(s_sc[j], __half2float(vh[static_cast<int64_t>(j) * hd + d]), acc);
    out[static_cast<int64_t>(h) * hd + d] = __float2half_rn(acc * inv);
  }
}

cudaError_t launch_decode_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads,
                                    int max_len, int hd, const int64_t* cache_len, float scale, uint16_t* out,
                                    cudaStream_t s) {
  const size_t smem = static_cast<size_t>(max_len) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(k_decode_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  k_decode_attention<<<static_cast<unsigned>(heads), kAttnThreads, smem, s>>>(
      reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k_cache),
      reinterpret_cast<const __half*>(v_cache), max_len, hd, cache_len, scale, reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

}  // namespace gemq
