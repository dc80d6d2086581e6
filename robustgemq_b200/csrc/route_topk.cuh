// Softmax + top-k of one token's router logits by one warp, shared by the router
// kernels (kernels_route.cu) and the one-token layer kernel (kernels_decode.cu).
// Reference: gemq/inference/moe_block.py:790-797 (fp32 softmax, top-k, optional
// renormalisation), 280-283 (Mixtral one-token: fp16 softmax / top-k / renorm).
#pragma once

#include <cuda_fp16.h>

#include <cfloat>
#include <cstdint>

namespace gemq {

constexpr int kMaxExperts = 256;

// Top-k of one token's probabilities v (slot i of lane l = expert 32 i + l; NV slots
// in use) by rank: a value's rank is the number of values ahead of it in the order
// "larger probability first, lower expert id on ties" (NaN ahead of every number:
// torch.topk's order), so the values of rank < k are the top k, in order. All
// comparisons run at once instead of k rounds of an argmax. The selected weights
// are summed in rank order (the order of the k-round selection), then lane r writes
// the rank-r expert and its (renormalised) weight.
template <int NV>
__device__ __forceinline__ void select_topk(const float (&v)[kMaxExperts / 32], int E, int k, int norm,
                                            int fp16_softmax, int32_t* __restrict__ idx_out,
                                            __half* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  auto key = [](float a) { return (a != a) ? FLT_MAX : a; };
  float m[NV];
  int rank[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    m[i] = key(v[i]);
    rank[i] = 0;
  }
#pragma unroll
  for (int jo = 0; jo < NV; ++jo) {
#pragma unroll 8
    for (int src = 0; src < 32; ++src) {
      const float o = __shfl_sync(0xffffffffu, m[jo], src);
      const int oe = jo * 32 + src;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int e = i * 32 + lane;
        rank[i] += (oe < E && (o > m[i] || (o == m[i] && oe < e))) ? 1 : 0;
      }
    }
  }
  float wsum = 0.f, myw = 0.f;
  int mye = 0;
  for (int r = 0; r < k; ++r) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const unsigned b = __ballot_sync(0xffffffffu, i * 32 + lane < E && rank[i] == r);
      if (b != 0u) {  // warp-uniform
        const int src = __ffs(b) - 1;
        const float val = __shfl_sync(0xffffffffu, v[i], src);
        wsum += val;
        if (lane == r) {
          myw = val;
          mye = i * 32 + src;
        }
        break;
      }
    }
  }
  if (lane < k) {
    if (fp16_softmax) wsum = __half2float(__float2half_rn(wsum));
    idx_out[lane] = mye;
    w_out[lane] = __float2half_rn(norm ? myw / wsum : myw);
  }
}

// Softmax + top-k + optional renormalisation of one token's logits by one warp.
// Softmax in fp32 with expf; selection takes the larger probability first and the
// lower expert id on ties; NaN ranks above every number (torch.topk's order), so
// the selected ids are always valid. fp16_softmax rounds the probabilities, their
// sum and the quotients to fp16 as the fp16 tensors of moe_block.py:280-283 do.
template <typename GetLogit>
__device__ __forceinline__ void topk_warp(GetLogit get, int E, int k, int norm, int fp16_softmax,
                                          int32_t* __restrict__ idx_out, __half* __restrict__ w_out) {
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
    if (fp16_softmax && e < E) pr = __half2float(__float2half_rn(pr));
    v[i] = pr;
  }
  const int nv = (E + 31) / 32;  // value slots per lane in use
  if (nv <= 1) select_topk<1>(v, E, k, norm, fp16_softmax, idx_out, w_out);
  else if (nv <= 2) select_topk<2>(v, E, k, norm, fp16_softmax, idx_out, w_out);
  else if (nv <= 4) select_topk<4>(v, E, k, norm, fp16_softmax, idx_out, w_out);
  else select_topk<8>(v, E, k, norm, fp16_softmax, idx_out, w_out);
}

// Gate logit of one token for expert row `g` (D fp16, D % 8 == 0) by one warp: lane
// l sums chunks l, l + 32, ... of 8 elements in order with fp32 fma, then the lanes'
// sums reduce by xor shuffles. The same order as k_gate_logits, so both give the same
// bits. `xs` holds the token's row as 16-byte chunks (shared memory).
__device__ __forceinline__ float gate_logit_warp(const uint4* xs, const __half* __restrict__ g, int d8, int lane) {
  const uint4* gr = reinterpret_cast<const uint4*>(g);
  float acc = 0.f;
  for (int c = lane; c < d8; c += 32) {
    const uint4 gv = __ldg(gr + c);
    const __half2* gh = reinterpret_cast<const __half2*>(&gv);
    const uint4 xv = xs[c];
    const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 gg = __half22float2(gh[j]);
      const float2 a = __half22float2(xh[j]);
      acc = fmaf(a.x, gg.x, acc);
      acc = fmaf(a.y, gg.y, acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace gemq
