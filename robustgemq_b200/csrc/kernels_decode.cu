// Decode GEMV family (CUDA cores, deterministic split-K), the one-token path of
// forward_one_token (moe_block.py:817-853) and the batch-1 dequant GEMV of
// dequant_gemv.py:118-156.
//
// part[mat][s][a][n] = split s of sum_k xin_a[k] * deq(W_{mat, idx[a]})[k, n] in fp32.
// A block covers 128 output features (4 per lane, 16-byte word loads) of one
// (matrix, row a) and one K split; its word rows are cut into 8 contiguous runs,
// one per warp, reduced through shared memory in a fixed order, so every result is
// bit-reproducible (the reference's fp16 atomics are not, dequant_gemv.py:115).
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

__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kGemvThreads) k_gemv(ProjDev w0, ProjDev w1, const int32_t* __restrict__ idx,
                                                       int rows_a, GemvSrc src, float* __restrict__ part, int splits) {
  extern __shared__ float s_x[];  // inputs of this split's k range
  __shared__ float s_red[8][kGemvCols];
  const int slab = blockIdx.x, s = blockIdx.y;
  const int mat = blockIdx.z / rows_a, a = blockIdx.z - mat * rows_a;
  const ProjDev& w = (mat == 0) ? w0 : w1;
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
  for (int kk = k0 + threadIdx.x; kk < k1; kk += blockDim.x) {
    float v;
    if (src.mode == kGemvX) {
      v = __half2float(src.x[a * src.x_stride + kk]);
    } else if (src.mode == kGemvSwiGLU) {
      v = silu_f32(__half2float(src.x[a * src.x_stride + kk])) * __half2float(src.x3[a * src.x_stride + kk]);
    } else {
      const int64_t mstride = static_cast<int64_t>(src.part_splits) * src.part_rows * src.part_n;
      float g1 = 0.f, g3 = 0.f;
      for (int q = 0; q < src.part_splits; ++q) {
        const int64_t off = (static_cast<int64_t>(q) * src.part_rows + a) * src.part_n + kk;
        g1 += src.part[off];
        g3 += src.part[mstride + off];
      }
      const float x1 = __half2float(__float2half_rn(g1));
      const float x3 = __half2float(__float2half_rn(g3));
      if (src.mode == kGemvPartF32) {
        v = silu_f32(x1) * x3;
      } else {
        v = __half2float(__float2half_rn(__half2float(__float2half_rn(silu_f32(x1))) * x3));
      }
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
      part[((static_cast<int64_t>(mat) * splits + s) * rows_a + a) * N + nn] = v;
    }
  }
}

__global__ void k_gemv_reduce(const float* __restrict__ part, int splits, int64_t count, __half* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= count) return;
  float v = 0.f;
  for (int s = 0; s < splits; ++s) v += part[s * count + i];
  out[i] = __float2half_rn(v);
}

// out[n] = fp16(sum_a w[a] * x2[a][n]) with x2 = fp16(sum_s part[s][a][n]): the fp32
// einsum combine of forward_one_token (moe_block.py:849-850); then the shared
// experts' fp16 output (moe_block.py:620) and an optional residual, each in fp16.
__global__ void k_decode_combine(const float* __restrict__ part, int splits, int A, int n, const __half* __restrict__ w,
                                 const float* __restrict__ shared_part, int shared_splits,
                                 const __half* __restrict__ residual, __half* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int a = 0; a < A; ++a) {
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += part[(static_cast<int64_t>(s) * A + a) * n + i];
    acc = fmaf(__half2float(w[a]), __half2float(__float2half_rn(v)), acc);
  }
  __half r = __float2half_rn(acc);
  if (shared_part != nullptr) {
    float v = 0.f;
    for (int s = 0; s < shared_splits; ++s) v += shared_part[static_cast<int64_t>(s) * n + i];
    r = __float2half_rn(__half2float(r) + __half2float(__float2half_rn(v)));
  }
  if (residual != nullptr) r = __float2half_rn(__half2float(r) + __half2float(residual[i]));
  out[i] = r;
}

}  // namespace

int gemv_default_splits(int k, int n, int rows_a, int num_sms) {
  const int ctas = ((n + kGemvCols - 1) / kGemvCols) * rows_a;
  int s = 1;
  while (ctas * s < 2 * num_sms && s < 16 && (k / (s * 2)) >= 256) s *= 2;
  return s;
}

cudaError_t launch_gemv(const ProjDev& w0, const ProjDev* w1, const int32_t* idx, int rows_a, const GemvSrc& src,
                        float* part, int splits, cudaStream_t s) {
  if (rows_a == 0) return cudaSuccess;
  const int nmat = (w1 != nullptr) ? 2 : 1;
  // a split covers at most cdiv(rows, splits) + 1 word rows of <= 32 codes each
  const size_t smem = sizeof(float) * static_cast<size_t>((w0.k + splits - 1) / splits + 64);
  static int smem_set = 48 * 1024;
  if (static_cast<int>(smem) > smem_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    smem_set = static_cast<int>(smem);
  }
  dim3 grid((w0.n + kGemvCols - 1) / kGemvCols, splits, nmat * rows_a);
  k_gemv<<<grid, kGemvThreads, smem, s>>>(w0, w1 != nullptr ? *w1 : w0, idx, rows_a, src, part, splits);
  return cudaGetLastError();
}

cudaError_t launch_gemv_reduce(const float* part, int splits, int rows_a, int n, uint16_t* out, cudaStream_t s) {
  const int64_t count = static_cast<int64_t>(rows_a) * n;
  if (count == 0) return cudaSuccess;
  k_gemv_reduce<<<static_cast<unsigned>((count + 255) / 256), 256, 0, s>>>(part, splits, count,
                                                                            reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

cudaError_t launch_decode_combine(const float* part, int splits, int A, int n, const uint16_t* w,
                                  const float* shared_part, int shared_splits, const uint16_t* residual, uint16_t* out,
                                  cudaStream_t s) {
  k_decode_combine<<<(n + 255) / 256, 256, 0, s>>>(part, splits, A, n, reinterpret_cast<const __half*>(w), shared_part,
                                                    shared_splits, reinterpret_cast<const __half*>(residual),
                                                    reinterpret_cast<__half*>(out));
  return cudaGetLastError();
}

}  // namespace gemq
