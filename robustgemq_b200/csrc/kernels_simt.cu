// CUDA-core grouped dequant GEMM: the generic path for shapes the tensor-core kernel
// does not take (k % 64, n % 128 or group % 64 non-zero) and a second, independent
// implementation the tests cross-check the tensor-core kernel against. Same
// segment/tile contract and epilogue rounding as kernels_tc.cu; tiles of 32 rows x
// 64 features, fp32 accumulation, bit-exact fp16 dequant in shared memory.
#include "gemq_common.cuh"
#include "gemq_internal.h"

namespace gemq {

namespace {

constexpr int kTM = 32;   // rows (tokens) per tile; segments must be built with nt == 32
constexpr int kTN = 64;   // features per tile
constexpr int kTK = 32;
constexpr int kThreadsS = 256;

__device__ __forceinline__ float silu_ref_s(float x) { return x / (1.f + expf(-x)); }

__device__ __forceinline__ __half deq_at(const ProjDev& w, int e, int nb, int k, int n) {
  const int eps = 32 / nb;
  const uint32_t word =
      static_cast<uint32_t>(w.wq[static_cast<int64_t>(w.wq_strides[e]) + static_cast<int64_t>(k / eps) * w.n + n]);
  const uint32_t q = (word >> ((k % eps) * nb)) & ((1u << nb) - 1u);
  const int64_t zi = static_cast<int64_t>(w.zs_strides[e]) + static_cast<int64_t>(k / w.group_size) * w.n + n;
  return dq_scalar(q, __ushort_as_half(w.scales[zi]), __ushort_as_half(w.zeros[zi]));
}

__global__ void __launch_bounds__(kThreadsS) k_moe_simt(GemmArgs a) {
  __shared__ __half sA[kTM][kTK + 2];
  __shared__ __half sB[2][kTK][kTN + 2];
  const bool dense = (a.mode == GemmMode::kDenseF16 || a.mode == GemmMode::kDenseF32);
  const int mats = (a.mode == GemmMode::kSwiGLU) ? 2 : 1;
  const int N = a.w0.n, K = a.w0.k;
  const int n_tiles = (N + kTN - 1) / kTN;
  const int total = a.tile_prefix[a.num_segs] * n_tiles;
  const int tr = (threadIdx.x / 16) * 2;  // 2 rows
  const int tc = (threadIdx.x % 16) * 4;  // 4 cols
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const int t = w / n_tiles, i = w - t * n_tiles;
    int lo = 0, hi = a.num_segs;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (a.tile_prefix[mid] <= t) lo = mid; else hi = mid;
    }
    const Seg sg = a.segs[lo];
    const int j = t - a.tile_prefix[lo];
    const int e = sg.x;
    const int act_row = sg.y + j * kTM, out_row = sg.z + j * kTM;
    const int rows = min(kTM, sg.w - j * kTM);
    const int n0 = i * kTN;
    const int nb = dense ? 0 : a.w0.nbits[e];
    if (!dense && (nb < 1 || nb > 4)) {
      if (threadIdx.x == 0) set_device_error(kDevBadBits);
      continue;
    }
    float acc[2][2][4] = {};
    for (int k0 = 0; k0 < K; k0 += kTK) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kTM * kTK; idx += kThreadsS) {
        const int r = idx / kTK, c = idx % kTK;
        __half v = __float2half(0.f);
        if (r < rows && k0 + c < K) v = __ushort_as_half(a.act[static_cast<int64_t>(act_row + r) * K + k0 + c]);
        sA[r][c] = v;
      }
      for (int m = 0; m < mats; ++m) {
        const ProjDev& wp = (m == 0) ? a.w0 : a.w1;
        for (int idx = threadIdx.x; idx < kTK * kTN; idx += kThreadsS) {
          const int kk = idx / kTN, nn = idx % kTN;
          __half v = __float2half(0.f);
          if (k0 + kk < K && n0 + nn < N) {
            if (dense)
              v = __ushort_as_half(a.dense_a[static_cast<int64_t>(n0 + nn) * K + k0 + kk]);
            else
              v = deq_at(wp, e, nb, k0 + kk, n0 + nn);
          }
          sB[m][kk][nn] = v;
        }
      }
      __syncthreads();
      for (int kk = 0; kk < kTK; ++kk) {
        const float x0 = __half2float(sA[tr][kk]);
        const float x1 = __half2float(sA[tr + 1][kk]);
        for (int m = 0; m < mats; ++m) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float b = __half2float(sB[m][kk][tc + c]);
            acc[m][0][c] = fmaf(x0, b, acc[m][0][c]);
            acc[m][1][c] = fmaf(x1, b, acc[m][1][c]);
          }
        }
      }
    }
    for (int r = 0; r < 2; ++r) {
      if (tr + r >= rows) continue;
      const int64_t row = out_row + tr + r;
      for (int c = 0; c < 4; ++c) {
        const int col = n0 + tc + c;
        if (col >= N) continue;
        const float a0 = acc[0][r][c];
        switch (a.mode) {
          case GemmMode::kSwiGLU: {
            const float x1 = __half2float(__float2half_rn(a0));
            const float x3 = __half2float(__float2half_rn(acc[1][r][c]));
            const float sl = __half2float(__float2half_rn(silu_ref_s(x1)));
            static_cast<__half*>(a.out)[row * a.out_ld + col] = __float2half_rn(sl * x3);
            break;
          }
          case GemmMode::kRouteWeight: {
            const float y = __half2float(__float2half_rn(a0));
            const float wv = __half2float(__ushort_as_half(a.row_weight[row]));
            static_cast<__half*>(a.out)[row * a.out_ld + col] = __float2half_rn(y * wv);
            break;
          }
          case GemmMode::kDenseF32:
            static_cast<float*>(a.out)[row * a.out_ld + col] = a0;
            break;
          default:
            static_cast<__half*>(a.out)[row * a.out_ld + col] = __float2half_rn(a0);
            break;
        }
      }
    }
  }
}

}  // namespace

cudaError_t launch_simt_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.nt != kTM) return cudaErrorInvalidValue;
  k_moe_simt<<<a.num_sms * 4, kThreadsS, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace gemq
