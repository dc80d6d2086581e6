// Internal declarations shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/gemq_b200.h"

namespace gemq {

// A contiguous run of activation rows that all use one expert:
// x = expert id, y = first activation row, z = first output row, w = row count.
using Seg = int4;

// Token-tile widths the tensor-core GEMM is instantiated for (UMMA N).
constexpr int kNtSmall = 32;
constexpr int kNtLarge = 128;

enum class GemmMode : int {
  kSwiGLU = 0,       // dual A (w1, w3): h = fp16(fp16(silu(fp16 g)) * fp16 u)   (moe_block.py:774-775)
  kRouteWeight = 1,  // y = fp16(fp16(acc) * w_row)                             (moe_block.py:811)
  kStoreF16 = 2,     // out = fp16(acc)                                          (dequant_group_gemm.py:138)
  kDenseF16 = 3,     // dense fp16 A (router gate) -> fp16 out                   (moe_block.py:790)
  kDenseF32 = 4,     // dense fp16 A (router gate) -> fp32 out                   (moe_block.py:549)
};

struct ProjDev {
  const int32_t* wq;
  const uint16_t* scales;
  const uint16_t* zeros;
  const int32_t* nbits;
  const int32_t* wq_strides;
  const int32_t* zs_strides;
  int64_t wq_rows;
  int num_experts, k, n, group_size;
};

// Everything a grouped-GEMM launch needs besides tensor maps.
struct GemmArgs {
  GemmMode mode;
  ProjDev w0;          // w1 (SwiGLU) or the single weight
  ProjDev w1;          // w3 for SwiGLU (nbits/strides of w0 are used, as the reference does at decode)
  const uint16_t* dense_a;  // kDense*: fp16 [n, k] row-major
  const uint16_t* act;      // fp16 activations [act_rows, k]
  int64_t act_rows;
  const Seg* segs;          // device [num_segs]
  const int32_t* tile_prefix;  // device [num_segs + 1], tiles of `nt` rows
  int num_segs;
  int nt;                   // token tile
  void* out;                // fp16 (or fp32) rows of length out_ld
  int64_t out_ld;
  int out_cols;             // valid output columns (n)
  const uint16_t* row_weight;  // kRouteWeight: fp16 per output row
  int num_sms;
};

// Tensor-core (tcgen05) grouped GEMM; returns cudaErrorNotSupported for shapes it
// does not handle (k % 64, n % 128, group % 64), for which callers use the SIMT GEMM.
bool tc_gemm_supported(const GemmArgs& a);
cudaError_t launch_tc_gemm(const GemmArgs& a, cudaStream_t stream);
cudaError_t launch_simt_gemm(const GemmArgs& a, cudaStream_t stream);

// Builds segments + tile prefix for a dequant_group_gemm call (one segment per index).
cudaError_t launch_build_index_segs(const int32_t* indices, int num_indices, int num_experts, int64_t m, int nt,
                                    Seg* segs, int32_t* tile_prefix, cudaStream_t stream);

// Routing / dispatch / combine.
cudaError_t launch_router_simt(const uint16_t* x, int64_t T, const uint16_t* gate, int E, int D, bool fp32_out,
                               void* logits, cudaStream_t stream);
cudaError_t launch_topk(const void* logits, bool logits_fp32, int64_t T, int E, int k, bool norm, bool fp16_softmax,
                        int32_t* topk_idx, uint16_t* topk_w, cudaStream_t stream);
cudaError_t launch_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t T, int k,
                            int E, int D, int nt, int32_t* counts, int32_t* cursor, Seg* segs, int32_t* tile_prefix,
                            int32_t* slot_pos, uint16_t* w_perm, uint16_t* x_perm, cudaStream_t stream);
cudaError_t launch_combine(const uint16_t* y_perm, const int32_t* slot_pos, const int32_t* topk_idx, int64_t T, int k,
                           int D, bool fp32_sum, const uint16_t* add, const uint16_t* residual, uint16_t* out,
                           cudaStream_t stream);

// Packing / dequant.
cudaError_t launch_pack(const uint8_t* codes, int64_t rows, int64_t cols, int nbits, int32_t* out, cudaStream_t s);
cudaError_t launch_unpack(const int32_t* packed, int64_t rows, int64_t pcols, int64_t ocols, int nbits, uint8_t* out,
                          cudaStream_t s);
cudaError_t launch_dequant_expert(const ProjDev& p, int expert, uint16_t* out, cudaStream_t s);

// Decode GEMV family (CUDA cores, deterministic split-K).
struct GemvPlan {
  int splits;  // K splits
};
size_t gemv_partial_floats(int rows_a, int n, int k);
// part[s][a][n] = sum over split s of x_a . deq(W_{idx[a]})[:, n]; x given as fp16 rows
// (x_stride 0 = the same x for every a), or as silu(x1)*x3 from fp16 x1/x3 (down).
cudaError_t launch_gemv_partials(const ProjDev& w, const int32_t* idx, int rows_a, const uint16_t* x, int64_t x_stride,
                                 const uint16_t* x3_for_swiglu, float* part, int splits, cudaStream_t s);
// out[a][n] = fp16(sum_s part[s][a][n]); optional second set for dual (x1,x3).
cudaError_t launch_gemv_reduce(const float* part, int splits, int rows_a, int n, uint16_t* out, cudaStream_t s);
// out[n] = fp16(sum_a w[a] * fp16 x2[a][n]) in fp32 (+ optional fp16 add).
cudaError_t launch_decode_combine(const uint16_t* x2, const uint16_t* w, int A, int n, const uint16_t* add,
                                  const uint16_t* residual, uint16_t* out, cudaStream_t s);
// fp16 SiLU*mul with the reference's fp16 rounding: h = fp16(fp16(silu(a)) * b).
cudaError_t launch_swiglu_f16(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* h, cudaStream_t s);
int gemv_default_splits(int k, int n, int rows_a, int num_sms);

int device_sm_count();
void set_error(const std::string& msg);

}  // namespace gemq
