// Internal declarations shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/gemq_b200.h"

namespace gemq {

// Launches `kernel` with programmatic stream serialization; the kernel calls
// grid_dep_wait() before it reads or writes global memory that other kernels use.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dep(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Devices whose raised shared-memory limits are remembered (a process on a larger
// machine still works: beyond this the limit is set on every call).
constexpr int kMaxDevices = 64;

// Raises `kernel`'s dynamic shared-memory limit to at least `bytes` on the current
// device. A limit set with cudaFuncSetAttribute belongs to the device that is current
// when it is set, so the largest size set so far is kept per device in `done`, and a
// process that drives several GPUs raises the limit on each of them. Sets are
// serialised, so the limit only grows. Call outside stream capture; once a device's
// limit covers `bytes` the call only reads an atomic.
template <typename... KArgs>
inline cudaError_t raise_smem_limit(void (*kernel)(KArgs...), size_t bytes, std::atomic<size_t> (&done)[kMaxDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kMaxDevices;
  if (tracked && done[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  static std::mutex m;
  std::lock_guard<std::mutex> lock(m);
  if (tracked && done[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess && tracked) done[dev].store(bytes, std::memory_order_release);
  return e;
}

// A contiguous run of activation rows that all use one expert:
// x = expert id, y = first activation row, z = first output row, w = row count.
using Seg = int4;

// Token-tile widths the tensor-core GEMM is instantiated for (UMMA N).
constexpr int kNtTiny = 16;  // decode GEMM, batches of at most 16 tokens (16 rows per expert at most)
constexpr int kNtSmall = 32;
constexpr int kNtMid = 64;   // tensor-memory dequant GEMM, prefill (more than 48 rows per expert)
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
  int sub_ok;  // every scale fits the tensor-memory GEMM's subnormal dequant (scale_exponents_ok)
};

// Everything a grouped-GEMM launch needs besides tensor maps.
struct GemmArgs {
  GemmMode mode;
  ProjDev w0;               // w1 (SwiGLU) or the single weight
  ProjDev w1;               // w3 for SwiGLU
  const uint16_t* dense_a;  // kDense*: fp16 [n, k] row-major
  const uint16_t* act;      // fp16 activations [act_rows, k]
  int64_t act_rows;
  const Seg* segs;             // device [num_segs]
  const int32_t* tile_prefix;  // device [num_segs + 1], tiles of `nt` rows
  int num_segs;
  int nt;                      // token tile
  void* out;                   // fp16 (or fp32) rows of length out_ld
  int64_t out_ld;
  int out_cols;                // valid output columns (n)
  const uint16_t* row_weight;  // kRouteWeight: fp16 per output row
  int num_sms;
  const int32_t* perm_out_nbits;  // decode GEMM, kSwiGLU: store h in the slot order of these bit-widths
  // decode GEMM, chained gate/up -> down of one forward (zeroed per forward by the
  // dispatch): per token tile, gate/up epilogue warps done; the down launch waits
  // for chain_target of them per tile
  int32_t* chain_done;
  int chain_target;
};

// Tensor-core (tcgen05) grouped GEMM; cudaErrorNotSupported for shapes it does not
// handle (k % 64, n % 128, group % 64), for which callers use the CUDA-core GEMM.
bool tc_gemm_supported(const GemmArgs& a);
cudaError_t launch_tc_gemm(const GemmArgs& a, cudaStream_t stream);
cudaError_t launch_simt_gemm(const GemmArgs& a, cudaStream_t stream);

// 1 when every scale of the projection is a normal fp16 number small enough that
// s * 2^(24 - o) stays finite for its expert's bit-width (b = 1: s < 1; 2, 4: s < 1/4;
// 3: s < 1/8): the condition of the subnormal dequant form. Synchronous (layer
// creation); uses a device word of the library, serialised by a host mutex.
cudaError_t scale_exponents_ok(const ProjDev& p, int* ok);

// Tensor-core GEMM with the dequantised weights in tensor memory (token tiles of
// 16 / 32 for decode batches, 64 for prefill; kernels_tcd.cu). Its activations are stored in the slot order of
// kperm.cuh for the expert's bit-width: dispatch with perm_nbits, and the gate/up
// launch's perm_out_nbits for the down projection.
bool tcd_gemm_supported(const GemmArgs& a);
cudaError_t launch_tcd_gemm(const GemmArgs& a, cudaStream_t stream);
int kperm_source_column(int nb, int k);

// One segment per index of dequant_group_gemm (invalid indices -> empty segments).
cudaError_t launch_build_index_segs(const int32_t* indices, int num_indices, int num_experts, int64_t m, int nt,
                                    Seg* segs, int32_t* tile_prefix, cudaStream_t stream);

// Routing / dispatch / combine.
// Gate logits of a small batch over many CTAs (then launch_topk).
cudaError_t launch_gate_logits(const uint16_t* x, int64_t T, int D, const uint16_t* gate, int E, bool fp32_logits,
                               void* logits, cudaStream_t stream);
// n_group > 1: group-limited greedy over n_group equal expert groups, keeping
// topk_group of them; scale multiplies the weights when not renormalising.
cudaError_t launch_topk(const void* logits, bool logits_fp32, int64_t T, int E, int k, bool norm, bool fp16_softmax,
                        int n_group, int topk_group, float scale, int32_t* topk_idx, uint16_t* topk_w,
                        cudaStream_t stream, int32_t* zero_buf = nullptr, int zero_n = 0);
bool small_dispatch_ok(int64_t P, int E);
// Segments of rows grouped as [group][expert] (n = groups * E counts, n <= 1024).
cudaError_t launch_group_segs(const int32_t* counts, int n, int E, int nt, Seg* segs, int32_t* tile_prefix,
                              cudaStream_t stream);
cudaError_t launch_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t T, int k,
                            int E, int D, int nt, int32_t* counts, int32_t* cursor, Seg* segs, int32_t* tile_prefix,
                            int32_t* slot_pos, uint16_t* w_perm, uint16_t* x_perm, const int32_t* perm_nbits,
                            const int32_t* order_nbits, int32_t* zero_buf, int zero_n, cudaStream_t stream);
cudaError_t launch_combine(const uint16_t* y_perm, const int32_t* slot_pos, const int32_t* topk_idx, int64_t T, int k,
                           int D, bool fp32_sum, const uint16_t* add, const uint16_t* residual, uint16_t* out,
                           cudaStream_t stream);

// Packing / dequant.
cudaError_t launch_pack(const uint8_t* codes, int64_t rows, int64_t cols, int nbits, int32_t* out, cudaStream_t s);
cudaError_t launch_unpack(const int32_t* packed, int64_t rows, int64_t pcols, int64_t ocols, int nbits, uint8_t* out,
                          cudaStream_t s);
cudaError_t launch_dequant_expert(const ProjDev& p, int expert, uint16_t* out, cudaStream_t s);
cudaError_t launch_swiglu_f16(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* h, cudaStream_t s);
cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, int64_t rows, int n, float eps, uint16_t* y,
                            cudaStream_t s);
cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t ld, int64_t rows, int n, int hd, const uint16_t* wq,
                                const uint16_t* wk, float eps, const uint16_t* cos_t, const uint16_t* sin_t,
                                uint16_t* q_out, uint16_t* k_out, uint16_t* k_cache, uint16_t* v_cache, int max_len,
                                int64_t* cache_len, cudaStream_t s);
cudaError_t launch_decode_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads,
                                    int max_len, int hd, const int64_t* cache_len, float scale, uint16_t* out,
                                    cudaStream_t s);

// Decode GEMV family (CUDA cores, deterministic split-K); see kernels_decode.cu.
enum GemvMode : int { kGemvX = 0, kGemvSwiGLU = 1, kGemvPartF32 = 2, kGemvPartF16 = 3 };
struct GemvSrc {
  int mode;
  const __half* x;      // kGemvX / kGemvSwiGLU: fp16 rows (x1 for SwiGLU)
  const __half* x3;     // kGemvSwiGLU: fp16 x3 rows
  int64_t x_stride;     // elements between rows a (0: one row shared by all a)
  const float* part;    // kGemvPart*: up partials [2][part_splits][part_rows][part_n]
  int part_splits, part_rows, part_n;
  // Chained one-token up -> down GEMVs (counters [rows], zeroed by the forward's
  // router): kGemvX adds 1 to done[a] per CTA once its partials are stored and lets
  // the down launch start at once; kGemvPartF32 waits for done_target on its row's
  // counter instead of the grid-completion wait before reading the partials.
  int32_t* done;
  int done_target;
};
// Split-K factor of a GEMV over rows_a rows and nmat matrices. Fewer matrices never
// give fewer splits, so a workspace sized with nmat = 1 also fits nmat = 2.
int gemv_default_splits(int k, int n, int rows_a, int num_sms, int nmat = 1);
// part[mat][s][a][n] for mat in {w0, w1 (optional)}
cudaError_t launch_gemv(const ProjDev& w0, const ProjDev* w1, const int32_t* idx, int rows_a, const GemvSrc& src,
                        float* part, int splits, cudaStream_t s);
// out[a][n] = fp16(sum_s part[s][a][n])
cudaError_t launch_gemv_reduce(const float* part, int splits, int rows_a, int n, uint16_t* out, cudaStream_t s);
// out[n] = fp16(sum_a w[a] * fp16(sum_s part[s][a][n])) (+ fp16 shared, + residual)
cudaError_t launch_decode_combine(const float* part, int splits, int A, int n, const uint16_t* w,
                                  const float* shared_part, int shared_splits, const uint16_t* residual, uint16_t* out,
                                  cudaStream_t s);

int device_sm_count();
void set_error(const std::string& msg);

}  // namespace gemq
