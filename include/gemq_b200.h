/*
 * gemq_b200.h -- C ABI of the B200 (sm_100a) real-quant mixed-bit MoE expert path.
 *
 * Drop-in for the GPU entry points of RobustGEMQ's quantized-MoE module
 * (gemq/inference/moe_block.py and gemq/triton_kernels/*.py). The reference binds
 * these through Python/Triton; here a Python host (robustgemq_b200) binds them with
 * ctypes, passing tensor.data_ptr() values and torch.cuda.current_stream().cuda_stream.
 *
 * Conventions
 *   - Every pointer argument is device memory unless its comment says "host".
 *   - fp16 data is passed as uint16_t bit patterns.
 *   - Every call is asynchronous on `stream` (a cudaStream_t) and returns a status;
 *     the library never aborts, traps or allocates device memory. Scratch space is
 *     passed in by the caller (sizes from the *_workspace_size queries).
 *   - Kernels bound every internal wait; an expired wait is recorded in a device
 *     error word read by gemq_get_device_error().
 *   - A layer handle is thread-compatible, not thread-safe.
 */
#ifndef GEMQ_B200_H
#define GEMQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEMQ_OK 0
#define GEMQ_ERR_INVALID_ARGUMENT 1 /* the reference raises AssertionError/ValueError here */
#define GEMQ_ERR_UNSUPPORTED 2
#define GEMQ_ERR_CUDA 3
#define GEMQ_ERR_WORKSPACE 4

/* Router flavours (moe_block.py:790 fp16 logits; moe_block.py:549,591 fp32 logits). */
#define GEMQ_ROUTER_FP16 0
#define GEMQ_ROUTER_FP32 1

/* gemq_moe_forward flags */
#define GEMQ_FWD_ONE_TOKEN 1u        /* forward_one_token rounding (moe_block.py:817-853); num_tokens == 1 */
#define GEMQ_FWD_GIVEN_ROUTING 2u    /* use topk_idx/topk_w instead of routing */
#define GEMQ_FWD_GIVEN_LOGITS 4u     /* router_logits is an input: skip the gate GEMM */
#define GEMQ_FWD_FP16_SOFTMAX 8u     /* Mixtral one-token router: fp16 softmax/top-k/renorm (moe_block.py:280-283) */
#define GEMQ_FWD_FP32_COMBINE 16u    /* one fp32 sum per token instead of per-expert fp16 rounding */
#define GEMQ_FWD_FORCE_SIMT 32u      /* use the CUDA-core grouped GEMM (cross-checking) */
#define GEMQ_FWD_RESIDUAL 64u        /* out = fp16(x + block(x)): the decoder layer's residual add, fused */
#define GEMQ_FWD_TIME_STAGES 128u    /* record CUDA events around each stage (read with gemq_layer_stage_times) */
#define GEMQ_FWD_SMEM_DEQUANT 256u   /* use the shared-memory dequant GEMM instead of the tensor-memory one (cross-checking) */
#define GEMQ_FWD_PERMUTED_ROWS 512u  /* gemq_moe_experts: rows are in the tensor-memory GEMM's K order (see there) */
#define GEMQ_FWD_NO_CHAIN 1024u      /* start the down GEMM after the gate/up GEMM completes, not on the SMs it
                                        leaves as its token tiles finish (cross-checking) */
#define GEMQ_FWD_TEST_WAIT_EXPIRY 2048u /* testing: the chained down GEMM of a decode batch waits for a tile count
                                        nothing reaches, so its bounded wait expires; the device error word
                                        then reads 11 and this forward's output is undefined */

/* Stage indices reported by gemq_layer_stage_times. */
#define GEMQ_STAGE_ROUTE 0    /* gate GEMM + softmax/top-k */
#define GEMQ_STAGE_DISPATCH 1 /* histogram, scan, permute (n-token path) */
#define GEMQ_STAGE_UP 2       /* gate/up projection with SiLU*mul */
#define GEMQ_STAGE_DOWN 3     /* down projection with routing weight */
#define GEMQ_STAGE_SHARED 4   /* DeepSeek shared experts */
#define GEMQ_STAGE_COMBINE 5  /* per-token combine (+ residual) */
#define GEMQ_NUM_STAGES 6

/*
 * One stacked packed projection: the w1/w3/w2 attribute set built by
 * QuantFused*MoEBlock.from_hf (moe_block.py:725-757, 178-209, 445-474, 955-987).
 *   wq        int32 [wq_rows, n], expert e's words start at element wq_strides[e];
 *             code (k, j) of expert e is bits ((k % eps)*b .. +b) of word row k / eps,
 *             eps = 32 / b (gemq/triton_kernels/utils.py:33-71)
 *   scales    fp16 [num_experts * k / group_size, n]
 *   zeros     fp16, additive zero z' = -zero*scale (w = fma(q, s, z'), utils.py:192-212)
 *   nbits, wq_strides, zs_strides   int32 [num_experts]
 * The shared experts of DeepSeek (moe_block.py:477-489) are projections with
 * num_experts == 1.
 */
typedef struct gemq_proj {
  const int32_t* wq;
  const uint16_t* scales;
  const uint16_t* zeros;
  const int32_t* nbits;
  const int32_t* wq_strides;
  const int32_t* zs_strides;
  int64_t wq_rows;
  int32_t num_experts;
  int32_t k;
  int32_t n;
  int32_t group_size;
} gemq_proj_t;

/* Block descriptor: the constructor arguments of QuantFused*MoEBlock (moe_block.py:688-713). */
typedef struct gemq_layer_desc {
  int32_t hidden;          /* D */
  int32_t inter;           /* F (per routed expert) */
  int32_t num_experts;     /* E */
  int32_t top_k;
  int32_t group_size;      /* block_group_size (moe_block.py:745-749) */
  int32_t norm_topk_prob;  /* renormalise the top-k weights (moe_block.py:794-795) */
  int32_t router;          /* GEMQ_ROUTER_FP16 | GEMQ_ROUTER_FP32 */
  const uint16_t* gate_weight; /* fp16 [E, D] */
  gemq_proj_t w1, w3, w2;  /* gate_proj, up_proj, down_proj */
  int32_t has_shared;      /* DeepSeek shared experts (moe_block.py:575, 617-620) */
  gemq_proj_t shared_w1, shared_w3, shared_w2;
} gemq_layer_desc_t;

typedef struct gemq_layer gemq_layer_t;

/* ---------------------------------------------------------------- status */
const char* gemq_last_error_string(void); /* host string, thread-local */
int gemq_version(void);
/* Synchronises the device, returns the device error word (0 = none) and clears it.
 * The first error recorded since the last call: 1-7 a bounded wait of the GEMM
 * pipeline expired (copies landed, stage freed, A stage written, A stage read,
 * accumulator full, accumulator free, drain), 8 an expert id out of range, 9 a
 * bit-width outside 1..4, 10 a KV-cache position past the cache, 11 a chained
 * down-projection item waited too long for its gate/up tiles. After an expired wait
 * the kernels of that forward drain and return; its outputs are undefined. */
int gemq_get_device_error(uint32_t* code_out /* host */);

/* ---------------------------------------------------------------- packing */
/* Replaces pack_weights_over_cols_triton (gemq/triton_kernels/utils.py:74-113).
 * codes uint8 [rows, cols] -> out int32 [rows, cdiv(cols, 32/nbits)] (the buffer
 * whose transpose the reference returns). */
int gemq_pack_weights_over_cols(const uint8_t* codes, int64_t rows, int64_t cols, int32_t nbits,
                                int32_t* out, void* stream);

/* Replaces unpack_over_cols_triton (gemq/triton_kernels/utils.py:149-189). */
int gemq_unpack_over_cols(const int32_t* packed, int64_t rows, int64_t packed_cols, int64_t out_cols,
                          int32_t nbits, uint8_t* out, void* stream);

/* The dequant of gemq/triton_kernels/utils.py:192-212 applied to one whole expert,
 * addressed as in dequant_group_gemm.py:71-81,118-130: out fp16 [k, n]. */
int gemq_dequant_expert(const gemq_proj_t* proj /* host struct */, int32_t expert, uint16_t* out,
                        void* stream);

/* ---------------------------------------------------------------- kernel-level GEMMs */
/* Replaces dequant_group_gemm_triton (dequant_group_gemm.py:155-202):
 * out[a] = x[m, k] @ deq(W[indices[a]]) -> fp16 [num_indices, m, n]. */
size_t gemq_group_gemm_workspace_size(int32_t num_indices);
int gemq_dequant_group_gemm(const gemq_proj_t* proj, const uint16_t* x, int64_t m, const int32_t* indices,
                            int32_t num_indices, uint16_t* out, void* workspace, size_t workspace_bytes,
                            void* stream);

/* gemq_dequant_group_gemm for callers that cannot allocate device memory: no
 * counterpart in the reference (its Triton launchers allocate through torch).
 * Meant for hosts whose device memory is fixed or owned by someone else, e.g. a
 * serving process that reserves its memory pool at start-up, or a plugin that must
 * not call its host's allocator: it takes no workspace and calls no cudaMalloc,
 * cudaFree or other allocating routine. The segment table lives in a 20 KiB array
 * in the library's device image, which every GPU that loads the library holds
 * until the process exits; num_indices above GEMQ_NOALLOC_MAX_INDICES is rejected
 * with GEMQ_ERR_INVALID_ARGUMENT. The first call on each device looks up that
 * array's address (cudaGetSymbolAddress), so make it before any stream capture.
 * Every call shares the one array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller. Each call
 * rewrites the entries it reads, so no clearing is needed between calls. The
 * looked-up address is kept for the life of the process: do not call
 * cudaDeviceReset on a device once this entry point has run there.
 * Both group GEMM entry points reject num_indices * m above 2^31 - 1 rows. */
#define GEMQ_NOALLOC_MAX_INDICES 1023
int gemq_dequant_group_gemm_noalloc(const gemq_proj_t* proj, const uint16_t* x, int64_t m, const int32_t* indices,
                                    int32_t num_indices, uint16_t* out, void* stream);

/* Replaces dequant_gemm_triton (dequant_gemm.py:150-193); proj->num_experts == 1. */
int gemq_dequant_gemm(const gemq_proj_t* proj, const uint16_t* x, int64_t m, uint16_t* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Replaces dequant_splitk_gemv_triton (dequant_gemv.py:118-156) with a deterministic
 * reduction (no fp16 atomics); x fp16 [1, k] -> out fp16 [1, n]. */
size_t gemq_gemv_workspace_size(const gemq_proj_t* proj, int32_t num_rows);
int gemq_dequant_gemv(const gemq_proj_t* proj, const uint16_t* x, uint16_t* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Replaces fused_dequant_up_proj_triton (fused_dequant_bmm.py:122-173):
 * x fp16 [1, k], idx int32 [num_idx] -> x1, x3 fp16 [1, num_idx * n]. w3 is read
 * with w1's nbits/strides as the reference does (check_w1_w3_aligned). */
int gemq_fused_up_proj(const gemq_proj_t* w1, const gemq_proj_t* w3, const uint16_t* x, const int32_t* idx,
                       int32_t num_idx, uint16_t* x1, uint16_t* x3, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Replaces fused_dequant_down_proj_triton (fused_dequant_bmm.py:264-312):
 * x1, x3 fp16 [1, num_idx * w2->k] -> x2 fp16 [1, num_idx * n], SiLU*mul in fp32. */
int gemq_fused_down_proj(const gemq_proj_t* w2, const uint16_t* x1, const uint16_t* x3, const int32_t* idx,
                         int32_t num_idx, uint16_t* x2, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---------------------------------------------------------------- MoE block */
/* Validates a block (moe_block.py:196-201 single group size, 69-80 w1/w3
 * alignment, 175-176 packed weights present) and prepares TMA descriptors.
 * Reads nbits/strides to the host once (synchronous). */
int gemq_layer_create(const gemq_layer_desc_t* desc /* host */, gemq_layer_t** out /* host */);
int gemq_layer_destroy(gemq_layer_t* layer);

size_t gemq_moe_workspace_size(const gemq_layer_t* layer, int64_t num_tokens, uint32_t flags);

/* Routing options beyond the block constructor's: DeepSeek-V2's group-limited greedy
 * selection and routed_scaling_factor, which the reference's fused block rejects
 * (gemq/inference/moe_block.py:18-66, check_deepseek_routing_supported and
 * check_deepseek_gate_matches). Selection as transformers'
 * DeepseekV2Moe.route_tokens_to_experts computes it: softmax in fp32; with
 * n_group > 1 the experts form n_group equal groups of consecutive ids, each scored
 * by its largest probability, the topk_group best groups are kept (lower group id on
 * ties) and every other expert's probability reads 0.0; then the top-k. Weights:
 * w / sum(w) when norm_topk_prob, else w * scale, rounded to fp16.
 * Limits: 1 <= n_group <= 32, num_experts % n_group == 0, 1 <= topk_group <= n_group,
 * topk_group * (num_experts / n_group) >= top_k, scale finite. */
typedef struct gemq_routing {
  int32_t norm_topk_prob;
  int32_t n_group;     /* 1 = plain greedy */
  int32_t topk_group;
  float scale;         /* routed_scaling_factor (1.0 = none) */
} gemq_routing_t;

/* Replaces the layer's routing options (default: the descriptor's norm_topk_prob,
 * n_group = topk_group = 1, scale = 1.0). Not to be called while a forward of the
 * layer is being enqueued on another thread. */
int gemq_layer_set_routing(gemq_layer_t* layer, const gemq_routing_t* routing /* host */);

/* Router of forward_n_tokens / forward_one_token (moe_block.py:790-797, 828-833,
 * 549-556, 280-283): logits (fp16, or fp32 for GEMQ_ROUTER_FP32) [T, E],
 * topk_idx int32 [T, k], topk_w fp16 [T, k]. Ties go to the lower expert id. */
int gemq_moe_route(gemq_layer_t* layer, const uint16_t* x, int64_t num_tokens, void* logits, int32_t* topk_idx,
                   uint16_t* topk_w, uint32_t flags, void* workspace, size_t workspace_bytes, void* stream);

/* The same router without a layer handle (the gate and routing options passed
 * directly): what an expert-parallel rank uses, whose layer holds only its own
 * experts while routing spans all of them (moe_block.py:790-797, 549-556).
 * workspace: at least GEMQ_ROUTE_WORKSPACE_BYTES. */
#define GEMQ_ROUTE_WORKSPACE_BYTES 1024
int gemq_route(const uint16_t* x, int64_t num_tokens, int32_t hidden, const uint16_t* gate_weight,
               int32_t num_experts, int32_t top_k, int32_t router, int32_t norm_topk_prob, uint32_t flags,
               void* logits, int32_t* topk_idx, uint16_t* topk_w, void* workspace, size_t workspace_bytes,
               void* stream);
/* gemq_route with the routing options of gemq_routing_t (NULL = plain greedy without
 * renormalisation). */
int gemq_route_ex(const uint16_t* x, int64_t num_tokens, int32_t hidden, const uint16_t* gate_weight,
                  int32_t num_experts, int32_t top_k, int32_t router, const gemq_routing_t* routing /* host */,
                  uint32_t flags, void* logits, int32_t* topk_idx, uint16_t* topk_w, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Combine of forward_n_tokens (moe_block.py:799-812) on already computed expert
 * outputs: out[t] = sum over the token's k slots of y[slot_row[t*k + j]], in
 * ascending expert id (topk_idx), every partial sum rounded to fp16 (one fp32 sum
 * with GEMQ_FWD_FP32_COMBINE), then + residual in fp16 when residual != NULL.
 * y fp16 [rows, hidden]; slot_row int32 [T*k] (-1 skips the slot). */
int gemq_moe_combine(const uint16_t* y, const int32_t* slot_row, const int32_t* topk_idx, int64_t num_tokens,
                     int32_t top_k, int32_t hidden, uint32_t flags, const uint16_t* residual, uint16_t* out,
                     void* stream);

/* Dispatch of forward_n_tokens (moe_block.py:804-810: one_hot / nonzero / where /
 * gather), exposed for expert parallelism: the T*k token-expert slots grouped by
 * expert id, ascending. expert_counts int32 [num_experts] (rows per expert, in row
 * order); slot_row int32 [T*k] (row of slot t*k + j, -1 for an expert id outside
 * [0, num_experts), which is also recorded in the device error word); w_rows fp16
 * [T*k] (routing weight of each row); x_rows fp16 [T*k, hidden] (the token's
 * activation row). Rows of one expert come in no particular order. */
size_t gemq_dispatch_workspace_size(int64_t num_tokens, int32_t top_k, int32_t num_experts);
int gemq_moe_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t num_tokens,
                      int32_t top_k, int32_t num_experts, int32_t hidden, const int32_t* perm_nbits,
                      int32_t* expert_counts, int32_t* slot_row, uint16_t* w_rows, uint16_t* x_rows, void* workspace,
                      size_t workspace_bytes, void* stream);
/* perm_nbits (device int32 [num_experts], or NULL): write each row in the K order the
 * tensor-memory GEMM reads for its expert's gate/up bit-width, for owners whose
 * gemq_moe_experts_row_order is 1 (the rows then go in with GEMQ_FWD_PERMUTED_ROWS).
 * Returns 1 when gemq_moe_experts runs this layer on the tensor-memory GEMM, whose
 * input rows must then be permuted (dispatch with perm_nbits = the gate/up bit-widths
 * of all experts) and flagged GEMQ_FWD_PERMUTED_ROWS; 0 when rows go in unpermuted. */
int gemq_moe_experts_row_order(const gemq_layer_t* layer);

/* forward_single_expert (moe_block.py:763-779) for every expert of the layer at once,
 * on rows already grouped by expert: rows fp16 [num_rows, hidden] ordered as
 * [group 0: expert 0 rows, expert 1 rows, ... | group 1: ...], with
 * group_counts int32 [num_groups * num_experts] (device) giving the row counts in
 * that order (an expert-parallel rank: one group per source rank). out fp16
 * [num_rows, hidden] in the same row order; each row fp16(fp16(y) * row_weight)
 * (moe_block.py:811) when row_weight (fp16 [num_rows]) is given, else fp16(y).
 * sm_budget > 0 caps the SMs the GEMMs use (leaves room for a concurrent
 * collective); 0 = all. num_groups * num_experts <= 1024. */
size_t gemq_moe_experts_workspace_size(const gemq_layer_t* layer, int64_t num_rows, int32_t num_groups);
int gemq_moe_experts(gemq_layer_t* layer, const uint16_t* rows, int64_t num_rows, const int32_t* group_counts,
                     int32_t num_groups, const uint16_t* row_weight, uint16_t* out, int32_t sm_budget,
                     uint32_t flags, void* workspace, size_t workspace_bytes, void* stream);

/* The whole block: replaces QuantFused*MoEBlock.forward -> forward_n_tokens /
 * forward_one_token (moe_block.py:781-858, 234-309, 540-628, 1011-1088).
 *   x fp16 [T, D] -> out fp16 [T, D]
 *   router_logits: output [T, E] (fp16 or fp32 per desc->router), may be NULL;
 *                  an input with GEMQ_FWD_GIVEN_LOGITS (fp32 accepted for both)
 *   topk_idx/topk_w: inputs with GEMQ_FWD_GIVEN_ROUTING, else NULL */
int gemq_moe_forward(gemq_layer_t* layer, const uint16_t* x, int64_t num_tokens, uint16_t* out,
                     void* router_logits, const int32_t* topk_idx, const uint16_t* topk_w, uint32_t flags,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Durations (ms, host array of GEMQ_NUM_STAGES; 0 for stages that did not run) of
 * the last gemq_moe_forward issued with GEMQ_FWD_TIME_STAGES; waits for it to finish.
 * No counterpart in the reference (it has no native timing hooks). */
int gemq_layer_stage_times(gemq_layer_t* layer, float* ms_out /* host */);

/* Dequant form the tensor-memory GEMM uses for w1, w3, w2 (host int32[3]): 1 = the
 * single-instruction form, taken when every scale of the projection is a normal fp16
 * number with s * 2^18 finite (2^16 for 1-bit experts, 2^19 for 3-bit: exponent field
 * at most 12 / 14 / 11); 0 = the general form. Both give bit-identical weights
 * (utils.py:206-210). Decided once, when the layer is created. No reference
 * counterpart (a diagnostic). */
int gemq_layer_dequant_forms(const gemq_layer_t* layer, int32_t* forms_out /* host */);

/* RMSNorm of the decoder layers around the MoE blocks (transformers' OlmoeRMSNorm):
 * out = fp16(weight * fp16(x * rsqrt(mean(x^2) + eps))) per row, x in fp32, in one
 * launch. x, out fp16 [rows, n], weight fp16 [n]; n % 8 == 0; pointers 16-byte
 * aligned. Not part of the reference's MoE path: the whole-model decode harness
 * (robustgemq_b200/inference/generate.py) uses it in place of the eager module's six
 * kernels per norm. */
int gemq_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t rows, int32_t n, float eps, uint16_t* out,
                  void* stream);

/* The attention prologue of transformers' OlmoeAttention after a fused q|k|v
 * projection, in one launch: per row of qkv (fp16 [rows, >= 2n], row stride ld),
 * q and k (the first two blocks of n values) each through RMSNorm with its own weight
 * (as gemq_rms_norm), then the rotary embedding of apply_rotary_pos_emb on fp16
 * tensors per head of head_dim values: out = fp16(fp16(x * cos) +
 * fp16(rotate_half(x) * sin)), cos / sin fp16 [rows, head_dim]. q_out, k_out fp16
 * [rows, n]. n % 8 == 0, ld % 8 == 0, qkv and the weights 16-byte aligned.
 * KV-cache write (k_cache != NULL; one row only): k after the rotation and v (the
 * third block of qkv) also go to position *cache_len (device int64) of k_cache /
 * v_cache (fp16 [n / head_dim heads][max_len][head_dim], batch 1), and *cache_len
 * advances by one: the update of a static KV cache (transformers' StaticLayer) in the
 * same launch. k_out may then be NULL. A position outside [0, max_len) writes nothing
 * and records a device error. Not part of the reference's MoE path: used by the
 * whole-model decode harness. */
int gemq_qk_norm_rope(const uint16_t* qkv, int64_t ld, int64_t rows, int32_t n, int32_t head_dim,
                      const uint16_t* q_norm_weight, const uint16_t* k_norm_weight, float eps, const uint16_t* cos,
                      const uint16_t* sin, uint16_t* q_out, uint16_t* k_out, uint16_t* k_cache, uint16_t* v_cache,
                      int32_t max_len, int64_t* cache_len, void* stream);

/* Attention of one query token of one sequence over a static KV cache:
 * out[h] = softmax(scale * q[h] K[h][0:L]^T) V[h][0:L] with L = *cache_len (device
 * int64, clamped to [0, max_len]), i.e. the causal mask of a one-token decode step,
 * which hides exactly the cache positions not yet written. q, out fp16 [heads,
 * head_dim]; k_cache, v_cache fp16 [heads][max_len][head_dim], 16-byte aligned;
 * head_dim % 8 == 0, at most 256; fp32 scores, softmax and sums, one rounding to fp16. Not part of the reference's MoE path: used by the
 * whole-model decode harness in place of the attention library call. */
int gemq_decode_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int32_t heads,
                          int32_t max_len, int32_t head_dim, const int64_t* cache_len, float scale, uint16_t* out,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GEMQ_B200_H */
