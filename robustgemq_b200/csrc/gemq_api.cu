// C ABI of gemq-b200: validation, workspace carving and the prefill / one-token
// pipelines of the quantized MoE block. See include/gemq_b200.h for the contract.
#include <cuda_fp16.h>

#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "gemq_common.cuh"
#include "gemq_internal.h"

namespace gemq {

namespace {
thread_local std::string t_last_error;

// Host-side NVTX range over one C-ABI call, named after the entry point, so a
// profiler timeline (nsys, ncu's NVTX filter) shows which call launched which
// kernels. NVTX records nothing unless a tool is attached.
struct TraceRange {
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};
}  // namespace

void set_error(const std::string& msg) { t_last_error = msg; }

int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

namespace {

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  set_error(std::string(where) + ": " + cudaGetErrorString(e));
  return GEMQ_ERR_CUDA;
}

#define GEMQ_CUDA(call, where)                                    \
  do {                                                            \
    cudaError_t _e = (call);                                      \
    if (_e != cudaSuccess) return cuda_fail(_e, where);           \
  } while (0)

ProjDev to_dev(const gemq_proj_t& p) {
  ProjDev d;
  d.wq = p.wq;
  d.scales = p.scales;
  d.zeros = p.zeros;
  d.nbits = p.nbits;
  d.wq_strides = p.wq_strides;
  d.zs_strides = p.zs_strides;
  d.wq_rows = p.wq_rows;
  d.num_experts = p.num_experts;
  d.k = p.k;
  d.n = p.n;
  d.group_size = p.group_size;
  d.sub_ok = 0;  // set by a layer's scale check; one-shot GEMM calls keep the general dequant
  return d;
}

// Shape checks every entry point shares (the reference asserts these implicitly).
int check_proj(const gemq_proj_t* p, const char* name) {
  if (p == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": null projection");
  if (p->wq == nullptr || p->scales == nullptr || p->zeros == nullptr || p->nbits == nullptr ||
      p->wq_strides == nullptr || p->zs_strides == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": null device pointer");
  if (p->num_experts <= 0 || p->k <= 0 || p->n <= 0 || p->group_size <= 0 || p->wq_rows <= 0)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": non-positive size");
  if (p->k % p->group_size != 0)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": k must be a multiple of group_size");
  if (p->n % 4 != 0) return fail(GEMQ_ERR_UNSUPPORTED, std::string(name) + ": n must be a multiple of 4");
  return GEMQ_OK;
}

int packed_rows(int k, int nb) {
  const int eps = 32 / nb;
  return (k + eps - 1) / eps;
}

// Reads nbits / strides to the host and checks they describe the from_hf layout
// (moe_block.py:737-757), so every kernel access stays inside wq / scales / zeros.
int validate_layout(const gemq_proj_t& p, const char* name, std::vector<int32_t>* nbits_out,
                    std::vector<int32_t>* wq_strides_out) {
  std::vector<int32_t> nb(p.num_experts), ws(p.num_experts), zs(p.num_experts);
  GEMQ_CUDA(cudaMemcpy(nb.data(), p.nbits, sizeof(int32_t) * p.num_experts, cudaMemcpyDeviceToHost), "copy nbits");
  GEMQ_CUDA(cudaMemcpy(ws.data(), p.wq_strides, sizeof(int32_t) * p.num_experts, cudaMemcpyDeviceToHost),
            "copy wq_strides");
  GEMQ_CUDA(cudaMemcpy(zs.data(), p.zs_strides, sizeof(int32_t) * p.num_experts, cudaMemcpyDeviceToHost),
            "copy zs_strides");
  int64_t wq_off = 0;
  const int64_t zs_per = static_cast<int64_t>(p.k / p.group_size) * p.n;
  for (int e = 0; e < p.num_experts; ++e) {
    if (nb[e] < 1 || nb[e] > 4)
      return fail(GEMQ_ERR_UNSUPPORTED, std::string(name) + ": bit-width must be 1, 2, 3 or 4 (utils.py:83)");
    if (ws[e] != wq_off)
      return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": wq_strides is not the exclusive cumsum of numel");
    if (zs[e] != e * zs_per)
      return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": zs_strides is not the exclusive cumsum of numel");
    wq_off += static_cast<int64_t>(packed_rows(p.k, nb[e])) * p.n;
  }
  if (wq_off > p.wq_rows * p.n)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, std::string(name) + ": wq has fewer rows than its experts need");
  if (wq_off > INT32_MAX)
    return fail(GEMQ_ERR_UNSUPPORTED, std::string(name) + ": int32 element offsets overflow (as in the reference)");
  if (nbits_out) *nbits_out = nb;
  if (wq_strides_out) *wq_strides_out = ws;
  return GEMQ_OK;
}

// Bump allocator over the caller's workspace (256-byte aligned pieces).
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~static_cast<size_t>(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += sizeof(T) * count;
    return p;
  }
};

int choose_nt(int64_t rows_per_expert) { return rows_per_expert > 48 ? kNtLarge : kNtSmall; }

// Up to this many tokens the router's gate logits run as a CUDA-core kernel spread
// over (expert group x token group) CTAs; beyond it, as a tensor-core GEMM. The
// top-k kernel follows either.
constexpr int64_t kSmallRouteTokens = 256;

// Runs one grouped GEMM, tensor cores when the shape allows, CUDA cores otherwise.
// The segments must have been built with the nt this returns through `nt_used`.
bool use_tc(const GemmArgs& a, bool force_simt) { return !force_simt && tc_gemm_supported(a); }

int run_gemm(GemmArgs a, bool force_simt, cudaStream_t s, const char* what) {
  cudaError_t e = use_tc(a, force_simt) ? launch_tc_gemm(a, s) : launch_simt_gemm(a, s);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return GEMQ_OK;
}

}  // namespace
}  // namespace gemq

using namespace gemq;

struct gemq_layer {
  gemq_layer_desc_t d;
  gemq_routing_t ro;  // norm_topk_prob (from d unless replaced), group-limited greedy, scale
  ProjDev w1, w3, w2, sw1, sw3, sw2;
  ProjDev w3_as_w1;  // w3 read with w1's nbits/strides (one-token path, fused_dequant_bmm.py:98)
  int num_sms;
  int shared_inter;
  // optional stage timing (GEMQ_FWD_TIME_STAGES)
  bool events_ready = false;
  cudaEvent_t ev[2 * GEMQ_NUM_STAGES];
  bool stage_ran[GEMQ_NUM_STAGES] = {};
};

namespace gemq {
namespace {
// Records events around pipeline stages when timing is requested.
struct StageTimer {
  gemq_layer_t* L;
  cudaStream_t s;
  bool on;
  StageTimer(gemq_layer_t* layer, cudaStream_t stream, uint32_t flags)
      : L(layer), s(stream), on((flags & GEMQ_FWD_TIME_STAGES) != 0) {
    if (!on) return;
    if (!L->events_ready) {
      for (auto& e : L->ev) cudaEventCreate(&e);
      L->events_ready = true;
    }
    for (bool& r : L->stage_ran) r = false;
  }
  void begin(int st) {
    if (on) cudaEventRecord(L->ev[2 * st], s);
  }
  void end(int st) {
    if (!on) return;
    cudaEventRecord(L->ev[2 * st + 1], s);
    L->stage_ran[st] = true;
  }
};
}  // namespace
}  // namespace gemq

extern "C" {

const char* gemq_last_error_string(void) { return t_last_error.c_str(); }

int gemq_version(void) { return 1; }

int gemq_get_device_error(uint32_t* code_out) {
  if (code_out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null output");
  GEMQ_CUDA(cudaDeviceSynchronize(), "synchronize");
  uint32_t v = 0;
  GEMQ_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)), "read device error");
  const uint32_t zero = 0;
  GEMQ_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)), "clear device error");
  GEMQ_CUDA(cudaMemcpyToSymbol(g_device_abort, &zero, sizeof(zero)), "clear device abort");
  *code_out = v;
  return GEMQ_OK;
}

int gemq_pack_weights_over_cols(const uint8_t* codes, int64_t rows, int64_t cols, int32_t nbits, int32_t* out,
                                void* stream) {
  TraceRange trace("gemq_pack_weights_over_cols");
  if (nbits < 1 || nbits > 4) return fail(GEMQ_ERR_INVALID_ARGUMENT, "Untested quantization bitwidth (utils.py:83)");
  if (rows < 0 || cols < 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "negative size");
  if (rows * cols > 0 && (codes == nullptr || out == nullptr)) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  GEMQ_CUDA(launch_pack(codes, rows, cols, nbits, out, static_cast<cudaStream_t>(stream)), "pack");
  return GEMQ_OK;
}

int gemq_unpack_over_cols(const int32_t* packed, int64_t rows, int64_t packed_cols, int64_t out_cols, int32_t nbits,
                          uint8_t* out, void* stream) {
  TraceRange trace("gemq_unpack_over_cols");
  if (nbits < 1 || nbits > 4) return fail(GEMQ_ERR_INVALID_ARGUMENT, "Untested quantization bitwidth (utils.py:83)");
  if (rows < 0 || out_cols < 0 || packed_cols < 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "negative size");
  const int eps = 32 / nbits;
  if ((out_cols + eps - 1) / eps > packed_cols)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "out_cols needs more packed columns than given");
  if (rows * out_cols > 0 && (packed == nullptr || out == nullptr)) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  GEMQ_CUDA(launch_unpack(packed, rows, packed_cols, out_cols, nbits, out, static_cast<cudaStream_t>(stream)), "unpack");
  return GEMQ_OK;
}

int gemq_dequant_expert(const gemq_proj_t* proj, int32_t expert, uint16_t* out, void* stream) {
  TraceRange trace("gemq_dequant_expert");
  if (int rc = check_proj(proj, "proj")) return rc;
  if (expert < 0 || expert >= proj->num_experts) return fail(GEMQ_ERR_INVALID_ARGUMENT, "expert out of range");
  if (out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null output");
  GEMQ_CUDA(launch_dequant_expert(to_dev(*proj), expert, out, static_cast<cudaStream_t>(stream)), "dequant");
  return GEMQ_OK;
}

size_t gemq_group_gemm_workspace_size(int32_t num_indices) {
  Carver c(nullptr);
  c.take<Seg>(num_indices > 0 ? num_indices : 1);
  c.take<int32_t>(num_indices + 1);
  return c.off + 256;
}

int gemq_dequant_group_gemm(const gemq_proj_t* proj, const uint16_t* x, int64_t m, const int32_t* indices,
                            int32_t num_indices, uint16_t* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  TraceRange trace("gemq_dequant_group_gemm");
  if (int rc = check_proj(proj, "proj")) return rc;
  if (num_indices <= 0 || num_indices > 1023) return fail(GEMQ_ERR_INVALID_ARGUMENT, "num_indices must be in [1, 1023]");
  if (m < 0 || m > INT32_MAX / 2) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad m");
  // output rows of index a start at a * m, held as a 32-bit row offset in the segment table
  if (static_cast<int64_t>(num_indices) * m > INT32_MAX)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "num_indices * m exceeds 2^31 - 1 output rows");
  if (m == 0) return GEMQ_OK;
  if (x == nullptr || out == nullptr || indices == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (workspace_bytes < gemq_group_gemm_workspace_size(num_indices) || workspace == nullptr)
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  Seg* segs = c.take<Seg>(num_indices);
  int32_t* tp = c.take<int32_t>(num_indices + 1);
  GemmArgs a{};
  a.mode = GemmMode::kStoreF16;
  a.w0 = to_dev(*proj);
  a.w1 = a.w0;
  a.act = x;
  a.act_rows = m;
  a.segs = segs;
  a.tile_prefix = tp;
  a.num_segs = num_indices;
  a.out = out;
  a.out_ld = proj->n;
  a.out_cols = proj->n;
  a.num_sms = device_sm_count();
  a.nt = choose_nt(m);
  if (!tc_gemm_supported(a)) a.nt = 32;
  GEMQ_CUDA(launch_build_index_segs(indices, num_indices, proj->num_experts, m, a.nt, segs, tp, s), "segments");
  return run_gemm(a, false, s, "dequant_group_gemm");
}

int gemq_dequant_gemm(const gemq_proj_t* proj, const uint16_t* x, int64_t m, uint16_t* out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_dequant_gemm");
  if (int rc = check_proj(proj, "proj")) return rc;
  if (proj->num_experts != 1) return fail(GEMQ_ERR_INVALID_ARGUMENT, "dequant_gemm takes a single weight");
  if (m <= 0) return m == 0 ? GEMQ_OK : fail(GEMQ_ERR_INVALID_ARGUMENT, "bad m");
  if (x == nullptr || out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (workspace_bytes < gemq_group_gemm_workspace_size(1) || workspace == nullptr)
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  Seg* segs = c.take<Seg>(1);
  int32_t* tp = c.take<int32_t>(2);
  GemmArgs a{};
  a.mode = GemmMode::kStoreF16;
  a.w0 = to_dev(*proj);
  a.w1 = a.w0;
  a.act = x;
  a.act_rows = m;
  a.segs = segs;
  a.tile_prefix = tp;
  a.num_segs = 1;
  a.out = out;
  a.out_ld = proj->n;
  a.out_cols = proj->n;
  a.num_sms = device_sm_count();
  a.nt = choose_nt(m);
  if (!tc_gemm_supported(a)) a.nt = 32;
  GEMQ_CUDA(launch_build_index_segs(nullptr, 1, 1, m, a.nt, segs, tp, s), "segments");
  return run_gemm(a, false, s, "dequant_gemm");
}

size_t gemq_gemv_workspace_size(const gemq_proj_t* proj, int32_t num_rows) {
  if (proj == nullptr || num_rows <= 0) return 0;
  const int splits = gemv_default_splits(proj->k, proj->n, num_rows, device_sm_count());
  Carver c(nullptr);
  c.take<float>(2ull * splits * num_rows * proj->n);
  return c.off + 256;
}

int gemq_dequant_gemv(const gemq_proj_t* proj, const uint16_t* x, uint16_t* out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_dequant_gemv");
  if (int rc = check_proj(proj, "proj")) return rc;
  if (proj->num_experts != 1) return fail(GEMQ_ERR_INVALID_ARGUMENT, "dequant_gemv takes a single weight");
  if (x == nullptr || out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (workspace == nullptr || workspace_bytes < gemq_gemv_workspace_size(proj, 1))
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int splits = gemv_default_splits(proj->k, proj->n, 1, device_sm_count());
  Carver c(workspace);
  float* part = c.take<float>(static_cast<size_t>(splits) * proj->n);
  GemvSrc src{kGemvX, reinterpret_cast<const __half*>(x), nullptr, 0, nullptr, 0, 0, 0};
  GEMQ_CUDA(launch_gemv(to_dev(*proj), nullptr, nullptr, 1, src, part, splits, s), "gemv");
  GEMQ_CUDA(launch_gemv_reduce(part, splits, 1, proj->n, out, s), "gemv reduce");
  return GEMQ_OK;
}

int gemq_fused_up_proj(const gemq_proj_t* w1, const gemq_proj_t* w3, const uint16_t* x, const int32_t* idx,
                       int32_t num_idx, uint16_t* x1, uint16_t* x3, void* workspace, size_t workspace_bytes,
                       void* stream) {
  TraceRange trace("gemq_fused_up_proj");
  if (int rc = check_proj(w1, "w1")) return rc;
  if (int rc = check_proj(w3, "w3")) return rc;
  if (w1->k != w3->k || w1->n != w3->n || w1->num_experts != w3->num_experts || w1->group_size != w3->group_size)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "w1 and w3 shapes differ");
  if (num_idx <= 0 || x == nullptr || idx == nullptr || x1 == nullptr || x3 == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad arguments");
  if (workspace == nullptr || workspace_bytes < gemq_gemv_workspace_size(w1, num_idx))
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int splits = gemv_default_splits(w1->k, w1->n, num_idx, device_sm_count(), 2);
  Carver c(workspace);
  float* p1 = c.take<float>(2ull * splits * num_idx * w1->n);  // [w1, w3][split][a][n]
  float* p3 = p1 + static_cast<size_t>(splits) * num_idx * w1->n;
  ProjDev d1 = to_dev(*w1), d3 = to_dev(*w3);
  d3.nbits = d1.nbits;            // fused_dequant_bmm.py:55-57: w3 read with w1's nbits
  d3.wq_strides = d1.wq_strides;  // and w1's word offsets (check_w1_w3_aligned)
  GemvSrc src{kGemvX, reinterpret_cast<const __half*>(x), nullptr, 0, nullptr, 0, 0, 0};
  GEMQ_CUDA(launch_gemv(d1, &d3, idx, num_idx, src, p1, splits, s), "up projection");
  GEMQ_CUDA(launch_gemv_reduce(p1, splits, num_idx, w1->n, x1, s), "reduce x1");
  GEMQ_CUDA(launch_gemv_reduce(p3, splits, num_idx, w1->n, x3, s), "reduce x3");
  return GEMQ_OK;
}

int gemq_fused_down_proj(const gemq_proj_t* w2, const uint16_t* x1, const uint16_t* x3, const int32_t* idx,
                         int32_t num_idx, uint16_t* x2, void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_fused_down_proj");
  if (int rc = check_proj(w2, "w2")) return rc;
  if (num_idx <= 0 || x1 == nullptr || x3 == nullptr || idx == nullptr || x2 == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad arguments");
  if (workspace == nullptr || workspace_bytes < gemq_gemv_workspace_size(w2, num_idx))
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int splits = gemv_default_splits(w2->k, w2->n, num_idx, device_sm_count());
  Carver c(workspace);
  float* p = c.take<float>(static_cast<size_t>(splits) * num_idx * w2->n);
  GemvSrc src{kGemvSwiGLU, reinterpret_cast<const __half*>(x1), reinterpret_cast<const __half*>(x3), w2->k,
              nullptr, 0, 0, 0};
  GEMQ_CUDA(launch_gemv(to_dev(*w2), nullptr, idx, num_idx, src, p, splits, s), "down");
  GEMQ_CUDA(launch_gemv_reduce(p, splits, num_idx, w2->n, x2, s), "reduce x2");
  return GEMQ_OK;
}

// ------------------------------------------------------------------ layer
int gemq_layer_create(const gemq_layer_desc_t* desc, gemq_layer_t** out) {
  TraceRange trace("gemq_layer_create");
  if (desc == nullptr || out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  const gemq_layer_desc_t& d = *desc;
  if (d.hidden <= 0 || d.inter <= 0 || d.num_experts <= 0 || d.top_k <= 0 || d.group_size <= 0)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "non-positive block dimension");
  if (d.top_k > d.num_experts || d.top_k > 16) return fail(GEMQ_ERR_UNSUPPORTED, "top_k must be <= min(E, 16)");
  if (d.num_experts > 256) return fail(GEMQ_ERR_UNSUPPORTED, "at most 256 experts");
  if (d.hidden % 8 != 0) return fail(GEMQ_ERR_UNSUPPORTED, "hidden size must be a multiple of 8");
  if (d.gate_weight == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null gate weight");
  if (d.router != GEMQ_ROUTER_FP16 && d.router != GEMQ_ROUTER_FP32)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "unknown router flavour");
  if (int rc = check_proj(&d.w1, "w1")) return rc;
  if (int rc = check_proj(&d.w3, "w3")) return rc;
  if (int rc = check_proj(&d.w2, "w2")) return rc;
  const gemq_proj_t* ps[3] = {&d.w1, &d.w3, &d.w2};
  for (const gemq_proj_t* p : ps) {
    if (p->num_experts != d.num_experts) return fail(GEMQ_ERR_INVALID_ARGUMENT, "projection expert count differs");
    if (p->group_size != d.group_size)
      return fail(GEMQ_ERR_INVALID_ARGUMENT, "Group sizes must be the same across all experts. (moe_block.py:200)");
  }
  if (d.w1.k != d.hidden || d.w1.n != d.inter || d.w3.k != d.hidden || d.w3.n != d.inter || d.w2.k != d.inter ||
      d.w2.n != d.hidden)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "projection shapes do not match hidden/inter");
  std::vector<int32_t> nb1, nb3, ws1, ws3;
  if (int rc = validate_layout(d.w1, "w1", &nb1, &ws1)) return rc;
  if (int rc = validate_layout(d.w3, "w3", &nb3, &ws3)) return rc;
  if (int rc = validate_layout(d.w2, "w2", nullptr, nullptr)) return rc;
  if (nb1 != nb3)
    return fail(GEMQ_ERR_INVALID_ARGUMENT,
                "w1 and w3 must share bit-widths: forward_one_token indexes w3 with w1's nbits (moe_block.py:75-77)");
  if (ws1 != ws3)
    return fail(GEMQ_ERR_INVALID_ARGUMENT,
                "w1 and w3 must share packed strides: forward_one_token reads w3 at w1's offsets (moe_block.py:78-80)");
  int shared_inter = 0;
  if (d.has_shared) {
    const gemq_proj_t* ss[3] = {&d.shared_w1, &d.shared_w3, &d.shared_w2};
    const char* names[3] = {"shared_w1", "shared_w3", "shared_w2"};
    for (int i = 0; i < 3; ++i) {
      if (int rc = check_proj(ss[i], names[i])) return rc;
      if (ss[i]->num_experts != 1) return fail(GEMQ_ERR_INVALID_ARGUMENT, "shared projections hold one weight");
      if (int rc = validate_layout(*ss[i], names[i], nullptr, nullptr)) return rc;
    }
    shared_inter = d.shared_w1.n;
    if (d.shared_w1.k != d.hidden || d.shared_w3.k != d.hidden || d.shared_w3.n != shared_inter ||
        d.shared_w2.k != shared_inter || d.shared_w2.n != d.hidden)
      return fail(GEMQ_ERR_INVALID_ARGUMENT, "shared expert shapes do not match");
  }
  gemq_layer_t* L = new gemq_layer();
  L->d = d;
  L->ro = gemq_routing_t{d.norm_topk_prob, 1, 1, 1.0f};
  L->w1 = to_dev(d.w1);
  L->w3 = to_dev(d.w3);
  L->w2 = to_dev(d.w2);
  for (ProjDev* pd : {&L->w1, &L->w3, &L->w2}) {
    const cudaError_t e = scale_exponents_ok(*pd, &pd->sub_ok);
    if (e != cudaSuccess) {
      delete L;
      return cuda_fail(e, "scale exponent check");
    }
  }
  L->w3_as_w1 = L->w3;
  L->w3_as_w1.nbits = L->w1.nbits;
  L->w3_as_w1.wq_strides = L->w1.wq_strides;
  if (d.has_shared) {
    L->sw1 = to_dev(d.shared_w1);
    L->sw3 = to_dev(d.shared_w3);
    L->sw2 = to_dev(d.shared_w2);
  }
  L->num_sms = device_sm_count();
  L->shared_inter = shared_inter;
  *out = L;
  return GEMQ_OK;
}

int gemq_layer_destroy(gemq_layer_t* layer) {
  if (layer != nullptr && layer->events_ready) {
    for (auto& e : layer->ev) cudaEventDestroy(e);
  }
  delete layer;
  return GEMQ_OK;
}

}  // extern "C"

namespace gemq {
namespace {

struct FwdBufs {
  void* logits = nullptr;
  int32_t* topk_idx = nullptr;
  uint16_t* topk_w = nullptr;
  int32_t *counts = nullptr, *cursor = nullptr, *tile_prefix = nullptr, *slot_pos = nullptr;
  int32_t* tile_done = nullptr;  // per token tile: gate/up epilogue warps done (chained launch)
  int n_tile_done = 0;
  int32_t* gemv_done = nullptr;  // one-token path, per routed row: up GEMV CTAs done (chained launch)
  Seg* segs = nullptr;
  Seg* one_seg = nullptr;
  int32_t* one_tp = nullptr;
  uint16_t *w_perm = nullptr, *x_perm = nullptr, *h_perm = nullptr, *y_perm = nullptr;
  uint16_t *s_h = nullptr, *s_out = nullptr;
  float *part_up = nullptr, *part_dn = nullptr, *part_s = nullptr, *part_s2 = nullptr;
  size_t bytes = 0;
  int splits_up = 1, splits_dn = 1, splits_s = 1, splits_s2 = 1;
};

// One carving routine both sizes (base == nullptr) and lays out the workspace.
FwdBufs carve(const gemq_layer_t* L, int64_t T, uint32_t flags, void* base, const void* given_logits) {
  const gemq_layer_desc_t& d = L->d;
  const int E = d.num_experts, k = d.top_k, D = d.hidden, F = d.inter, Fs = L->shared_inter;
  const int64_t P = T * k;
  FwdBufs b;
  Carver c(base);
  const bool given_routing = (flags & GEMQ_FWD_GIVEN_ROUTING) != 0;
  (void)given_logits;
  b.logits = c.take<float>(static_cast<size_t>(T) * E);
  if (!given_routing) {
    b.topk_idx = c.take<int32_t>(P);
    b.topk_w = c.take<uint16_t>(P);
  }
  b.one_seg = c.take<Seg>(1);
  b.one_tp = c.take<int32_t>(2);
  if (flags & GEMQ_FWD_ONE_TOKEN) {
    b.splits_up = gemv_default_splits(D, F, k, L->num_sms, 2);
    b.splits_dn = gemv_default_splits(F, D, k, L->num_sms);
    b.part_up = c.take<float>(2ull * b.splits_up * k * F);  // [w1, w3][split][a][F]
    b.part_dn = c.take<float>(static_cast<size_t>(b.splits_dn) * k * D);
    b.gemv_done = c.take<int32_t>(k);
    if (d.has_shared) {
      b.splits_s = gemv_default_splits(D, Fs, 1, L->num_sms, 2);
      b.splits_s2 = gemv_default_splits(Fs, D, 1, L->num_sms);
      b.part_s = c.take<float>(2ull * b.splits_s * Fs);
      b.part_s2 = c.take<float>(static_cast<size_t>(b.splits_s2) * D);
    }
  } else {
    b.counts = c.take<int32_t>(E);
    b.cursor = c.take<int32_t>(E);
    b.segs = c.take<Seg>(E);
    b.tile_prefix = c.take<int32_t>(E + 1);
    // token tiles of at least 16 rows: at most P / 16 + E of them
    b.n_tile_done = static_cast<int>(P / kNtTiny + E + 1);
    b.tile_done = c.take<int32_t>(b.n_tile_done);
    b.slot_pos = c.take<int32_t>(P);
    b.w_perm = c.take<uint16_t>(P);
    b.x_perm = c.take<uint16_t>(static_cast<size_t>(P) * D);
    b.h_perm = c.take<uint16_t>(static_cast<size_t>(P) * F);
    b.y_perm = c.take<uint16_t>(static_cast<size_t>(P) * D);
    if (d.has_shared) {
      b.s_h = c.take<uint16_t>(static_cast<size_t>(T) * Fs);
      b.s_out = c.take<uint16_t>(static_cast<size_t>(T) * D);
    }
  }
  b.bytes = c.off + 256;
  return b;
}

// logits -> top-k (or nothing when routing is given)
// Checks routing options against the layer shape (limits of gemq_routing_t).
int check_routing(const gemq_routing_t& r, int E, int k) {
  if (r.n_group < 1 || r.n_group > 32 || E % r.n_group != 0)
    return fail(GEMQ_ERR_UNSUPPORTED, "n_group must be in [1, 32] and divide num_experts");
  if (r.topk_group < 1 || r.topk_group > r.n_group)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "topk_group must be in [1, n_group]");
  if (static_cast<int64_t>(r.topk_group) * (E / r.n_group) < k)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "the kept groups hold fewer than top_k experts");
  if (!std::isfinite(r.scale)) return fail(GEMQ_ERR_INVALID_ARGUMENT, "routing scale must be finite");
  return GEMQ_OK;
}

int run_router(const gemq_layer_desc_t& d, const gemq_routing_t& ro, int num_sms, const uint16_t* x, int64_t T,
               void* logits_out, bool logits_given, int32_t* idx, uint16_t* w, uint32_t flags, Seg* one_seg,
               int32_t* one_tp, cudaStream_t s, StageTimer* tm = nullptr, int32_t* zero_buf = nullptr,
               int zero_n = 0) {
  if (tm) tm->begin(GEMQ_STAGE_ROUTE);
  const bool fp32_logits = logits_given || d.router == GEMQ_ROUTER_FP32;
  const bool norm = ro.norm_topk_prob != 0;
  const bool fp16_softmax = (flags & GEMQ_FWD_FP16_SOFTMAX) != 0;
  if (!logits_given && T <= kSmallRouteTokens) {
    // small batches: gate dot products spread over (expert group x token group) CTAs
    GEMQ_CUDA(launch_gate_logits(x, T, d.hidden, d.gate_weight, d.num_experts, d.router == GEMQ_ROUTER_FP32,
                                 logits_out, s),
              "router");
  } else if (!logits_given) {
    GemmArgs a{};
    a.mode = d.router == GEMQ_ROUTER_FP32 ? GemmMode::kDenseF32 : GemmMode::kDenseF16;
    a.w0.k = d.hidden;
    a.w0.n = d.num_experts;
    a.w0.num_experts = 1;
    a.w0.group_size = 64;
    a.w1 = a.w0;
    a.dense_a = d.gate_weight;
    a.act = x;
    a.act_rows = T;
    a.num_segs = 1;
    a.segs = one_seg;
    a.tile_prefix = one_tp;
    a.out = logits_out;
    a.out_ld = d.num_experts;
    a.out_cols = d.num_experts;
    a.num_sms = num_sms;
    a.nt = choose_nt(T);
    const bool tc = !(flags & GEMQ_FWD_FORCE_SIMT) && tc_gemm_supported(a);
    if (tc) {
      GEMQ_CUDA(launch_build_index_segs(nullptr, 1, 1, T, a.nt, one_seg, one_tp, s), "router segments");
      GEMQ_CUDA(launch_tc_gemm(a, s), "router gemm");
    } else {
      a.nt = 32;
      GEMQ_CUDA(launch_build_index_segs(nullptr, 1, 1, T, a.nt, one_seg, one_tp, s), "router segments");
      GEMQ_CUDA(launch_simt_gemm(a, s), "router gemm");
    }
  }
  GEMQ_CUDA(launch_topk(logits_out, fp32_logits, T, d.num_experts, d.top_k, norm, fp16_softmax, ro.n_group,
                        ro.topk_group, ro.scale, idx, w, s, zero_buf, zero_n),
            "topk");
  if (tm) tm->end(GEMQ_STAGE_ROUTE);
  return GEMQ_OK;
}

int forward_one_token(gemq_layer_t* L, const uint16_t* x, uint16_t* out, const int32_t* idx, const uint16_t* w,
                      uint32_t flags, FwdBufs& b, cudaStream_t s, StageTimer& tm) {
  const uint16_t* residual = (flags & GEMQ_FWD_RESIDUAL) ? x : nullptr;
  const gemq_layer_desc_t& d = L->d;
  const int k = d.top_k, D = d.hidden, F = d.inter;
  // up: w1 and w3 (read with w1's nbits/offsets, fused_dequant_bmm.py:98) in one launch
  // Chained launch (the router of this forward zeroed the counters; not with a given
  // routing): the down GEMV starts at once, on the SM slots the up GEMV leaves free,
  // streams its words and scales, and waits per routed row for the up partials.
  // Measured on B200 (old and new library back to back): the batch-1 pass of the
  // 16-layer OLMoE stack 0.574 -> 0.556 ms, whole-model decode 695 -> 712 tokens/s.
  const bool chain = (flags & (GEMQ_FWD_NO_CHAIN | GEMQ_FWD_GIVEN_ROUTING)) == 0;
  tm.begin(GEMQ_STAGE_UP);
  GemvSrc xs{kGemvX, reinterpret_cast<const __half*>(x), nullptr, 0, nullptr, 0, 0, 0};
  if (chain) xs.done = b.gemv_done;
  GEMQ_CUDA(launch_gemv(L->w1, &L->w3_as_w1, idx, k, xs, b.part_up, b.splits_up, s), "up projection");
  tm.end(GEMQ_STAGE_UP);
  // down: reduces the up partials to fp16 x1/x3 and forms fp32 silu(x1)*x3 itself
  tm.begin(GEMQ_STAGE_DOWN);
  GemvSrc hs{kGemvPartF32, nullptr, nullptr, 0, b.part_up, b.splits_up, k, F};
  if (chain) {
    hs.done = b.gemv_done;
    hs.done_target = ((F + 127) / 128) * b.splits_up * 2;  // the row's up CTAs: slabs x splits x (w1, w3)
  }
  GEMQ_CUDA(launch_gemv(L->w2, nullptr, idx, k, hs, b.part_dn, b.splits_dn, s), "down projection");
  tm.end(GEMQ_STAGE_DOWN);
  const float* shared_part = nullptr;
  if (d.has_shared) {
    const int Fs = L->shared_inter;
    tm.begin(GEMQ_STAGE_SHARED);
    const GemvSrc sx{kGemvX, reinterpret_cast<const __half*>(x), nullptr, 0, nullptr, 0, 0, 0};  // unchained
    GEMQ_CUDA(launch_gemv(L->sw1, &L->sw3, nullptr, 1, sx, b.part_s, b.splits_s, s), "shared up");
    const GemvSrc ss{kGemvPartF16, nullptr, nullptr, 0, b.part_s, b.splits_s, 1, Fs};
    GEMQ_CUDA(launch_gemv(L->sw2, nullptr, nullptr, 1, ss, b.part_s2, b.splits_s2, s), "shared down");
    tm.end(GEMQ_STAGE_SHARED);
    shared_part = b.part_s2;
  }
  tm.begin(GEMQ_STAGE_COMBINE);
  GEMQ_CUDA(launch_decode_combine(b.part_dn, b.splits_dn, k, D, w, shared_part, b.splits_s2, residual, out, s),
            "combine");
  tm.end(GEMQ_STAGE_COMBINE);
  return GEMQ_OK;
}

int forward_n_tokens(gemq_layer_t* L, const uint16_t* x, int64_t T, uint16_t* out, const int32_t* idx,
                     const uint16_t* w, uint32_t flags, FwdBufs& b, cudaStream_t s, StageTimer& tm) {
  const gemq_layer_desc_t& d = L->d;
  const int E = d.num_experts, k = d.top_k, D = d.hidden, F = d.inter;
  const int64_t P = T * k;
  const bool force_simt = (flags & GEMQ_FWD_FORCE_SIMT) != 0;
  GemmArgs up{};
  up.mode = GemmMode::kSwiGLU;
  up.w0 = L->w1;
  up.w1 = L->w3;
  up.act = b.x_perm;
  up.act_rows = P;
  up.segs = b.segs;
  up.tile_prefix = b.tile_prefix;
  up.num_segs = E;
  up.out = b.h_perm;
  up.out_ld = F;
  up.out_cols = F;
  up.num_sms = L->num_sms;
  up.nt = choose_nt(P / E);
  GemmArgs dn = up;
  dn.mode = GemmMode::kRouteWeight;
  dn.w0 = L->w2;
  dn.w1 = L->w2;
  dn.act = b.h_perm;
  dn.out = b.y_perm;
  dn.out_ld = D;
  dn.out_cols = D;
  dn.row_weight = b.w_perm;
  const bool tc = !force_simt && tc_gemm_supported(up) && tc_gemm_supported(dn);
  if (!tc) up.nt = dn.nt = 32;
  // the tensor-memory dequant GEMM, with activations in its K order, wherever it
  // takes the shapes: 16 / 32-token tiles for decode batches, 64 for prefill
  bool dec = false;
  if (tc && (flags & GEMQ_FWD_SMEM_DEQUANT) == 0) {
    GemmArgs u2 = up, d2 = dn;
    if (up.nt == kNtLarge) u2.nt = d2.nt = kNtMid;
    if (tcd_gemm_supported(u2) && tcd_gemm_supported(d2)) {
      dec = true;
      up.nt = dn.nt = u2.nt;
    }
  }
  if (dec) up.perm_out_nbits = L->w2.nbits;
  // Token tiles of 16 halve the MMA width. With at most 16 tokens no expert gets more
  // than 16 rows (a token picks an expert once); up to about 10 rows per expert on
  // average the few experts that need a second tile (and stream their weights twice)
  // cost less than the wider MMAs of 32-row tiles, measured on B200.
  if (dec && up.nt == kNtSmall && (T <= kNtTiny || P <= 10 * static_cast<int64_t>(E))) up.nt = dn.nt = kNtTiny;
  // Few slots per expert (well under three waves of work items): order the segments
  // by dequant cost so the decode GEMM's last wave holds its cheapest items. With
  // more waves a mix of bit-widths on the SMs at any time measured faster.
  const bool sort_segs = dec && P <= 2 * static_cast<int64_t>(E);
  // Chained launch: the down GEMM starts on the SMs the gate/up GEMM's CTAs leave and
  // takes each token tile once all of its gate/up items stored their h columns (the
  // counters are zeroed by the dispatch of this forward). With stage events between
  // the launches the down launch follows the gate/up completion and finds every
  // counter full. Decode batches only (16 / 32-token tiles, a few waves of items, where
  // the gate/up tail left SMs idle): measured on B200, the OLMoE decode stack 2-3%
  // faster, the Qwen3-shaped prefill (26 waves, 64-token tiles) 3% slower.
  const bool chain = dec && up.nt != kNtMid && (flags & GEMQ_FWD_NO_CHAIN) == 0;
  if (chain) {
    up.chain_done = dn.chain_done = b.tile_done;
    dn.chain_target = (F / 128) * 4;  // gate/up feature tiles x epilogue warps per tile
    if (flags & GEMQ_FWD_TEST_WAIT_EXPIRY) dn.chain_target = INT32_MAX;  // a count no tile reaches
  }
  tm.begin(GEMQ_STAGE_DISPATCH);
  GEMQ_CUDA(launch_dispatch(idx, w, x, T, k, E, D, up.nt, b.counts, b.cursor, b.segs, b.tile_prefix, b.slot_pos,
                            b.w_perm, b.x_perm, dec ? L->w1.nbits : nullptr, sort_segs ? L->w1.nbits : nullptr,
                            chain ? b.tile_done : nullptr, chain ? b.n_tile_done : 0, s),
            "dispatch");
  tm.end(GEMQ_STAGE_DISPATCH);
  tm.begin(GEMQ_STAGE_UP);
  if (dec) {
    GEMQ_CUDA(launch_tcd_gemm(up, s), "up projection");
  } else if (int rc = run_gemm(up, !tc, s, "up projection")) {
    return rc;
  }
  tm.end(GEMQ_STAGE_UP);
  tm.begin(GEMQ_STAGE_DOWN);
  if (dec) {
    GEMQ_CUDA(launch_tcd_gemm(dn, s), "down projection");
  } else if (int rc = run_gemm(dn, !tc, s, "down projection")) {
    return rc;
  }
  tm.end(GEMQ_STAGE_DOWN);
  const uint16_t* add = nullptr;
  if (d.has_shared) {
    const int Fs = L->shared_inter;
    GemmArgs su{};
    su.mode = GemmMode::kSwiGLU;
    su.w0 = L->sw1;
    su.w1 = L->sw3;
    su.act = x;
    su.act_rows = T;
    su.segs = b.one_seg;
    su.tile_prefix = b.one_tp;
    su.num_segs = 1;
    su.out = b.s_h;
    su.out_ld = Fs;
    su.out_cols = Fs;
    su.num_sms = L->num_sms;
    su.nt = choose_nt(T);
    GemmArgs sd = su;
    sd.mode = GemmMode::kStoreF16;
    sd.w0 = sd.w1 = L->sw2;
    sd.act = b.s_h;
    sd.out = b.s_out;
    sd.out_ld = D;
    sd.out_cols = D;
    const bool stc = !force_simt && tc_gemm_supported(su) && tc_gemm_supported(sd);
    if (!stc) su.nt = sd.nt = 32;
    tm.begin(GEMQ_STAGE_SHARED);
    GEMQ_CUDA(launch_build_index_segs(nullptr, 1, 1, T, su.nt, b.one_seg, b.one_tp, s), "shared segments");
    if (int rc = run_gemm(su, !stc, s, "shared up")) return rc;
    if (int rc = run_gemm(sd, !stc, s, "shared down")) return rc;
    tm.end(GEMQ_STAGE_SHARED);
    add = b.s_out;
  }
  tm.begin(GEMQ_STAGE_COMBINE);
  GEMQ_CUDA(launch_combine(b.y_perm, b.slot_pos, idx, T, k, D, (flags & GEMQ_FWD_FP32_COMBINE) != 0, add,
                           (flags & GEMQ_FWD_RESIDUAL) ? x : nullptr, out, s),
            "combine");
  tm.end(GEMQ_STAGE_COMBINE);
  return GEMQ_OK;
}

}  // namespace
}  // namespace gemq

extern "C" {

size_t gemq_moe_workspace_size(const gemq_layer_t* layer, int64_t num_tokens, uint32_t flags) {
  if (layer == nullptr || num_tokens < 0) return 0;
  return carve(layer, num_tokens, flags, nullptr, nullptr).bytes;
}

int gemq_moe_route(gemq_layer_t* layer, const uint16_t* x, int64_t num_tokens, void* logits, int32_t* topk_idx,
                   uint16_t* topk_w, uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_moe_route");
  if (layer == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null layer");
  if (num_tokens < 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "negative token count");
  if (num_tokens == 0) return GEMQ_OK;
  if (x == nullptr || logits == nullptr || topk_idx == nullptr || topk_w == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  Carver c(workspace);
  Seg* seg = c.take<Seg>(1);
  int32_t* tp = c.take<int32_t>(2);
  if (workspace == nullptr || workspace_bytes < c.off + 256) return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  return run_router(layer->d, layer->ro, layer->num_sms, x, num_tokens, logits,
                    (flags & GEMQ_FWD_GIVEN_LOGITS) != 0, topk_idx, topk_w, flags, seg, tp,
                    static_cast<cudaStream_t>(stream));
}

int gemq_moe_forward(gemq_layer_t* layer, const uint16_t* x, int64_t num_tokens, uint16_t* out, void* router_logits,
                     const int32_t* topk_idx, const uint16_t* topk_w, uint32_t flags, void* workspace,
                     size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_moe_forward");
  if (layer == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null layer");
  if (num_tokens < 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "negative token count");
  if (num_tokens == 0) return GEMQ_OK;  // empty batch: nothing to read or write (pointers may be null)
  if (x == nullptr || out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(GEMQ_ERR_UNSUPPORTED, "x and out must be 16-byte aligned");
  const bool one = (flags & GEMQ_FWD_ONE_TOKEN) != 0;
  if (one && num_tokens != 1)
    return fail(GEMQ_ERR_INVALID_ARGUMENT,
                "This function only supports single token forward (moe_block.py:825)");
  const bool given_routing = (flags & GEMQ_FWD_GIVEN_ROUTING) != 0;
  const bool given_logits = (flags & GEMQ_FWD_GIVEN_LOGITS) != 0;
  if (given_routing && (topk_idx == nullptr || topk_w == nullptr))
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "GEMQ_FWD_GIVEN_ROUTING needs topk_idx and topk_w");
  if (given_logits && router_logits == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "GEMQ_FWD_GIVEN_LOGITS needs router_logits");
  if (num_tokens * layer->d.top_k > INT32_MAX / 2) return fail(GEMQ_ERR_UNSUPPORTED, "too many tokens");
  FwdBufs b = carve(layer, num_tokens, flags, workspace, router_logits);
  if (workspace == nullptr || workspace_bytes < b.bytes) return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StageTimer tm(layer, s, flags);
  const int32_t* idx = topk_idx;
  const uint16_t* w = topk_w;
  if (!given_routing) {
    void* logits = (router_logits != nullptr) ? router_logits : b.logits;
    // the one-token path's chained GEMV counters are zeroed by the top-k launch
    const bool chain_gemv = one && (flags & GEMQ_FWD_NO_CHAIN) == 0;
    if (int rc = run_router(layer->d, layer->ro, layer->num_sms, x, num_tokens, logits, given_logits, b.topk_idx,
                            b.topk_w, flags, b.one_seg, b.one_tp, s, &tm, chain_gemv ? b.gemv_done : nullptr,
                            chain_gemv ? layer->d.top_k : 0))
      return rc;
    idx = b.topk_idx;
    w = b.topk_w;
  }
  if (one) return forward_one_token(layer, x, out, idx, w, flags, b, s, tm);
  return forward_n_tokens(layer, x, num_tokens, out, idx, w, flags, b, s, tm);
}

int gemq_route(const uint16_t* x, int64_t num_tokens, int32_t hidden, const uint16_t* gate_weight,
               int32_t num_experts, int32_t top_k, int32_t router, int32_t norm_topk_prob, uint32_t flags,
               void* logits, int32_t* topk_idx, uint16_t* topk_w, void* workspace, size_t workspace_bytes,
               void* stream) {
  const gemq_routing_t r{norm_topk_prob, 1, 1, 1.0f};
  return gemq_route_ex(x, num_tokens, hidden, gate_weight, num_experts, top_k, router, &r, flags, logits, topk_idx,
                       topk_w, workspace, workspace_bytes, stream);
}

int gemq_route_ex(const uint16_t* x, int64_t num_tokens, int32_t hidden, const uint16_t* gate_weight,
                  int32_t num_experts, int32_t top_k, int32_t router, const gemq_routing_t* routing, uint32_t flags,
                  void* logits, int32_t* topk_idx, uint16_t* topk_w, void* workspace, size_t workspace_bytes,
                  void* stream) {
  TraceRange trace("gemq_route");
  if (num_tokens < 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "negative token count");
  if (num_tokens == 0) return GEMQ_OK;
  if (x == nullptr || gate_weight == nullptr || logits == nullptr || topk_idx == nullptr || topk_w == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if (hidden <= 0 || hidden % 8 != 0) return fail(GEMQ_ERR_UNSUPPORTED, "hidden size must be a positive multiple of 8");
  if (num_experts <= 0 || num_experts > 256 || top_k <= 0 || top_k > num_experts || top_k > 16)
    return fail(GEMQ_ERR_UNSUPPORTED, "need 0 < top_k <= min(num_experts, 16), num_experts <= 256");
  if (router != GEMQ_ROUTER_FP16 && router != GEMQ_ROUTER_FP32)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "unknown router flavour");
  if (reinterpret_cast<uintptr_t>(x) & 15u) return fail(GEMQ_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const gemq_routing_t ro = routing ? *routing : gemq_routing_t{0, 1, 1, 1.0f};
  if (int rc = check_routing(ro, num_experts, top_k)) return rc;
  Carver c(workspace);
  Seg* seg = c.take<Seg>(1);
  int32_t* tp = c.take<int32_t>(2);
  static_assert(GEMQ_ROUTE_WORKSPACE_BYTES >= 256 + 8 + 256, "router workspace constant");
  if (workspace == nullptr || workspace_bytes < GEMQ_ROUTE_WORKSPACE_BYTES)
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  gemq_layer_desc_t d{};
  d.hidden = hidden;
  d.num_experts = num_experts;
  d.top_k = top_k;
  d.norm_topk_prob = ro.norm_topk_prob;
  d.router = router;
  d.gate_weight = gate_weight;
  return run_router(d, ro, device_sm_count(), x, num_tokens, logits, (flags & GEMQ_FWD_GIVEN_LOGITS) != 0, topk_idx,
                    topk_w, flags, seg, tp, static_cast<cudaStream_t>(stream));
}

int gemq_layer_set_routing(gemq_layer_t* layer, const gemq_routing_t* routing) {
  if (layer == nullptr || routing == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if (int rc = check_routing(*routing, layer->d.num_experts, layer->d.top_k)) return rc;
  layer->ro = *routing;
  layer->d.norm_topk_prob = routing->norm_topk_prob;
  return GEMQ_OK;
}

int gemq_moe_combine(const uint16_t* y, const int32_t* slot_row, const int32_t* topk_idx, int64_t num_tokens,
                     int32_t top_k, int32_t hidden, uint32_t flags, const uint16_t* residual, uint16_t* out,
                     void* stream) {
  TraceRange trace("gemq_moe_combine");
  if (num_tokens < 0 || top_k <= 0 || top_k > 16) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad token or top_k count");
  if (num_tokens == 0) return GEMQ_OK;
  if (y == nullptr || slot_row == nullptr || topk_idx == nullptr || out == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if (hidden <= 0 || hidden % 8 != 0) return fail(GEMQ_ERR_UNSUPPORTED, "hidden size must be a positive multiple of 8");
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15u)
    return fail(GEMQ_ERR_UNSUPPORTED, "y, out and residual must be 16-byte aligned");
  GEMQ_CUDA(launch_combine(y, slot_row, topk_idx, num_tokens, top_k, hidden, (flags & GEMQ_FWD_FP32_COMBINE) != 0,
                           nullptr, residual, out, static_cast<cudaStream_t>(stream)),
            "combine");
  return GEMQ_OK;
}

size_t gemq_dispatch_workspace_size(int64_t num_tokens, int32_t top_k, int32_t num_experts) {
  (void)num_tokens;
  (void)top_k;
  if (num_experts <= 0) return 0;
  Carver c(nullptr);
  c.take<int32_t>(num_experts);  // cursor
  c.take<Seg>(num_experts);
  c.take<int32_t>(num_experts + 1);
  return c.off + 256;
}

int gemq_moe_dispatch(const int32_t* topk_idx, const uint16_t* topk_w, const uint16_t* x, int64_t num_tokens,
                      int32_t top_k, int32_t num_experts, int32_t hidden, const int32_t* perm_nbits,
                      int32_t* expert_counts, int32_t* slot_row, uint16_t* w_rows, uint16_t* x_rows, void* workspace,
                      size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_moe_dispatch");
  if (num_tokens < 0 || top_k <= 0 || top_k > 16) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad token or top_k count");
  if (num_experts <= 0 || num_experts > 256) return fail(GEMQ_ERR_UNSUPPORTED, "num_experts must be in [1, 256]");
  if (hidden <= 0 || hidden % 8 != 0) return fail(GEMQ_ERR_UNSUPPORTED, "hidden size must be a positive multiple of 8");
  if (num_tokens * top_k > INT32_MAX / 2) return fail(GEMQ_ERR_UNSUPPORTED, "too many tokens");
  if (expert_counts == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_tokens == 0) {
    GEMQ_CUDA(cudaMemsetAsync(expert_counts, 0, sizeof(int32_t) * num_experts, s), "zero counts");
    return GEMQ_OK;
  }
  if (topk_idx == nullptr || topk_w == nullptr || x == nullptr || slot_row == nullptr || w_rows == nullptr ||
      x_rows == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x_rows)) & 15u)
    return fail(GEMQ_ERR_UNSUPPORTED, "x and x_rows must be 16-byte aligned");
  if (perm_nbits != nullptr && hidden % 128 != 0)
    return fail(GEMQ_ERR_UNSUPPORTED, "permuted rows need a hidden size that is a multiple of 128");
  if (workspace == nullptr || workspace_bytes < gemq_dispatch_workspace_size(num_tokens, top_k, num_experts))
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  Carver c(workspace);
  int32_t* cursor = c.take<int32_t>(num_experts);
  Seg* segs = c.take<Seg>(num_experts);
  int32_t* tp = c.take<int32_t>(num_experts + 1);
  GEMQ_CUDA(launch_dispatch(topk_idx, topk_w, x, num_tokens, top_k, num_experts, hidden, kNtLarge, expert_counts,
                            cursor, segs, tp, slot_row, w_rows, x_rows, perm_nbits, nullptr, nullptr, 0, s),
            "dispatch");
  return GEMQ_OK;
}

size_t gemq_moe_experts_workspace_size(const gemq_layer_t* layer, int64_t num_rows, int32_t num_groups) {
  if (layer == nullptr || num_rows < 0 || num_groups <= 0) return 0;
  const int n = num_groups * layer->d.num_experts;
  Carver c(nullptr);
  c.take<Seg>(n);
  c.take<int32_t>(n + 1);
  c.take<uint16_t>(static_cast<size_t>(num_rows > 0 ? num_rows : 1) * layer->d.inter);
  return c.off + 256;
}

}  // extern "C"

namespace gemq {
namespace {
// The two GEMMs of gemq_moe_experts for a layer, tile width and row order chosen the
// same way whatever the row counts, so that the row order a sender must use
// (gemq_moe_experts_row_order) depends on the layer alone.
void experts_args(const gemq_layer_t* layer, int32_t sm_budget, GemmArgs& up, GemmArgs& dn, bool& tc, bool& tmem) {
  const gemq_layer_desc_t& d = layer->d;
  up = GemmArgs{};
  up.mode = GemmMode::kSwiGLU;
  up.w0 = layer->w1;
  up.w1 = layer->w3;
  up.out_ld = d.inter;
  up.out_cols = d.inter;
  up.num_sms = (sm_budget > 0 && sm_budget < layer->num_sms) ? sm_budget : layer->num_sms;
  up.num_segs = 1;
  up.nt = kNtLarge;
  dn = up;
  dn.mode = GemmMode::kRouteWeight;
  dn.w0 = dn.w1 = layer->w2;
  dn.out_ld = d.hidden;
  dn.out_cols = d.hidden;
  up.act = dn.act = reinterpret_cast<const uint16_t*>(uintptr_t{256});  // alignment check only
  tc = tc_gemm_supported(up) && tc_gemm_supported(dn);
  GemmArgs u2 = up, d2 = dn;
  u2.nt = d2.nt = kNtMid;
  tmem = tc && tcd_gemm_supported(u2) && tcd_gemm_supported(d2);
}
}  // namespace
}  // namespace gemq

extern "C" {

int gemq_moe_experts_row_order(const gemq_layer_t* layer) {
  if (layer == nullptr) return 0;
  GemmArgs up, dn;
  bool tc = false, tmem = false;
  experts_args(layer, 0, up, dn, tc, tmem);
  return tmem ? 1 : 0;
}

int gemq_moe_experts(gemq_layer_t* layer, const uint16_t* rows, int64_t num_rows, const int32_t* group_counts,
                     int32_t num_groups, const uint16_t* row_weight, uint16_t* out, int32_t sm_budget,
                     uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("gemq_moe_experts");
  if (layer == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null layer");
  if (num_rows < 0 || num_groups <= 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad row or group count");
  if (num_rows == 0) return GEMQ_OK;
  if (num_rows > INT32_MAX / 2) return fail(GEMQ_ERR_UNSUPPORTED, "too many rows");
  const gemq_layer_desc_t& d = layer->d;
  const int E = d.num_experts;
  if (static_cast<int64_t>(num_groups) * E > 1024) return fail(GEMQ_ERR_UNSUPPORTED, "num_groups * experts > 1024");
  if (rows == nullptr || group_counts == nullptr || out == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  if ((reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(GEMQ_ERR_UNSUPPORTED, "rows and out must be 16-byte aligned");
  if (workspace == nullptr || workspace_bytes < gemq_moe_experts_workspace_size(layer, num_rows, num_groups))
    return fail(GEMQ_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = num_groups * E;
  Carver c(workspace);
  Seg* segs = c.take<Seg>(n);
  int32_t* tp = c.take<int32_t>(n + 1);
  uint16_t* h = c.take<uint16_t>(static_cast<size_t>(num_rows) * d.inter);
  GemmArgs up, dn;
  bool tc = false, tmem = false;
  experts_args(layer, sm_budget, up, dn, tc, tmem);
  const bool permuted = (flags & GEMQ_FWD_PERMUTED_ROWS) != 0;
  if (permuted != tmem)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, tmem ? "this layer takes rows in the tensor-memory GEMM's K order "
                                                  "(dispatch with perm_nbits, flag GEMQ_FWD_PERMUTED_ROWS)"
                                                : "this layer takes unpermuted rows");
  if (row_weight == nullptr && tmem) return fail(GEMQ_ERR_UNSUPPORTED, "the tensor-memory GEMM needs row weights");
  up.act = rows;
  up.act_rows = num_rows;
  up.segs = segs;
  up.tile_prefix = tp;
  up.num_segs = n;
  up.out = h;
  dn.mode = row_weight != nullptr ? GemmMode::kRouteWeight : GemmMode::kStoreF16;
  dn.act = h;
  dn.act_rows = num_rows;
  dn.segs = segs;
  dn.tile_prefix = tp;
  dn.num_segs = n;
  dn.out = out;
  dn.row_weight = row_weight;
  if (tmem) {
    // 16 / 32 / 64-token tiles by rows per segment, h written in w2's K order
    const int64_t per = num_rows / n;
    up.nt = per > 48 ? kNtMid : (per > 10 ? kNtSmall : kNtTiny);
    up.perm_out_nbits = layer->w2.nbits;
  } else {
    up.nt = tc ? choose_nt(num_rows / n) : 32;
  }
  dn.nt = up.nt;
  GEMQ_CUDA(launch_group_segs(group_counts, n, E, up.nt, segs, tp, s), "segments");
  if (tmem) {
    if (!tcd_gemm_supported(up) || !tcd_gemm_supported(dn)) return fail(GEMQ_ERR_UNSUPPORTED, "expert GEMM shape");
    GEMQ_CUDA(launch_tcd_gemm(up, s), "up projection");
    GEMQ_CUDA(launch_tcd_gemm(dn, s), "down projection");
    return GEMQ_OK;
  }
  if (int rc = run_gemm(up, !tc, s, "up projection")) return rc;
  return run_gemm(dn, !tc, s, "down projection");
}

int gemq_layer_stage_times(gemq_layer_t* layer, float* ms_out) {
  if (layer == nullptr || ms_out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  for (int st = 0; st < GEMQ_NUM_STAGES; ++st) ms_out[st] = 0.f;
  if (!layer->events_ready) return GEMQ_OK;
  for (int st = 0; st < GEMQ_NUM_STAGES; ++st) {
    if (!layer->stage_ran[st]) continue;
    GEMQ_CUDA(cudaEventSynchronize(layer->ev[2 * st + 1]), "stage event");
    GEMQ_CUDA(cudaEventElapsedTime(&ms_out[st], layer->ev[2 * st], layer->ev[2 * st + 1]), "stage time");
  }
  return GEMQ_OK;
}

int gemq_layer_dequant_forms(const gemq_layer_t* layer, int32_t* forms_out) {
  if (layer == nullptr || forms_out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null argument");
  forms_out[0] = layer->w1.sub_ok;
  forms_out[1] = layer->w3.sub_ok;
  forms_out[2] = layer->w2.sub_ok;
  return GEMQ_OK;
}

int gemq_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t rows, int32_t n, float eps, uint16_t* out,
                  void* stream) {
  TraceRange trace("gemq_rms_norm");
  if (rows < 0 || rows > INT32_MAX || n <= 0 || n % 8 != 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad rows or n");
  if (rows == 0) return GEMQ_OK;
  if (x == nullptr || weight == nullptr || out == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out)) &
       15u) != 0)
    return fail(GEMQ_ERR_UNSUPPORTED, "x, weight and out must start on a 16-byte boundary");
  GEMQ_CUDA(launch_rms_norm(x, weight, rows, n, eps, out, static_cast<cudaStream_t>(stream)), "rms norm");
  return GEMQ_OK;
}

int gemq_qk_norm_rope(const uint16_t* qkv, int64_t ld, int64_t rows, int32_t n, int32_t head_dim,
                      const uint16_t* q_norm_weight, const uint16_t* k_norm_weight, float eps, const uint16_t* cos,
                      const uint16_t* sin, uint16_t* q_out, uint16_t* k_out, uint16_t* k_cache, uint16_t* v_cache,
                      int32_t max_len, int64_t* cache_len, void* stream) {
  TraceRange trace("gemq_qk_norm_rope");
  if (rows < 0 || rows > INT32_MAX || n <= 0 || n % 8 != 0 || head_dim <= 0 || head_dim % 2 != 0 ||
      n % head_dim != 0 || ld < 2 * static_cast<int64_t>(n) || ld % 8 != 0)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad rows, n, head_dim or ld");
  if (rows == 0) return GEMQ_OK;
  if (qkv == nullptr || q_norm_weight == nullptr || k_norm_weight == nullptr || cos == nullptr || sin == nullptr ||
      q_out == nullptr || (k_out == nullptr && k_cache == nullptr))
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (k_cache != nullptr && (v_cache == nullptr || cache_len == nullptr || max_len <= 0 || rows != 1))
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "a cache write takes one row, both caches, max_len and the length");
  if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q_norm_weight) |
        reinterpret_cast<uintptr_t>(k_norm_weight)) & 15u) != 0)
    return fail(GEMQ_ERR_UNSUPPORTED, "qkv and the norm weights must start on a 16-byte boundary");
  GEMQ_CUDA(launch_qk_norm_rope(qkv, ld, rows, n, head_dim, q_norm_weight, k_norm_weight, eps, cos, sin, q_out, k_out,
                                k_cache, v_cache, max_len, cache_len, static_cast<cudaStream_t>(stream)),
            "q/k norm + rotary");
  return GEMQ_OK;
}

int gemq_decode_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int32_t heads,
                          int32_t max_len, int32_t head_dim, const int64_t* cache_len, float scale, uint16_t* out,
                          void* stream) {
  TraceRange trace("gemq_decode_attention");
  if (heads <= 0 || max_len <= 0 || head_dim <= 0 || head_dim > 256 || head_dim % 8 != 0 || max_len > 1 << 16)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad heads, max_len or head_dim (head_dim % 8 == 0, <= 256)");
  if (((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u) != 0)
    return fail(GEMQ_ERR_UNSUPPORTED, "k_cache and v_cache must start on a 16-byte boundary");
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || cache_len == nullptr || out == nullptr)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  GEMQ_CUDA(launch_decode_attention(q, k_cache, v_cache, heads, max_len, head_dim, cache_len, scale, out,
                                    static_cast<cudaStream_t>(stream)),
            "decode attention");
  return GEMQ_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free group GEMM
// gemq_dequant_group_gemm keeps its segment table and tile prefix in caller
// workspace. Hosts that cannot allocate device memory of their own (an
// inference server whose memory pool is fixed when it starts, a plugin running
// inside a host whose allocator it must not call, a caller with no cudaMalloc
// binding) use gemq_dequant_group_gemm_noalloc instead: the same table lives in
// the file-scope array below, part of the library's device image.
namespace gemq {
namespace {

constexpr int kNoallocMaxDevices = 64;
constexpr size_t kNoallocSegBytes = sizeof(Seg) * 1024;                    // segments [0, 1023)
constexpr size_t kNoallocScratchBytes = kNoallocSegBytes + sizeof(int32_t) * 1024;  // + tile prefix [0, 1023]
static_assert(GEMQ_NOALLOC_MAX_INDICES < 1024, "static scratch sized for 1023 indices");

// Every GPU that loads the library holds these 20 KiB until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoallocMaxDevices] = {};

// The device address of g_noalloc_scratch on the current device, looked up once
// per device (host code cannot use the symbol itself as a pointer).
int noalloc_scratch(void** out) {
  int dev = 0;
  GEMQ_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kNoallocMaxDevices) return fail(GEMQ_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    GEMQ_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(static scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return GEMQ_OK;
}

}  // namespace
}  // namespace gemq

extern "C" int gemq_dequant_group_gemm_noalloc(const gemq_proj_t* proj, const uint16_t* x, int64_t m,
                                               const int32_t* indices, int32_t num_indices, uint16_t* out,
                                               void* stream) {
  TraceRange trace("gemq_dequant_group_gemm_noalloc");
  if (int rc = check_proj(proj, "proj")) return rc;
  if (num_indices > GEMQ_NOALLOC_MAX_INDICES)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "num_indices " + std::to_string(num_indices) +
                                               " exceeds GEMQ_NOALLOC_MAX_INDICES (" +
                                               std::to_string(GEMQ_NOALLOC_MAX_INDICES) +
                                               "), the capacity of the library's static segment table");
  if (num_indices <= 0) return fail(GEMQ_ERR_INVALID_ARGUMENT, "num_indices must be positive");
  if (m < 0 || m > INT32_MAX / 2) return fail(GEMQ_ERR_INVALID_ARGUMENT, "bad m");
  if (static_cast<int64_t>(num_indices) * m > INT32_MAX)
    return fail(GEMQ_ERR_INVALID_ARGUMENT, "num_indices * m exceeds 2^31 - 1 output rows");
  if (m == 0) return GEMQ_OK;
  if (x == nullptr || out == nullptr || indices == nullptr) return fail(GEMQ_ERR_INVALID_ARGUMENT, "null pointer");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The segment kernel rewrites every entry the GEMM reads (segments [0, A) and
  // tile prefix [0, A]), so the previous call's contents need no clearing.
  Seg* segs = static_cast<Seg*>(scratch);
  int32_t* tp = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + kNoallocSegBytes);
  GemmArgs a{};
  a.mode = GemmMode::kStoreF16;
  a.w0 = to_dev(*proj);
  a.w1 = a.w0;
  a.act = x;
  a.act_rows = m;
  a.segs = segs;
  a.tile_prefix = tp;
  a.num_segs = num_indices;
  a.out = out;
  a.out_ld = proj->n;
  a.out_cols = proj->n;
  a.num_sms = device_sm_count();
  a.nt = choose_nt(m);
  if (!tc_gemm_supported(a)) a.nt = 32;
  GEMQ_CUDA(launch_build_index_segs(indices, num_indices, proj->num_experts, m, a.nt, segs, tp, s), "segments");
  return run_gemm(a, false, s, "dequant_group_gemm_noalloc");
}
