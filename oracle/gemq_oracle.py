"""CPU restatement of RobustGEMQ's real-quant mixed-bit MoE expert path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker (or the timed CPU baseline). The product path in
``robustgemq_b200`` never calls it.

Every function cites the reference file:line it restates (paths relative to the
reference project root). Integer work (pack / unpack / code extraction) is exact
numpy. The fp16 dequant ``w = fma(fp16(q), s, z')`` is restated exactly: fp16
values are integer multiples of 2**-24, so ``q*S + Z`` is formed in int64 and
rounded to fp16 once (``fma="single"``, the ``fma.rn.f16`` that ``tl.fma``
lowers to on NVIDIA GPUs). ``fma="double"`` restates the Triton CPU
interpreter's ``x*y + z`` in numpy float16 (two roundings); it exists only so
the restatement can be pinned bit-for-bit against interpreted reference
kernels. Matrix products are formed in float64 and rounded to the storage type
of the reference (fp16 outputs); the reference accumulates in fp32, so these
agree to within an fp16 rounding flip.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

F16 = np.float16
F32 = np.float32
F64 = np.float64


def elements_per_word(nbits: int) -> int:
    """Codes per int32 word: ``32 // nbits`` (utils.py:85, dequant_group_gemm.py:106)."""
    if nbits not in (1, 2, 3, 4):
        raise ValueError(f"unsupported bit-width {nbits}")
    return 32 // nbits


def packed_rows(K: int, nbits: int) -> int:
    """Words along K: ``cdiv(K, 32 // nbits)`` (utils.py:88)."""
    eps = elements_per_word(nbits)
    return (K + eps - 1) // eps


# --------------------------------------------------------------------------- packing
def pack_weights_over_cols(codes: np.ndarray, nbits: int, transpose: bool = True) -> np.ndarray:
    """uint8 codes ``[N, K]`` -> int32 words; restates utils.py:33-113.

    Word ``c`` of row ``n`` holds codes ``K[c*eps : c*eps+eps]`` with code ``j``
    at bits ``[j*nbits, j*nbits+nbits)`` (utils.py:54-66). A ragged tail (3-bit:
    ten codes per word and two high bits left zero) is zero-padded (utils.py:55,63).
    The reference returns the transposed view ``[cdiv(K, eps), N]`` (utils.py:110-111).
    """
    codes = np.asarray(codes)
    if codes.ndim != 2:
        raise ValueError("codes must be 2-D [N, K]")
    N, K = codes.shape
    eps = elements_per_word(nbits)
    ncols = packed_rows(K, nbits)
    padded = np.zeros((N, ncols * eps), dtype=np.uint64)
    padded[:, :K] = codes.astype(np.uint64) & ((1 << nbits) - 1)
    padded = padded.reshape(N, ncols, eps)
    shifts = (np.arange(eps, dtype=np.uint64) * np.uint64(nbits))
    words = np.bitwise_or.reduce(padded << shifts, axis=2).astype(np.uint32).view(np.int32)
    return words.T if transpose else words


def unpack_over_cols(packed: np.ndarray, nbits: int, num_output_cols: int) -> np.ndarray:
    """int32 words ``[rows, cols]`` -> uint8 codes ``[rows, num_output_cols]``; restates utils.py:116-189.

    ``out[r, c] = (packed[r, c // eps] >> ((c % eps) * nbits)) & mask`` (utils.py:134-142).
    """
    packed = np.asarray(packed).astype(np.int32)
    eps = elements_per_word(nbits)
    c = np.arange(num_output_cols)
    words = packed[:, c // eps].view(np.uint32)
    shifts = ((c % eps) * nbits).astype(np.uint32)
    return ((words >> shifts) & np.uint32((1 << nbits) - 1)).astype(np.uint8)


# --------------------------------------------------------------------------- dequant
def fma_f16(q: np.ndarray, s: np.ndarray, z: np.ndarray, fma: str = "single") -> np.ndarray:
    """``fma(float16(q), s, z)`` from utils.py:206-210.

    ``single``: exact ``q*s + z`` rounded once to fp16. fp16 numbers are integer
    multiples of 2**-24, so ``q*S + Z`` (S = s*2**24, Z = z*2**24) is exact in
    int64 (|.| < 2**45) and exact again in float64 before the one rounding.
    ``double``: numpy float16 ``q*s`` then ``+ z`` exactly as the Triton CPU
    interpreter evaluates ``tl.fma`` (two roundings).
    """
    q = np.asarray(q)
    s = np.asarray(s, dtype=F16)
    z = np.asarray(z, dtype=F16)
    if fma == "double":
        return (q.astype(F16) * s) + z
    if fma != "single":
        raise ValueError(fma)
    S = (s.astype(F64) * 2.0 ** 24).astype(np.int64)
    Z = (z.astype(F64) * 2.0 ** 24).astype(np.int64)
    exact = q.astype(np.int64) * S + Z
    return (exact.astype(F64) * 2.0 ** -24).astype(F16)


@dataclass
class PackedProj:
    """One stacked projection of a QuantFused block (moe_block.py:725-757).

    ``wq``: int32 ``[sum_e cdiv(K, eps_e), N]`` row-major; ``scales``/``zeros``:
    fp16 ``[E*K/g, N]`` with the additive zero ``z' = -zero*scale``;
    ``wq_strides``/``zs_strides``: exclusive cumsum of per-expert numel
    (moe_block.py:751-757).
    """

    wq: np.ndarray
    scales: np.ndarray
    zeros: np.ndarray
    nbits: np.ndarray
    group_sizes: np.ndarray
    wq_strides: np.ndarray
    zs_strides: np.ndarray
    K: int
    N: int

    @property
    def num_experts(self) -> int:
        return int(self.nbits.shape[0])

    @property
    def group_size(self) -> int:
        g = np.unique(self.group_sizes)
        if g.size != 1:
            raise ValueError("group sizes must be the same across all experts (moe_block.py:745-749)")
        return int(g[0])


def dequantize_expert(proj: PackedProj, e: int, fma: str = "single") -> np.ndarray:
    """Dequantised weight ``[K, N]`` fp16 of expert ``e``.

    Addressing follows dequant_group_gemm.py:71-81,118-130: the expert's words
    start at element ``wq_strides[e]`` with row stride N; code ``(k, n)`` sits in
    word row ``k // eps`` at shift ``(k % eps) * nbits``; scale/zero row ``k // g``
    starting at element ``zs_strides[e]``.

    ``single`` (the GPU's ``fma.rn.f16``): every fp16 value is an integer multiple
    of 2**-24 below 2**16, and the code is below 2**4, so ``q*s + z`` spans at
    most 45 bits and is exact in float64; the one rounding is the float64 -> fp16
    conversion (round to nearest even), the same result as ``fma_f16``.
    """
    nb = int(proj.nbits[e])
    g = int(proj.group_sizes[e])
    eps = elements_per_word(nb)
    K, N = proj.K, proj.N
    rows = packed_rows(K, nb)
    w0 = int(proj.wq_strides[e])
    words = proj.wq.reshape(-1)[w0: w0 + rows * N].reshape(rows, N).view(np.uint32)
    shifts = (np.arange(eps, dtype=np.uint32) * np.uint32(nb))[None, :, None]
    # code k = r*eps + j of word row r sits at bit j*nb (utils.py:134-142)
    q = ((words[:, None, :] >> shifts) & np.uint32((1 << nb) - 1)).reshape(rows * eps, N)[:K]
    ng = K // g
    z0 = int(proj.zs_strides[e])
    s = proj.scales.reshape(-1)[z0: z0 + ng * N].reshape(ng, 1, N)
    z = proj.zeros.reshape(-1)[z0: z0 + ng * N].reshape(ng, 1, N)
    qg = q.reshape(ng, g, N)
    if fma == "double":
        return fma_f16(qg, s, z, fma).reshape(K, N)
    if fma != "single":
        raise ValueError(fma)
    w = qg.astype(F64) * s.astype(F64) + z.astype(F64)
    return w.reshape(K, N).astype(F16)


def matmul_f16_out(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """fp16 x fp16 product with wide accumulation, rounded to fp16 (dequant_group_gemm.py:133-138)."""
    return (np.asarray(a).astype(F64) @ np.asarray(b).astype(F64)).astype(F16)


# --------------------------------------------------------------------------- kernel-level mirrors
def dequant_group_gemm(x: np.ndarray, indices: Sequence[int], proj: PackedProj, fma: str = "single") -> np.ndarray:
    """``out[a] = x @ deq(W[indices[a]])`` -> fp16 ``[A, M, N]``; restates dequant_group_gemm.py:155-202."""
    return np.stack([matmul_f16_out(x, dequantize_expert(proj, int(e), fma)) for e in indices])


def dequant_gemm(x: np.ndarray, proj: PackedProj, fma: str = "single") -> np.ndarray:
    """Single packed weight (shared experts): dequant_gemm.py:150-193."""
    return matmul_f16_out(x, dequantize_expert(proj, 0, fma))


def dequant_gemv(x: np.ndarray, proj: PackedProj, fma: str = "single") -> np.ndarray:
    """Batch-1 GEMV of dequant_gemv.py:118-156.

    The reference sums split-K partials with fp16 atomics in arrival order
    (dequant_gemv.py:115,137), so its output varies run to run; the restatement
    rounds the exact sum once, the centre of that spread.
    """
    return matmul_f16_out(x, dequantize_expert(proj, 0, fma))


def silu_f32(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=F64)
    return (v / (1.0 + np.exp(-v))).astype(F32)


def fused_up_proj(x: np.ndarray, idx: Sequence[int], w1: PackedProj, w3: PackedProj, fma: str = "single"):
    """Decode gate/up for the selected experts; restates fused_dequant_bmm.py:25-173.

    Returns ``x1, x3`` fp16 ``[1, A*N]``: fp32-accumulated dot products stored to
    fp16 buffers (fused_dequant_bmm.py:93,111,118-119,152-153). w3 is addressed
    with w1's nbits/strides (fused_dequant_bmm.py:55-57,98), which
    ``check_w1_w3_aligned`` makes safe.
    """
    x = np.asarray(x).reshape(1, -1)
    x1 = np.concatenate([matmul_f16_out(x, dequantize_expert(w1, int(e), fma)) for e in idx], axis=1)
    x3 = np.concatenate([matmul_f16_out(x, dequantize_expert(w3, int(e), fma)) for e in idx], axis=1)
    return x1, x3


def fused_down_proj(x1: np.ndarray, x3: np.ndarray, idx: Sequence[int], w2: PackedProj, fma: str = "single"):
    """Decode down projection; restates fused_dequant_bmm.py:181-312.

    ``h = silu(fp32(x1)) * fp32(x3)`` stays fp32 (fused_dequant_bmm.py:237-239);
    the product with the dequantised fp16 weight is accumulated in fp32 and stored
    as fp16 (fused_dequant_bmm.py:255,261,292).
    """
    A = len(idx)
    K = w2.K
    x1 = np.asarray(x1).reshape(A, K)
    x3 = np.asarray(x3).reshape(A, K)
    outs = []
    for a, e in enumerate(idx):
        h = silu_f32(x1[a].astype(F32)).astype(F64) * x3[a].astype(F64)
        h = h.astype(F32)
        outs.append((h.astype(F64)[None, :] @ dequantize_expert(w2, int(e), fma).astype(F64)).astype(F16))
    return np.concatenate(outs, axis=1)


# --------------------------------------------------------------------------- routing
def softmax_f32(logits: np.ndarray) -> np.ndarray:
    v = np.asarray(logits, dtype=F64)
    v = v - v.max(axis=-1, keepdims=True)
    ev = np.exp(v)
    return (ev / ev.sum(axis=-1, keepdims=True)).astype(F32)


def topk_desc(values: np.ndarray, k: int):
    """Top-k along the last axis, descending; equal values keep the lower index first."""
    order = np.argsort(-np.asarray(values, dtype=F64), axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(values, order, axis=-1), order


@dataclass
class Routing:
    logits: np.ndarray      # [T, E] (fp16, or fp32 for the DeepSeek router)
    topk_idx: np.ndarray    # [T, k] int64
    topk_w: np.ndarray      # [T, k] fp16


def group_limit(p: np.ndarray, n_group: int, topk_group: int) -> np.ndarray:
    """DeepSeek-V2's group-limited greedy mask (transformers
    ``DeepseekV2Moe.route_tokens_to_experts``, ``topk_method == "group_limited_greedy"``):
    each of the ``n_group`` groups of consecutive experts is scored by its largest
    probability, the ``topk_group`` best groups are kept (lower group id first on
    ties), and every other expert's probability is replaced by 0.0 (``masked_fill``)."""
    T, E = p.shape
    gs = p.reshape(T, n_group, E // n_group).max(axis=-1)
    _, keep = topk_desc(gs, topk_group)
    mask = np.zeros((T, n_group), dtype=bool)
    np.put_along_axis(mask, keep, True, axis=-1)
    return np.where(np.repeat(mask, E // n_group, axis=-1), p, np.zeros_like(p))


def route(x: np.ndarray, gate_w: Optional[np.ndarray], top_k: int, norm_topk_prob: bool,
          router_fp32: bool = False, logits: Optional[np.ndarray] = None,
          softmax_fp16: bool = False, n_group: int = 1, topk_group: int = 1,
          scale: float = 1.0) -> Routing:
    """Router of forward_n_tokens / forward_one_token.

    fp16 logits ``x @ Wg^T`` (moe_block.py:790,828); DeepSeek forms them in fp32
    (moe_block.py:549,591). Softmax in fp32 (moe_block.py:792), top-k, renormalise
    when ``norm_topk_prob`` (moe_block.py:794-795), cast to fp16 (moe_block.py:797).
    ``softmax_fp16`` restates Mixtral's one-token router, whose softmax, top-k and
    renormalisation run on fp16 tensors (moe_block.py:280-283).
    ``logits`` may be given directly (the skewed-load benchmark configs).
    Beyond the reference's fused block, which rejects them (moe_block.py:18-66):
    ``n_group > 1`` restricts the top-k to the best groups (``group_limit``), and
    without renormalisation the weights are multiplied by ``scale`` in fp32
    (``routed_scaling_factor``, as the HF and official DeepSeek gates do) before the
    fp16 cast.
    """
    if logits is None:
        if router_fp32:
            logits = (np.asarray(x, F64) @ np.asarray(gate_w, F64).T).astype(F32)
        else:
            logits = matmul_f16_out(x, np.asarray(gate_w).T)
    if softmax_fp16:
        p = softmax_f32(logits.astype(F32)).astype(F16)
        w, idx = topk_desc(p, top_k)
        if norm_topk_prob:
            ssum = w.astype(F64).sum(axis=-1, keepdims=True).astype(F16)
            w = (w.astype(F64) / ssum.astype(F64)).astype(F16)
        return Routing(logits, idx.astype(np.int64), w.astype(F16))
    p = softmax_f32(logits.astype(F32))
    if n_group > 1:
        p = group_limit(p, n_group, topk_group)
    w, idx = topk_desc(p, top_k)
    if norm_topk_prob:
        w = (w.astype(F64) / w.astype(F64).sum(axis=-1, keepdims=True)).astype(F32)
    elif scale != 1.0:
        w = (w.astype(F32) * F32(scale)).astype(F32)
    return Routing(logits, idx.astype(np.int64), w.astype(F16))


# --------------------------------------------------------------------------- block forward
@dataclass
class BlockWeights:
    """Packed MoE block: the attribute set of QuantFused*MoEBlock (moe_block.py:688-761)."""

    gate_w: np.ndarray            # fp16 [E, D]
    w1: PackedProj                # gate_proj  [D -> F]
    w3: PackedProj                # up_proj    [D -> F]
    w2: PackedProj                # down_proj  [F -> D]
    top_k: int
    norm_topk_prob: bool
    router_fp32: bool = False     # DeepSeek (moe_block.py:549)
    shared_w1: Optional[PackedProj] = None   # DeepSeek shared experts (moe_block.py:477-489)
    shared_w3: Optional[PackedProj] = None
    shared_w2: Optional[PackedProj] = None
    n_group: int = 1              # DeepSeek-V2 group-limited greedy (1 = greedy)
    topk_group: int = 1
    route_scale: float = 1.0      # routed_scaling_factor when not renormalising
    dequant_cache: dict = field(default_factory=dict)

    def deq(self, name: str, e: int, fma: str = "single") -> np.ndarray:
        key = (name, e, fma)
        if key not in self.dequant_cache:
            self.dequant_cache[key] = dequantize_expert(getattr(self, name), e, fma)
        return self.dequant_cache[key]


def expert_ffn_n_tokens(blk: BlockWeights, e: int, xe: np.ndarray, fma: str = "single") -> np.ndarray:
    """forward_single_expert (moe_block.py:763-779): fp16 x1, x3; ``F.silu(x1) * x3`` on fp16
    tensors (each op computed in fp32, rounded to fp16); fp16 x2."""
    x1 = matmul_f16_out(xe, blk.deq("w1", e, fma))
    x3 = matmul_f16_out(xe, blk.deq("w3", e, fma))
    h = (silu_f32(x1.astype(F32)).astype(F16).astype(F32) * x3.astype(F32)).astype(F16)
    return matmul_f16_out(h, blk.deq("w2", e, fma))


def shared_ffn(blk: BlockWeights, x: np.ndarray, fma: str = "single") -> np.ndarray:
    """DeepSeek shared experts via dequant_gemm (moe_block.py:511-522): same fp16 rounding points."""
    x1 = matmul_f16_out(x, blk.deq("shared_w1", 0, fma))
    x3 = matmul_f16_out(x, blk.deq("shared_w3", 0, fma))
    h = (silu_f32(x1.astype(F32)).astype(F16).astype(F32) * x3.astype(F32)).astype(F16)
    return matmul_f16_out(h, blk.deq("shared_w2", 0, fma))


def moe_forward_n_tokens(blk: BlockWeights, x: np.ndarray, routing: Optional[Routing] = None,
                         fma: str = "single"):
    """forward_n_tokens (moe_block.py:781-815; DeepSeek 540-578).

    Experts are visited in ascending id order (``expert_hit`` from ``nonzero``,
    moe_block.py:807). Each expert's fp16 output is multiplied by its fp16 routing
    weight (fp16 result) and ``index_add_``-ed into an fp16 accumulator that starts
    at zero (moe_block.py:799-812), so every token's sum is rounded to fp16 after
    each expert, in ascending expert order. DeepSeek then adds the shared experts
    in fp16 (moe_block.py:575). Returns ``(out[T, D] fp16, routing)``.
    """
    x = np.asarray(x, dtype=F16)
    T, D = x.shape
    if routing is None:
        routing = route(x, blk.gate_w, blk.top_k, blk.norm_topk_prob, blk.router_fp32, n_group=blk.n_group,
                        topk_group=blk.topk_group, scale=blk.route_scale)
    out = np.zeros((T, D), dtype=F16)
    idx = routing.topk_idx
    for e in np.unique(idx):
        tok, slot = np.nonzero(idx == e)
        y = expert_ffn_n_tokens(blk, int(e), x[tok], fma)
        yw = (y.astype(F32) * routing.topk_w[tok, slot].astype(F32)[:, None]).astype(F16)
        out[tok] = (out[tok].astype(F32) + yw.astype(F32)).astype(F16)
    if blk.shared_w1 is not None:
        out = (out.astype(F32) + shared_ffn(blk, x, fma).astype(F32)).astype(F16)
    return out, routing


def moe_forward_one_token(blk: BlockWeights, x: np.ndarray, routing: Optional[Routing] = None,
                          fma: str = "single", mixtral: bool = False):
    """forward_one_token (moe_block.py:817-853; Mixtral 269-304; DeepSeek 580-623).

    x1/x3 from fused_up_proj (fp16), x2 from fused_down_proj (fp32 SiLU*mul, fp16
    store), then ``einsum("tai,ta->ti")`` of fp16 x2 with fp16 weights: one fp32
    sum rounded to fp16. DeepSeek adds shared experts computed by split-K GEMVs
    with fp16 ``F.silu(x1) * x3`` (moe_block.py:617-620), added in fp16.
    """
    x = np.asarray(x, dtype=F16).reshape(1, -1)
    if routing is None:
        routing = route(x, blk.gate_w, blk.top_k, blk.norm_topk_prob or mixtral, blk.router_fp32,
                        softmax_fp16=mixtral, n_group=blk.n_group, topk_group=blk.topk_group,
                        scale=blk.route_scale)
    idx = [int(e) for e in routing.topk_idx[0]]
    x1, x3 = fused_up_proj(x, idx, blk.w1, blk.w3, fma)
    x2 = fused_down_proj(x1, x3, idx, blk.w2, fma).reshape(len(idx), -1)
    out = (routing.topk_w[0].astype(F64) @ x2.astype(F64)).astype(F16)[None, :]
    if blk.shared_w1 is not None:
        s1 = dequant_gemv(x, blk.shared_w1, fma)
        s3 = dequant_gemv(x, blk.shared_w3, fma)
        h = (silu_f32(s1.astype(F32)).astype(F16).astype(F32) * s3.astype(F32)).astype(F16)
        s2 = dequant_gemv(h, blk.shared_w2, fma)
        out = (out.astype(F32) + s2.astype(F32)).astype(F16)
    return out, routing


# --------------------------------------------------------------------------- synthetic producers
def rtn_quantize(W: np.ndarray, nbits: int, group_size: int):
    """Min-max asymmetric RTN along the input dim; restates rtn.py:15-55 (nbits >= 2)
    and rtn.py:36-40 (nbits == 1). Returns (Q [N, K] uint8, scale [N*K/g, 1], zero [N*K/g, 1])
    in the dtype of W (the reference quantises in the weight's dtype)."""
    W = np.asarray(W)
    dt = W.dtype
    N, K = W.shape
    Wg = W.reshape(-1, group_size).astype(F64)
    if nbits == 1:
        Q = (Wg >= 0).astype(F64)
        scales = (np.abs(Wg).mean(axis=1, keepdims=True) * 2).astype(dt)
        zeros = np.full_like(scales, 0.5)
        return Q.reshape(N, K).astype(np.uint8), scales, zeros
    max_int = 2 ** nbits - 1
    mx = Wg.max(axis=1, keepdims=True).astype(dt)
    mn = Wg.min(axis=1, keepdims=True).astype(dt)
    scales = (np.maximum((mx.astype(F32) - mn.astype(F32)).astype(dt), dt.type(1e-5)).astype(F32) / max_int).astype(dt)
    zeros = np.clip(-np.round((mn.astype(F32) / scales.astype(F32)).astype(dt).astype(F32)), 0, max_int).astype(dt)
    Q = np.clip(np.round((Wg.astype(dt).astype(F32) / scales.astype(F32)).astype(dt).astype(F32)) + zeros.astype(F32), 0, max_int)
    return Q.reshape(N, K).astype(np.uint8), scales, zeros


def kernel_scale_zero(scales: np.ndarray, zeros: np.ndarray, N: int, K: int, group_size: int):
    """(scale, zero) ``[N*K/g, 1]`` -> kernel layout ``[K/g, N]`` fp16 with the additive
    zero ``z' = fp16(-zero*scale)`` formed in fp32: the convention the reference's
    ``dequantize`` assumes of GemLite's repack (test_quant_linear_equiv.py:6-9)."""
    s = np.asarray(scales, F32).reshape(N, K // group_size)
    z = np.asarray(zeros, F32).reshape(N, K // group_size)
    return s.T.astype(F16).copy(), (-(z * s)).T.astype(F16).copy()


def stack_projection(codes: Sequence[np.ndarray], scales: Sequence[np.ndarray], zeros: Sequence[np.ndarray],
                     nbits: Sequence[int], group_size: int, K: int, N: int) -> PackedProj:
    """Stack per-expert packed weights exactly as ``from_hf`` does (moe_block.py:725-757):
    ``torch.cat`` of each expert's ``[cdiv(K, eps), N]`` words and ``[K/g, N]`` meta,
    exclusive-cumsum numel offsets."""
    wqs = [np.ascontiguousarray(pack_weights_over_cols(c, int(b))) for c, b in zip(codes, nbits)]
    sz = [kernel_scale_zero(s, z, N, K, group_size) for s, z in zip(scales, zeros)]
    wq = np.concatenate(wqs, axis=0)
    sc = np.concatenate([a for a, _ in sz], axis=0)
    ze = np.concatenate([b for _, b in sz], axis=0)
    wq_strides = np.concatenate([[0], np.cumsum([w.size for w in wqs])[:-1]]).astype(np.int32)
    zs_strides = np.concatenate([[0], np.cumsum([a.size for a, _ in sz])[:-1]]).astype(np.int32)
    E = len(wqs)
    return PackedProj(wq=wq, scales=sc, zeros=ze, nbits=np.asarray(nbits, np.int32),
                      group_sizes=np.full(E, group_size, np.int32), wq_strides=wq_strides,
                      zs_strides=zs_strides, K=K, N=N)
