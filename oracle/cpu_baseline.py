"""CPU fake-quant baseline: the reference's dequantise + torch-matmul path, timed.

TEST / BASELINE INFRASTRUCTURE ONLY: used by ``bench.py``'s ``cpu_baseline`` leg
and ``--impl reference`` arm, never by the product path.

Restates ``forward_n_tokens`` (gemq/inference/moe_block.py:781-815) with each hit
expert's packed weights dequantised to fp32 (``w = q*s + z'``, the math of
gemq/triton_kernels/utils.py:192-212) and ``F.linear`` in fp32 on all host cores.
Bytes are counted the way the GPU arm counts them: packed words + fp16 scales and
zeros of every hit expert, the fp16 gate weight, and fp16 activations in/out.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import gemq_oracle as O


@dataclass
class CpuLayer:
    D: int
    F: int
    E: int
    k: int
    gate: np.ndarray  # fp16 [E, D]
    w1: O.PackedProj
    w3: O.PackedProj
    w2: O.PackedProj
    norm: bool = False

    def expert_bytes(self, e: int) -> int:
        total = 0
        for p in (self.w1, self.w3, self.w2):
            rows = O.packed_rows(p.K, int(p.nbits[e]))
            total += 4 * rows * p.N + 2 * 2 * (p.K // p.group_size) * p.N
        return total


def _proj_np(blk, name: str, K: int) -> O.PackedProj:
    g = lambda a: getattr(blk, f"{name}_{a}").cpu().numpy()  # noqa: E731
    return O.PackedProj(wq=g("wq"), scales=g("scales"), zeros=g("zeros"), nbits=g("nbits"),
                        group_sizes=g("group_sizes"), wq_strides=g("wq_strides"), zs_strides=g("zs_strides"), K=K,
                        N=getattr(blk, f"{name}_wq").shape[1])


def layer_from_block(blk) -> CpuLayer:
    D, Fd = blk.hidden_dim, blk.ffn_dim
    return CpuLayer(D=D, F=Fd, E=blk.num_experts, k=blk.top_k, gate=blk.gate.weight.detach().cpu().numpy(),
                    w1=_proj_np(blk, "w1", D), w3=_proj_np(blk, "w3", D), w2=_proj_np(blk, "w2", Fd),
                    norm=blk.norm_topk_prob)


def synthetic_layer(seed: int = 0, D: int = 2048, Fd: int = 1024, E: int = 64, k: int = 8, g: int = 64) -> CpuLayer:
    """OLMoE-shaped layer with the bench's bit mix (mean 2.5: 5/8 two-bit, 1/4
    three-bit, 1/8 four-bit), random codes and RTN-like scales, built on the CPU."""
    rng = np.random.default_rng(seed)
    counts = {2: 40, 3: 16, 4: 8} if E == 64 else {2: E * 5 // 8, 3: E // 4, 4: E - E * 5 // 8 - E // 4}
    bits = [b for b, c in counts.items() for _ in range(c)]
    rng.shuffle(bits)

    def proj(K, N):
        codes, scs, zes = [], [], []
        for b in bits:
            codes.append(rng.integers(0, 2 ** b, size=(N, K), dtype=np.uint8))
            scs.append((0.1 / (2 ** b - 1) * (0.75 + 0.5 * rng.random((N * K // g, 1)))).astype(np.float16))
            zes.append(rng.integers(0, 2 ** b, size=(N * K // g, 1)).astype(np.float16))
        return O.stack_projection(codes, scs, zes, bits, g, K, N)

    return CpuLayer(D=D, F=Fd, E=E, k=k, gate=(rng.standard_normal((E, D)) * 0.02).astype(np.float16),
                    w1=proj(D, Fd), w3=proj(D, Fd), w2=proj(Fd, D))


def dequant_fp32(p: O.PackedProj, e: int) -> np.ndarray:
    """Fake-quant weight ``[K, N]`` in fp32: ``q * s + z'`` (no fp16 rounding)."""
    nb = int(p.nbits[e])
    eps = O.elements_per_word(nb)
    rows = O.packed_rows(p.K, nb)
    w0 = int(p.wq_strides[e])
    words = p.wq.reshape(-1)[w0: w0 + rows * p.N].reshape(rows, p.N).view(np.uint32)
    q = np.empty((rows, eps, p.N), dtype=np.float32)
    for j in range(eps):
        q[:, j, :] = (words >> np.uint32(j * nb)) & np.uint32((1 << nb) - 1)
    q = q.reshape(rows * eps, p.N)[: p.K]
    ng = p.K // p.group_size
    z0 = int(p.zs_strides[e])
    s = p.scales.reshape(-1)[z0: z0 + ng * p.N].reshape(ng, 1, p.N).astype(np.float32)
    z = p.zeros.reshape(-1)[z0: z0 + ng * p.N].reshape(ng, 1, p.N).astype(np.float32)
    return (q.reshape(ng, p.group_size, p.N) * s + z).reshape(p.K, p.N)


def dequant_fp32_torch(p: O.PackedProj, e: int) -> torch.Tensor:
    """``dequant_fp32`` with torch CPU ops (which use all the host threads torch is given)."""
    nb = int(p.nbits[e])
    eps = O.elements_per_word(nb)
    rows = O.packed_rows(p.K, nb)
    w0 = int(p.wq_strides[e])
    words = torch.from_numpy(p.wq.reshape(-1)[w0: w0 + rows * p.N].reshape(rows, p.N).view(np.int32).astype(np.int64))
    words = words & 0xFFFFFFFF
    shifts = torch.arange(eps, dtype=torch.int64).view(1, eps, 1) * nb
    q = ((words.view(rows, 1, p.N) >> shifts) & ((1 << nb) - 1)).reshape(rows * eps, p.N)[: p.K].float()
    ng = p.K // p.group_size
    z0 = int(p.zs_strides[e])
    s = torch.from_numpy(p.scales.reshape(-1)[z0: z0 + ng * p.N].reshape(ng, 1, p.N).astype(np.float32))
    z = torch.from_numpy(p.zeros.reshape(-1)[z0: z0 + ng * p.N].reshape(ng, 1, p.N).astype(np.float32))
    return (q.view(ng, p.group_size, p.N) * s + z).reshape(p.K, p.N)


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def block_prefill(layer: CpuLayer, x: torch.Tensor, weights=None) -> torch.Tensor:
    """``forward_n_tokens`` (moe_block.py:781-815) in fp32 on the CPU: router, then per hit
    expert (ascending id) SwiGLU with ``F.linear``-equivalent matmuls and ``index_add_``.
    ``weights`` maps expert -> (W1, W3, W2) fp32 already dequantised (the matmul-only
    leg); without it every hit expert is dequantised inside the call."""
    logits = x @ torch.from_numpy(layer.gate.astype(np.float32)).T
    p = torch.softmax(logits, dim=-1)
    w, idx = torch.topk(p, layer.k, dim=-1)
    if layer.norm:
        w = w / w.sum(dim=-1, keepdim=True)
    out = torch.zeros_like(x)
    for e in torch.unique(idx).tolist():
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        if weights is not None:
            W1, W3, W2 = weights[e]
        else:
            W1, W3, W2 = (dequant_fp32_torch(layer.w1, e), dequant_fp32_torch(layer.w3, e),
                          dequant_fp32_torch(layer.w2, e))
        xe = x[tok]
        h = F.silu(xe @ W1) * (xe @ W3)
        out.index_add_(0, tok, (h @ W2) * w[tok, slot, None])
    return out


def time_block_prefill(layer: CpuLayer, x: np.ndarray, reps: int = 3) -> dict:
    """Config 0 on the host: one OLMoE-shaped block over ``x`` [T, D] in fp32, timed
    twice: dequantise + matmul (weights dequantised inside every pass) and matmul only
    (weights dequantised once beforehand). Median of ``reps`` passes after a warm-up."""
    xt = torch.from_numpy(np.asarray(x, dtype=np.float32))
    T = xt.shape[0]
    flops = T * layer.k * 6 * layer.D * layer.F + 2 * T * layer.D * layer.E
    res = {}
    block_prefill(layer, xt)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        block_prefill(layer, xt)
        ts.append(time.perf_counter() - t0)
    res["dequant_matmul_ms"] = round(1e3 * float(np.median(ts)), 1)
    weights = {e: (dequant_fp32_torch(layer.w1, e), dequant_fp32_torch(layer.w3, e), dequant_fp32_torch(layer.w2, e))
               for e in range(layer.E)}
    block_prefill(layer, xt, weights)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        block_prefill(layer, xt, weights)
        ts.append(time.perf_counter() - t0)
    res["matmul_only_ms"] = round(1e3 * float(np.median(ts)), 1)
    res["dequant_matmul_tokens_per_s"] = round(T / (res["dequant_matmul_ms"] * 1e-3), 1)
    res["matmul_only_tokens_per_s"] = round(T / (res["matmul_only_ms"] * 1e-3), 1)
    res["matmul_only_gflops"] = round(flops / (res["matmul_only_ms"] * 1e-3) / 1e9, 1)
    return res


def decode_layer(layer: CpuLayer, x: np.ndarray) -> int:
    """One fake-quant forward of the layer on x [B, D]; returns the algorithmic bytes."""
    xt = torch.from_numpy(np.asarray(x, dtype=np.float32))
    logits = xt @ torch.from_numpy(layer.gate.astype(np.float32)).T
    p = torch.softmax(logits, dim=-1)
    w, idx = torch.topk(p, layer.k, dim=-1)
    if layer.norm:
        w = w / w.sum(dim=-1, keepdim=True)
    out = torch.zeros_like(xt)
    hit = torch.unique(idx).tolist()
    for e in hit:
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        W1 = dequant_fp32_torch(layer.w1, e)
        W3 = dequant_fp32_torch(layer.w3, e)
        W2 = dequant_fp32_torch(layer.w2, e)
        xe = xt[tok]
        h = F.silu(xe @ W1) * (xe @ W3)
        out.index_add_(0, tok, (h @ W2) * w[tok, slot, None])
    B = x.shape[0]
    return sum(layer.expert_bytes(e) for e in hit) + layer.E * layer.D * 2 + 3 * B * layer.D * 2


def time_decode(layer: CpuLayer, xs: dict, seconds: float) -> dict:
    """Cycle batch sizes until ``seconds`` of CPU work; GB/s over the whole sample."""
    torch.set_num_threads(torch.get_num_threads())
    batches = sorted(xs)
    decode_layer(layer, xs[batches[0]])  # warm-up
    t0 = time.perf_counter()
    total = 0
    passes = 0
    while True:
        B = batches[passes % len(batches)]
        total += decode_layer(layer, xs[B])
        passes += 1
        if time.perf_counter() - t0 > seconds and passes >= len(batches):
            break
    dt = time.perf_counter() - t0
    return {"value": round(total / dt / 1e9, 4), "unit": "GB/s", "kind": "port",
            "sample": f"{passes} single-layer fake-quant decode passes (batches {batches}) of one OLMoE-shaped "
                      f"layer of the benchmarked stack: dequantise hit experts to fp32 + torch matmul, {dt:.1f} s"}
