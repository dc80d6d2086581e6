"""Seeded synthetic MoE layers for benchmarks and large-shape tests (built on the GPU).

Bit mixes use exact counts that hit the mean bit-width, permuted per layer by a
seeded generator (mean 2.5 -> {2: 5/8, 3: 1/4, 4: 1/8} of E; 2.75 -> {2: 1/2,
3: 1/4, 4: 1/4}; 3.0 -> {2: 1/4, 3: 1/2, 4: 1/4}). Weights are N(0, 0.02) in
fp16, quantised per group with the reference's min-max RTN and stored in the
packed layout of ``quant.PackedLinear`` / ``QuantFused*.from_hf``.
"""

from __future__ import annotations

from types import SimpleNamespace
from typing import Dict, List, Optional

import torch

from .quant import PackedLinear, pack_linear, rtn_quantize

BIT_MIX = {
    2.5: {2: 5 / 8, 3: 1 / 4, 4: 1 / 8},
    2.75: {2: 1 / 2, 3: 1 / 4, 4: 1 / 4},
    3.0: {2: 1 / 4, 3: 1 / 2, 4: 1 / 4},
}


def bit_mix(num_experts: int, mean_bits: float, seed: int) -> List[int]:
    frac = BIT_MIX[mean_bits]
    counts = {b: int(round(f * num_experts)) for b, f in frac.items()}
    counts[2] += num_experts - sum(counts.values())
    bits = [b for b, c in sorted(counts.items()) for _ in range(c)]
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_experts, generator=g).tolist()
    return [bits[i] for i in perm]


def random_packed_linear(out_features: int, in_features: int, nbits: int, group_size: int, gen: torch.Generator,
                         device) -> PackedLinear:
    """N(0, 0.02) fp16 weights, min-max RTN per group along the input dim, packed."""
    W = (torch.randn((out_features, in_features), generator=gen, device=device) * 0.02).half()
    Q, s, z = rtn_quantize(W, nbits, group_size)
    return pack_linear(Q, s, z, nbits, group_size)


def random_block(family_cls, config, hidden: int, inter: int, num_experts: int, mean_bits: float, group_size: int,
                 seed: int, device, shared_inter: int = 0, shared_bits: int = 4):
    """A QuantFused* block with synthetic packed experts (and DeepSeek shared experts)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    bits = bit_mix(num_experts, mean_bits, seed)
    w1 = [random_packed_linear(inter, hidden, b, group_size, gen, device) for b in bits]
    w3 = [random_packed_linear(inter, hidden, b, group_size, gen, device) for b in bits]
    w2 = [random_packed_linear(hidden, inter, b, group_size, gen, device) for b in bits]
    gate = (torch.randn((num_experts, hidden), generator=gen, device=device) * 0.02).half()
    shared = None
    if shared_inter:
        shared = (random_packed_linear(shared_inter, hidden, shared_bits, group_size, gen, device),
                  random_packed_linear(shared_inter, hidden, shared_bits, group_size, gen, device),
                  random_packed_linear(hidden, shared_inter, shared_bits, group_size, gen, device))
    blk = family_cls.from_packed(config, gate, w1, w3, w2, shared=shared)
    blk.gate.to(device)
    blk.bits = bits
    return blk


def random_block_experts(family_cls, config, hidden: int, inter: int, num_experts: int, mean_bits: float,
                         group_size: int, seed: int, device, experts=None):
    """A block holding only ``experts`` (default: all) of a synthetic layer whose experts
    are each drawn from their own generator (seed, expert), so any subset, on any rank,
    equals the same experts of the whole layer. The config's expert count must match
    ``len(experts)``; the gate ``[num_experts, hidden]`` of the whole layer is returned
    beside the block."""
    experts = list(range(num_experts)) if experts is None else list(experts)
    bits = bit_mix(num_experts, mean_bits, seed)
    w1, w3, w2 = [], [], []
    for e in experts:
        gen = torch.Generator(device=device).manual_seed(seed * 100003 + e)
        w1.append(random_packed_linear(inter, hidden, bits[e], group_size, gen, device))
        w3.append(random_packed_linear(inter, hidden, bits[e], group_size, gen, device))
        w2.append(random_packed_linear(hidden, inter, bits[e], group_size, gen, device))
    g = torch.Generator(device=device).manual_seed(seed * 100003 + num_experts)
    gate = (torch.randn((num_experts, hidden), generator=g, device=device) * 0.02).half()
    blk = family_cls.from_packed(config, gate[experts[0]:experts[0] + len(experts)], w1, w3, w2)
    blk.gate.to(device)
    blk.bits = [bits[e] for e in experts]
    return blk, gate


# ----------------------------------------------------------------------------- configs
def olmoe_config():
    """OLMoE-1B-7B-shaped block (BASELINE configs 0/1)."""
    return SimpleNamespace(hidden_size=2048, intermediate_size=1024, num_experts=64, num_experts_per_tok=8,
                           norm_topk_prob=False), dict(hidden=2048, inter=1024, num_experts=64, mean_bits=2.5,
                                                       group_size=64)


def qwen3_config():
    """Qwen3-30B-A3B-shaped block."""
    return SimpleNamespace(hidden_size=2048, moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
                           norm_topk_prob=True), dict(hidden=2048, inter=768, num_experts=128, mean_bits=2.5,
                                                      group_size=128)


def deepseek_config():
    """DeepSeek-V2-Lite-shaped block: 2 shared experts = one 2816-wide SwiGLU."""
    return SimpleNamespace(hidden_size=2048, moe_intermediate_size=1408, n_routed_experts=64, n_shared_experts=2,
                           num_experts_per_tok=6, norm_topk_prob=False, topk_method="greedy",
                           scoring_func="softmax", routed_scaling_factor=1.0), dict(
        hidden=2048, inter=1408, num_experts=64, mean_bits=2.75, group_size=64, shared_inter=2816)


def mixtral_config():
    """Mixtral-8x7B-shaped block."""
    return SimpleNamespace(hidden_size=4096, intermediate_size=14336, num_local_experts=8,
                           num_experts_per_tok=2), dict(hidden=4096, inter=14336, num_experts=8, mean_bits=3.0,
                                                        group_size=128)


def zipf_logits(tokens: int, num_experts: int, seed: int, device, s: float = 1.1, c: float = 2.0) -> torch.Tensor:
    """Router logits N(0, 1) + c * rank^-s over a seeded expert permutation (skewed load)."""
    g = torch.Generator(device=device).manual_seed(seed)
    perm = torch.randperm(num_experts, generator=g, device=device)
    bias = torch.empty(num_experts, device=device)
    bias[perm] = c * torch.arange(1, num_experts + 1, device=device, dtype=torch.float32).pow(-s)
    return torch.randn((tokens, num_experts), generator=g, device=device) + bias[None, :]


def expert_bytes(blk, e: int) -> int:
    """Packed words + fp16 scales/zeros of expert e across w1, w3, w2 (what a forward reads)."""
    total = 0
    for name in ("w1", "w3", "w2"):
        wq = getattr(blk, f"{name}_wq")
        strides = getattr(blk, f"{name}_wq_strides")
        n_words = (int(strides[e + 1]) if e + 1 < strides.numel() else wq.numel()) - int(strides[e])
        sc = getattr(blk, f"{name}_scales")
        total += 4 * n_words + 2 * 2 * (sc.numel() // blk.num_experts)
    return total


def layer_expert_bytes(blk) -> List[int]:
    cpu = SimpleNamespace(num_experts=blk.num_experts)
    for name in ("w1", "w3", "w2"):
        setattr(cpu, f"{name}_wq", getattr(blk, f"{name}_wq"))
        setattr(cpu, f"{name}_wq_strides", getattr(blk, f"{name}_wq_strides").cpu())
        setattr(cpu, f"{name}_scales", getattr(blk, f"{name}_scales"))
    return [expert_bytes(cpu, e) for e in range(blk.num_experts)]
