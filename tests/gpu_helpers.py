"""Helpers shared by the GPU tests: golden vectors -> CUDA tensors -> blocks."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import torch

from conftest import load_golden

PROJ_FIELDS = ("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides", "zs_strides")


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def proj_tensors(d: dict, prefix: str) -> dict:
    return {f: cuda(d[f"{prefix}_{f}"]) for f in PROJ_FIELDS}


def family_config(family: str, d: dict):
    D, F, k = int(d["D"]), int(d["F"]), int(d["top_k"])
    E = int(d["w1_nbits"].shape[0])
    norm = bool(d["norm_topk_prob"])
    if family == "mixtral":
        return SimpleNamespace(hidden_size=D, intermediate_size=F, num_local_experts=E, num_experts_per_tok=k)
    if family == "olmoe":
        return SimpleNamespace(hidden_size=D, intermediate_size=F, num_experts=E, num_experts_per_tok=k,
                               norm_topk_prob=norm)
    if family == "qwen3":
        return SimpleNamespace(hidden_size=D, moe_intermediate_size=F, num_experts=E, num_experts_per_tok=k,
                               norm_topk_prob=norm)
    return SimpleNamespace(hidden_size=D, moe_intermediate_size=F, n_routed_experts=E, n_shared_experts=2,
                           num_experts_per_tok=k, norm_topk_prob=norm, topk_method="greedy", scoring_func="softmax",
                           routed_scaling_factor=1.0)


def block_from_golden(family: str, d: dict = None):
    from robustgemq_b200.inference import moe_block as mb

    if d is None:
        d = load_golden(f"block_{family}.npz")
    cls = {"olmoe": mb.QuantFusedOlmoeMoEBlock, "qwen3": mb.QuantFusedQwen3MoeMoEBlock,
           "mixtral": mb.QuantFusedMixtralMoEBlock, "deepseek": mb.QuantFusedDeepseekV2MoEBlock}[family]
    blk = cls(family_config(family, d))
    blk.gate.weight.data = cuda(d["gate_w"])
    blk.gate.cuda().half()
    for name in ("w1", "w2", "w3"):
        for f, t in proj_tensors(d, name).items():
            setattr(blk, f"{name}_{f}", t)
    blk.block_group_size = int(d["group_size"])
    if family == "deepseek":
        for name in ("shared_w1", "shared_w2", "shared_w3"):
            for f in ("wq", "scales", "zeros"):
                setattr(blk, f"{name}_{f}", cuda(d[f"{name}_{f}"]))
        blk.shared_nbits = int(d["shared_w1_nbits"][0])
        blk.shared_group_size = int(d["shared_w1_group_sizes"][0])
    blk.invalidate()
    return blk, d
