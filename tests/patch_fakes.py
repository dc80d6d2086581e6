"""Stand-ins for an HQQ-quantised HF model, for the model-patching tests.

``FakeHQQLinear`` has the part of hqq's ``HQQLinear`` interface that
``create_gemlite_from_hqq`` reads (gemq/inference/patch.py:27-50): ``meta`` with
``shape``, ``nbits``, ``group_size``, ``axis``, ``scale`` and ``zero``; ``unpack``
returning uint8 codes with one row per quantisation group (3-bit rows padded to a
multiple of ten, as HQQ's ten-per-word packing leaves them); ``W_q``; ``bias``.
The codes come from the oracle's min-max RTN quantiser on seeded N(0, 0.02)
weights, and every projection's (codes, scale, zero) is kept so tests can build
the expected packed layout with the oracle.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import torch
from torch import nn

from oracle import gemq_oracle as O

# small shapes that keep the 3-bit padding in play: N*K/g rows not a multiple of ten
HIDDEN, INTER, EXPERTS, TOP_K, GROUP = 256, 128, 8, 2, 64
EXPERT_BITS = [2, 3, 4, 2, 3, 1, 2, 3]


class FakeHQQLinear(nn.Module):
    def __init__(self, Q: np.ndarray, scale: np.ndarray, zero: np.ndarray, nbits: int, group_size: int,
                 bias=None, device="cpu"):
        super().__init__()
        N, K = Q.shape
        self.meta = {"shape": (N, K), "nbits": nbits, "group_size": group_size, "axis": 1,
                     "scale": torch.from_numpy(scale).to(device), "zero": torch.from_numpy(zero).to(device)}
        self.W_q = torch.zeros(1, dtype=torch.uint8, device=device)  # only its device is read
        self.bias = bias
        self._codes = torch.from_numpy(Q).to(device)

    def unpack(self, reshape=False, dtype=torch.uint8):
        assert reshape is False
        g = self.meta["group_size"]
        rows = self._codes.reshape(-1, g)
        if self.meta["nbits"] == 3:
            pad = (-rows.shape[0]) % 10
            # non-zero padding, so a caller that forgets to drop it fails loudly
            rows = torch.cat([rows, torch.full((pad, g), 5, dtype=rows.dtype, device=rows.device)])
        return rows.to(dtype)


def quantised(rng: np.random.Generator, out_f: int, in_f: int, nbits: int, group_size: int = GROUP):
    W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float16)
    Q, s, z = O.rtn_quantize(W, nbits, group_size)
    return Q, s.astype(np.float16), z.astype(np.float16)


class _Expert(nn.Module):
    pass


def _expert(rng, names, nbits, device, record):
    ex = _Expert()
    n1, n3, n2 = names
    for name, (o, i), key in ((n1, (INTER, HIDDEN), "w1"), (n3, (INTER, HIDDEN), "w3"), (n2, (HIDDEN, INTER), "w2")):
        Q, s, z = quantised(rng, o, i, nbits)
        record[key].append((Q, s, z, nbits))
        setattr(ex, name, FakeHQQLinear(Q, s, z, nbits, GROUP, device=device))
    return ex


def family_config(family: str):
    if family == "mixtral":
        return SimpleNamespace(hidden_size=HIDDEN, intermediate_size=INTER, num_local_experts=EXPERTS,
                               num_experts_per_tok=TOP_K)
    if family == "olmoe":
        return SimpleNamespace(hidden_size=HIDDEN, intermediate_size=INTER, num_experts=EXPERTS,
                               num_experts_per_tok=TOP_K, norm_topk_prob=False)
    if family == "qwen3":
        return SimpleNamespace(hidden_size=HIDDEN, moe_intermediate_size=INTER, num_experts=EXPERTS,
                               num_experts_per_tok=TOP_K, norm_topk_prob=True)
    return SimpleNamespace(hidden_size=HIDDEN, moe_intermediate_size=INTER, n_routed_experts=EXPERTS,
                           n_shared_experts=2, num_experts_per_tok=TOP_K, norm_topk_prob=False,
                           topk_method="greedy", scoring_func="softmax", routed_scaling_factor=1.0)


MODEL_NAME = {"mixtral": "mistralai/Mixtral-8x7B-v0.1", "olmoe": "allenai/OLMoE-1B-7B-0924",
              "qwen3": "Qwen/Qwen3-30B-A3B", "deepseek": "deepseek-ai/DeepSeek-V2-Lite"}


def fake_model(family: str, num_layers: int = 3, seed: int = 0, device="cpu"):
    """An HF-shaped causal LM whose linears are ``FakeHQQLinear``.

    Returns ``(model, records)``: ``records[i]`` holds, for MoE layer i, the gate weight
    and each projection's per-expert (codes, scale, zero, nbits) in expert order, plus
    the attention projection's. DeepSeek's layer 0 and Qwen3's last layer are dense.
    """
    rng = np.random.default_rng(seed)
    names = ("w1", "w3", "w2") if family == "mixtral" else ("gate_proj", "up_proj", "down_proj")
    attr = "block_sparse_moe" if family == "mixtral" else "mlp"
    layers, records = nn.ModuleList(), {}
    for i in range(num_layers):
        layer = nn.Module()
        layer.self_attn = nn.Module()
        Qa, sa, za = quantised(rng, HIDDEN, HIDDEN, 4)
        bias = torch.from_numpy((rng.standard_normal(HIDDEN) * 0.1).astype(np.float16)).to(device)
        layer.self_attn.q_proj = FakeHQQLinear(Qa, sa, za, 4, GROUP, bias=bias, device=device)
        Qo, so, zo = quantised(rng, HIDDEN, HIDDEN, 3)
        layer.self_attn.o_proj = FakeHQQLinear(Qo, so, zo, 3, GROUP, device=device)
        rec = {"q_proj": (Qa, sa, za, 4, bias), "o_proj": (Qo, so, zo, 3, None)}
        dense = (family == "deepseek" and i == 0) or (family == "qwen3" and i == num_layers - 1)
        if dense:
            mlp = nn.Module()
            Qd, sd, zd = quantised(rng, HIDDEN, HIDDEN, 4)
            mlp.down_proj = FakeHQQLinear(Qd, sd, zd, 4, GROUP, device=device)
            rec["dense_down_proj"] = (Qd, sd, zd, 4, None)
        else:
            mlp = nn.Module()
            gate = nn.Linear(HIDDEN, EXPERTS, bias=False).to(device=device, dtype=torch.float16)
            with torch.no_grad():
                gate.weight.copy_(torch.from_numpy((rng.standard_normal((EXPERTS, HIDDEN)) * 0.02)
                                                   .astype(np.float16)))
            mlp.gate = gate
            rec.update(gate=gate.weight.detach().cpu().numpy(), w1=[], w3=[], w2=[])
            mlp.experts = nn.ModuleList([_expert(rng, names, b, device, rec) for b in EXPERT_BITS])
            if family == "deepseek":
                rec.update(sw1=[], sw3=[], sw2=[])
                sh = {"w1": rec["sw1"], "w3": rec["sw3"], "w2": rec["sw2"]}
                mlp.shared_experts = _expert(rng, names, 4, device, sh)
        setattr(layer, attr, mlp)
        layers.append(layer)
        records[i] = rec
    model = nn.Module()
    model.model = nn.Module()
    model.model.layers = layers
    model.config = family_config(family)
    return model, records


def expected_projection(entries, K: int, N: int):
    """The oracle's stacked packing (from_hf's layout) of per-expert (codes, scale, zero, nbits)."""
    return O.stack_projection([e[0] for e in entries], [e[1] for e in entries], [e[2] for e in entries],
                              [e[3] for e in entries], GROUP, K, N)
