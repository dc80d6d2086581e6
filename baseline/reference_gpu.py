"""The reference's own GPU path, for side-by-side parity and timing.

MEASUREMENT AND TEST INFRASTRUCTURE ONLY. Nothing under ``robustgemq_b200/``
imports this file. It is used by ``tests/golden/make_ref_gpu.py``, which records
fixtures of the reference's GPU outputs, and by ``bench.py``'s ``reference_gpu``
sub-object.

The reference (RobustGEMQ's ``gemq`` package) is installed unmodified into
``baseline/_ref`` with ``pip install --no-deps --target baseline/_ref``. Its MoE
blocks (``gemq/inference/moe_block.py``) run their Triton kernels, JIT-compiled
for the B200 by the image's triton, with the reference's own autotune
configurations. Two of its module-level imports do not resolve in this image, so
they are given stand-ins before the import:

* ``gemlite.core.GemLiteLinearTriton`` is used only in an ``isinstance`` check
  inside ``from_hf`` (moe_block.py:10, 181-182);
* ``transformers``' ``DeepseekV2MoE`` is only a type annotation (moe_block.py:7).

A reference block is built with the reference class's own constructor. Every
packed tensor of one of this library's blocks is then assigned to it unchanged,
which gives the same attribute set ``from_hf`` produces (moe_block.py:166-213,
429-506, 715-761). Both implementations therefore read the same weights.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path
from types import SimpleNamespace

import torch

REF_ROOT = Path(__file__).resolve().parent / "_ref"

PROJ_ATTRS = ("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides", "zs_strides")


def available() -> bool:
    """True when the installed reference, triton and a CUDA device are all present."""
    if not (REF_ROOT / "gemq" / "inference" / "moe_block.py").exists():
        return False
    if not torch.cuda.is_available():
        return False
    try:
        import triton  # noqa: F401
    except Exception:
        return False
    return True


_MB = None


def load():
    """Import ``gemq.inference.moe_block`` from ``baseline/_ref`` (once per process)."""
    global _MB
    if _MB is not None:
        return _MB
    if not available():
        raise RuntimeError("the reference is not installed in baseline/_ref, or triton / CUDA is missing")
    if "gemlite" not in sys.modules:
        gl = types.ModuleType("gemlite")
        glc = types.ModuleType("gemlite.core")

        class GemLiteLinearTriton:  # isinstance target only
            pass

        glc.GemLiteLinearTriton = GemLiteLinearTriton
        gl.core = glc
        sys.modules["gemlite"] = gl
        sys.modules["gemlite.core"] = glc
    import transformers.models.deepseek_v2.modeling_deepseek_v2 as ds

    if not hasattr(ds, "DeepseekV2MoE"):
        ds.DeepseekV2MoE = type("DeepseekV2MoE", (torch.nn.Module,), {})
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("ignore", SyntaxWarning)
        from gemq.inference import moe_block as mb
    _MB = mb
    return mb


def _family(ours) -> str:
    name = type(ours).__name__
    for fam in ("Olmoe", "Qwen3", "Mixtral", "Deepseek"):
        if fam in name:
            return fam
    raise ValueError(f"no reference block for {name}")


def reference_block(ours):
    """The reference's QuantFused block of the same family, holding ``ours``'s tensors."""
    mb = load()
    fam = _family(ours)
    D, F, E, k = ours.hidden_dim, ours.ffn_dim, ours.num_experts, ours.top_k
    if fam == "Olmoe":
        cfg = SimpleNamespace(hidden_size=D, intermediate_size=F, num_experts=E, num_experts_per_tok=k,
                              norm_topk_prob=bool(ours.norm_topk_prob))
        ref = mb.QuantFusedOlmoeMoEBlock(cfg)
    elif fam == "Qwen3":
        cfg = SimpleNamespace(hidden_size=D, moe_intermediate_size=F, num_experts=E, num_experts_per_tok=k,
                              norm_topk_prob=bool(ours.norm_topk_prob))
        ref = mb.QuantFusedQwen3MoeMoEBlock(cfg)
    elif fam == "Mixtral":
        cfg = SimpleNamespace(hidden_size=D, intermediate_size=F, num_local_experts=E, num_experts_per_tok=k)
        ref = mb.QuantFusedMixtralMoEBlock(cfg)
    else:
        cfg = SimpleNamespace(hidden_size=D, moe_intermediate_size=F, n_routed_experts=E,
                              n_shared_experts=ours.num_shared_experts, num_experts_per_tok=k,
                              norm_topk_prob=bool(ours.norm_topk_prob), topk_method="greedy", scoring_func="softmax")
        ref = mb.QuantFusedDeepseekV2MoEBlock(cfg)
    ref.gate.weight.data = ours.gate.weight.data
    for name in ("w1", "w2", "w3"):
        for a in PROJ_ATTRS:
            setattr(ref, f"{name}_{a}", getattr(ours, f"{name}_{a}"))
    ref.block_group_size = ours.block_group_size
    if fam == "Deepseek":
        for name in ("shared_w1", "shared_w2", "shared_w3"):
            for a in ("wq", "scales", "zeros"):
                setattr(ref, f"{name}_{a}", getattr(ours, f"{name}_{a}"))
        ref.shared_nbits = ours.shared_nbits
        ref.shared_group_size = ours.shared_group_size
    mb.check_w1_w3_aligned(ref)
    return ref


class FixedLogits(torch.nn.Module):
    """Stands in for the gate so that ``forward_n_tokens`` routes from given logits
    (the skewed-load configuration feeds its logits straight to softmax / top-k)."""

    def __init__(self, logits: torch.Tensor):
        super().__init__()
        self.logits = logits

    def forward(self, x):
        assert x.shape[0] == self.logits.shape[0]
        return self.logits


def output(ret) -> torch.Tensor:
    """The hidden-state output of a block call (OLMoE / Qwen3 / Mixtral return a tuple)."""
    return ret[0] if isinstance(ret, tuple) else ret
