"""Model patching for quantised inference: the counterpart of gemq/inference/patch.py.

=================================================  ===================================
reference (gemq/...)                                here
=================================================  ===================================
inference/patch.py:27-72   create_gemlite_from_hqq  create_linear_from_hqq (alias kept)
inference/patch.py:75-83   replace_linear_recursive replace_linear_recursive
inference/patch.py:86-162  replace_moe_blocks       replace_moe_blocks
inference/patch.py:165-181 prepare_for_inference    prepare_for_inference
utils/model_utils.py:22-50 ModelType, NAME_TO_MODEL ModelType, NAME_TO_MODEL
utils/model_utils.py:131-143 get_blocks             get_blocks
=================================================  ===================================

A quantised model is prepared in two passes, as in the reference: every HQQ linear
becomes a ``QuantLinear`` (packed words, fp16 scales and additive zeros), then each
MoE block becomes the family's ``QuantFused*MoEBlock`` built by ``from_hf`` from those
linears. HQQ linears are recognised by type when the ``hqq`` package is importable
and otherwise by their interface: a ``meta`` dict with ``shape``, ``nbits``,
``group_size``, ``axis``, ``scale`` and ``zero``, and an ``unpack`` method returning
the uint8 codes. The codes come from the layer's own ``unpack``, so the on-disk
packing stays the HQQ layer's business.

The reference's fp16 path (``is_fp=True``: unquantised ``Fused*MoEBlock``) is not
part of this library and raises ``NotImplementedError``.
"""

from __future__ import annotations

import gc
from enum import Enum, auto

import torch
from torch import nn

from .linear import QuantLinear
from .moe_block import (
    QuantFusedDeepseekV2MoEBlock,
    QuantFusedMixtralMoEBlock,
    QuantFusedOlmoeMoEBlock,
    QuantFusedQwen3MoeMoEBlock,
)


class ModelType(Enum):
    """Model families the reference knows (model_utils.py:22-31)."""

    LLAMA2 = auto()
    QWEN3 = auto()
    MIXTRAL = auto()
    DEEPSEEKV2 = auto()
    OLMOE = auto()
    QWEN3MOE = auto()


# checkpoint name -> family (model_utils.py:42-50)
NAME_TO_MODEL = {
    "meta-llama/Llama-2-7b-hf": ModelType.LLAMA2,
    "Qwen/Qwen3-8B": ModelType.QWEN3,
    "mistralai/Mixtral-8x7B-v0.1": ModelType.MIXTRAL,
    "deepseek-ai/DeepSeek-V2-Lite": ModelType.DEEPSEEKV2,
    "allenai/OLMoE-1B-7B-0924": ModelType.OLMOE,
    "Qwen/Qwen3-30B-A3B": ModelType.QWEN3MOE,
}

# family -> (attribute of a decoder layer holding the MoE block, fused block class)
_MOE_FAMILIES = {
    ModelType.MIXTRAL: ("block_sparse_moe", QuantFusedMixtralMoEBlock),
    ModelType.DEEPSEEKV2: ("mlp", QuantFusedDeepseekV2MoEBlock),
    ModelType.OLMOE: ("mlp", QuantFusedOlmoeMoEBlock),
    ModelType.QWEN3MOE: ("mlp", QuantFusedQwen3MoeMoEBlock),
}


def get_blocks(model, model_name: str):
    """The decoder layers of an HF causal LM of a known family (model_utils.py:131-143)."""
    NAME_TO_MODEL[model_name]  # unknown names raise KeyError, as in the reference
    return model.model.layers


_HQQ_META_KEYS = ("shape", "nbits", "group_size", "axis", "scale", "zero")


def is_hqq_linear(module) -> bool:
    """True for ``hqq.core.quantize.HQQLinear`` and for modules with its interface."""
    try:
        from hqq.core.quantize import HQQLinear
    except ImportError:
        HQQLinear = None
    if HQQLinear is not None and isinstance(module, HQQLinear):
        return True
    meta = getattr(module, "meta", None)
    return isinstance(meta, dict) and all(k in meta for k in _HQQ_META_KEYS) and callable(
        getattr(module, "unpack", None))


def create_linear_from_hqq(hqq_layer, **kwargs) -> QuantLinear:
    """An HQQ linear -> ``QuantLinear`` (patch.py:27-72).

    Keyword arguments as in the reference: ``device`` (default: the layer's ``W_q``
    device) and ``dtype`` (default: the dtype of the layer's scales). The kernels
    compute in fp16, so ``dtype`` must be ``torch.float16``."""
    meta = hqq_layer.meta
    w_q_attr = getattr(hqq_layer, "W_q", None)
    device = kwargs.get("device", w_q_attr.device if w_q_attr is not None else meta["scale"].device)
    out_features, in_features = meta["shape"]
    nbits = meta["nbits"]
    group_size = meta["group_size"]
    assert meta["axis"] == 1, "Only axis==1 is supported."

    W_q = hqq_layer.unpack(reshape=False, dtype=torch.uint8)
    if nbits == 3:
        # 3-bit HQQ packs ten rows per word, so the unpacked rows are padded to a multiple of 10
        W_q = W_q[:out_features * in_features // group_size]
    W_q = W_q.reshape(out_features, in_features)
    scales = meta["scale"].clone()
    zeros = meta["zero"].clone()
    bias = hqq_layer.bias.clone() if getattr(hqq_layer, "bias", None) is not None else None

    dtype = kwargs.get("dtype", scales.dtype)
    assert scales.dtype in (torch.float16, torch.bfloat16, torch.float32), (
        "Invalid scales.dtype, should floating point.")
    if dtype != torch.float16:
        raise NotImplementedError(f"the packed kernels compute in float16, got dtype={dtype}")

    W_q = W_q.to(device)
    scales = scales.to(dtype=dtype, device=device)
    zeros = zeros.to(dtype=dtype, device=device)
    if bias is not None:
        bias = bias.to(device=device, dtype=dtype)

    return QuantLinear(nbits, group_size, in_features, out_features).pack(W_q, scales, zeros, bias=bias,
                                                                           packing_bitwidth=32)


create_gemlite_from_hqq = create_linear_from_hqq


def replace_linear_recursive(module: nn.Module, **kwargs) -> None:
    """Replace every HQQ linear below ``module`` with a ``QuantLinear`` (patch.py:75-83)."""
    for name, child in module.named_children():
        if is_hqq_linear(child):
            setattr(module, name, create_linear_from_hqq(child, **kwargs))
        else:
            replace_linear_recursive(child, **kwargs)


def _is_moe_block(block) -> bool:
    # dense layers of a MoE model (Qwen3's mlp_only_layers / decoder_sparse_step) have no experts
    return block is not None and hasattr(block, "experts") and hasattr(block, "gate")


def _release(del_orig: bool) -> None:
    if del_orig:
        gc.collect()
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.empty_cache()


def replace_moe_blocks(model, model_name: str, config, is_fp: bool = False) -> None:
    """Replace the MoE block of every decoder layer with the family's fused block (patch.py:86-162).

    DeepSeek-V2's first layer is dense and stays as it is; Qwen3-MoE layers whose MLP is
    dense (no experts) stay as they are. The expert linears must already be packed
    (``replace_linear_recursive``)."""
    if is_fp:
        raise NotImplementedError("the unquantised fp16 Fused*MoEBlock path is not part of this library")
    model_type = NAME_TO_MODEL[model_name]
    if model_type not in _MOE_FAMILIES:
        raise NotImplementedError
    attr, cls = _MOE_FAMILIES[model_type]
    layers = get_blocks(model, model_name)
    for i in range(len(layers)):
        layer = layers[i]
        if model_type == ModelType.DEEPSEEKV2 and i == 0:
            continue  # the first layer of this model is a dense layer
        org_block = getattr(layer, attr)
        if model_type == ModelType.QWEN3MOE and not _is_moe_block(org_block):
            continue
        setattr(layer, attr, cls.from_hf(config, org_block))
        del org_block
        _release(True)


def prepare_for_inference(model, model_name: str, is_fp: bool = False):
    """Pack every HQQ linear, then fuse the MoE blocks (patch.py:165-181). Returns ``model``."""
    if is_fp:
        replace_moe_blocks(model, model_name, model.config, is_fp=True)
    else:
        replace_linear_recursive(model)
        replace_moe_blocks(model, model_name, model.config, is_fp=False)
    _release(True)
    return model
