"""Packed low-bit linear layer: what the reference puts in place of each HQQ linear.

The reference turns every ``HQQLinear`` of a quantised model into a GemLite
``GemLiteLinearTriton`` (gemq/inference/patch.py:27-83). Attention and dense MLP
projections then run through GemLite's Triton kernels, and the expert projections
are stacked by ``QuantFused*MoEBlock.from_hf``, which reads ``W_q``, ``scales``,
``zeros``, ``W_nbits`` and ``group_size`` off each linear (moe_block.py:725-742).

``QuantLinear`` stores the same attribute set in the layout the fused blocks stack
(``quant.PackedLinear``), so patched expert linears go straight into ``from_hf``.
Its ``forward`` runs the sm_100a kernels of this library:

* one input row: the split-K dequant GEMV (the batch-1 path of dequant_gemv.py:118-156);
* more rows: the tensor-core dequant GEMM (dequant_gemm.py:150-193).

Both compute in fp16 with fp32 accumulation and return fp16. The bias is added
after the product in fp16.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn

from .. import ops
from ..quant import pack_linear


class QuantLinear(nn.Module):
    """``y = x @ deq(W)^T (+ bias)`` over a packed ``W_nbits``-bit weight ``[out_features, in_features]``."""

    def __init__(self, W_nbits: int, group_size: int, in_features: int, out_features: int) -> None:
        super().__init__()
        if W_nbits not in (1, 2, 3, 4):
            raise ValueError(f"W_nbits must be 1, 2, 3 or 4, got {W_nbits}")
        if group_size <= 0 or group_size % 32 != 0:
            raise ValueError(f"group_size must be a positive multiple of 32, got {group_size}")
        if in_features % group_size != 0:
            raise ValueError(f"in_features ({in_features}) must be a multiple of group_size ({group_size})")
        if out_features % 4 != 0:
            raise ValueError(f"out_features ({out_features}) must be a multiple of 4")
        self.W_nbits = int(W_nbits)
        self.group_size = int(group_size)
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        # plain attributes, like the reference's packed tensors (moe_block.py:152-164)
        self.W_q: Optional[Tensor] = None
        self.scales: Optional[Tensor] = None
        self.zeros: Optional[Tensor] = None
        self.bias: Optional[Tensor] = None

    def pack(self, W_q: Tensor, scales: Tensor, zeros: Tensor, bias: Optional[Tensor] = None,
             packing_bitwidth: int = 32) -> "QuantLinear":
        """Pack uint8 codes ``W_q [out, in]`` with their per-group ``scales`` and ``zeros``.

        ``scales`` / ``zeros`` hold one value per group of ``group_size`` inputs of a row,
        in row-major group order (HQQ's ``[out * in / g, 1]`` or ``[out, in / g]``). The
        kernels read ``scales`` fp16 ``[in / g, out]`` and the additive zero
        ``z' = fp16(-zero * scale)`` (formed in fp32) in the same layout, and the codes as
        int32 words ``[cdiv(in, 32 // b), out]``. Packing runs on the codes' device,
        which must be a CUDA device."""
        if packing_bitwidth != 32:
            raise ValueError(f"only 32-bit packing words are supported, got {packing_bitwidth}")
        if tuple(W_q.shape) != (self.out_features, self.in_features):
            raise ValueError(f"W_q must be [{self.out_features}, {self.in_features}], got {list(W_q.shape)}")
        groups = self.out_features * self.in_features // self.group_size
        for name, t in (("scales", scales), ("zeros", zeros)):
            if t.numel() != groups:
                raise ValueError(f"{name} must hold {groups} values (one per group), got {t.numel()}")
        p = pack_linear(W_q.to(torch.uint8).contiguous(), scales, zeros, self.W_nbits, self.group_size)
        self.W_q, self.scales, self.zeros = p.W_q, p.scales, p.zeros
        self.bias = None if bias is None else bias.detach().to(device=p.W_q.device, dtype=torch.float16).contiguous()
        return self

    def forward(self, x: Tensor) -> Tensor:
        if self.W_q is None:
            raise RuntimeError("QuantLinear has no weights: call pack() first")
        if x.dtype != torch.float16:
            raise TypeError(f"QuantLinear computes in fp16, got input of dtype {x.dtype}")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected {self.in_features} input features, got {x.shape[-1]}")
        lead = x.shape[:-1]
        rows = x.reshape(-1, self.in_features)
        if rows.shape[0] == 1:
            y = ops.dequant_splitk_gemv(rows, self.W_q, self.scales, self.zeros, self.W_nbits, self.group_size)
        else:
            y = ops.dequant_gemm(rows, self.W_q, self.scales, self.zeros, self.W_nbits, self.group_size)
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, W_nbits={self.W_nbits}, "
                f"group_size={self.group_size}, bias={self.bias is not None}")
