"""Producer of the packed checkpoint layout the fused blocks consume.

``PackedLinear`` carries the attribute set ``QuantFused*MoEBlock.from_hf`` reads
off a repacked linear (``W_q``, ``scales``, ``zeros``, ``W_nbits``,
``group_size``; gemq/inference/patch.py:57-70, moe_block.py:725-742):

* ``W_q``     int32 ``[cdiv(K, 32 // b), N]`` -- the transposed view the reference
  packer returns (gemq/triton_kernels/utils.py:110-111), made contiguous;
* ``scales``  fp16 ``[K / g, N]``;
* ``zeros``   fp16 ``[K / g, N]``, the additive zero ``z' = -zero * scale`` the
  reference's ``dequantize`` expects (w = q*s + z', utils.py:206-210). It is formed
  in fp32 and rounded once to fp16.

``rtn_quantize`` restates the min-max RTN quantiser of gemq/quantizers/rtn.py:15-55,
used to make synthetic (Q, scale, zero) exactly as the reference's tests do
(tests/conftest.py:117-131).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class PackedLinear:
    W_q: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    W_nbits: int
    group_size: int
    in_features: int
    out_features: int


def rtn_quantize(W: torch.Tensor, nbits: int, group_size: int):
    """Min-max asymmetric RTN along the input dim (rtn.py:15-55; 1-bit: rtn.py:36-40).

    Returns ``(Q [N, K] uint8, scale [N*K/g, 1], zero [N*K/g, 1])`` in W's dtype.
    """
    N, K = W.shape
    if K % group_size:
        raise ValueError(f"w_shape: {K} | groupsize: {group_size}")
    Wg = W.reshape(-1, group_size)
    if nbits == 1:
        Q = torch.where(Wg >= 0, 1, 0).to(W.dtype)
        scales = torch.mean(torch.abs(Wg), dim=1, keepdim=True) * 2
        zeros = 0.5 * torch.ones_like(scales)
        return Q.reshape(N, K).to(torch.uint8), scales, zeros
    max_int = 2 ** nbits - 1
    mx = Wg.amax(dim=1, keepdim=True)
    mn = Wg.amin(dim=1, keepdim=True)
    scales = (mx - mn).clamp(min=1e-5) / max_int
    zeros = (-torch.round(mn / scales)).clamp_(0, max_int)
    Q = torch.clamp(torch.round(Wg / scales) + zeros, 0, max_int)
    return Q.reshape(N, K).to(torch.uint8), scales, zeros


def dequant_reference_fp16(Q: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group_size: int) -> torch.Tensor:
    """The fake-quant weight ``(Q - zero) * scale`` of rtn.py:57-61 (what the
    reference's dequantised HF blocks hold), in the scales' dtype."""
    N, K = Q.shape
    Qg = Q.reshape(-1, group_size).to(scales.dtype)
    return ((Qg - zeros) * scales).reshape(N, K)


def pack_codes(codes: torch.Tensor, nbits: int) -> torch.Tensor:
    """uint8 ``[N, K]`` (CUDA) -> int32 ``[cdiv(K, 32//b), N]`` contiguous via the CUDA packer."""
    from .ops import pack_weights_over_cols

    packed, _ = pack_weights_over_cols(codes, nbits)
    return packed.contiguous()


def pack_linear(Q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, nbits: int, group_size: int) -> PackedLinear:
    """(Q, scale, zero) from the RTN quantiser -> the repacked layout the kernels read."""
    N, K = Q.shape
    s = scale.float().reshape(N, K // group_size)
    z = zero.float().reshape(N, K // group_size)
    scales = s.t().contiguous().half()
    zeros = (-(z * s)).t().contiguous().half()
    return PackedLinear(W_q=pack_codes(Q.contiguous(), nbits), scales=scales, zeros=zeros, W_nbits=int(nbits),
                        group_size=int(group_size), in_features=K, out_features=N)


def quantize_linear(W: torch.Tensor, nbits: int, group_size: int):
    """RTN-quantise and pack ``W [N, K]``; returns ``(PackedLinear, W_fake_fp16)``."""
    Q, s, z = rtn_quantize(W, nbits, group_size)
    return pack_linear(Q, s, z, nbits, group_size), dequant_reference_fp16(Q, s, z, group_size).to(W.dtype)


