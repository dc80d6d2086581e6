"""Kernel-level operators: the entry points of ``gemq/triton_kernels/*.py`` with the
same argument meaning, run by the sm_100a kernels of ``libgemq_b200.so``.

=============================================  ========================================
reference (gemq/triton_kernels/...)             here
=============================================  ========================================
utils.pack_weights_over_cols_triton (74-113)    pack_weights_over_cols
utils.unpack_over_cols_triton (149-189)         unpack_over_cols
dequant_group_gemm.dequant_group_gemm_triton    dequant_group_gemm
dequant_gemm.dequant_gemm_triton                dequant_gemm
dequant_gemv.dequant_splitk_gemv_triton         dequant_splitk_gemv (deterministic)
fused_dequant_bmm.fused_dequant_up_proj_triton  fused_dequant_up_proj
fused_dequant_bmm.fused_dequant_down_proj_...   fused_dequant_down_proj
=============================================  ========================================

The reference names (with their ``_triton`` suffix) are kept as aliases so code
written against the reference imports unchanged. Outputs are allocated with
``torch.empty`` on the input's device and the work runs on the current stream,
as in the reference.
"""

from __future__ import annotations

import ctypes
from typing import Tuple

import torch

from . import _lib
from ._lib import ProjT, check, on_input_device, ptr, stream_ptr


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path)")


def _i32(values, device) -> torch.Tensor:
    return torch.as_tensor(values, dtype=torch.int32, device=device)


def make_proj(wq: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, nbits: torch.Tensor,
              wq_strides: torch.Tensor, zs_strides: torch.Tensor, k: int, group_size: int) -> ProjT:
    """C struct for one stacked projection (pointers stay owned by the tensors)."""
    for t, name in ((wq, "wq"), (scales, "scales"), (zeros, "zeros")):
        _cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if wq.dtype != torch.int32 or scales.dtype != torch.float16 or zeros.dtype != torch.float16:
        raise ValueError("wq must be int32 and scales/zeros float16")
    p = ProjT()
    p.wq, p.scales, p.zeros = wq.data_ptr(), scales.data_ptr(), zeros.data_ptr()
    p.nbits, p.wq_strides, p.zs_strides = nbits.data_ptr(), wq_strides.data_ptr(), zs_strides.data_ptr()
    p.wq_rows = wq.shape[0]
    p.num_experts = nbits.shape[0]
    p.k = int(k)
    p.n = wq.shape[1]
    p.group_size = int(group_size)
    return p


# ------------------------------------------------------------------ packing
@on_input_device
def pack_weights_over_cols(W_q: torch.Tensor, W_nbits: int, packing_bitwidth: int = 32,
                           transpose: bool = True) -> Tuple[torch.Tensor, int]:
    """uint8 codes ``[N, K]`` -> int32 words; returns ``(words, 32 // W_nbits)`` where
    ``words`` is the ``[cdiv(K, eps), N]`` transposed view when ``transpose``
    (utils.py:74-113)."""
    assert packing_bitwidth == 32, "Unsuported bitpacking width"
    assert W_nbits in [4, 3, 2, 1], f"Untested quantization bitwidth: {W_nbits}"
    _cuda(W_q, "W_q")
    W_q = W_q.contiguous()
    if W_q.dtype != torch.uint8:
        W_q = W_q.to(torch.uint8)
    eps = packing_bitwidth // W_nbits
    rows, cols = W_q.shape
    out = torch.empty((rows, (cols + eps - 1) // eps), dtype=torch.int32, device=W_q.device)
    check(_lib.load().gemq_pack_weights_over_cols(ptr(W_q), rows, cols, W_nbits, ptr(out), stream_ptr(W_q.device)))
    return (out.t() if transpose else out), eps


@on_input_device
def unpack_over_cols(W_q_packed: torch.Tensor, W_nbits: int, packing_bitwidth: int, num_output_cols: int,
                     dtype: torch.dtype = torch.uint8) -> torch.Tensor:
    """Inverse of the packer on the ``[N, cdiv(K, eps)]`` buffer (utils.py:149-189)."""
    _cuda(W_q_packed, "W_q_packed")
    assert packing_bitwidth == 32
    W_q_packed = W_q_packed.contiguous()
    rows, pcols = W_q_packed.shape
    out = torch.empty((rows, num_output_cols), dtype=torch.uint8, device=W_q_packed.device)
    check(_lib.load().gemq_unpack_over_cols(ptr(W_q_packed), rows, pcols, num_output_cols, W_nbits, ptr(out),
                                            stream_ptr(W_q_packed.device)))
    return out if dtype == torch.uint8 else out.to(dtype)


@on_input_device
def dequantize_expert(wq, scales, zeros, nbits, wq_strides, zs_strides, K: int, group_size: int,
                      expert: int) -> torch.Tensor:
    """Dequantised ``[K, N]`` fp16 weight of one expert: the reference's ``dequantize``
    (utils.py:192-212) over a whole expert, bit-exact."""
    p = make_proj(wq, scales, zeros, nbits, wq_strides, zs_strides, K, group_size)
    out = torch.empty((K, wq.shape[1]), dtype=torch.float16, device=wq.device)
    check(_lib.load().gemq_dequant_expert(ctypes.byref(p), int(expert), ptr(out), stream_ptr(wq.device)))
    return out


# ------------------------------------------------------------------ GEMMs
@on_input_device
def dequant_group_gemm(x: torch.Tensor, indices: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                       zeros: torch.Tensor, nbits: torch.Tensor, group_sizes: torch.Tensor, wq_strides: torch.Tensor,
                       zs_strides: torch.Tensor, compute_dtype=torch.float16) -> torch.Tensor:
    """``output[a] = x @ dequantize(wq[indices[a]])`` -> ``[A, M, N]`` (dequant_group_gemm.py:155-202)."""
    if compute_dtype != torch.float16:
        raise ValueError("compute dtype is fixed to float16, as in the reference kernels")
    _cuda(x, "x")
    if x.dtype != torch.float16:
        raise ValueError("x must be float16")
    x = x.contiguous()
    M, K = x.shape
    idx = indices.reshape(-1).to(device=x.device, dtype=torch.int32).contiguous()
    A = idx.shape[0]
    g = torch.unique(group_sizes)
    if g.numel() != 1:
        raise ValueError("group sizes must be the same across all experts")
    p = make_proj(wq, scales, zeros, nbits, wq_strides, zs_strides, K, int(g.item()))
    out = torch.empty((A, M, wq.shape[1]), dtype=torch.float16, device=x.device)
    lib = _lib.load()
    ws = torch.empty(lib.gemq_group_gemm_workspace_size(A), dtype=torch.uint8, device=x.device)
    check(lib.gemq_dequant_group_gemm(ctypes.byref(p), ptr(x), M, ptr(idx), A, ptr(out), ptr(ws), ws.numel(),
                                      stream_ptr(x.device)))
    return out


class _SingleMeta:
    """Device-side nbits/strides for a single (non-stacked) weight, cached per value."""

    cache: dict = {}

    @classmethod
    def get(cls, nbits: int, device: torch.device):
        key = (int(nbits), str(device))
        if key not in cls.cache:
            cls.cache[key] = (_i32([nbits], device), _i32([0], device), _i32([0], device))
        return cls.cache[key]


@on_input_device
def dequant_gemm(x: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, nbits: int,
                 group_size: int) -> torch.Tensor:
    """``x @ dequantize(w_q)`` for one packed weight (dequant_gemm.py:150-193)."""
    _cuda(x, "x")
    x = x.contiguous()
    M, K = x.shape
    nb, ws_, zs_ = _SingleMeta.get(nbits, x.device)
    p = make_proj(w_q.contiguous(), scales.contiguous(), zeros.contiguous(), nb, ws_, zs_, K, group_size)
    out = torch.empty((M, w_q.shape[1]), dtype=torch.float16, device=x.device)
    lib = _lib.load()
    ws = torch.empty(lib.gemq_group_gemm_workspace_size(1), dtype=torch.uint8, device=x.device)
    check(lib.gemq_dequant_gemm(ctypes.byref(p), ptr(x), M, ptr(out), ptr(ws), ws.numel(), stream_ptr(x.device)))
    return out


@on_input_device
def dequant_splitk_gemv(x: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, nbits: int,
                        group_size: int) -> torch.Tensor:
    """Batch-1 ``x @ dequantize(w_q)`` (dequant_gemv.py:118-156). The split-K partial
    sums are reduced in a fixed order instead of fp16 atomics, so repeated calls are
    bit-identical."""
    _cuda(x, "x")
    x = x.contiguous()
    M, K = x.shape
    if M != 1:
        raise ValueError("dequant_splitk_gemv takes a single row")
    nb, ws_, zs_ = _SingleMeta.get(nbits, x.device)
    p = make_proj(w_q.contiguous(), scales.contiguous(), zeros.contiguous(), nb, ws_, zs_, K, group_size)
    out = torch.empty((1, w_q.shape[1]), dtype=torch.float16, device=x.device)
    lib = _lib.load()
    ws = torch.empty(lib.gemq_gemv_workspace_size(ctypes.byref(p), 1), dtype=torch.uint8, device=x.device)
    check(lib.gemq_dequant_gemv(ctypes.byref(p), ptr(x), ptr(out), ptr(ws), ws.numel(), stream_ptr(x.device)))
    return out


def _stacked_zs(E: int, K: int, group_size: int, N: int, device) -> torch.Tensor:
    # fused_dequant_bmm.py:62,218 address scales at idx * (K // group_size) rows
    return torch.arange(E, dtype=torch.int32, device=device) * ((K // group_size) * N)


@on_input_device
def fused_dequant_up_proj(x: torch.Tensor, idx: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor,
                          w1_scales: torch.Tensor, w1_zeros: torch.Tensor, w3_scales: torch.Tensor,
                          w3_zeros: torch.Tensor, nbits: torch.Tensor, w_strides: torch.Tensor, group_size: int):
    """``x1 = x @ deq(w1[e])``, ``x3 = x @ deq(w3[e])`` for e in idx, fp16 ``[1, A*N]``
    (fused_dequant_bmm.py:122-173). w3 is read with w1's nbits/strides."""
    _cuda(x, "x")
    x = x.contiguous()
    _, K = x.shape
    N = w1.shape[1]
    idx = idx.reshape(-1).to(device=x.device, dtype=torch.int32).contiguous()
    A = idx.shape[0]
    E = nbits.shape[0]
    zs = _stacked_zs(E, K, group_size, N, x.device)
    p1 = make_proj(w1, w1_scales, w1_zeros, nbits, w_strides, zs, K, group_size)
    p3 = make_proj(w3, w3_scales, w3_zeros, nbits, w_strides, zs, K, group_size)
    x1 = torch.empty((1, A * N), dtype=torch.float16, device=x.device)
    x3 = torch.empty((1, A * N), dtype=torch.float16, device=x.device)
    lib = _lib.load()
    ws = torch.empty(lib.gemq_gemv_workspace_size(ctypes.byref(p1), A), dtype=torch.uint8, device=x.device)
    check(lib.gemq_fused_up_proj(ctypes.byref(p1), ctypes.byref(p3), ptr(x), ptr(idx), A, ptr(x1), ptr(x3), ptr(ws),
                                 ws.numel(), stream_ptr(x.device)))
    return x1, x3


@on_input_device
def fused_dequant_down_proj(x1: torch.Tensor, x3: torch.Tensor, idx: torch.Tensor, w2: torch.Tensor,
                            w2_scales: torch.Tensor, w2_zeros: torch.Tensor, nbits: torch.Tensor,
                            w_strides: torch.Tensor, group_size: int) -> torch.Tensor:
    """``x2 = (silu(x1) * x3) @ deq(w2[e])`` per selected expert, SiLU*mul in fp32,
    fp16 ``[1, A*N]`` (fused_dequant_bmm.py:264-312)."""
    _cuda(x1, "x1")
    x1 = x1.contiguous()
    x3 = x3.contiguous()
    idx = idx.reshape(-1).to(device=x1.device, dtype=torch.int32).contiguous()
    A = idx.shape[0]
    K = x1.shape[1] // A
    N = w2.shape[1]
    E = nbits.shape[0]
    zs = _stacked_zs(E, K, group_size, N, x1.device)
    p = make_proj(w2, w2_scales, w2_zeros, nbits, w_strides, zs, K, group_size)
    x2 = torch.empty((1, A * N), dtype=torch.float16, device=x1.device)
    lib = _lib.load()
    ws = torch.empty(lib.gemq_gemv_workspace_size(ctypes.byref(p), A), dtype=torch.uint8, device=x1.device)
    check(lib.gemq_fused_down_proj(ctypes.byref(p), ptr(x1), ptr(x3), ptr(idx), A, ptr(x2), ptr(ws), ws.numel(),
                                   stream_ptr(x1.device)))
    return x2


# reference names, for drop-in imports
pack_weights_over_cols_triton = pack_weights_over_cols
unpack_over_cols_triton = unpack_over_cols
dequant_group_gemm_triton = dequant_group_gemm
dequant_gemm_triton = dequant_gemm
dequant_splitk_gemv_triton = dequant_splitk_gemv
fused_dequant_up_proj_triton = fused_dequant_up_proj
fused_dequant_down_proj_triton = fused_dequant_down_proj
