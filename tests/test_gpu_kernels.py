"""Kernel-level parity of the sm_100a kernels with the reference (``-m gpu``).

Bit-exact: packing, unpacking and dequantised weights against the golden vectors
recorded from the reference kernels (single-rounding fma semantics). Products:
rel-L2 against the same vectors; the reference accumulates in fp32 in its own
order, so agreement is to within fp16 rounding flips (tolerance written below).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, proj_from, rel_l2
from gpu_helpers import cuda, proj_tensors
from oracle import gemq_oracle as O

pytestmark = pytest.mark.gpu

PRODUCT_REL_TOL = 2e-3


@pytest.fixture(autouse=True)
def _no_device_error(cuda_device):
    from robustgemq_b200 import _lib

    _lib.device_error()
    yield
    assert _lib.device_error() == 0, "a kernel recorded a device-side error"


def test_pack_and_unpack_bit_exact():
    from robustgemq_b200 import ops

    d = load_golden("pack.npz")
    for key in sorted(k[:-6] for k in d if k.endswith("_codes")):
        nb = int(key[1])
        codes = cuda(d[f"{key}_codes"])
        packed, eps = ops.pack_weights_over_cols(codes, nb)
        assert eps == 32 // nb
        assert tuple(packed.shape) == d[f"{key}_packed"].shape
        assert np.array_equal(packed.cpu().numpy(), d[f"{key}_packed"]), key
        back = ops.unpack_over_cols(packed.t().contiguous(), nb, 32, codes.shape[1])
        assert torch.equal(back, codes), key


@pytest.mark.parametrize("g", [64, 128])
def test_dequant_bit_exact(g):
    from robustgemq_b200 import ops

    d = load_golden("group_gemm.npz")
    sub = {k[len(f"g{g}_"):]: v for k, v in d.items() if k.startswith(f"g{g}_")}
    t = proj_tensors(sub, "w")
    K = int(sub["w_K"])
    for e in range(t["nbits"].shape[0]):
        deq = ops.dequantize_expert(t["wq"], t["scales"], t["zeros"], t["nbits"], t["wq_strides"], t["zs_strides"], K,
                                    g, e)
        ref = sub["deq_gpu"][e]
        assert np.array_equal(deq.cpu().numpy().view(np.uint16), ref.view(np.uint16)), (g, e)


@pytest.mark.parametrize("g", [64, 128])
def test_group_gemm_matches_reference(g):
    """Tensor-core grouped GEMM (the shapes are tcgen05-eligible) on every expert,
    dequantised through the in-smem fma: the identity input recovers the dequantised
    weights exactly, which pins the swizzled A-tile layout bit for bit."""
    from robustgemq_b200 import ops

    d = load_golden("group_gemm.npz")
    sub = {k[len(f"g{g}_"):]: v for k, v in d.items() if k.startswith(f"g{g}_")}
    t = proj_tensors(sub, "w")
    E = t["nbits"].shape[0]
    idx = torch.arange(E, dtype=torch.int32, device="cuda")
    y = ops.dequant_group_gemm(cuda(sub["x"]), idx, t["wq"], t["scales"], t["zeros"], t["nbits"], t["group_sizes"],
                               t["wq_strides"], t["zs_strides"])
    assert rel_l2(y.cpu().numpy(), sub["y_gpu"]) < PRODUCT_REL_TOL
    eye = torch.eye(int(sub["w_K"]), dtype=torch.float16, device="cuda")
    deq = ops.dequant_group_gemm(eye, idx, t["wq"], t["scales"], t["zeros"], t["nbits"], t["group_sizes"],
                                 t["wq_strides"], t["zs_strides"])
    assert np.array_equal(deq.cpu().numpy().view(np.uint16), sub["deq_gpu"].view(np.uint16))


def test_group_gemm_single_index_and_reverse_order():
    from robustgemq_b200 import ops

    d = load_golden("group_gemm.npz")
    sub = {k[len("g64_"):]: v for k, v in d.items() if k.startswith("g64_")}
    t = proj_tensors(sub, "w")
    x = cuda(sub["x"])
    for order in ([3], [5, 0, 2]):
        idx = torch.tensor(order, dtype=torch.int32, device="cuda")
        y = ops.dequant_group_gemm(x, idx, t["wq"], t["scales"], t["zeros"], t["nbits"], t["group_sizes"],
                                   t["wq_strides"], t["zs_strides"]).cpu().numpy()
        assert rel_l2(y, sub["y_gpu"][order]) < PRODUCT_REL_TOL


def test_decode_kernels_match_reference():
    from robustgemq_b200 import ops

    d = load_golden("decode_kernels.npz")
    w1, w3, w2 = proj_tensors(d, "w1"), proj_tensors(d, "w3"), proj_tensors(d, "w2")
    idx = cuda(d["idx"])
    g = int(d["w1_group_sizes"][0])
    x1, x3 = ops.fused_dequant_up_proj(cuda(d["x"]), idx, w1["wq"], w3["wq"], w1["scales"], w1["zeros"], w3["scales"],
                                       w3["zeros"], w1["nbits"], w1["wq_strides"], g)
    assert rel_l2(x1.cpu().numpy(), d["x1_gpu"]) < PRODUCT_REL_TOL
    assert rel_l2(x3.cpu().numpy(), d["x3_gpu"]) < PRODUCT_REL_TOL
    x2 = ops.fused_dequant_down_proj(cuda(d["x1_gpu"]), cuda(d["x3_gpu"]), idx, w2["wq"], w2["scales"], w2["zeros"],
                                     w2["nbits"], w2["wq_strides"], g)
    assert rel_l2(x2.cpu().numpy(), d["x2_gpu"]) < PRODUCT_REL_TOL
    sh = proj_tensors(d, "sh")
    y = ops.dequant_gemm(cuda(d["xs"]), sh["wq"], sh["scales"], sh["zeros"], 4, g)
    assert rel_l2(y.cpu().numpy(), d["gemm_gpu"]) < PRODUCT_REL_TOL
    v = ops.dequant_splitk_gemv(cuda(d["x"]), sh["wq"], sh["scales"], sh["zeros"], 4, g)
    assert rel_l2(v.cpu().numpy(), d["gemv_gpu"]) < PRODUCT_REL_TOL
    sh2 = proj_tensors(d, "sh2")
    v2 = ops.dequant_splitk_gemv(cuda(d["h2"]), sh2["wq"], sh2["scales"], sh2["zeros"], 3, g)
    assert rel_l2(v2.cpu().numpy(), d["gemv2_gpu"]) < PRODUCT_REL_TOL


def test_gemv_is_deterministic():
    """The reference's split-K GEMV is not bit-reproducible (fp16 atomics,
    test_decode_nan_hunt.py:241-277); this one is."""
    from robustgemq_b200 import ops

    d = load_golden("decode_kernels.npz")
    sh = proj_tensors(d, "sh")
    g = int(d["w1_group_sizes"][0])
    x = cuda(d["x"])
    runs = [ops.dequant_splitk_gemv(x, sh["wq"], sh["scales"], sh["zeros"], 4, g) for _ in range(5)]
    assert all(torch.equal(runs[0], r) for r in runs[1:])


@pytest.mark.parametrize("nbits", [1, 2, 3, 4])
@pytest.mark.parametrize("K,N,M", [(256, 128, 7), (512, 256, 130), (320, 384, 33)])
def test_group_gemm_vs_oracle_shapes(nbits, K, N, M):
    """Ragged token counts (M not a multiple of the tile), K not a multiple of the
    3-bit word (K % 10 != 0), several N tiles; both group sizes."""
    from robustgemq_b200 import ops

    rng = np.random.default_rng(1000 + nbits * 7 + K)
    g = 64
    codes = [rng.integers(0, 2 ** nbits, size=(N, K), dtype=np.uint8) for _ in range(2)]
    scs = [(rng.random((N * K // g, 1)) * 0.01 + 0.001).astype(np.float16) for _ in range(2)]
    zes = [rng.integers(0, 2 ** nbits, size=(N * K // g, 1)).astype(np.float16) for _ in range(2)]
    proj = O.stack_projection(codes, scs, zes, [nbits, nbits], g, K, N)
    x = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    ref = O.dequant_group_gemm(x, [1, 0], proj)
    t = {f: cuda(getattr(proj, f)) for f in ("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides",
                                             "zs_strides")}
    y = ops.dequant_group_gemm(cuda(x), torch.tensor([1, 0], dtype=torch.int32, device="cuda"), t["wq"], t["scales"],
                               t["zeros"], t["nbits"], t["group_sizes"], t["wq_strides"], t["zs_strides"])
    assert rel_l2(y.cpu().numpy(), ref) < PRODUCT_REL_TOL


def test_argument_errors_raise_like_the_reference():
    from robustgemq_b200 import ops

    codes = torch.zeros((4, 16), dtype=torch.uint8, device="cuda")
    with pytest.raises(AssertionError):
        ops.pack_weights_over_cols(codes, 5)
    with pytest.raises(AssertionError):
        ops.pack_weights_over_cols(codes, 4, packing_bitwidth=16)
