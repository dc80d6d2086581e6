"""gemq_dequant_group_gemm_noalloc: the grouped dequant GEMM for callers that
cannot allocate device memory.

Some hosts of this library own all device memory themselves (a serving process
that reserves its pool at start-up, a plugin inside a host whose allocator it may
not call) and so cannot hand over a workspace. The allocation-free entry point
keeps its segment table in a fixed array inside the library instead. These tests
call it through the C ABI and compare it with gemq_dequant_group_gemm, which
takes caller workspace, on two calls in a row with different index lists: the
second call must not see the first call's table. The file name makes pytest
collect it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2

pytestmark = pytest.mark.gpu

PRODUCT_REL_TOL = 2e-3  # the tolerance of the other GEMM tests


def _proj(t: dict, K: int, g: int):
    from robustgemq_b200 import ops

    return ops.make_proj(t["wq"], t["scales"], t["zeros"], t["nbits"], t["wq_strides"], t["zs_strides"], K, g)


def _with_workspace(lib, p, x, idx, n):
    from robustgemq_b200._lib import check, ptr, stream_ptr

    out = torch.empty((idx.numel(), x.shape[0], n), dtype=torch.float16, device=x.device)
    ws = torch.empty(lib.gemq_group_gemm_workspace_size(idx.numel()), dtype=torch.uint8, device=x.device)
    check(lib.gemq_dequant_group_gemm(ctypes.byref(p), ptr(x), x.shape[0], ptr(idx), idx.numel(), ptr(out),
                                      ptr(ws), ws.numel(), stream_ptr(x.device)))
    return out


def _no_alloc(lib, p, x, idx, out):
    from robustgemq_b200._lib import check, ptr, stream_ptr

    check(lib.gemq_dequant_group_gemm_noalloc(ctypes.byref(p), ptr(x), x.shape[0], ptr(idx), idx.numel(), ptr(out),
                                              stream_ptr(x.device)))
    return out


def test_no_alloc_group_gemm_matches_workspace_version():
    from robustgemq_b200 import _lib
    from gpu_helpers import cuda, proj_tensors

    lib = _lib.load()
    d = load_golden("group_gemm.npz")
    sub = {k[len("g64_"):]: v for k, v in d.items() if k.startswith("g64_")}
    t = proj_tensors(sub, "w")
    K, N = int(sub["w_K"]), int(t["wq"].shape[1])
    p = _proj(t, K, 64)
    E = t["nbits"].shape[0]
    x = cuda(sub["x"])
    rng = np.random.default_rng(7)
    # call 1: every expert plus repeats; call 2: a shorter list in another order and
    # a different token count, so stale segments from call 1 would show
    calls = [(x, torch.tensor(list(range(E)) + [2, 5, 5], dtype=torch.int32, device="cuda")),
             (torch.from_numpy(rng.standard_normal((37, K)).astype(np.float16)).cuda(),
              torch.tensor([4, 1], dtype=torch.int32, device="cuda"))]
    for xc, idx in calls:
        ref = _with_workspace(lib, p, xc, idx, N)
        out = torch.full((idx.numel(), xc.shape[0], N), float("nan"), dtype=torch.float16, device="cuda")
        got = _no_alloc(lib, p, xc, idx, out)
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < PRODUCT_REL_TOL
        assert torch.equal(got, ref)  # same kernels on the same inputs: bit-identical
    assert _lib.device_error() == 0


def test_no_alloc_group_gemm_beyond_256_indices():
    """257-1023 indices run the CUDA-core grouped GEMM (the tensor-core kernel
    takes up to 256 segments); two calls in a row, 300 then 1023 indices."""
    from conftest import proj_from
    from gpu_helpers import proj_tensors
    from oracle import gemq_oracle as O
    from robustgemq_b200 import _lib

    lib = _lib.load()
    d = load_golden("group_gemm.npz")
    sub = {k[len("g64_"):]: v for k, v in d.items() if k.startswith("g64_")}
    t = proj_tensors(sub, "w")
    K, N = int(sub["w_K"]), int(t["wq"].shape[1])
    p = _proj(t, K, 64)
    E = t["nbits"].shape[0]
    rng = np.random.default_rng(11)
    for A, M in ((300, 3), (1023, 2)):
        xc = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16)).cuda()
        idx = torch.from_numpy(rng.integers(0, E, size=A).astype(np.int32)).cuda()
        ref = _with_workspace(lib, p, xc, idx, N)
        out = torch.full((A, M, N), float("nan"), dtype=torch.float16, device="cuda")
        got = _no_alloc(lib, p, xc, idx, out)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
        # and against the per-index products of the oracle for a few indices
        op = proj_from(sub, "w")
        for a in (0, A // 2, A - 1):
            e = int(idx[a])
            yo = O.dequant_group_gemm(xc.cpu().numpy(), [e], op)[0]
            assert rel_l2(got[a].cpu().numpy(), yo) < PRODUCT_REL_TOL
    assert _lib.device_error() == 0


def test_no_alloc_rejects_more_indices_than_the_static_table():
    from robustgemq_b200 import _lib
    from gpu_helpers import proj_tensors

    lib = _lib.load()
    d = load_golden("group_gemm.npz")
    sub = {k[len("g64_"):]: v for k, v in d.items() if k.startswith("g64_")}
    t = proj_tensors(sub, "w")
    K, N = int(sub["w_K"]), int(t["wq"].shape[1])
    p = _proj(t, K, 64)
    x = torch.zeros((1, K), dtype=torch.float16, device="cuda")
    idx = torch.zeros(1024, dtype=torch.int32, device="cuda")
    out = torch.empty((1024, 1, N), dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.GemqArgumentError, match="GEMQ_NOALLOC_MAX_INDICES"):
        _no_alloc(lib, p, x, idx, out)
