"""Chained gate/up -> down launches of the decode GEMM and of the one-token GEMVs (``-m gpu``).

The down-projection GEMM starts on the SMs the gate/up GEMM leaves and takes each
token tile once a per-tile counter shows all of its gate/up items stored (the
counters are zeroed by each forward's dispatch). Its results must not depend on
that: every test compares the chained forward bit for bit with the forward whose
down launch waits for the gate/up completion (``GEMQ_FWD_NO_CHAIN``), over decode
batches (16- and 32-token tiles), a prefill (64-token tiles, the large-batch
dispatch), repeated forwards and CUDA-graph replays.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _block(cfg_fn, seed=3):
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock, QuantFusedQwen3MoeMoEBlock

    cfg, shp = cfg_fn()
    cls = QuantFusedOlmoeMoEBlock if cfg_fn is synth.olmoe_config else QuantFusedQwen3MoeMoEBlock
    return synth.random_block(cls, cfg, shp["hidden"], shp["inter"], shp["num_experts"], shp["mean_bits"],
                              shp["group_size"], seed=seed, device=torch.device("cuda"))


def _fwd(blk, x, chain: bool):
    from robustgemq_b200 import _lib

    blk._fwd_flags = 0 if chain else _lib.FWD_NO_CHAIN
    try:
        return blk.forward_n_tokens(x.unsqueeze(0))[0][0]
    finally:
        blk._fwd_flags = 0


@pytest.mark.parametrize("T", [2, 8, 24, 64, 200, 512])  # 16 / 32-token tiles (512: 64-token, unchained)
def test_chained_down_launch_is_bit_identical_olmoe(T):
    from robustgemq_b200 import _lib, synth

    blk = _block(synth.olmoe_config)
    x = torch.randn((T, blk.hidden_dim), generator=torch.Generator(device="cuda").manual_seed(T),
                    device="cuda").half()
    ref = _fwd(blk, x, chain=False)
    for _ in range(3):  # the counters are zeroed by every forward's dispatch
        assert torch.equal(_fwd(blk, x, chain=True), ref)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_chained_down_launch_is_bit_identical_qwen3_prefill():
    """4096 tokens x top-8: the large-batch dispatch (histogram, scan, scatter); the
    prefill tiles run unchained, so both flags take the same path here."""
    from robustgemq_b200 import _lib, synth

    blk = _block(synth.qwen3_config)
    x = torch.randn((4096, blk.hidden_dim), generator=torch.Generator(device="cuda").manual_seed(1),
                    device="cuda").half()
    ref = _fwd(blk, x, chain=False)
    assert torch.equal(_fwd(blk, x, chain=True), ref)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_chained_down_launch_in_a_cuda_graph():
    from robustgemq_b200 import _lib, synth

    blk = _block(synth.olmoe_config)
    x = torch.randn((64, blk.hidden_dim), generator=torch.Generator(device="cuda").manual_seed(9),
                    device="cuda").half()
    ref = _fwd(blk, x, chain=False)
    xs = x.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _fwd(blk, xs, chain=True)  # warm-up outside capture (workspace, smem attributes)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = blk.forward_n_tokens(xs.unsqueeze(0))[0][0]
    for i in range(3):
        xs.copy_(x)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"replay {i}"
    assert _lib.device_error() == 0


def test_expired_wait_is_reported_and_the_context_stays_usable():
    """A wait that runs out (the chained down GEMM waits for a tile count nothing
    reaches, GEMQ_FWD_TEST_WAIT_EXPIRY) ends the forward within its time bound with
    a wait-expiry error recorded; the next forward on the same context is correct."""
    import time

    from robustgemq_b200 import _lib, synth

    blk = _block(synth.olmoe_config)
    x = torch.randn((64, blk.hidden_dim), generator=torch.Generator(device="cuda").manual_seed(5),
                    device="cuda").half()
    ref = _fwd(blk, x, chain=True)
    assert _lib.device_error() == 0
    blk._fwd_flags = _lib.FWD_TEST_WAIT_EXPIRY
    try:
        t0 = time.monotonic()
        blk.forward_n_tokens(x.unsqueeze(0))
        code = _lib.device_error()  # synchronises
        waited = time.monotonic() - t0
    finally:
        blk._fwd_flags = 0
    # 11: the chained wait; a pipeline wait of the same kernel (1-7) may run out a
    # moment earlier and be the one recorded
    assert code & 0xFF in (1, 2, 3, 4, 5, 6, 7, 11), code
    assert waited < 20.0
    assert torch.equal(_fwd(blk, x, chain=True), ref)
    assert _lib.device_error() == 0


def _fwd_one(blk, x, chain: bool):
    from robustgemq_b200 import _lib

    blk._fwd_flags = 0 if chain else _lib.FWD_NO_CHAIN
    try:
        out = blk.forward_one_token(x.view(1, 1, -1))
        return out[0] if isinstance(out, tuple) else out
    finally:
        blk._fwd_flags = 0


@pytest.mark.parametrize("family", ["olmoe", "deepseek"])
def test_chained_one_token_gemvs_are_bit_identical(family):
    """One-token path: the down GEMV starts with the up GEMV and waits per routed row
    for its partials; the output equals the unchained forward's, bit for bit, over
    several tokens and repeated calls (DeepSeek: the unchained shared experts after)."""
    from types import SimpleNamespace

    from robustgemq_b200 import _lib, synth
    from robustgemq_b200.inference import QuantFusedDeepseekV2MoEBlock

    if family == "olmoe":
        blk = _block(synth.olmoe_config)
    else:
        cfg = SimpleNamespace(hidden_size=2048, moe_intermediate_size=1408, n_routed_experts=64,
                              n_shared_experts=2, num_experts_per_tok=6, norm_topk_prob=False,
                              topk_method="greedy", scoring_func="softmax", routed_scaling_factor=1.0)
        blk = synth.random_block(QuantFusedDeepseekV2MoEBlock, cfg, 2048, 1408, 64, 2.75, 64, seed=4,
                                 device=torch.device("cuda"), shared_inter=2816)
    g = torch.Generator(device="cuda").manual_seed(17)
    for i in range(4):
        x = torch.randn((1, blk.hidden_dim), generator=g, device="cuda").half()
        ref = _fwd_one(blk, x, chain=False)
        for _ in range(2):
            assert torch.equal(_fwd_one(blk, x, chain=True), ref), i
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_chained_one_token_gemvs_in_a_cuda_graph():
    from robustgemq_b200 import _lib, synth

    blk = _block(synth.olmoe_config)
    x = torch.randn((1, blk.hidden_dim), generator=torch.Generator(device="cuda").manual_seed(2),
                    device="cuda").half()
    ref = _fwd_one(blk, x, chain=False)
    xs = x.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _fwd_one(blk, xs, chain=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = blk.forward_one_token(xs.view(1, 1, -1))[0]
    for i in range(3):
        xs.copy_(x)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"replay {i}"
    assert _lib.device_error() == 0
