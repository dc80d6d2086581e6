"""Chained gate/up -> down launch of the decode GEMM (``-m gpu``).

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
