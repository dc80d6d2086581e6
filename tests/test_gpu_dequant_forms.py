"""The tensor-memory GEMM's two dequant forms give bit-identical blocks (``-m gpu``).

A layer whose scales all fit the single-instruction (subnormal-operand) form uses it;
one scale outside its range sends that projection back to the general form. Both
compute fp16(q * s + z) with one rounding (gemq/triton_kernels/utils.py:206-210), and
the GEMM's summation order does not depend on the form, so a block whose only change
is one scale of an expert no token is routed to must give the same bits. Every
bit-width (1-4) meets both forms, at decode (token tiles 16 / 32) and prefill (64)
sizes and in the one-token GEMV path; the outputs are also checked against the
oracle's dequantised weights.
"""

from __future__ import annotations

import ctypes
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

HIDDEN, INTER, E, TOPK, G = 1024, 512, 9, 4, 64
BITS = [1, 2, 3, 4, 1, 2, 3, 4, 2]  # expert E - 1 is never routed to


def _block():
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg = SimpleNamespace(hidden_size=HIDDEN, intermediate_size=INTER, num_experts=E, num_experts_per_tok=TOPK,
                          norm_topk_prob=False)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(23)
    w1 = [synth.random_packed_linear(INTER, HIDDEN, b, G, gen, dev) for b in BITS]
    w3 = [synth.random_packed_linear(INTER, HIDDEN, b, G, gen, dev) for b in BITS]
    w2 = [synth.random_packed_linear(HIDDEN, INTER, b, G, gen, dev) for b in BITS]
    gate = (torch.randn((E, HIDDEN), generator=gen, device=dev) * 0.02).half()
    blk = QuantFusedOlmoeMoEBlock.from_packed(cfg, gate, w1, w3, w2)
    blk.gate.to(dev)
    return blk


def _forms(blk):
    from robustgemq_b200 import _lib

    out = (ctypes.c_int32 * 3)()
    _lib.check(_lib.load().gemq_layer_dequant_forms(blk.layer_handle(), out))
    return list(out)


def _routing(T: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E - 1, generator=g)[:TOPK] for _ in range(T)]).to(torch.int32)
    w = (torch.rand((T, TOPK), generator=g) * 0.5 + 0.1).half()
    return idx.cuda(), w.cuda()


@pytest.mark.parametrize("proj", ["w1", "w3", "w2"])
def test_dequant_forms_bit_identical(proj):
    from robustgemq_b200 import _lib

    blk = _block()
    assert _forms(blk) == [1, 1, 1], "synthetic RTN scales should all fit the single-instruction form"
    cases = []
    for T, seed in ((3, 1), (12, 2), (40, 3), (300, 4)):
        x = torch.randn((T, HIDDEN), generator=torch.Generator(device="cuda").manual_seed(seed), device="cuda").half()
        idx, w = _routing(T, seed)
        cases.append((x, idx, w))
    _lib.device_error()
    one_x = torch.randn((1, HIDDEN), generator=torch.Generator(device="cuda").manual_seed(9), device="cuda").half()
    one_idx, one_w = _routing(1, 9)
    y_sub = [blk.forward_routed(x, idx, w) for x, idx, w in cases]
    y_sub.append(blk.forward_routed(one_x, one_idx, one_w, one_token=True))  # the one-token GEMV path
    # one scale of the unrouted expert out of the single-instruction range (exponent 15)
    scales = getattr(blk, f"{proj}_scales")
    z0 = int(getattr(blk, f"{proj}_zs_strides")[E - 1].item())
    scales.view(-1)[z0] = 1024.0
    blk.invalidate()
    forms = _forms(blk)
    assert forms == [int(p != proj) for p in ("w1", "w3", "w2")]
    y_gen = [blk.forward_routed(x, idx, w) for x, idx, w in cases]
    y_gen.append(blk.forward_routed(one_x, one_idx, one_w, one_token=True))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for a, b in zip(y_sub, y_gen):
        assert torch.equal(a, b)


def test_dequant_form_against_oracle():
    """The single-instruction form against the oracle's fp16 block (float64 sums)."""
    from robustgemq_b200 import _lib
    from oracle import gemq_oracle as O
    from oracle.cpu_baseline import _proj_np

    blk = _block()
    assert _forms(blk) == [1, 1, 1]
    T = 40
    x = torch.randn((T, HIDDEN), generator=torch.Generator(device="cuda").manual_seed(7), device="cuda").half()
    idx, w = _routing(T, 7)
    y = blk.forward_routed(x, idx, w).float().cpu().numpy()
    assert _lib.device_error() == 0
    ob = O.BlockWeights(gate_w=blk.gate.weight.detach().cpu().numpy(), w1=_proj_np(blk, "w1", HIDDEN),
                        w3=_proj_np(blk, "w3", HIDDEN), w2=_proj_np(blk, "w2", INTER), top_k=TOPK,
                        norm_topk_prob=False)
    ref, _ = O.moe_forward_n_tokens(ob, x.cpu().numpy(), O.Routing(None, idx.cpu().numpy().astype(np.int64),
                                                                   w.cpu().numpy()))
    assert rel_l2(y, ref.astype(np.float32)) <= 1e-3
