"""Full-size shapes of the benchmark configs against the CPU oracle (``-m gpu``).

One synthetic OLMoE-shaped layer (D 2048, F 1024, 64 experts, top-8, g 64, mean
2.5 bits) at decode batches 1 / 8 / 64 and a 512-token prefill, plus a
Qwen3-shaped layer (128 experts, F 768, g 128) with Zipf-skewed logits; outputs
compared with the oracle on the same routing at rel-L2 <= 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import gemq_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(autouse=True)
def _no_device_error(cuda_device):
    from robustgemq_b200 import _lib

    _lib.device_error()
    yield
    assert _lib.device_error() == 0, "a kernel recorded a device-side error"


def _oracle_block(blk):
    from oracle.cpu_baseline import _proj_np

    return O.BlockWeights(gate_w=blk.gate.weight.detach().cpu().numpy(), w1=_proj_np(blk, "w1", blk.hidden_dim),
                          w3=_proj_np(blk, "w3", blk.hidden_dim), w2=_proj_np(blk, "w2", blk.ffn_dim),
                          top_k=blk.top_k, norm_topk_prob=blk.norm_topk_prob)


@pytest.fixture(scope="module")
def olmoe_layer():
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg, s = synth.olmoe_config()
    blk = synth.random_block(QuantFusedOlmoeMoEBlock, cfg, s["hidden"], s["inter"], s["num_experts"], s["mean_bits"],
                             s["group_size"], 1234, torch.device("cuda"))
    return blk, _oracle_block(blk)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_olmoe_decode_batches(olmoe_layer, B):
    blk, ob = olmoe_layer
    g = torch.Generator(device="cuda").manual_seed(B)
    x = torch.randn((B, blk.hidden_dim), generator=g, device="cuda").half()
    logits, idx, w = blk.route(x)
    assert torch.isfinite(logits.float()).all()
    assert int(idx.min()) >= 0 and int(idx.max()) < blk.num_experts
    xn = x.cpu().numpy()
    routing = O.Routing(None, idx.cpu().numpy().astype(np.int64), w.cpu().numpy())
    if B == 1:
        y = blk.forward_routed(x, idx, w, one_token=True)
        yo, _ = O.moe_forward_one_token(ob, xn, routing)
    else:
        y = blk.forward_routed(x, idx, w)
        yo, _ = O.moe_forward_n_tokens(ob, xn, routing)
    assert torch.isfinite(y).all()
    err = rel_l2(y.cpu().numpy(), yo)
    print(f"\n[olmoe B={B}] rel-L2 {err:.3e}")
    assert err <= TOL
    # the residual flag adds x in fp16 after the block (decoder residual)
    from robustgemq_b200 import _lib

    flags = _lib.FWD_RESIDUAL | (_lib.FWD_ONE_TOKEN if B == 1 else 0)
    yr, _ = blk._run(x, flags, want_logits=False, topk_idx=idx, topk_w=w)
    ref = (y.float() + x.float()).half()
    assert torch.equal(yr, ref)


def test_olmoe_prefill_512(olmoe_layer):
    blk, ob = olmoe_layer
    g = torch.Generator(device="cuda").manual_seed(512)
    x = torch.randn((512, blk.hidden_dim), generator=g, device="cuda").half()
    out, logits = blk.forward_n_tokens(x[None])
    _, idx, w = blk.route(x)
    routing = O.Routing(None, idx.cpu().numpy().astype(np.int64), w.cpu().numpy())
    yo, _ = O.moe_forward_n_tokens(ob, x.cpu().numpy(), routing)
    err = rel_l2(out[0].cpu().numpy(), yo)
    print(f"\n[olmoe prefill 512] rel-L2 {err:.3e}")
    assert err <= TOL


def test_qwen3_prefill_zipf():
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedQwen3MoeMoEBlock

    cfg, s = synth.qwen3_config()
    blk = synth.random_block(QuantFusedQwen3MoeMoEBlock, cfg, s["hidden"], s["inter"], s["num_experts"],
                             s["mean_bits"], s["group_size"], 77, torch.device("cuda"))
    T = 384
    logits = synth.zipf_logits(T, s["num_experts"], 3, torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn((T, s["hidden"]), generator=g, device="cuda").half()
    y = blk.forward_logits(x, logits)
    ob = _oracle_block(blk)
    r = O.route(None, None, blk.top_k, True, logits=logits.cpu().numpy())
    yo, _ = O.moe_forward_n_tokens(ob, x.cpu().numpy(), r)
    err = rel_l2(y.cpu().numpy(), yo)
    print(f"\n[qwen3 prefill zipf] rel-L2 {err:.3e}")
    assert err <= TOL
