"""Decode-batch tensor-memory GEMM on shapes where the two dequant warp groups see
different scale chunks (``-m gpu``).

The decode GEMM's dequant warps take alternate 128-k stages; scale/zero rows come in
chunks of 16 groups (8 stages at g = 64). With K = 1152 an item has 9 stages and its
last chunk holds a single stage, which only one of the two groups reads; the other
must still release it or the next item's scale load would wait forever. The down
projection (K = inter) meets this at inter = 1152 or 2176; the gate/up projection
cannot, as the decode GEMM needs hidden % 256 == 0 for the down projection. The results
must agree with the shared-memory dequant GEMM (same exact dequantised weights,
another fp32 summation order) and no kernel may record a device error.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hidden,inter,tokens", [(2048, 1152, 8), (2048, 1152, 40), (1024, 2176, 16)])
def test_decode_gemm_single_stage_last_chunk(hidden, inter, tokens):
    from robustgemq_b200 import _lib, synth
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg = SimpleNamespace(hidden_size=hidden, intermediate_size=inter, num_experts=16, num_experts_per_tok=4,
                          norm_topk_prob=False)
    blk = synth.random_block(QuantFusedOlmoeMoEBlock, cfg, hidden, inter, 16, 2.5, 64, 5, torch.device("cuda"))
    gen = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((tokens, hidden), generator=gen, device="cuda").half()
    _lib.device_error()
    _, idx, w = blk.route(x)
    y_tmem = blk.forward_routed(x, idx, w).float()
    blk._fwd_flags = _lib.FWD_SMEM_DEQUANT
    y_smem = blk.forward_routed(x, idx, w).float()
    blk._fwd_flags = 0
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.isfinite(y_tmem).all()
    assert rel_l2(y_tmem.cpu().numpy(), y_smem.cpu().numpy()) <= 5e-4
