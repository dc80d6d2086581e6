"""Model patching on the GPU (``-m gpu``): HQQ-style linears -> ``QuantLinear`` and
fused MoE blocks, run through the sm_100a kernels.

* ``QuantLinear`` (the GemLite linear's counterpart, patch.py:27-72) against the
  oracle's dequant product, for one row (split-K GEMV) and several rows (tensor-core
  GEMM), with and without bias;
* the packed tensors the CUDA packer produced are bit-identical to the oracle's;
* a patched OLMoE-shaped model's MoE layer returns exactly what a block built
  directly from the same codes returns, for prefill and one-token decode.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import gemq_oracle as O
from patch_fakes import HIDDEN, INTER, MODEL_NAME, expected_projection, fake_model, family_config

pytestmark = pytest.mark.gpu

PRODUCT_REL_TOL = 2e-3  # fp16 output against the oracle's exact product rounded once


@pytest.fixture(autouse=True)
def _no_device_error(cuda_device):
    from robustgemq_b200 import _lib

    _lib.device_error()
    yield
    assert _lib.device_error() == 0, "a kernel recorded a device-side error"


@pytest.fixture(scope="module")
def patched():
    from robustgemq_b200.inference import patch

    model, records = fake_model("olmoe", num_layers=2, seed=3, device="cuda")
    patch.prepare_for_inference(model, MODEL_NAME["olmoe"])
    return model, records


def test_quant_linear_matches_oracle(patched):
    model, records = patched
    rng = np.random.default_rng(7)
    for name in ("q_proj", "o_proj"):
        Q, s, z, nbits, bias = records[0][name]
        lin = getattr(model.model.layers[0].self_attn, name)
        want = expected_projection([(Q, s, z, nbits)], HIDDEN, HIDDEN)
        assert np.array_equal(lin.W_q.cpu().numpy(), want.wq), name
        assert np.array_equal(lin.scales.cpu().numpy(), want.scales), name
        assert np.array_equal(lin.zeros.cpu().numpy(), want.zeros), name
        for rows in (1, 5, 130):
            x = rng.standard_normal((rows, HIDDEN)).astype(np.float16)
            ref = O.dequant_gemm(x, want).astype(np.float64)
            if bias is not None:
                ref = ref + bias.cpu().numpy().astype(np.float64)
            y = lin(torch.from_numpy(x).cuda().reshape(1, rows, HIDDEN))
            assert y.shape == (1, rows, HIDDEN) and y.dtype == torch.float16
            assert rel_l2(y.reshape(rows, HIDDEN).cpu().numpy(), ref) < PRODUCT_REL_TOL, (name, rows)


def test_patched_moe_layer_equals_direct_block(patched):
    from robustgemq_b200.inference import moe_block as mb
    from robustgemq_b200.quant import pack_linear

    model, records = patched
    rec = records[1]
    blk = model.model.layers[1].mlp
    assert isinstance(blk, mb.QuantFusedOlmoeMoEBlock)
    blk.gate.cuda()

    def packed(entries):
        return [pack_linear(torch.from_numpy(Q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(z).cuda(),
                            nb, blk.block_group_size) for Q, s, z, nb in entries]

    direct = mb.QuantFusedOlmoeMoEBlock.from_packed(family_config("olmoe"), torch.from_numpy(rec["gate"]).cuda(),
                                                     packed(rec["w1"]), packed(rec["w3"]), packed(rec["w2"]))
    direct.gate.cuda()
    for f in ("wq", "scales", "zeros", "nbits", "wq_strides", "zs_strides"):
        for name, K, N in (("w1", HIDDEN, INTER), ("w3", HIDDEN, INTER), ("w2", INTER, HIDDEN)):
            assert np.array_equal(getattr(blk, f"{name}_{f}").cpu().numpy(),
                                  getattr(expected_projection(rec[name], K, N), f)), (name, f)
    g = torch.Generator(device="cuda").manual_seed(11)
    for shape in ((2, 9, HIDDEN), (1, 1, HIDDEN)):
        h = torch.randn(shape, generator=g, device="cuda").half()
        out, logits = blk(h)
        ref, ref_logits = direct(h)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), shape
        if logits is not None:
            assert torch.equal(logits, ref_logits), shape
