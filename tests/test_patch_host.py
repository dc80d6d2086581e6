"""Model patching on the host: the two passes of gemq/inference/patch.py:165-181.

The CUDA packer is replaced by the oracle's packer here (these tests run without a
GPU), so what is checked is the plumbing: which modules get replaced, the 3-bit
padding of HQQ's unpacked codes, the scale / zero layout, and that each fused block
stacks its experts exactly as the oracle's ``stack_projection`` does. The GPU run
of the same flow is in test_gpu_patch.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import gemq_oracle as O
from patch_fakes import (EXPERTS, GROUP, HIDDEN, INTER, MODEL_NAME, FakeHQQLinear, expected_projection, fake_model,
                         quantised)


def _cpu_pack_linear(Q, scale, zero, nbits, group_size):
    from robustgemq_b200.quant import PackedLinear

    N, K = Q.shape
    words = np.ascontiguousarray(O.pack_weights_over_cols(Q.cpu().numpy(), nbits))
    s, z = O.kernel_scale_zero(scale.cpu().numpy(), zero.cpu().numpy(), N, K, group_size)
    return PackedLinear(W_q=torch.from_numpy(words), scales=torch.from_numpy(s), zeros=torch.from_numpy(z),
                        W_nbits=int(nbits), group_size=int(group_size), in_features=K, out_features=N)


@pytest.fixture
def cpu_packer(monkeypatch):
    from robustgemq_b200.inference import linear

    monkeypatch.setattr(linear, "pack_linear", _cpu_pack_linear)


def test_name_table_and_layers():
    from robustgemq_b200.inference import patch

    assert patch.NAME_TO_MODEL["allenai/OLMoE-1B-7B-0924"] is patch.ModelType.OLMOE
    assert patch.NAME_TO_MODEL["mistralai/Mixtral-8x7B-v0.1"] is patch.ModelType.MIXTRAL
    model, _ = fake_model("olmoe", num_layers=2)
    assert patch.get_blocks(model, "allenai/OLMoE-1B-7B-0924") is model.model.layers
    with pytest.raises(KeyError):
        patch.get_blocks(model, "unknown/model")


def test_hqq_linears_recognised_by_interface():
    from robustgemq_b200.inference import patch

    Q, s, z = quantised(np.random.default_rng(0), 64, 128, 4)
    assert patch.is_hqq_linear(FakeHQQLinear(Q, s, z, 4, GROUP))
    assert not patch.is_hqq_linear(nn.Linear(4, 4))
    assert not patch.is_hqq_linear(nn.Module())


def test_replace_linear_recursive_reaches_nested_children(monkeypatch):
    from robustgemq_b200.inference import patch

    seen = []

    def fake_create(layer, **kwargs):
        seen.append((layer.meta["shape"], kwargs))
        return nn.Identity()

    monkeypatch.setattr(patch, "create_linear_from_hqq", fake_create)
    model, _ = fake_model("olmoe", num_layers=2)
    keep = model.model.layers[0].mlp.gate
    patch.replace_linear_recursive(model, device="cpu")
    # per layer: q_proj, o_proj and 3 projections of each expert
    assert len(seen) == 2 * (2 + 3 * EXPERTS)
    assert all(kw == {"device": "cpu"} for _, kw in seen)
    assert isinstance(model.model.layers[1].self_attn.q_proj, nn.Identity)
    assert isinstance(model.model.layers[1].mlp.experts[3].down_proj, nn.Identity)
    assert model.model.layers[0].mlp.gate is keep  # a plain linear stays


def test_create_linear_guards():
    from robustgemq_b200.inference import patch

    Q, s, z = quantised(np.random.default_rng(1), 64, 128, 4)
    lin = FakeHQQLinear(Q, s, z, 4, GROUP)
    lin.meta["axis"] = 0
    with pytest.raises(AssertionError, match="axis==1"):
        patch.create_linear_from_hqq(lin)
    lin.meta["axis"] = 1
    with pytest.raises(NotImplementedError, match="float16"):
        patch.create_linear_from_hqq(lin, dtype=torch.bfloat16)


def test_quant_linear_argument_checks():
    from robustgemq_b200.inference.linear import QuantLinear

    with pytest.raises(ValueError):
        QuantLinear(5, 64, 128, 64)
    with pytest.raises(ValueError):
        QuantLinear(4, 48, 96, 64)  # group size not a multiple of 32
    with pytest.raises(ValueError):
        QuantLinear(4, 64, 96, 64)  # in_features not a multiple of the group
    with pytest.raises(ValueError):
        QuantLinear(4, 64, 128, 66)
    lin = QuantLinear(4, 64, 128, 64)
    with pytest.raises(RuntimeError, match="pack"):
        lin(torch.zeros(1, 128, dtype=torch.float16))
    with pytest.raises(ValueError):
        lin.pack(torch.zeros(64, 64, dtype=torch.uint8), torch.ones(128), torch.zeros(128))


def test_create_linear_packs_like_the_oracle(cpu_packer):
    from robustgemq_b200.inference import patch
    from robustgemq_b200.inference.linear import QuantLinear

    rng = np.random.default_rng(2)
    for nbits in (1, 2, 3, 4):
        Q, s, z = quantised(rng, 128, 256, nbits)  # 512 groups: 3-bit rows come back padded
        bias = torch.arange(128, dtype=torch.float16)
        lin = patch.create_linear_from_hqq(FakeHQQLinear(Q, s, z, nbits, GROUP, bias=bias))
        assert isinstance(lin, QuantLinear)
        want = expected_projection([(Q, s, z, nbits)], 256, 128)
        assert np.array_equal(lin.W_q.numpy(), want.wq), nbits
        assert np.array_equal(lin.scales.numpy(), want.scales), nbits
        assert np.array_equal(lin.zeros.numpy(), want.zeros), nbits
        assert torch.equal(lin.bias, bias)
        assert (lin.W_nbits, lin.group_size, lin.in_features, lin.out_features) == (nbits, GROUP, 256, 128)


@pytest.mark.parametrize("family", ["olmoe", "qwen3", "mixtral", "deepseek"])
def test_prepare_for_inference_stacks_experts_like_the_oracle(family, cpu_packer):
    from robustgemq_b200.inference import moe_block as mb
    from robustgemq_b200.inference import patch
    from robustgemq_b200.inference.linear import QuantLinear

    cls = {"olmoe": mb.QuantFusedOlmoeMoEBlock, "qwen3": mb.QuantFusedQwen3MoeMoEBlock,
           "mixtral": mb.QuantFusedMixtralMoEBlock, "deepseek": mb.QuantFusedDeepseekV2MoEBlock}[family]
    attr = "block_sparse_moe" if family == "mixtral" else "mlp"
    model, records = fake_model(family, num_layers=3)
    out = patch.prepare_for_inference(model, MODEL_NAME[family])
    assert out is model
    for i, layer in enumerate(model.model.layers):
        assert isinstance(layer.self_attn.q_proj, QuantLinear)
        assert isinstance(layer.self_attn.o_proj, QuantLinear)
        rec = records[i]
        block = getattr(layer, attr)
        if "dense_down_proj" in rec:  # DeepSeek's first layer, Qwen3's dense layer
            assert not isinstance(block, mb._QuantFusedMoEBlock)
            assert isinstance(block.down_proj, QuantLinear)
            continue
        assert isinstance(block, cls)
        assert np.array_equal(block.gate.weight.detach().numpy(), rec["gate"])
        for name, K, N in (("w1", HIDDEN, INTER), ("w3", HIDDEN, INTER), ("w2", INTER, HIDDEN)):
            want = expected_projection(rec[name], K, N)
            for f in ("wq", "scales", "zeros", "nbits", "wq_strides", "zs_strides"):
                assert np.array_equal(getattr(block, f"{name}_{f}").numpy(), getattr(want, f)), (i, name, f)
        assert block.block_group_size == GROUP
        if family == "deepseek":
            for name, key in (("shared_w1", "sw1"), ("shared_w3", "sw3"), ("shared_w2", "sw2")):
                K, N = (INTER, HIDDEN) if name == "shared_w2" else (HIDDEN, INTER)
                want = expected_projection(rec[key], K, N)
                assert np.array_equal(getattr(block, f"{name}_wq").numpy(), want.wq), name
                assert np.array_equal(getattr(block, f"{name}_zeros").numpy(), want.zeros), name
            assert block.shared_nbits == 4


def test_unsupported_models_and_fp_path_raise():
    from robustgemq_b200.inference import patch

    model, _ = fake_model("olmoe", num_layers=1)
    with pytest.raises(NotImplementedError):
        patch.replace_moe_blocks(model, "meta-llama/Llama-2-7b-hf", model.config)
    with pytest.raises(NotImplementedError):
        patch.prepare_for_inference(model, "allenai/OLMoE-1B-7B-0924", is_fp=True)
    with pytest.raises(KeyError):
        patch.replace_moe_blocks(model, "unknown/model", model.config)
