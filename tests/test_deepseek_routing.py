"""DeepSeek-V2 routing beyond the reference's fused block: group-limited greedy
selection and ``routed_scaling_factor``.

The reference's fused block rejects both (gemq/inference/moe_block.py:18-66); the
block it replaces computes them as transformers' ``DeepseekV2Moe.route_tokens_to_experts``
does (softmax in fp32; groups scored by their largest probability, the best
``topk_group`` kept, the rest masked to 0.0; top-k; weights times the scale). The
oracle's restatement is pinned here against that HF function on CPU; the ``-m gpu``
tests check the router kernel and the whole block against the oracle.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import rel_l2

E, K, NG, TG = 64, 6, 8, 3  # DeepSeek-V2-shaped selection at a smaller expert count


def _hf_moe(topk_method: str, scale: float, n_group: int = NG, topk_group: int = TG, k: int = K):
    from transformers import DeepseekV2Config
    from transformers.models.deepseek_v2.modeling_deepseek_v2 import DeepseekV2Moe

    cfg = DeepseekV2Config(hidden_size=32, moe_intermediate_size=16, n_routed_experts=E, n_shared_experts=1,
                           num_experts_per_tok=k, topk_method=topk_method, n_group=n_group, topk_group=topk_group,
                           routed_scaling_factor=scale, norm_topk_prob=False)
    moe = DeepseekV2Moe(cfg)
    # the group-limited branch reads self.num_experts, which this transformers version's
    # __init__ never sets (it raises AttributeError as shipped): give it the routed count
    moe.num_experts = E
    return moe


@pytest.mark.parametrize("topk_method,scale,n_group,topk_group,k", [
    ("group_limited_greedy", 16.0, NG, TG, K), ("group_limited_greedy", 1.0, 4, 1, 8),
    ("group_limited_greedy", 2.5, 32, 4, 6), ("greedy", 2.5, NG, TG, K),
])
def test_oracle_routing_matches_transformers(topk_method, scale, n_group, topk_group, k):
    from oracle import gemq_oracle as O

    moe = _hf_moe(topk_method, scale, n_group, topk_group, k)
    g = torch.Generator().manual_seed(5)
    logits = torch.randn((1, 257, E), generator=g) * 2.0
    with torch.no_grad():
        hf_idx, hf_w = moe.route_tokens_to_experts(logits)
    ng, tg = (n_group, topk_group) if topk_method == "group_limited_greedy" else (1, 1)
    r = O.route(None, None, k, False, router_fp32=True, logits=logits[0].numpy(), n_group=ng, topk_group=tg,
                scale=scale)
    hi = hf_idx.numpy()
    order_hf = np.argsort(hi, axis=-1)
    order_or = np.argsort(r.topk_idx, axis=-1)
    np.testing.assert_array_equal(np.take_along_axis(hi, order_hf, -1), np.take_along_axis(r.topk_idx, order_or, -1))
    w_hf = np.take_along_axis(hf_w.numpy(), order_hf, -1).astype(np.float16)
    w_or = np.take_along_axis(r.topk_w, order_or, -1)
    # fp32 softmax against the oracle's float64-then-fp32 one: at most one fp16 ulp apart
    assert np.all(np.abs(w_hf.astype(np.float32) - w_or.astype(np.float32))
                  <= np.spacing(np.maximum(np.abs(w_hf), np.abs(w_or))).astype(np.float32))
    if topk_method == "group_limited_greedy":
        greedy = O.route(None, None, k, False, router_fp32=True, logits=logits[0].numpy())
        assert (np.sort(greedy.topk_idx, -1) != np.sort(r.topk_idx, -1)).any(axis=-1).mean() > 0.2
        # every selected expert lies in one of the kept groups
        assert (np.unique(r.topk_idx // (E // n_group), axis=None).size <= n_group)
        assert max(len(set((row // (E // n_group)).tolist())) for row in r.topk_idx) <= topk_group


# ----------------------------------------------------------------------------- GPU
def _ds_block(norm: bool = False, scale: float = 16.0):
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedDeepseekV2MoEBlock

    cfg = SimpleNamespace(hidden_size=1024, moe_intermediate_size=512, n_routed_experts=E, n_shared_experts=2,
                          num_experts_per_tok=K, norm_topk_prob=norm, topk_method="group_limited_greedy",
                          n_group=NG, topk_group=TG, scoring_func="softmax", routed_scaling_factor=scale)
    blk = synth.random_block(QuantFusedDeepseekV2MoEBlock, cfg, 1024, 512, E, 2.75, 64, seed=31,
                             device=torch.device("cuda"), shared_inter=1024)
    blk.set_routing(norm_topk_prob=norm, routed_scaling_factor=scale)
    return blk


def _oracle_block(blk, scale: float):
    from oracle import gemq_oracle as O
    from oracle.cpu_baseline import _proj_np

    D, F = blk.hidden_dim, blk.ffn_dim
    sh = lambda n, k: O.PackedProj(  # noqa: E731
        wq=getattr(blk, f"shared_{n}_wq").cpu().numpy(), scales=getattr(blk, f"shared_{n}_scales").cpu().numpy(),
        zeros=getattr(blk, f"shared_{n}_zeros").cpu().numpy(), nbits=np.array([blk.shared_nbits], np.int32),
        group_sizes=np.array([blk.shared_group_size], np.int32), wq_strides=np.zeros(1, np.int32),
        zs_strides=np.zeros(1, np.int32), K=k, N=getattr(blk, f"shared_{n}_wq").shape[1])
    Fs = blk.shared_w1_wq.shape[1]
    return O.BlockWeights(gate_w=blk.gate.weight.detach().cpu().numpy(), w1=_proj_np(blk, "w1", D),
                          w3=_proj_np(blk, "w3", D), w2=_proj_np(blk, "w2", F), top_k=blk.top_k,
                          norm_topk_prob=blk.norm_topk_prob, router_fp32=True, shared_w1=sh("w1", D),
                          shared_w3=sh("w3", D), shared_w2=sh("w2", Fs), n_group=NG, topk_group=TG,
                          route_scale=scale)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 40, 300])  # one-token router, small-batch router, tensor-core router
@pytest.mark.parametrize("norm,scale", [(False, 16.0), (True, 1.0)])
def test_group_limited_router_matches_oracle(T, norm, scale):
    from oracle import gemq_oracle as O
    from robustgemq_b200 import _lib

    blk = _ds_block(norm, scale)
    x = torch.randn((T, 1024), generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").half()
    logits, idx, w = blk.route(x)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    lg = logits.cpu().numpy()
    ref_logits = (x.double().cpu().numpy() @ blk.gate.weight.detach().double().cpu().numpy().T)
    assert rel_l2(lg, ref_logits) <= 1e-5
    r = O.route(None, None, K, norm, router_fp32=True, logits=lg, n_group=NG, topk_group=TG, scale=scale)
    np.testing.assert_array_equal(idx.cpu().numpy(), r.topk_idx)
    wg = w.float().cpu().numpy()
    wr = r.topk_w.astype(np.float32)
    assert np.all(np.abs(wg - wr) <= np.spacing(np.maximum(np.abs(wg), np.abs(wr)).astype(np.float16)))
    if T >= 40:
        greedy = O.route(None, None, K, norm, router_fp32=True, logits=lg)
        assert (np.sort(greedy.topk_idx, -1) != np.sort(r.topk_idx, -1)).any(axis=-1).mean() > 0.2


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 40, 300])
def test_group_limited_block_matches_oracle(T):
    """The whole block (prefill path for T > 1, the one-token path for T = 1) against
    the oracle fed the GPU's fp32 logits, so both select the same experts."""
    from oracle import gemq_oracle as O
    from robustgemq_b200 import _lib

    scale = 16.0
    blk = _ds_block(False, scale)
    x = torch.randn((T, 1024), generator=torch.Generator(device="cuda").manual_seed(100 + T), device="cuda").half()
    logits, _, _ = blk.route(x)
    out = blk.forward(x.view(1, T, 1024) if T == 1 else x.view(T, 1, 1024))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ob = _oracle_block(blk, scale)
    r = O.route(None, None, K, False, router_fp32=True, logits=logits.cpu().numpy(), n_group=NG, topk_group=TG,
                scale=scale)
    xn = x.cpu().numpy()
    if T == 1:
        ref, _ = O.moe_forward_one_token(ob, xn, r)
    else:
        ref, _ = O.moe_forward_n_tokens(ob, xn, r)
    assert rel_l2(out.reshape(T, -1).float().cpu().numpy(), ref.reshape(T, -1).astype(np.float32)) <= 1e-3


def test_expert_parallel_carries_the_group_routing():
    """An expert-parallel wrapper routes over all experts with the block's group-limited
    selection and scale (``gemq_route_ex`` options), built on CPU without weights."""
    from robustgemq_b200.inference import QuantFusedDeepseekV2MoEBlock
    from robustgemq_b200.inference.expert_parallel import ExpertParallelMoE

    cfg = SimpleNamespace(hidden_size=64, moe_intermediate_size=32, n_routed_experts=E, n_shared_experts=1,
                          num_experts_per_tok=K, norm_topk_prob=False, topk_method="group_limited_greedy",
                          n_group=NG, topk_group=TG, scoring_func="softmax", routed_scaling_factor=16.0)
    blk = QuantFusedDeepseekV2MoEBlock(cfg)
    assert (blk.n_group, blk.topk_group) == (NG, TG)
    blk.set_routing(routed_scaling_factor=16.0)
    ep = ExpertParallelMoE(blk)
    assert ep.routing == (False, NG, TG, 16.0)
    r = blk.routing_options()
    assert (r.norm_topk_prob, r.n_group, r.topk_group, r.scale) == (0, NG, TG, 16.0)
