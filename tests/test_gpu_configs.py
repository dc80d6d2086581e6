"""Parity at the benchmark configurations' full shapes (``-m gpu``).

These run the exact paths the benchmark numbers come from, against the CPU
oracle on the same seeded inputs and the device's own routing:

* Qwen3-30B-A3B-shaped prefill at T=4096 with Zipf-skewed logits (g 128): 32768
  token-expert slots, so dispatch takes the histogram / scan / scatter kernels
  and the grouped GEMM its 128-token tiles;
* the tensor-core gate (T > 256 tokens) against the oracle's router: logits
  within fp16 rounding, and top-k ids / weights exactly the oracle's top-k of the
  device logits (ties to the lower expert id, as the reference's ``torch.topk``
  on equal values does in the golden fixtures);
* DeepSeek-V2-Lite-shaped prefill at T=2048 and decode batch 16, shared experts
  included;
* a Mixtral-8x7B-shaped layer on one GPU at T=2304 (4608 slots).

The reference's rel-L2 bar for the block (``north_star``: rel-L2 <= 1e-3) is the
tolerance. Reference: gemq/inference/moe_block.py:781-815 (n-token path),
549-578 (DeepSeek), tests/test_moe_block_equiv.py:342-416 (the reference's ladder).
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


def _np_proj(blk, name: str, K: int) -> O.PackedProj:
    from oracle.cpu_baseline import _proj_np

    return _proj_np(blk, name, K)


def _shared_np(blk, name: str, K: int) -> O.PackedProj:
    f = lambda a: getattr(blk, f"{name}_{a}").cpu().numpy()  # noqa: E731
    wq = f("wq")
    return O.PackedProj(wq=wq, scales=f("scales"), zeros=f("zeros"),
                        nbits=np.array([blk.shared_nbits], np.int32),
                        group_sizes=np.array([blk.shared_group_size], np.int32),
                        wq_strides=np.zeros(1, np.int32), zs_strides=np.zeros(1, np.int32), K=K, N=wq.shape[1])


def _oracle_block(blk) -> O.BlockWeights:
    ob = O.BlockWeights(gate_w=blk.gate.weight.detach().cpu().numpy(), w1=_np_proj(blk, "w1", blk.hidden_dim),
                        w3=_np_proj(blk, "w3", blk.hidden_dim), w2=_np_proj(blk, "w2", blk.ffn_dim),
                        top_k=blk.top_k, norm_topk_prob=bool(blk.norm_topk_prob or blk.always_normalize),
                        router_fp32=bool(blk.router_fp32))
    if getattr(blk, "has_shared", False):
        fs = blk.shared_w1_wq.shape[1]
        ob.shared_w1 = _shared_np(blk, "shared_w1", blk.hidden_dim)
        ob.shared_w3 = _shared_np(blk, "shared_w3", blk.hidden_dim)
        ob.shared_w2 = _shared_np(blk, "shared_w2", fs)
    return ob


def _device_routing(blk, x):
    _, idx, w = blk.route(x)
    return O.Routing(None, idx.cpu().numpy().astype(np.int64), w.cpu().numpy())


def _block(which: str, seed: int):
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import (QuantFusedDeepseekV2MoEBlock, QuantFusedMixtralMoEBlock,
                                           QuantFusedOlmoeMoEBlock, QuantFusedQwen3MoeMoEBlock)

    cls, (cfg, s) = {
        "olmoe": (QuantFusedOlmoeMoEBlock, synth.olmoe_config()),
        "qwen3": (QuantFusedQwen3MoeMoEBlock, synth.qwen3_config()),
        "deepseek": (QuantFusedDeepseekV2MoEBlock, synth.deepseek_config()),
        "mixtral": (QuantFusedMixtralMoEBlock, synth.mixtral_config()),
    }[which]
    return synth.random_block(cls, cfg, s["hidden"], s["inter"], s["num_experts"], s["mean_bits"], s["group_size"],
                              seed, torch.device("cuda"), shared_inter=s.get("shared_inter", 0)), s


def _x(T: int, D: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((T, D), generator=g, device="cuda").half()


def test_qwen3_prefill_t4096_zipf_large_dispatch():
    """Config 2 at its benchmark shape: T 4096, Zipf(1.1) logits, g 128."""
    from robustgemq_b200 import synth

    blk, s = _block("qwen3", 2024)
    T = 4096
    logits = synth.zipf_logits(T, s["num_experts"], 5, torch.device("cuda"))
    x = _x(T, s["hidden"], 6)
    y = blk.forward_logits(x, logits)
    torch.cuda.synchronize()
    r = O.route(None, None, blk.top_k, True, logits=logits.cpu().numpy())
    counts = np.bincount(r.topk_idx.ravel(), minlength=s["num_experts"])
    assert counts.max() > 4 * counts.mean(), "logits are not skewed"  # hot experts take many tiles
    yo, _ = O.moe_forward_n_tokens(_oracle_block(blk), x.cpu().numpy(), r)
    err = rel_l2(y.cpu().numpy(), yo)
    print(f"\n[qwen3 T=4096 zipf] rel-L2 {err:.3e}, max expert load {counts.max()}")
    assert err <= TOL


@pytest.mark.parametrize("which,T", [("olmoe", 512), ("qwen3", 4096), ("deepseek", 2048)])
def test_tensor_core_router_matches_oracle(which, T):
    """Gate logits from the tensor-core GEMM (T > 256), then top-k."""
    blk, s = _block(which, 31)
    x = _x(T, s["hidden"], 32)
    logits, idx, w = blk.route(x)
    torch.cuda.synchronize()
    ob = _oracle_block(blk)
    xr = x.cpu().numpy()
    ro = O.route(xr, ob.gate_w, blk.top_k, ob.norm_topk_prob, ob.router_fp32)
    lg = logits.float().cpu().numpy()
    assert rel_l2(lg, ro.logits.astype(np.float32)) <= 2e-3
    # logits agree to one fp16 rounding (different fp32 summation order)
    tol = 2.0 ** -10 * np.maximum(np.abs(ro.logits.astype(np.float64)), 2.0 ** -4)
    assert np.all(np.abs(lg - ro.logits.astype(np.float64)) <= 2 * tol + 1e-6)
    # top-k of the device logits: ids exact (equal probabilities -> lower id first)
    rd = O.route(None, None, blk.top_k, ob.norm_topk_prob, logits=logits.cpu().numpy())
    ids = idx.cpu().numpy().astype(np.int64)
    assert np.array_equal(ids, rd.topk_idx), f"{(ids != rd.topk_idx).any(axis=1).sum()} tokens differ"
    assert np.abs(w.float().cpu().numpy() - rd.topk_w.astype(np.float32)).max() <= 1e-3
    # against the oracle's own logits, ids differ only where the k-th and (k+1)-th
    # oracle probabilities are within the logits' rounding of each other
    p = O.softmax_f32(ro.logits.astype(np.float32)).astype(np.float64)
    ps = -np.sort(-p, axis=1)
    gap = ps[:, blk.top_k - 1] - ps[:, blk.top_k]
    differ = ~np.all(np.sort(ids, 1) == np.sort(ro.topk_idx, 1), axis=1)
    assert np.all(gap[differ] <= 4e-3 * ps[differ, blk.top_k - 1]), "a clear top-k choice differs"
    print(f"\n[{which} router T={T}] {differ.sum()} near-tie tokens differ from the oracle's logits")


def test_deepseek_prefill_t2048_and_decode_b16():
    """Config 3: 64 routed experts top-6 + 2 shared (one 2816-wide 4-bit SwiGLU), g 64."""
    blk, s = _block("deepseek", 303)
    ob = _oracle_block(blk)
    for T, seed in ((2048, 1), (16, 2)):
        x = _x(T, s["hidden"], seed)
        y = blk(x[None])[0]
        torch.cuda.synchronize()
        yo, _ = O.moe_forward_n_tokens(ob, x.cpu().numpy(), _device_routing(blk, x))
        err = rel_l2(y.cpu().numpy(), yo)
        print(f"\n[deepseek T={T}] rel-L2 {err:.3e}")
        assert err <= TOL
    # one token: fused GEMVs + split-K shared GEMVs
    x1 = _x(1, s["hidden"], 3)
    y1 = blk(x1[None])
    yo1, _ = O.moe_forward_one_token(ob, x1.cpu().numpy(), _device_routing(blk, x1))
    assert rel_l2(y1.reshape(1, -1).cpu().numpy(), yo1) <= TOL


def test_mixtral_layer_one_gpu_t2304():
    """Config 4's layer on one GPU: D 4096, F 14336, 8 experts top-2, g 128, mean 3 bits;
    2304 tokens = 4608 slots (the large-dispatch path)."""
    blk, s = _block("mixtral", 404)
    T = 2304
    x = _x(T, s["hidden"], 7)
    y, _ = blk(x[None])
    torch.cuda.synchronize()
    yo, _ = O.moe_forward_n_tokens(_oracle_block(blk), x.cpu().numpy(), _device_routing(blk, x))
    err = rel_l2(y[0].cpu().numpy(), yo)
    print(f"\n[mixtral T={T}] rel-L2 {err:.3e}")
    assert err <= TOL
