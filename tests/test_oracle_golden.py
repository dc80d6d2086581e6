"""Pin the CPU oracle against golden vectors recorded from the reference itself.

The vectors come from ``tests/golden/make_golden.py``, which ran the reference's
Triton kernels and ``QuantFused*MoEBlock`` forwards under the Triton CPU
interpreter (``*_interp``: the interpreter's two-rounding fma; ``*_gpu``: the
single-rounding ``fma.rn.f16`` of the GPU lowering). Integer results and the
dequantised weights must agree bit for bit; products accumulate in fp32 in the
reference and in float64 here, so they agree to within fp16 rounding flips.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, proj_from, rel_l2
from oracle import gemq_oracle as O

# fp32-vs-float64 accumulation differs by at most a few fp16 rounding flips
PRODUCT_REL_TOL = 2e-3


def test_pack_matches_reference_kernel():
    d = load_golden("pack.npz")
    keys = sorted(k[:-6] for k in d if k.endswith("_codes"))
    assert len(keys) == 16
    for key in keys:
        nb = int(key[1])
        codes = d[f"{key}_codes"]
        packed = O.pack_weights_over_cols(codes, nb)
        assert packed.dtype == np.int32
        assert np.array_equal(packed, d[f"{key}_packed"]), key
        # round trip through the restated unpack (untransposed [N, words] buffer)
        assert np.array_equal(O.unpack_over_cols(packed.T, nb, codes.shape[1]), codes), key
        if f"{key}_unpacked" in d:
            assert np.array_equal(O.unpack_over_cols(packed.T, nb, codes.shape[1]), d[f"{key}_unpacked"]), key


def test_pack_ragged_three_bit_pads_high_bits_zero():
    codes = np.full((3, 13), 7, dtype=np.uint8)  # 13 = 10 + 3: second word holds 3 codes
    packed = O.pack_weights_over_cols(codes, 3, transpose=False).view(np.uint32)
    assert packed.shape == (3, 2)
    assert np.all(packed[:, 0] == (1 << 30) - 1)   # ten codes, bits 30-31 zero
    assert np.all(packed[:, 1] == (1 << 9) - 1)    # three codes, rest zero-padded


@pytest.mark.parametrize("g", [64, 128])
@pytest.mark.parametrize("mode", ["gpu", "interp"])
def test_dequant_bit_exact_against_reference(g, mode):
    d = load_golden("group_gemm.npz")
    proj = proj_from({k[len(f"g{g}_"):]: v for k, v in d.items() if k.startswith(f"g{g}_")}, "w")
    deq_ref = d[f"g{g}_deq_{mode}"]
    fma = "single" if mode == "gpu" else "double"
    for e in range(proj.num_experts):
        ours = O.dequantize_expert(proj, e, fma)
        assert ours.dtype == np.float16
        assert np.array_equal(ours.view(np.uint16), deq_ref[e].view(np.uint16)), (g, mode, e, int(proj.nbits[e]))


def test_single_and_double_rounding_differ_somewhere():
    """The two fma semantics are distinguishable on these inputs, so the bit-exact
    test above really pins the single-rounding one."""
    d = load_golden("group_gemm.npz")
    assert not np.array_equal(d["g64_deq_gpu"], d["g64_deq_interp"])


@pytest.mark.parametrize("g", [64, 128])
def test_group_gemm_matches_reference(g):
    d = load_golden("group_gemm.npz")
    sub = {k[len(f"g{g}_"):]: v for k, v in d.items() if k.startswith(f"g{g}_")}
    proj = proj_from(sub, "w")
    y = O.dequant_group_gemm(sub["x"], range(proj.num_experts), proj)
    assert rel_l2(y, sub["y_gpu"]) < PRODUCT_REL_TOL
    # max one fp16 ulp apart
    diff = np.abs(y.astype(np.float64) - sub["y_gpu"].astype(np.float64))
    ulp = np.spacing(np.abs(sub["y_gpu"]).astype(np.float16)).astype(np.float64)
    assert np.all(diff <= ulp + 1e-12)


def test_decode_kernels_match_reference():
    d = load_golden("decode_kernels.npz")
    w1, w3, w2 = proj_from(d, "w1"), proj_from(d, "w3"), proj_from(d, "w2")
    idx = [int(i) for i in d["idx"]]
    x1, x3 = O.fused_up_proj(d["x"], idx, w1, w3)
    assert rel_l2(x1, d["x1_gpu"]) < PRODUCT_REL_TOL
    assert rel_l2(x3, d["x3_gpu"]) < PRODUCT_REL_TOL
    # feed the reference's own fp16 x1/x3 to isolate the down projection
    x2 = O.fused_down_proj(d["x1_gpu"], d["x3_gpu"], idx, w2)
    assert rel_l2(x2, d["x2_gpu"]) < PRODUCT_REL_TOL
    sh, sh2 = proj_from(d, "sh"), proj_from(d, "sh2")
    assert rel_l2(O.dequant_gemm(d["xs"], sh), d["gemm_gpu"]) < PRODUCT_REL_TOL
    assert rel_l2(O.dequant_gemv(d["x"], sh), d["gemv_gpu"]) < PRODUCT_REL_TOL
    assert rel_l2(O.dequant_gemv(d["h2"], sh2), d["gemv2_gpu"]) < PRODUCT_REL_TOL


def block_weights(d: dict, family: str) -> O.BlockWeights:
    blk = O.BlockWeights(gate_w=d["gate_w"], w1=proj_from(d, "w1"), w3=proj_from(d, "w3"),
                         w2=proj_from(d, "w2"), top_k=int(d["top_k"]),
                         norm_topk_prob=bool(d["norm_topk_prob"]), router_fp32=(family == "deepseek"))
    if "shared_w1_wq" in d:
        blk.shared_w1, blk.shared_w3, blk.shared_w2 = (proj_from(d, n) for n in ("shared_w1", "shared_w3", "shared_w2"))
    return blk


FAMILIES = ["olmoe", "qwen3", "mixtral", "deepseek"]


@pytest.mark.parametrize("family", FAMILIES)
def test_block_prefill_matches_reference(family):
    d = load_golden(f"block_{family}.npz")
    blk = block_weights(d, family)
    routing = O.Routing(d["route_logits"], d["route_idx"].astype(np.int64), d["route_w"])
    y, _ = O.moe_forward_n_tokens(blk, d["x"], routing)
    assert rel_l2(y, d["y_ntok_gpu"]) < 1e-3
    y_i, _ = O.moe_forward_n_tokens(blk, d["x"], routing, fma="double")
    assert rel_l2(y_i, d["y_ntok_interp"]) < 1e-3


@pytest.mark.parametrize("family", FAMILIES)
def test_block_decode_matches_reference(family):
    d = load_golden(f"block_{family}.npz")
    blk = block_weights(d, family)
    routing = O.Routing(None, d["route1_idx"].astype(np.int64), d["route1_w"])
    y, _ = O.moe_forward_one_token(blk, d["x_one"], routing)
    assert rel_l2(y, d["y_one_gpu"]) < 1e-3


@pytest.mark.parametrize("family", FAMILIES)
def test_router_matches_reference(family):
    """The restated router picks the reference's experts and weights (ties broken
    toward the lower expert id; none occur in these vectors)."""
    d = load_golden(f"block_{family}.npz")
    blk = block_weights(d, family)
    r = O.route(d["x"], blk.gate_w, blk.top_k, blk.norm_topk_prob or family == "mixtral", blk.router_fp32)
    assert np.array_equal(r.topk_idx, d["route_idx"])
    assert np.abs(r.topk_w.astype(np.float32) - d["route_w"].astype(np.float32)).max() <= 1e-3
    r1 = O.route(d["x_one"], blk.gate_w, blk.top_k, blk.norm_topk_prob or family == "mixtral", blk.router_fp32,
                 softmax_fp16=(family == "mixtral"))
    assert np.array_equal(r1.topk_idx, d["route1_idx"])
    assert np.abs(r1.topk_w.astype(np.float32) - d["route1_w"].astype(np.float32)).max() <= 1e-3
