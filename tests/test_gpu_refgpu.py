"""Parity with the reference's own GPU path at the benchmark configurations (``-m gpu``).

``tests/golden/make_ref_gpu.py`` ran the reference's Triton MoE blocks
(gemq/inference/moe_block.py:781-858, its kernels JIT-compiled for the B200) on
seeded synthetic layers and recorded 32 sampled output rows per case, with the
experts the reference routed them to. This test regenerates the same layer and
input, runs this library through the public block API and compares those rows.
The bar is ``north_star``'s: rel-L2 <= 1e-3 against the reference's GPU path.

Rows whose expert set differs between the two routers (fp16 gate logits that
round differently at a near tie) are excluded from the rel-L2 and counted; at
most one such row per sample is allowed.

Where the reference is not deterministic (DeepSeek's shared experts at one token
go through its split-K GEMV, which adds fp16 partial sums atomically in arrival
order, dequant_gemv.py:115), no implementation can sit closer to it than its own
run-to-run spread, recorded in the fixture; the bar there is 1e-3 plus twice that
spread. This library rounds the exact sum once (the centre of that spread) and
is checked against the CPU oracle at 1e-3 on the same path
(tests/test_gpu_configs.py).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3
FIXTURES = sorted(p.name for p in GOLDEN.glob("refgpu_*.npz"))


def _load(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


@pytest.mark.parametrize("fixture", FIXTURES)
def test_block_matches_reference_gpu_path(fixture, cuda_device):
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_ref_gpu as M
    from robustgemq_b200 import _lib, synth

    d = _load(fixture)
    family = str(d["family"])
    blk, s = M.make_layer(family, int(d["layer_seed"]))
    np.testing.assert_allclose(M.weight_checksums(blk), d["weights_checksum"], rtol=1e-9, atol=0,
                               err_msg="regenerated weights differ from the fixture's (not a kernel error)")
    i = 0
    while f"c{i}_T" in d:
        k = f"c{i}"
        T = int(d[f"{k}_T"])
        x = M.make_input(T, s["hidden"], int(d[f"{k}_x_seed"]))
        zseed = int(d[f"{k}_zipf_seed"])
        rows = torch.from_numpy(d[f"{k}_rows"]).cuda()
        if zseed >= 0:
            logits = synth.zipf_logits(T, s["num_experts"], zseed, torch.device("cuda"))
            y = blk.forward_logits(x, logits)
            ids = torch.topk(torch.softmax(logits, 1), blk.top_k, dim=-1)[1]
        else:
            y = blk(x[None])
            y = (y[0] if isinstance(y, tuple) else y).reshape(T, -1)
            ids = blk.route(x)[1]
        got = y[rows].cpu().numpy()
        ids = ids[rows].cpu().numpy()
        same = np.all(np.sort(ids, 1) == np.sort(d[f"{k}_ids_ref"], 1), axis=1)
        err = rel_l2(got[same], d[f"{k}_y_ref"][same])
        label = str(d[f"{k}_label"])
        print(f"\n[{family} {label}] rel-L2 vs reference GPU {err:.3e} over {same.sum()} rows "
              f"(recorded full-output {float(d[f'{k}_rel_l2_same_routing']):.2e})")
        spread = float(d.get(f"{k}_ref_spread", 0.0))
        tol = TOL + 2 * spread
        assert (~same).sum() <= 1, f"{label}: {(~same).sum()} sampled rows routed differently"
        assert err <= tol, f"{label}: {err:.3e} (reference spread {spread:.1e})"
        assert float(d[f"{k}_rel_l2_same_routing"]) <= tol, label
        i += 1
    assert i > 0
    assert _lib.device_error() == 0
