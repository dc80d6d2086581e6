"""Record the reference's own GPU outputs at the benchmark configurations.

Run on a B200 box whose checkout has the reference installed in ``baseline/_ref``
(``pip install --no-deps --target baseline/_ref <RobustGEMQ checkout>``)::

    python tests/golden/make_ref_gpu.py [--cases olmoe,qwen3,deepseek,mixtral] [--summary out.md]

For each case it builds one seeded synthetic layer with ``robustgemq_b200.synth``
on the GPU and hands the same packed tensors to the reference block
(``baseline/reference_gpu.py``). It then runs the reference's Triton path (its own
autotune, JIT-compiled for sm_100a) and this library's path on the same seeded
input. It writes ``tests/golden/refgpu_<case>.npz``, which holds:

* the seeds and shape, and checksums of the packed weights, so the GPU test can
  tell regenerated weights from a kernel change;
* 32 sampled output rows of the reference, with the expert ids the reference
  routed those rows to;
* the full-output rel-L2 between the two paths and the count of tokens whose
  expert sets differ (near ties of the two routers), both measured here;
* the reference's own run-to-run spread (max rel-L2 between repeated calls): its
  split-K GEMV, used for DeepSeek's shared experts at one token, adds fp16
  partial sums atomically in arrival order (dequant_gemv.py:115), so that path
  differs from itself from call to call.

``tests/test_gpu_refgpu.py`` regenerates each layer and input, runs this library,
and compares the sampled rows; no reference code is needed at test time. Timings
of both paths (CUDA events, after warm-up) are printed as a markdown table.

The one-token path of the reference asserts ``N % BLOCK_SIZE_N == 0`` on the
device (fused_dequant_bmm.py:51, 207). Its autotune block sizes are at most 128,
and every shape here has N divisible by 128 (checked before the call).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from baseline import reference_gpu as RG  # noqa: E402
from robustgemq_b200 import synth  # noqa: E402
from robustgemq_b200.inference import (QuantFusedDeepseekV2MoEBlock, QuantFusedMixtralMoEBlock,  # noqa: E402
                                       QuantFusedOlmoeMoEBlock, QuantFusedQwen3MoeMoEBlock)

SAMPLE_ROWS = 32

# case -> (family, layer seed, [(label, tokens, input seed, zipf logits seed or None)])
CASES = {
    "olmoe": ("olmoe", 1234, [("prefill T=512 (config 0)", 512, 11, None), ("decode B=1 (config 1)", 1, 12, None),
                              ("decode B=8 (config 1)", 8, 13, None), ("decode B=64 (config 1)", 64, 14, None)]),
    "qwen3": ("qwen3", 2024, [("prefill T=4096 Zipf (config 2)", 4096, 6, 5)]),
    "deepseek": ("deepseek", 303, [("prefill T=2048 (config 3)", 2048, 1, None), ("decode B=16 (config 3)", 16, 2, None),
                                   ("decode B=1", 1, 3, None)]),
    "mixtral": ("mixtral", 404, [("prefill T=2304 (config 4 layer)", 2304, 7, None), ("decode B=1", 1, 8, None)]),
}

FAMILY = {
    "olmoe": (QuantFusedOlmoeMoEBlock, synth.olmoe_config),
    "qwen3": (QuantFusedQwen3MoeMoEBlock, synth.qwen3_config),
    "deepseek": (QuantFusedDeepseekV2MoEBlock, synth.deepseek_config),
    "mixtral": (QuantFusedMixtralMoEBlock, synth.mixtral_config),
}


def make_layer(family: str, seed: int):
    cls, cfg_fn = FAMILY[family]
    cfg, s = cfg_fn()
    blk = synth.random_block(cls, cfg, s["hidden"], s["inter"], s["num_experts"], s["mean_bits"], s["group_size"],
                             seed, torch.device("cuda"), shared_inter=s.get("shared_inter", 0))
    return blk, s


def make_input(T: int, D: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((T, D), generator=g, device="cuda").half()


def weight_checksums(blk) -> np.ndarray:
    """Sums of the packed words (int64) and of the scales and zeros (float64), per projection."""
    out = []
    for name in ("w1", "w3", "w2"):
        out.append(float(getattr(blk, f"{name}_wq").to(torch.int64).sum().item()))
        out.append(float(getattr(blk, f"{name}_scales").double().sum().item()))
        out.append(float(getattr(blk, f"{name}_zeros").double().sum().item()))
    return np.array(out, dtype=np.float64)


def time_ms(fn, reps: int = 5) -> float:
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return float(np.median(times))


def reference_ids(ref, x: torch.Tensor, logits) -> np.ndarray:
    """The expert ids the reference's forward selects (the same torch ops, moe_block.py:790-793, 549-551)."""
    with torch.no_grad():
        if logits is not None:
            lg = logits
        elif type(ref).__name__.startswith("QuantFusedDeepseek"):
            lg = torch.nn.functional.linear(x.float(), ref.gate.weight.float())
        else:
            lg = ref.gate(x)
        p = torch.softmax(lg, dim=1, dtype=torch.float)
        return torch.topk(p, ref.top_k, dim=-1)[1].cpu().numpy()


def run_case(name: str, out_dir: Path, rows: list) -> None:
    family, seed, items = CASES[name]
    blk, s = make_layer(family, seed)
    ref = RG.reference_block(blk)
    data = {"family": np.array(family), "layer_seed": np.int64(seed), "weights_checksum": weight_checksums(blk)}
    assert s["inter"] % 128 == 0 and s["hidden"] % 128 == 0
    for i, (label, T, xseed, zseed) in enumerate(items):
        x = make_input(T, s["hidden"], xseed)
        logits = None if zseed is None else synth.zipf_logits(T, s["num_experts"], zseed, torch.device("cuda"))
        gate = ref.gate
        if logits is not None:
            ref.gate = RG.FixedLogits(logits)
        with torch.no_grad():
            ref_fn = lambda: RG.output(ref(x[None]))  # noqa: E731
            ours_fn = (lambda: blk.forward_logits(x, logits)) if logits is not None else \
                (lambda: RG.output(blk(x[None])))  # noqa: E731
            y_ref = ref_fn()  # first call: JIT + autotune
            ms_ref = time_ms(ref_fn)
            y_ref = ref_fn().reshape(T, -1)
            # the reference's own run-to-run spread (its split-K GEMV adds fp16 partials
            # atomically in arrival order, dequant_gemv.py:115; the other paths repeat exactly)
            spread = 0.0
            for _ in range(3):
                y2 = ref_fn().reshape(T, -1).double()
                spread = max(spread, float((y2 - y_ref.double()).norm() / y_ref.double().norm()))
            y_ours = ours_fn()
            ms_ours = time_ms(ours_fn)
            y_ours = ours_fn().reshape(T, -1)
        torch.cuda.synchronize()
        ids_ref = reference_ids(ref, x, logits)
        ref.gate = gate
        if logits is not None:
            ids_ours = torch.topk(torch.softmax(logits, 1), blk.top_k, dim=-1)[1].cpu().numpy()
        else:
            ids_ours = blk.route(x)[1].cpu().numpy()
        differ = ~np.all(np.sort(ids_ref, 1) == np.sort(ids_ours, 1), axis=1)
        a, b = y_ours.double(), y_ref.double()
        err = float((a - b).norm() / b.norm())
        same = torch.from_numpy(~differ).cuda()
        err_same = float((a[same] - b[same]).norm() / b[same].norm())
        rng = np.random.default_rng(1000 + i)
        sel = np.sort(rng.choice(T, size=min(SAMPLE_ROWS, T), replace=False))
        key = f"c{i}"
        data.update({f"{key}_label": np.array(label), f"{key}_T": np.int64(T), f"{key}_x_seed": np.int64(xseed),
                     f"{key}_zipf_seed": np.int64(-1 if zseed is None else zseed),
                     f"{key}_rows": sel.astype(np.int64),
                     f"{key}_y_ref": y_ref[torch.from_numpy(sel).cuda()].cpu().numpy(),
                     f"{key}_ids_ref": ids_ref[sel].astype(np.int32),
                     f"{key}_rel_l2_full": np.float64(err), f"{key}_rel_l2_same_routing": np.float64(err_same),
                     f"{key}_tokens_routed_differently": np.int64(differ.sum()),
                     f"{key}_ms_ref": np.float64(ms_ref), f"{key}_ms_ours": np.float64(ms_ours),
                     f"{key}_ref_spread": np.float64(spread)})
        rows.append((family, label, T, err, err_same, int(differ.sum()), ms_ref, ms_ours, spread))
        print(f"{family:8s} {label:32s} rel-L2 {err:.3e} (same routing {err_same:.3e}, {differ.sum()} tokens "
              f"routed differently, reference spread {spread:.1e})  ref {ms_ref:.3f} ms  ours {ms_ours:.3f} ms  "
              f"x{ms_ref / ms_ours:.1f}", flush=True)
    np.savez_compressed(out_dir / f"refgpu_{name}.npz", **data)
    del blk, ref
    torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", default=",".join(CASES))
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--summary", default=None, help="write the markdown table here")
    args = ap.parse_args()
    import triton

    rows = []
    for name in args.cases.split(","):
        run_case(name, Path(args.out), rows)
    lines = [f"triton {triton.__version__}, torch {torch.__version__}, {torch.cuda.get_device_name(0)}", "",
             "| family | case | tokens | rel-L2 ours vs reference GPU | same-routing rel-L2 | tokens routed "
             "differently | reference run-to-run spread | reference ms | ours ms | speed-up |",
             "|---|---|---|---|---|---|---|---|---|---|"]
    for fam, label, T, err, err_same, nd, mr, mo, sp in rows:
        lines.append(f"| {fam} | {label} | {T} | {err:.2e} | {err_same:.2e} | {nd} | {sp:.1e} | {mr:.3f} | "
                     f"{mo:.3f} | {mr / mo:.0f}x |")
    text = "\n".join(lines)
    print(text)
    if args.summary:
        Path(args.summary).write_text(text + "\n")


if __name__ == "__main__":
    main()
