#!/usr/bin/env python
"""Benchmark of the fused mixed-bit MoE path (one JSON line on rank 0).

Headline workload: OLMoE-shaped 16-layer MoE stack, decode at
batch 1, 8, 32 and 64. One step = one pass of the 16-layer stack at each batch
size, each batch size replayed as one CUDA graph; layer l reads its own seeded
N(0, 1) input (the normalised hidden state a decoder feeds its MoE; chaining
un-normalised MoE outputs would overflow fp16), rotated over 4 input sets so the
routing changes from step to step. ``value`` =
algorithmic HBM bytes of all passes (packed weights + fp16 scales/zeros of every
expert the routing hits, the gate weights, activations in/out) / device time, in
GB/s, summed over ranks (``--gpus N`` runs N independent replicas: weak scaling).

Also reported: per-batch GB/s and tokens/s, Qwen3-30B-A3B-shaped prefill (BASELINE
config 2, Zipf-skewed router logits) tokens/s and TFLOP/s, the dominant stage's
roofline from library stage timers, ``e2e`` through the public block API with
pinned host buffers, the CPU fake-quant baseline (``cpu_baseline``), clocks.
``--impl reference`` times the reference's CPU fake-quant path instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer prefill tokens/s + decode HBM GB/s (% roofline) at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batches", default="1,8,32,64")
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--prefill-layers", type=int, default=48)
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--ep-layers", type=int, default=2)
    ap.add_argument("--ep-tokens", type=int, default=8192)
    ap.add_argument("--no-ep", action="store_true")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="token chunks of the expert-parallel forward (exchanges overlap the previous chunk's GEMMs)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-configs", action="store_true", help="skip the config 0 / config 3 sub-objects")
    ap.add_argument("--no-generate", action="store_true", help="skip the whole-model decode sub-object")
    ap.add_argument("--reference-gpu", default="prefill", choices=["none", "prefill", "all"],
                    help="time the reference's own Triton path beside ours (N=1, when baseline/_ref is installed)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ----------------------------------------------------------------------------- clocks
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        # the samples go to GEMQ_BENCH_CLOCKS_CSV when it is set (to keep them), else
        # to a fresh temporary file
        keep = os.environ.get("GEMQ_BENCH_CLOCKS_CSV")
        if keep:
            self.path = Path(keep)
        else:
            fd, name = tempfile.mkstemp(prefix="gemq_bench_clocks_", suffix=".csv")
            os.close(fd)
            self.path = Path(name)

    def start(self):
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # the timed region starts only once the sampler is producing rows
        deadline = time.time() + 5.0
        while time.time() < deadline:
            self.f.flush()
            if self.path.exists() and self.path.stat().st_size > 0:
                break
            time.sleep(0.02)

    def stop(self, gpus):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.f.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in gpus:
                continue
            rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        loaded = [v for v in sm if v > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ----------------------------------------------------------------------------- our arm
def build_stack(n_layers, device, seed0):
    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg, shp = synth.olmoe_config()
    blocks = []
    for l in range(n_layers):
        blocks.append(synth.random_block(QuantFusedOlmoeMoEBlock, cfg, shp["hidden"], shp["inter"],
                                         shp["num_experts"], shp["mean_bits"], shp["group_size"], seed0 + l, device))
    return blocks


def stack_forward(blocks, xs, one_token, time_stages=False, outs=None):
    """Layer l reads its own input xs[l] (a normalised hidden state stands in for the
    residual stream after RMSNorm, which an un-normalised MoE chain lacks) and
    writes outs[l]. Returns the stacked outputs."""
    from robustgemq_b200 import _lib

    flags = _lib.FWD_ONE_TOKEN if one_token else 0
    if time_stages:
        flags |= _lib.FWD_TIME_STAGES
    res = []
    for l, blk in enumerate(blocks):
        y, _ = blk._run(xs[l], flags, want_logits=False)
        res.append(y)
    return res


def stage_times(blk):
    import ctypes

    from robustgemq_b200 import _lib

    arr = (ctypes.c_float * 6)()
    _lib.check(_lib.load().gemq_layer_stage_times(blk.layer_handle(), arr))
    return list(arr)


def decode_bytes(blocks, expert_bytes, xs):
    """Algorithmic HBM bytes of one stack pass from its actual routing (untimed):
    hit experts' packed words + scales/zeros, gate weights, activations in/out."""
    import torch

    B, D = xs[0].shape
    total = 0
    for l, (blk, eb) in enumerate(zip(blocks, expert_bytes)):
        _, idx, _ = blk.route(xs[l])
        hit = torch.unique(idx).tolist()
        assert 0 <= min(hit) and max(hit) < blk.num_experts
        total += sum(eb[e] for e in hit) + blk.num_experts * D * 2 + 2 * B * D * 2
    return total


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from robustgemq_b200 import _lib, synth

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    hbm_peak, bf16_peak, bf16_sus, peak_src = peaks()
    batches = [int(b) for b in args.batches.split(",")]
    t0 = time.time()
    blocks = build_stack(args.layers, device, 1000)
    expert_bytes = [synth.layer_expert_bytes(b) for b in blocks]
    D = blocks[0].hidden_dim
    n_sets = 4
    gen = torch.Generator(device=device).manual_seed(7 + rank)
    L = args.layers
    # n_sets input sets per batch size, each [L, B, D]: layer l's normalised input
    inputs = {B: [torch.randn((L, B, D), generator=gen, device=device).half() for _ in range(n_sets)]
              for B in batches}
    # per-batch algorithmic bytes, averaged over the input sets
    bytes_per_pass = {B: sum(decode_bytes(blocks, expert_bytes, xs) for xs in inputs[B]) / n_sets for B in batches}
    # warm the workspaces, then capture one graph per batch size
    static_in = {B: inputs[B][0].clone() for B in batches}
    graphs, static_out = {}, {}
    for B in batches:
        for _ in range(2):
            stack_forward(blocks, static_in[B], B == 1)
    torch.cuda.synchronize()
    for B in batches:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static_out[B] = stack_forward(blocks, static_in[B], B == 1)
        graphs[B] = g
    torch.cuda.synchronize()
    setup_s = time.time() - t0

    def step(i):
        for B in batches:
            static_in[B].copy_(inputs[B][i % n_sets])
            graphs[B].replay()

    for i in range(args.warmup):
        step(i)
    # per-batch timing (outside the timed region; for the breakdown)
    per_b = {}
    for B in batches:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, args.steps // 2)
        torch.cuda.synchronize()
        s.record()
        for i in range(reps):
            static_in[B].copy_(inputs[B][i % n_sets])
            graphs[B].replay()
        e.record()
        torch.cuda.synchronize()
        per_b[B] = s.elapsed_time(e) / reps

    clocks = Clocks() if rank == 0 else None
    if clocks:
        clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        step(i)
    stop.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(stop)
    clk = clocks.stop(list(range(world)) if world > 1 else [torch.cuda.current_device()]) if clocks else None
    ms_t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    step_bytes = sum(bytes_per_pass.values())
    value = world * step_bytes * args.steps / (ms_max * 1e-3) / 1e9

    # e2e through the block API: every step copies its per-layer inputs from pinned
    # host memory and reads every layer's output back (eager calls)
    host_in = {B: [t.cpu().pin_memory() for t in inputs[B]] for B in batches}
    host_out = {B: torch.empty((L, B, D), dtype=torch.float16).pin_memory() for B in batches}
    dev_in = {B: torch.empty((L, B, D), dtype=torch.float16, device=device) for B in batches}

    def e2e_step(i):
        for B in batches:
            dev_in[B].copy_(host_in[B][i % n_sets], non_blocking=True)
            outs = stack_forward(blocks, dev_in[B], B == 1)
            host_out[B].copy_(torch.stack(outs), non_blocking=True)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    e_steps = max(3, args.steps // 2)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    for i in range(e_steps):
        e2e_step(i)
    ee.record()
    torch.cuda.synchronize()
    e2e_ms = es.elapsed_time(ee) / e_steps
    h2d = sum(L * B * D * 2 for B in batches)

    # stage breakdown + dominant-stage roofline (eager, stage events)
    stage_ms = {}
    for B in batches:
        acc = [0.0] * 6
        reps = 3
        for i in range(reps):
            xs = inputs[B][i % n_sets]
            for l, blk in enumerate(blocks):
                stack_forward([blk], xs[l:l + 1], B == 1, time_stages=True)
                st = stage_times(blk)
                acc = [a + s for a, s in zip(acc, st)]
        stage_ms[B] = [a / reps for a in acc]
    names = _lib.STAGES
    dom_b, dom_s = max(((B, s) for B in batches for s in range(6)), key=lambda bs: stage_ms[bs[0]][bs[1]])
    # algorithmic bytes of the up/down stages for that batch: the hit experts' matrices
    dom_bytes = None
    if names[dom_s] in ("up", "down"):
        share = {"up": 2.0 / 3.0, "down": 1.0 / 3.0}[names[dom_s]]  # w1+w3 vs w2 of each expert (equal shapes)
        weights = bytes_per_pass[dom_b] - args.layers * (blocks[0].num_experts * D * 2 + 2 * dom_b * D * 2)
        dom_bytes = weights * share / args.layers
    dom_ms = stage_ms[dom_b][dom_s] / args.layers
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9 if dom_bytes else None

    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(args, device, bf16_peak, bf16_sus)
    ep = None
    if not args.no_ep:
        ep = run_ep(args, rank, world, device, bf16_sus)
    configs = None
    if not args.no_configs:
        configs = run_configs(blocks[0], device, hbm_peak, bf16_peak)
    cpu = cpu0 = None
    if rank == 0 and not args.no_cpu:
        cpu = cpu_baseline(blocks[0], inputs, args.cpu_seconds)
        cpu0 = cpu_config0(blocks[0])
    ref_gpu = None
    if world == 1 and args.reference_gpu != "none":
        ref_gpu = optional(lambda: run_reference_gpu(args, blocks[0], device))
    gen = None
    if not args.no_generate:
        gen = optional(lambda: run_generate(blocks, device))
    launches = kernel_launches(blocks, batches)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "olmoe-16-layer-moe-stack-decode (BASELINE config 1)",
                   "batches": batches, "layers": args.layers, "hidden": D, "inter": blocks[0].ffn_dim,
                   "experts": blocks[0].num_experts, "top_k": blocks[0].top_k, "group_size": 64,
                   "mean_bits": 2.5, "parallelism": f"replicas x{world}",
                   "l2": "per-step weight working set 0.3-2.5 GB per batch size > 126 MB L2",
                   "graph": "one CUDA graph per batch size"},
        "decode_per_batch": {str(B): {"ms_per_pass": round(per_b[B], 4),
                                      "gbs": round(bytes_per_pass[B] / (per_b[B] * 1e-3) / 1e9, 1),
                                      "tokens_per_s": round(B / (per_b[B] * 1e-3), 1),
                                      "frac_hbm": round(bytes_per_pass[B] / (per_b[B] * 1e-3) / 1e9 / hbm_peak, 3),
                                      "stage_ms_per_layer": [round(v / args.layers, 5) for v in stage_ms[B]]}
                             for B in batches},
        "stages": list(names),
        "roofline": {"bound": "hbm", "kernel": f"{names[dom_s]} stage at batch {dom_b}",
                     "achieved": round(achieved, 1) if achieved else None, "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 3) if achieved else None,
                     "traffic": profiled_traffic(names[dom_s], dom_b),
                     "algorithmic_bytes": round(dom_bytes) if dom_bytes else None,
                     "peak_source": peak_src},
        "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d,
                "path": "QuantFusedOlmoeMoEBlock per layer (eager C-ABI calls), pinned host in/out every step"},
        "gpu_launches": launches * args.steps,
        "clocks": clk, "setup_s": round(setup_s, 1),
    }
    if prefill:
        line["prefill"] = prefill
    if ep:
        line["expert_parallel"] = ep
    if cpu:
        line["cpu_baseline"] = cpu
    if configs:
        line.update(configs)
    if cpu0:
        line["cpu_config0"] = cpu0
    if ref_gpu:
        line["reference_gpu"] = ref_gpu
    if gen:
        line["generate"] = gen
    return line


def kernel_launches(blocks, batches):
    """Kernels of ours per step, counted from the pipeline: one-token path 5 per layer
    (gate logits, top-k, gate/up GEMV, down GEMV reducing the up partials, combine
    reducing the down partials); n-token path at these batch sizes 6 (gate logits,
    top-k, one-launch dispatch, gate/up GEMM, down GEMM, combine)."""
    return sum(len(blocks) * (5 if B == 1 else 6) for B in batches)


def profiled_traffic(kernel: str, batch: int):
    """DRAM bytes per launch of the dominant kernel from one ncu capture, kept as data in
    profiles/ncu_traffic.json (the capture and its command are summarised beside it),
    or None when no capture covers it."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    try:
        table = json.loads(path.read_text())["dram_bytes_per_launch"]
    except (OSError, ValueError, KeyError):
        return None
    v = table.get(f"{kernel}_b{batch}")
    return int(v) if v is not None else None


def run_prefill(args, device, bf16_peak, bf16_sus):
    import torch

    from robustgemq_b200 import _lib, synth
    from robustgemq_b200.inference import QuantFusedQwen3MoeMoEBlock

    cfg, shp = synth.qwen3_config()
    L, T = args.prefill_layers, args.prefill_tokens
    blocks = [synth.random_block(QuantFusedQwen3MoeMoEBlock, cfg, shp["hidden"], shp["inter"], shp["num_experts"],
                                 shp["mean_bits"], shp["group_size"], 5000 + l, device) for l in range(L)]
    logits = [synth.zipf_logits(T, shp["num_experts"], 9000 + l, device) for l in range(L)]
    x0 = torch.randn((T, shp["hidden"]), device=device).half()

    def fwd(x, time_stages=False):
        # every layer reads the same normalised input (routing comes from the given
        # per-layer logits); outputs are written and discarded
        flags = _lib.FWD_TIME_STAGES if time_stages else 0
        y = None
        for blk, lg in zip(blocks, logits):
            y, _ = blk._run(x, flags, want_logits=False, logits_in=lg)
        return y

    for _ in range(2):
        fwd(x0)
    torch.cuda.synchronize()
    reps = max(2, args.steps // 4)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fwd(x0)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    D, F, E, k = shp["hidden"], shp["inter"], shp["num_experts"], cfg.num_experts_per_tok
    flops = L * T * k * 6 * D * F  # routed experts (router logits are given)
    # stage times on the first layer
    x = x0
    blk = blocks[0]
    blk._run(x, _lib.FWD_TIME_STAGES, want_logits=False, logits_in=logits[0])
    st = stage_times(blk)
    up_flops = T * k * 4 * D * F
    dn_flops = T * k * 2 * D * F
    return {"workload": "qwen3-30b-a3b-shaped prefill, 48 layers, 4096 tokens, Zipf(1.1) router logits (config 2)",
            "layers": L, "tokens": T, "ms_per_pass": round(ms, 3), "tokens_per_s": round(T / (ms * 1e-3), 1),
            "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "frac_bf16_peak": round(flops / (ms * 1e-3) / 1e12 / bf16_peak, 3),
            "peak_tflops_used": bf16_peak,
            "frac_bf16_sustained": round(flops / (ms * 1e-3) / 1e12 / bf16_sus, 3),
            "stage_ms_layer0": [round(v, 4) for v in st],
            "up_tflops": round(up_flops / (st[2] * 1e-3) / 1e12, 1) if st[2] > 0 else None,
            "down_tflops": round(dn_flops / (st[3] * 1e-3) / 1e12, 1) if st[3] > 0 else None}


def run_ep(args, rank, world, device, bf16_sus):
    """Mixtral-shaped prefill with expert parallelism over all ranks:
    each rank builds and holds only its E / world experts (``ExpertParallelMoE.from_shard``)
    and routes its own ``ep_tokens`` tokens (weak scaling); tokens reach their experts'
    ranks and return by NCCL all-to-all. Also reported: the per-step breakdown (max over
    ranks) and the sharded forward's parity with the whole layer run on one GPU."""
    from types import SimpleNamespace

    import torch
    import torch.distributed as dist

    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedMixtralMoEBlock
    from robustgemq_b200.inference.expert_parallel import STAGES, ExpertParallelMoE

    cfg, shp = synth.mixtral_config()
    L, T = args.ep_layers, args.ep_tokens
    E = shp["num_experts"]
    epr = E // world
    mine = range(rank * epr, (rank + 1) * epr)
    local_cfg = SimpleNamespace(**{**vars(cfg), "num_local_experts": epr})
    layers = []
    for l in range(L):
        blk, gate = synth.random_block_experts(QuantFusedMixtralMoEBlock, local_cfg, shp["hidden"], shp["inter"], E,
                                               shp["mean_bits"], shp["group_size"], 7000 + l, device, experts=mine)
        layers.append(ExpertParallelMoE.from_shard(blk, gate, E, time_stages=True))
    gen = torch.Generator(device=device).manual_seed(900 + rank)
    x = torch.randn((T, shp["hidden"]), generator=gen, device=device).half()

    chunks = max(1, args.ep_chunks)

    def run(ep, xx):
        return ep.forward_tokens_chunked(xx, chunks) if chunks > 1 else ep.forward_tokens(xx)

    def fwd():
        for ep in layers:  # every layer reads the same input; outputs are discarded
            run(ep, x)

    for _ in range(2):
        fwd()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    reps = 3
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fwd()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / reps], device=device)
    # per-step breakdown of the last layer of the last pass, max over ranks
    st = layers[-1].stage_times()  # not recorded by the chunked forward: zeros then
    brk = torch.tensor([st.get(n, 0.0) for n in STAGES], device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(brk, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    # parity (untimed): layer 0 sharded against the whole layer 0 built on this GPU
    # (every expert from its own generator, so identical to the union of the shards),
    # on 256 of this rank's tokens; every rank takes the same collective steps
    full_cfg = cfg
    full0, _ = synth.random_block_experts(QuantFusedMixtralMoEBlock, full_cfg, shp["hidden"], shp["inter"], E,
                                          shp["mean_bits"], shp["group_size"], 7000, device)
    xp = x[:256].contiguous()
    y_ep, _ = run(layers[0], xp)
    y_full = full0(xp[None])[0][0]
    err = ((y_ep.double() - y_full.double()).norm() / y_full.double().norm()).reshape(1)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    del full0
    torch.cuda.empty_cache()
    D, F, k = shp["hidden"], shp["inter"], cfg.num_experts_per_tok
    flops = world * T * L * k * 6 * D * F
    return {"workload": f"mixtral-8x7b-shaped prefill, {L} layers, {T} tokens per rank, experts sharded over "
                        f"{world} rank(s), NCCL all-to-all dispatch/combine (config 4)",
            "layers": L, "tokens_per_rank": T, "n_ranks": world, "chunks": chunks, "ms_per_pass": round(ms, 3),
            "tokens_per_s": round(world * T / (ms * 1e-3), 1), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "frac_bf16_peak_per_gpu": round(flops / world / (ms * 1e-3) / 1e12 / bf16_sus, 3),
            "peak_tflops_used": bf16_sus,
            "stage_ms_per_layer_max_over_ranks": {n: round(float(v), 4) for n, v in zip(STAGES, brk.tolist())},
            "parity_rel_l2": float(f"{float(err.item()):.3e}"),
            "parity": "layer 0, 256 tokens per rank: sharded forward vs the whole layer on one GPU, max over ranks"}


def _time_ms(fn, reps):
    import torch

    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def run_configs(olmoe_blk, device, hbm_peak, bf16_peak):
    """Configs 0 and 3 on one GPU, eager through the block API (router included).

    config 0: one OLMoE-shaped layer (a layer of the decode stack), prefill of 512 tokens;
    config 3: one DeepSeek-V2-Lite-shaped layer (64 routed experts top-6 + 2 shared,
    F 1408, g 64, mean 2.75 bits, shared 4-bit), prefill of 2048 tokens and decode of 16."""
    import torch

    from robustgemq_b200 import synth
    from robustgemq_b200.inference import QuantFusedDeepseekV2MoEBlock

    out = {}
    g = torch.Generator(device=device).manual_seed(4242)
    D = olmoe_blk.hidden_dim
    x0 = torch.randn((1, 512, D), generator=g, device=device).half()
    ms = _time_ms(lambda: olmoe_blk(x0), 10)
    F, E, k = olmoe_blk.ffn_dim, olmoe_blk.num_experts, olmoe_blk.top_k
    flops = 512 * k * 6 * D * F + 2 * 512 * D * E
    out["config0"] = {"workload": "olmoe-shaped MoE block, prefill of 512 tokens, device router (config 0)",
                      "ms": round(ms, 4), "tokens_per_s": round(512 / (ms * 1e-3), 1),
                      "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                      "frac_bf16_peak": round(flops / (ms * 1e-3) / 1e12 / bf16_peak, 3)}
    cfg, s = synth.deepseek_config()
    blk = synth.random_block(QuantFusedDeepseekV2MoEBlock, cfg, s["hidden"], s["inter"], s["num_experts"],
                             s["mean_bits"], s["group_size"], 303, device, shared_inter=s["shared_inter"])
    D, F, E, k, Fs = s["hidden"], s["inter"], s["num_experts"], cfg.num_experts_per_tok, s["shared_inter"]
    xp = torch.randn((1, 2048, D), generator=g, device=device).half()
    ms_p = _time_ms(lambda: blk(xp), 10)
    flops_p = 2048 * (k * 6 * D * F + 6 * D * Fs + 2 * D * E)
    xd = torch.randn((16, D), generator=g, device=device).half()
    ms_d = _time_ms(lambda: blk(xd[None]), 20)
    eb = synth.layer_expert_bytes(blk)
    _, idx, _ = blk.route(xd)
    shared_bytes = sum(getattr(blk, f"shared_{n}_wq").numel() * 4 + 2 * 2 * getattr(blk, f"shared_{n}_scales").numel()
                       for n in ("w1", "w3", "w2"))
    bytes_d = sum(eb[e] for e in torch.unique(idx).tolist()) + shared_bytes + E * D * 2 + 2 * 16 * D * 2
    out["config3"] = {"workload": "deepseek-v2-lite-shaped MoE layer with 2 shared experts (config 3)",
                      "prefill_tokens": 2048, "prefill_ms": round(ms_p, 4),
                      "prefill_tokens_per_s": round(2048 / (ms_p * 1e-3), 1),
                      "prefill_tflops": round(flops_p / (ms_p * 1e-3) / 1e12, 1),
                      "prefill_frac_bf16_peak": round(flops_p / (ms_p * 1e-3) / 1e12 / bf16_peak, 3),
                      "decode_batch": 16, "decode_ms": round(ms_d, 4),
                      "decode_gbs": round(bytes_d / (ms_d * 1e-3) / 1e9, 1),
                      "decode_frac_hbm": round(bytes_d / (ms_d * 1e-3) / 1e9 / hbm_peak, 3),
                      "decode_path": "eager block call (no CUDA graph)"}
    del blk
    torch.cuda.empty_cache()
    return out


def run_reference_gpu(args, blk, device):
    """The reference's own GPU path (its Triton kernels JIT-compiled for this B200 with
    its own autotune, from the unmodified package in baseline/_ref) beside ours on the
    same OLMoE-shaped layer and inputs: prefill of 512 tokens (config 0), and with
    ``--reference-gpu all`` the one-token decode path (config 1, batch 1)."""
    import torch

    from baseline import reference_gpu as RG

    if not RG.available():
        return {"unavailable": "the reference is not installed in baseline/_ref (or triton is missing)"}
    ref = RG.reference_block(blk)
    g = torch.Generator(device=device).manual_seed(512)
    res = {"source": "baseline/_ref (unmodified gemq package), Triton JIT + autotune on this GPU"}
    cases = [("prefill_512", 512)] + ([("decode_b1", 1)] if args.reference_gpu == "all" else [])
    for name, T in cases:
        x = torch.randn((1, T, blk.hidden_dim), generator=g, device=device).half()
        t0 = time.time()
        with torch.no_grad():
            RG.output(ref(x))
        torch.cuda.synchronize()
        first_s = time.time() - t0
        with torch.no_grad():
            ms_ref = _time_ms(lambda: RG.output(ref(x)), 5)
            y_ref = RG.output(ref(x)).reshape(T, -1).double()
        ms_ours = _time_ms(lambda: RG.output(blk(x)), 20)
        y = RG.output(blk(x)).reshape(T, -1).double()
        res[name] = {"tokens": T, "reference_ms": round(ms_ref, 4), "ours_ms": round(ms_ours, 4),
                     "speedup": round(ms_ref / ms_ours, 1),
                     "reference_tokens_per_s": round(T / (ms_ref * 1e-3), 1),
                     "ours_tokens_per_s": round(T / (ms_ours * 1e-3), 1),
                     "rel_l2_ours_vs_reference": float(f"{float((y - y_ref).norm() / y_ref.norm()):.3e}"),
                     "reference_first_call_s": round(first_s, 1)}
    return res


def optional(fn):
    """Runs an optional sub-measurement; a failure is reported in the line, not raised."""
    try:
        return fn()
    except Exception as exc:  # the headline measurement must not depend on it
        import torch

        torch.cuda.synchronize()
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def run_generate(blocks, device):
    """Whole-model decode: an OLMoE-1B-7B-shaped transformers model whose 16 MoE blocks
    are the decode stack's layers, 4-bit attention projections, static KV cache, the
    decode step replayed as one CUDA graph; the reference's protocol (9-token prompt,
    64 new tokens, 3 rounds, benchmark_generate.py:160-230), greedy tokens."""
    import torch

    from robustgemq_b200.inference.generate import StaticDecoder, synthetic_olmoe

    model = synthetic_olmoe(num_layers=len(blocks), device=device, seed=11, blocks=blocks,
                            max_position_embeddings=256)
    prompt = torch.randint(0, model.config.vocab_size, (9,), generator=torch.Generator().manual_seed(9)).to(device)
    dec = StaticDecoder(model, max_cache_len=9 + 64)
    dec.generate(prompt, 64)  # capture + warm-up round
    rounds = [dec.generate(prompt, 64)[1] for _ in range(3)]
    dec_tps = sorted(r["decode_tokens_per_s"] for r in rounds)[1]
    pre_tps = sorted(r["prefill_tokens_per_s"] for r in rounds)[1]
    for layer in model.model.layers:  # the blocks stay owned by the decode stack
        layer.mlp = None
    del dec, model
    torch.cuda.empty_cache()
    return {"workload": "olmoe-1b-7b-shaped model, 16 MoE layers of this library, 4-bit attention (one q|k|v "
                        "projection, q/k norm + rotary in one launch), fused fp16 RMSNorms, fp16 embeddings / LM "
                        "head; 9-token prompt, 64 new tokens, greedy; median of 3 rounds",
            "decode_tokens_per_s": round(dec_tps, 1), "prefill_tokens_per_s": round(pre_tps, 1),
            "decode_path": "static KV cache, decode step replayed as one CUDA graph"}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_config0(blk):
    """Config 0 on the host cores: the reference's fake-quant block (dequantise to fp32 +
    torch matmul, the forward_n_tokens control flow) over 512 tokens, both with the
    dequant inside the timed pass and with pre-dequantised weights (matmul only)."""
    import numpy as np
    import torch

    from oracle import cpu_baseline as cb

    torch.set_num_threads(os.cpu_count() or 1)
    layer = cb.layer_from_block(blk)
    x = np.random.default_rng(512).standard_normal((512, layer.D)).astype(np.float16)
    r = cb.time_block_prefill(layer, x, reps=3)
    r.update({"workload": "olmoe-shaped MoE block, prefill of 512 tokens, fp32 (config 0)", "kind": "port",
              "cores": torch.get_num_threads(), "cpu_model": cb.cpu_model()})
    return r


def cpu_baseline(blk, inputs, seconds):
    """The reference's CPU fake-quant path (dequantise + torch fp32 matmul) on one OLMoE
    layer, timed on this host's cores; sample: one layer at each batch size."""
    import numpy as np
    import torch

    from oracle import cpu_baseline as cb

    torch.set_num_threads(os.cpu_count() or 1)  # torchrun sets OMP_NUM_THREADS=1
    layer = cb.layer_from_block(blk)
    xs = {B: v[0][0].float().cpu().numpy() for B, v in inputs.items()}
    r = cb.time_decode(layer, xs, seconds)
    r["cores"] = torch.get_num_threads()
    r["cpu_model"] = cb.cpu_model()
    return r


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    import numpy as np
    import torch

    from oracle import cpu_baseline as cb

    layer = cb.synthetic_layer(seed=1000)
    batches = [int(b) for b in args.batches.split(",")]
    rng = np.random.default_rng(7)
    xs = {B: rng.standard_normal((B, layer.D)).astype(np.float16) for B in batches}
    for i in range(args.warmup):
        B = batches[i % len(batches)]
        cb.decode_layer(layer, xs[B])
    t0 = time.perf_counter()
    total_bytes = 0
    for i in range(args.steps):
        B = batches[i % len(batches)]
        total_bytes += cb.decode_layer(layer, xs[B])
    dt = time.perf_counter() - t0
    v = total_bytes / dt / 1e9
    cores = torch.get_num_threads()
    sample = (f"{args.steps} single-layer decode passes of the OLMoE-shaped layer cycling batch "
              f"{batches}, dequantise hit experts to fp32 + torch matmul (the reference's fake-quant path)")
    return {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "olmoe-16-layer-moe-stack-decode (BASELINE config 1), CPU sample"},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample,
                             "cpu_model": cb.cpu_model()},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def claim_stdout():
    """Point file descriptor 1 at stderr for the rest of the run; return a stream on the real stdout.

    Native libraries print to the C-level stdout (NCCL its version banner when NCCL_DEBUG is
    set in the environment), which would put text before the result line. After this call
    everything written to fd 1 lands on stderr, and the result line alone goes to the stream
    returned here. dup2 shares the open file, so a log that holds both streams is not reopened
    or truncated."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        print(json.dumps(run_reference(args)))
        return
    result_out = claim_stdout()
    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    line = run_ours(args, rank, world, local_rank)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), file=result_out, flush=True)


if __name__ == "__main__":
    main()
