"""Expert parallelism: slot bookkeeping, expert slicing and the all-to-all exchange.

CPU tests run two gloo ranks; the router, the local experts and the combine are the
oracle's (the exchange, the send order and the slot -> row mapping are the module's
own), and every rank's output must equal the 1-process oracle block's on its tokens,
bit for bit. Failure tests (gloo, CPU) make the failure on the host: one rank's
router returns an expert id past E, or one rank never joins the exchange; every
waiting rank must end with ``ExpertParallelError``, not hang. GPU tests run the CUDA
defaults: one rank against the block itself, and two NCCL ranks when the machine has
two GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from conftest import load_golden, proj_from, rel_l2

F16, F32 = np.float16, np.float32


def _golden_block(device="cpu"):
    from gpu_helpers import family_config
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    d = load_golden("block_olmoe.npz")
    blk = QuantFusedOlmoeMoEBlock(family_config("olmoe", d))
    blk.gate.weight.data = torch.from_numpy(d["gate_w"]).to(device)
    for name in ("w1", "w2", "w3"):
        for f in ("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides", "zs_strides"):
            setattr(blk, f"{name}_{f}", torch.from_numpy(np.ascontiguousarray(d[f"{name}_{f}"])).to(device))
    blk.block_group_size = int(d["group_size"])
    return blk, d


def _oracle_weights(d):
    from oracle import gemq_oracle as O

    return O.BlockWeights(gate_w=d["gate_w"], w1=proj_from(d, "w1"), w3=proj_from(d, "w3"), w2=proj_from(d, "w2"),
                          top_k=int(d["top_k"]), norm_topk_prob=bool(d["norm_topk_prob"]))


def cpu_dispatch(idx, w, x, num_experts):
    """Slots grouped by expert id (stable), as gemq_moe_dispatch groups them; an id
    outside [0, E) gets no row and slot_row -1."""
    k = idx.shape[1]
    flat = idx.reshape(-1).to(torch.int64)
    valid = (flat >= 0) & (flat < num_experts)
    order = torch.argsort(torch.where(valid, flat, num_experts), stable=True)
    nvalid = int(valid.sum())
    counts = torch.bincount(flat[valid], minlength=num_experts).to(torch.int32)
    slot_row = torch.full((flat.numel(),), -1, dtype=torch.int32)
    slot_row[order[:nvalid]] = torch.arange(nvalid, dtype=torch.int32)
    sel = order[:nvalid]
    return counts, slot_row, w.reshape(-1)[sel], x[torch.div(sel, k, rounding_mode="floor")]


def test_cpu_dispatch_groups_slots_by_expert():
    idx = torch.tensor([[5, 0], [2, 7], [3, 4], [0, 9]], dtype=torch.int32)
    w = torch.arange(8, dtype=torch.float16).reshape(4, 2)
    x = torch.arange(4, dtype=torch.float16).reshape(4, 1).expand(4, 8).contiguous()
    counts, slot_row, w_rows, x_rows = cpu_dispatch(idx, w, x, 8)
    assert counts.tolist() == [2, 0, 1, 1, 1, 1, 0, 1]
    assert slot_row.tolist() == [5, 0, 2, 6, 3, 4, 1, -1]
    assert w_rows.tolist() == [1, 6, 2, 4, 5, 0, 3]
    assert x_rows[:, 0].tolist() == [0, 3, 1, 2, 2, 0, 1]


def test_slice_projection_keeps_each_experts_dequant():
    from oracle import gemq_oracle as O
    from robustgemq_b200.inference.expert_parallel import slice_projection

    blk, d = _golden_block()
    full = proj_from(d, "w2")
    sl = slice_projection(blk, "w2", 3, 7, int(d["w2_K"]))
    part = O.PackedProj(wq=sl["wq"].numpy(), scales=sl["scales"].numpy(), zeros=sl["zeros"].numpy(),
                        nbits=sl["nbits"].numpy(), group_sizes=sl["group_sizes"].numpy(),
                        wq_strides=sl["wq_strides"].numpy(), zs_strides=sl["zs_strides"].numpy(), K=full.K, N=full.N)
    for j in range(4):
        assert np.array_equal(O.dequantize_expert(part, j).view(np.uint16),
                              O.dequantize_expert(full, 3 + j).view(np.uint16))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_ep(route_hook=None, placement=None):
    """An ExpertParallelMoE on the golden OLMoE block whose router, local experts and
    combine are the oracle's; ``route_hook(idx)`` may rewrite the routed expert ids."""
    from oracle import gemq_oracle as O
    from robustgemq_b200.inference.expert_parallel import ExpertParallelMoE

    blk, d = _golden_block()
    ow = _oracle_weights(d)
    k = ow.top_k
    ep = None

    def route_fn(x):
        r = O.route(x.numpy(), ow.gate_w, k, ow.norm_topk_prob)
        idx = r.topk_idx.astype(np.int32)
        if route_hook is not None:
            idx = route_hook(idx)
        return torch.from_numpy(r.logits), torch.from_numpy(idx), torch.from_numpy(r.topk_w)

    def dispatch_fn(idx, w, x):
        return cpu_dispatch(idx, w, x, ow.w1.num_experts)

    def experts_fn(rows, group_counts, wts):
        # rows arrive grouped as [source rank][local expert]
        rows_np, gc, w_np = rows.numpy(), group_counts.numpy(), wts.numpy()
        y = np.zeros_like(rows_np)
        off = 0
        for g in range(gc.shape[0]):
            for e in range(gc.shape[1]):
                c = int(gc[g, e])
                if c:
                    ye = O.expert_ffn_n_tokens(ow, ep.local_experts[e], rows_np[off:off + c])
                    y[off:off + c] = (ye.astype(F32) * w_np[off:off + c].astype(F32)[:, None]).astype(F16)
                off += c
        return torch.from_numpy(y)

    def combine_fn(y, slot_row, idx, residual):
        y_np, sr, ix = y.numpy(), slot_row.numpy(), idx.numpy()
        T = ix.shape[0]
        out = np.zeros((T, y_np.shape[1]), dtype=F16)
        for t in range(T):
            for j in np.argsort(ix[t], kind="stable"):
                out[t] = (out[t].astype(F32) + y_np[sr[t * k + j]].astype(F32)).astype(F16)
        return torch.from_numpy(out)

    ep = ExpertParallelMoE(blk, route_fn=route_fn, experts_fn=experts_fn, combine_fn=combine_fn,
                           dispatch_fn=dispatch_fn, placement=placement)
    return ep, ow, d


def _matches_oracle(ep, ow, d, rank, world):
    from oracle import gemq_oracle as O

    mine = np.ascontiguousarray(d["x"].astype(F16)[rank::world])
    out, _ = ep.forward_tokens(torch.from_numpy(mine))
    ref, _ = O.moe_forward_n_tokens(ow, mine)
    return bool(np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16)))


def _cpu_rank(rank, world, port, results, placement=None):
    import torch.distributed as dist
    from oracle import gemq_oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ep, ow, d = _cpu_ep(placement=placement)
        ok = _matches_oracle(ep, ow, d, rank, world)
        # the measured load, summed over ranks, counts every rank's routed slots
        load = ep.measured_load().numpy()
        x = d["x"].astype(F16)
        want = np.zeros(ow.w1.num_experts, dtype=np.int64)
        for r in range(world):
            idx = O.route(np.ascontiguousarray(x[r::world]), ow.gate_w, ow.top_k, ow.norm_topk_prob).topk_idx
            want += np.bincount(idx.reshape(-1), minlength=ow.w1.num_experts)
        results[rank] = (ok, bool(np.array_equal(load, want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("placement", [None, "shuffled"])
def test_expert_parallel_two_gloo_ranks_match_the_single_block(placement):
    """Contiguous expert ranges, and a shuffled placement (rank 0 holds the odd-indexed
    half of a permutation): both bit-identical to the 1-process block."""
    import torch.multiprocessing as mp

    if placement == "shuffled":
        E = int(load_golden("block_olmoe.npz")["w1_nbits"].shape[0])
        placement = [int(e) for e in np.random.default_rng(3).permutation(E)]
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, 2, port, results, placement)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}


def _chunked_rank(rank, world, port, results, chunks, placement):
    import torch.distributed as dist
    from oracle import gemq_oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ep, ow, d = _cpu_ep(placement=placement)
        mine = np.ascontiguousarray(d["x"].astype(F16)[rank::world])
        out, _ = ep.forward_tokens_chunked(torch.from_numpy(mine), chunks)
        ref, _ = O.moe_forward_n_tokens(ow, mine)
        results[rank] = bool(np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks,shuffled", [(2, False), (3, True)])
def test_chunked_exchange_two_gloo_ranks_match_the_single_block(chunks, shuffled):
    """Chunked forward (asynchronous exchanges of chunk c + 1 beside chunk c's experts):
    bit-identical to the 1-process block on both ranks."""
    import torch.multiprocessing as mp

    placement = None
    if shuffled:
        E = int(load_golden("block_olmoe.npz")["w1_nbits"].shape[0])
        placement = [int(e) for e in np.random.default_rng(5).permutation(E)]
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_chunked_rank, args=(r, 2, port, results, chunks, placement)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: True, 1: True}


def test_chunked_forward_single_process():
    from oracle import gemq_oracle as O

    ep, ow, d = _cpu_ep()
    x = np.ascontiguousarray(d["x"].astype(F16))
    ref, _ = O.moe_forward_n_tokens(ow, x)
    for chunks in (1, 2, 5):
        out, _ = ep.forward_tokens_chunked(torch.from_numpy(x), chunks)
        assert np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16)), chunks


def test_balanced_placement():
    from robustgemq_b200.inference.expert_parallel import balanced_placement

    load = [90, 5, 5, 40, 40, 10, 10, 0]
    order = balanced_placement(load, 2)
    assert sorted(order) == list(range(8))
    halves = [order[:4], order[4:]]
    assert all(h == sorted(h) for h in halves)
    totals = sorted(sum(load[e] for e in h) for h in halves)
    assert totals == [100, 100]  # {0, 1, 2, 7} and {3, 4, 5, 6}
    # contiguous ranges would give 140 / 60; one expert per rank is the identity
    assert balanced_placement(load, 8) == sorted(range(8), key=lambda e: (-load[e], e))
    with pytest.raises(ValueError):
        balanced_placement(load, 3)


def test_gather_projection_keeps_each_experts_dequant():
    from oracle import gemq_oracle as O
    from robustgemq_b200.inference.expert_parallel import gather_projection

    blk, d = _golden_block()
    full = proj_from(d, "w1")
    experts = [5, 0, 3, 6]
    sl = gather_projection(blk, "w1", experts, int(d["w1_K"]))
    part = O.PackedProj(wq=sl["wq"].numpy(), scales=sl["scales"].numpy(), zeros=sl["zeros"].numpy(),
                        nbits=sl["nbits"].numpy(), group_sizes=sl["group_sizes"].numpy(),
                        wq_strides=sl["wq_strides"].numpy(), zs_strides=sl["zs_strides"].numpy(), K=full.K, N=full.N)
    for j, e in enumerate(experts):
        assert np.array_equal(O.dequantize_expert(part, j).view(np.uint16),
                              O.dequantize_expert(full, e).view(np.uint16))


def _bad_routing_rank(rank, world, port, results):
    """Rank 1's router returns an expert id past E on the first forward only."""
    import torch.distributed as dist
    from robustgemq_b200.inference.expert_parallel import ExpertParallelError

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        calls = {"n": 0}

        def hook(idx):
            calls["n"] += 1
            if rank == 1 and calls["n"] == 1:
                idx = idx.copy()
                idx[0, 0] = 1000
            return idx

        ep, ow, d = _cpu_ep(route_hook=hook)
        mine = torch.from_numpy(np.ascontiguousarray(d["x"].astype(F16)[rank::world]))
        try:
            ep.forward_tokens(mine)
            raised = ""
        except ExpertParallelError as exc:
            raised = str(exc)
        # every rank learned of rank 1's table in the counts exchange, and the group
        # is still usable: the next forward runs and matches the oracle
        results[rank] = ("rank(s) [1]" in raised, _matches_oracle(ep, ow, d, rank, world))
    finally:
        dist.destroy_process_group()


def test_invalid_routing_on_one_rank_fails_every_rank_and_keeps_the_group():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_bad_routing_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}


def _absent_peer_rank(rank, world, port, results, release):
    """Rank 1 joins the group but never runs a forward; rank 0's exchange must fail
    within the group's short timeout instead of waiting for ever."""
    import time
    from datetime import timedelta

    import torch.distributed as dist
    from robustgemq_b200.inference.expert_parallel import ExpertParallelError

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=3))
    try:
        if rank == 1:
            release.wait(90)
            results[rank] = True
            return
        ep, ow, d = _cpu_ep()
        mine = torch.from_numpy(np.ascontiguousarray(d["x"].astype(F16)[0::world]))
        t0 = time.monotonic()
        first = second = ""
        try:
            ep.forward_tokens(mine)
        except ExpertParallelError as exc:
            first = str(exc)
        waited = time.monotonic() - t0
        try:
            ep.forward_tokens(mine)  # refused on the host: no collective after a failed one
        except ExpertParallelError as exc:
            second = str(exc)
        results[rank] = ("counts" in first, waited < 60, "earlier exchange failed" in second)
        release.set()
    finally:
        dist.destroy_process_group()


def test_absent_peer_ends_the_exchange_with_an_error():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    release = manager.Event()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_rank, args=(r, 2, port, results, release)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(150)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert procs[0].exitcode == 0, [p.exitcode for p in procs]
    assert results.get(0) == (True, True, True), dict(results)


@pytest.mark.gpu
def test_expert_parallel_one_rank_matches_block_on_gpu():
    from robustgemq_b200 import _lib
    from robustgemq_b200.inference.expert_parallel import ExpertParallelMoE

    blk, d = _golden_block("cuda")
    x = torch.from_numpy(d["x"].astype(F16)).cuda()
    ref, ref_logits = blk.forward_n_tokens(x.unsqueeze(0))
    ep = ExpertParallelMoE(blk, time_stages=True)
    out, logits = ep.forward_tokens(x)
    torch.cuda.synchronize()
    # the received rows go through the grouped GEMM (the block's decode-batch GEMM
    # reads K in another order): equal up to fp32 summation order
    assert rel_l2(out.cpu().numpy(), ref[0].cpu().numpy()) < 1e-3
    assert torch.equal(logits, ref_logits)
    st = ep.stage_times()
    assert set(st) == {"route", "dispatch", "counts", "rows_out", "experts", "rows_back", "combine"}
    assert all(v >= 0 for v in st.values())
    # a shard built from this rank's experts alone gives the same result
    from robustgemq_b200.inference.expert_parallel import slice_projection
    from gpu_helpers import family_config
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg = family_config("olmoe", d)
    loc = QuantFusedOlmoeMoEBlock(cfg)
    for name, kk in (("w1", blk.hidden_dim), ("w3", blk.hidden_dim), ("w2", blk.ffn_dim)):
        for key, t in slice_projection(blk, name, 0, blk.num_experts, kk).items():
            setattr(loc, f"{name}_{key}", t)
    loc.block_group_size = blk.block_group_size
    ep2 = ExpertParallelMoE.from_shard(loc, blk.gate.weight, blk.num_experts)
    out2, _ = ep2.forward_tokens(x)
    assert torch.equal(out2, out)
    # a shuffled placement (the local experts gathered in its order, slots dispatched
    # by position, the combine by expert id) gives the same bits
    perm = [int(e) for e in np.random.default_rng(4).permutation(blk.num_experts)]
    ep3 = ExpertParallelMoE(blk, placement=perm)
    out3, _ = ep3.forward_tokens(x)
    assert torch.equal(out3, out)
    counts = torch.bincount(ep3.route_fn(x)[1].reshape(-1).long(), minlength=blk.num_experts)
    assert torch.equal(ep3.measured_load().cpu(), counts.cpu())
    assert _lib.device_error() == 0


def _nccl_rank(rank, world, port, results):
    import torch.distributed as dist
    from robustgemq_b200.inference.expert_parallel import ExpertParallelMoE

    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        blk, d = _golden_block(f"cuda:{rank}")
        x = torch.from_numpy(d["x"].astype(F16)).cuda(rank)
        ref, _ = blk.forward_n_tokens(x.unsqueeze(0))
        ep = ExpertParallelMoE(blk)
        mine = x[rank::world].contiguous()
        out, _ = ep.forward_tokens(mine)
        torch.cuda.synchronize()
        results[rank] = rel_l2(out.cpu().numpy(), ref[0][rank::world].cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_expert_parallel_two_nccl_ranks_match_the_single_block():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert all(results[r] < 1e-3 for r in range(2)), dict(results)


def test_balanced_placement_properties():
    """Random loads: a permutation of the experts, each rank's slice ascending, no
    rank above the list-scheduling bound (mean load per rank + the largest expert
    load), never worse than contiguous ranges."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    from robustgemq_b200.inference.expert_parallel import balanced_placement

    @settings(max_examples=60, deadline=None, derandomize=True)
    @given(st.sampled_from([(8, 1), (8, 2), (8, 4), (8, 8), (64, 4), (64, 8), (128, 8), (160, 8)]),
           st.integers(min_value=0, max_value=2**31 - 1))
    def check(shape, seed):
        E, world = shape
        load = np.random.default_rng(seed).zipf(1.3, size=E).astype(float)
        order = balanced_placement(load.tolist(), world)
        assert sorted(order) == list(range(E))
        epr = E // world
        slices = [order[r * epr:(r + 1) * epr] for r in range(world)]
        assert all(sl == sorted(sl) for sl in slices)
        worst = max(load[sl].sum() for sl in slices)
        assert worst <= load.sum() / world + load.max() + 1e-9
        contiguous = max(load[r * epr:(r + 1) * epr].sum() for r in range(world))
        assert worst <= contiguous + 1e-9

    check()
