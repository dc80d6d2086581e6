"""Expert parallelism for the quantized MoE block over ``torch.distributed``.

Rank ``r`` of ``P`` holds experts ``[r * E / P, (r + 1) * E / P)`` of every
projection (the stacked packed layout of ``from_hf``, sliced by expert with its
strides rebased, or built from the rank's experts alone with ``from_shard``). A
forward on a rank's own tokens:

1. routes them over all ``E`` experts (``gemq_route_ex``; the gate is replicated);
2. groups the ``T * k`` token-expert slots by expert id on the device
   (``gemq_moe_dispatch``: histogram, scan, scatter of the activation rows and
   routing weights). Experts are contiguous per rank, so the rows come out grouped
   by destination rank and, inside each destination, by its local expert. Each row
   is written in the K order the owner's tensor-memory GEMM reads for that expert's
   bit-width (``gemq_moe_experts_row_order``; every rank knows all experts' gate/up
   bit-widths, gathered once by ``from_shard``);
3. exchanges the per-expert row counts (with this rank's routing status) in one
   ``all_to_all_single`` and reads them to the host: the one host synchronisation
   of the forward, which sizes the exchanges that follow;
4. sends the activation rows and their routing weights to their owners;
5. the owner runs its experts on the rows it received, grouped as [source rank]
   [local expert] (``gemq_moe_experts``: the segment table built on the device from
   the received counts, then the gate/up and down GEMMs; each output row is exactly
   ``fp16(fp16(y) * w)``, the down projection's route-weight epilogue);
6. sends the rows back with the reverse ``all_to_all_single``;
7. combines each token's ``k`` rows in ascending expert id with fp16 rounding after
   every add (``gemq_moe_combine``): the fp16 ``index_add_`` order of
   ``forward_n_tokens`` (moe_block.py:799-812), so a rank's output equals the 1-GPU
   block's on the same tokens whenever the per-row GEMM results do.

``placement`` (a permutation of the expert ids) replaces the contiguous ranges: rank
``r`` then holds experts ``placement[r * E / P:(r + 1) * E / P]``, and the dispatch
groups slots by an expert's position in ``placement`` (one gather of the routed ids),
so rows still come out grouped by destination rank. The combine reads the original
ids, so its ascending-expert order, and with it the output, does not depend on the
placement. ``balanced_placement`` builds one from per-expert loads (the token counts
every forward accumulates in ``expert_load``, or any other estimate), largest load
first onto the least loaded rank that still has room.

DeepSeek's shared experts are replicated and run on the token's own rank; their
output is added in fp16 after the combine (moe_block.py:575).

``time_stages=True`` records CUDA events around steps 1-7 (route, dispatch, counts,
rows out, experts, rows back, combine); ``stage_times()`` returns their durations.

Failures end in ``ExpertParallelError`` on every rank, never in a hang:

* an invalid routing table on one rank (an expert id outside ``[0, E)``) travels
  with the counts of step 3 as a per-peer status, so every rank learns of it in
  the same exchange and raises before any row is sent; all ranks took the same
  collective steps, so the group stays usable for the next forward;
* a rank that is gone or never joins ends the others' pending exchange through
  the process group's timeout (or the closed connection); the error names the
  step, and the wrapper refuses further forwards, since the group's state is no
  longer known (rebuild the group and the wrapper).

With NCCL the exchange runs over NVLink; with gloo (CPU tests) the router, the
dispatch, the local expert compute and the combine can be replaced by callables
(``route_fn``, ``dispatch_fn``, ``experts_fn``, ``combine_fn``) so the exchange
bookkeeping is tested without a GPU. The defaults are the CUDA kernels; there is
no CPU fallback.
"""

from __future__ import annotations

import ctypes

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor, nn

from .. import _lib
from .._lib import check, ptr, stream_ptr
from .moe_block import _QuantFusedMoEBlock


class ExpertParallelError(RuntimeError):
    """An expert-parallel forward failed: invalid routing on some rank, or a failed exchange."""


def slice_projection(block: _QuantFusedMoEBlock, name: str, e0: int, e1: int, k: int) -> dict:
    """Experts ``[e0, e1)`` of a stacked projection, strides rebased to the slice."""
    wq = getattr(block, f"{name}_wq")
    scales, zeros = getattr(block, f"{name}_scales"), getattr(block, f"{name}_zeros")
    nbits = getattr(block, f"{name}_nbits")
    wqs = getattr(block, f"{name}_wq_strides").to(torch.int64).cpu()
    zss = getattr(block, f"{name}_zs_strides").to(torch.int64).cpu()
    n = wq.shape[1]
    E = nbits.shape[0]
    w_end = int(wqs[e1]) if e1 < E else wq.numel()
    z_end = int(zss[e1]) if e1 < E else scales.numel()
    w0, z0 = int(wqs[e0]), int(zss[e0])
    return {
        "wq": wq[w0 // n:w_end // n].contiguous(),
        "scales": scales[z0 // n:z_end // n].contiguous(),
        "zeros": zeros[z0 // n:z_end // n].contiguous(),
        "nbits": nbits[e0:e1].contiguous(),
        "group_sizes": getattr(block, f"{name}_group_sizes")[e0:e1].contiguous(),
        "wq_strides": (wqs[e0:e1] - w0).to(device=wq.device, dtype=torch.int32),
        "zs_strides": (zss[e0:e1] - z0).to(device=wq.device, dtype=torch.int32),
    }


def gather_projection(block: _QuantFusedMoEBlock, name: str, experts: Sequence[int], k: int) -> dict:
    """Experts ``experts`` (any order) of a stacked projection, in that order, strides
    rebased; a contiguous ascending run is one slice."""
    experts = [int(e) for e in experts]
    if experts == list(range(experts[0], experts[0] + len(experts))):
        return slice_projection(block, name, experts[0], experts[0] + len(experts), k)
    parts = [slice_projection(block, name, e, e + 1, k) for e in experts]
    out = {key: torch.cat([p[key] for p in parts]).contiguous()
           for key in ("wq", "scales", "zeros", "nbits", "group_sizes")}
    n = out["wq"].shape[1]
    dev = out["wq"].device
    w_sizes = [p["wq"].numel() for p in parts]
    z_sizes = [p["scales"].numel() for p in parts]
    out["wq_strides"] = torch.tensor([sum(w_sizes[:i]) for i in range(len(parts))], dtype=torch.int32, device=dev)
    out["zs_strides"] = torch.tensor([sum(z_sizes[:i]) for i in range(len(parts))], dtype=torch.int32, device=dev)
    assert all(int(v) % n == 0 for v in out["wq_strides"].tolist())
    return out


def balanced_placement(load: Sequence[float], world: int) -> List[int]:
    """An expert order whose ``world`` equal slices (one per rank) have balanced total
    load. Experts go by decreasing load (lower id first on ties) onto the rank with the
    least load so far among those with a free slot (lower rank on ties); then, while
    it lowers the heaviest rank's load, the best swap of one of its experts with a
    lighter expert of another rank is made. Returns the concatenation of the ranks'
    expert lists, each ascending."""
    load = [float(v) for v in load]
    E = len(load)
    if world <= 0 or E % world != 0:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    epr = E // world
    bins: List[List[int]] = [[] for _ in range(world)]
    tot = [0.0] * world
    for e in sorted(range(E), key=lambda i: (-load[i], i)):
        r = min((r for r in range(world) if len(bins[r]) < epr), key=lambda r: (tot[r], r))
        bins[r].append(e)
        tot[r] += load[e]
    for _ in range(E * E):
        h = max(range(world), key=lambda r: (tot[r], -r))
        best = None  # (new max of the pair, a, r, b)
        for r in range(world):
            if r == h:
                continue
            for a in bins[h]:
                for b in bins[r]:
                    d = load[a] - load[b]
                    if d > 0:
                        m = max(tot[h] - d, tot[r] + d)
                        if m < tot[h] and (best is None or m < best[0]):
                            best = (m, a, r, b)
        if best is None:
            break
        _, a, r, b = best
        d = load[a] - load[b]
        bins[h][bins[h].index(a)] = b
        bins[r][bins[r].index(b)] = a
        tot[h] -= d
        tot[r] += d
    return [e for b in bins for e in sorted(b)]


class _LocalExperts(_QuantFusedMoEBlock):
    """A rank's slice of the routed experts, run with given routing and ``top_k = 1``."""

    def __init__(self, hidden: int, ffn: int, num_experts: int):
        nn.Module.__init__(self)
        self._init_common(hidden, ffn, num_experts, 1, False)


STAGES = ("route", "dispatch", "counts", "rows_out", "experts", "rows_back", "combine")


class ExpertParallelMoE(nn.Module):
    """Expert-parallel wrapper of a ``QuantFused*MoEBlock`` (see the module docstring)."""

    def __init__(self, block: Optional[_QuantFusedMoEBlock], group=None, route_fn: Optional[Callable] = None,
                 experts_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None,
                 dispatch_fn: Optional[Callable] = None, time_stages: bool = False, sm_budget: int = 0,
                 placement: Optional[Sequence[int]] = None, _shard: Optional[tuple] = None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if _shard is not None:
            local_block, gate_weight, E = _shard
            src = local_block
        else:
            src = block
            E = block.num_experts
            gate_weight = block.gate.weight
        if E % self.world != 0:
            raise ValueError(f"{E} experts do not split evenly over {self.world} ranks")
        self.num_experts, self.top_k = E, src.top_k
        self.hidden_dim, self.ffn_dim = src.hidden_dim, src.ffn_dim
        self.experts_per_rank = E // self.world
        self.e0 = self.rank * self.experts_per_rank  # first slot of this rank in the placement
        order = list(range(E)) if placement is None else [int(e) for e in placement]
        if sorted(order) != list(range(E)):
            raise ValueError(f"placement must be a permutation of the {E} expert ids")
        self.placement = order
        self.local_experts = order[self.e0:self.e0 + self.experts_per_rank]  # global ids, slot order
        self._identity = order == list(range(E))
        self._slot_of = None  # device int32 [E]: expert id -> position in the placement
        self.expert_load = None  # token-expert slots routed to each expert (device int64 [E])
        self.router_fp32 = src.router_fp32
        self.norm = bool(src.norm_topk_prob or src.always_normalize)
        # group-limited selection and the routing scale span all E experts
        self.routing = (self.norm, src.n_group, src.topk_group, src.routed_scaling_factor)
        self.returns_logits = src.returns_logits
        self.gate_weight = gate_weight.detach().to(torch.float16).contiguous()
        self.shared = src if getattr(src, "has_shared", False) else None
        if _shard is not None:
            if local_block.num_experts != self.experts_per_rank:
                raise ValueError(f"a shard holds {self.experts_per_rank} experts, got {local_block.num_experts}")
            self.local = _LocalExperts(src.hidden_dim, src.ffn_dim, self.experts_per_rank)
            for name in ("w1", "w2", "w3"):
                for key in ("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides", "zs_strides"):
                    setattr(self.local, f"{name}_{key}", getattr(local_block, f"{name}_{key}"))
            self.local.block_group_size = local_block.block_group_size
            self.local.invalidate()
        else:
            self.local = _LocalExperts(block.hidden_dim, block.ffn_dim, self.experts_per_rank)
            if block.w1_wq is not None:
                self._load_local(block)
        # gate/up bit-widths of all E experts (the dispatch writes each row in the K
        # order its owner's tensor-memory GEMM reads); a shard gathers them once
        if _shard is None:
            self.w1_nbits_all = block.w1_nbits if self._identity else block.w1_nbits[torch.tensor(
                order, device=block.w1_nbits.device)]
        elif self.world > 1:
            nb = local_block.w1_nbits.to(torch.int32).contiguous()
            allnb = nb.new_empty(E)
            dist.all_gather_into_tensor(allnb, nb, group=group)
            self.w1_nbits_all = allnb
        else:
            self.w1_nbits_all = local_block.w1_nbits
        self._rows_permuted = None  # decided by the local layer on the first forward
        self.route_fn = route_fn or self._route
        self.dispatch_fn = dispatch_fn or self._dispatch
        self.experts_fn = experts_fn or self._experts
        self.combine_fn = combine_fn or self._combine
        self.time_stages = time_stages
        self.sm_budget = int(sm_budget)
        self._events = None
        self._broken: Optional[str] = None  # set when an exchange failed

    @classmethod
    def from_shard(cls, local_block: _QuantFusedMoEBlock, gate_weight: Tensor, num_experts: int, group=None,
                   **kw) -> "ExpertParallelMoE":
        """Build from this rank's experts alone: ``local_block`` holds experts
        ``[rank * E / P, (rank + 1) * E / P)`` (its own gate is not used), and
        ``gate_weight`` is the full ``[E, hidden]`` router weight. No rank ever holds
        the whole layer. With ``placement=...`` the block holds experts
        ``placement[rank * E / P:(rank + 1) * E / P]`` in that order."""
        return cls(None, group=group, _shard=(local_block, gate_weight, num_experts), **kw)

    def _load_local(self, block: _QuantFusedMoEBlock):
        for name, k in (("w1", block.hidden_dim), ("w3", block.hidden_dim), ("w2", block.ffn_dim)):
            for key, t in gather_projection(block, name, self.local_experts, k).items():
                setattr(self.local, f"{name}_{key}", t)
        self.local.block_group_size = block.block_group_size
        self.local.invalidate()

    # ------------------------------------------------------------------ CUDA defaults
    def _route(self, x: Tensor):
        T = x.shape[0]
        gw = self.gate_weight.to(x.device)
        logits = torch.empty((T, self.num_experts), device=x.device,
                             dtype=torch.float32 if self.router_fp32 else torch.float16)
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.top_k), dtype=torch.float16, device=x.device)
        ws = torch.empty(_lib.ROUTE_WORKSPACE_BYTES, dtype=torch.uint8, device=x.device)
        router = _lib.GEMQ_ROUTER_FP32 if self.router_fp32 else _lib.GEMQ_ROUTER_FP16
        r = _lib.RoutingT(int(self.routing[0]), *self.routing[1:])
        check(_lib.load().gemq_route_ex(ptr(x), T, self.hidden_dim, ptr(gw), self.num_experts, self.top_k, router,
                                        ctypes.byref(r), 0, ptr(logits), ptr(idx), ptr(w), ptr(ws), ws.numel(),
                                        stream_ptr(x.device)))
        return logits, idx, w

    def _count_load(self, counts: Tensor) -> None:
        c = counts.to(torch.int64)
        if self.expert_load is None or self.expert_load.device != c.device:
            self.expert_load = torch.zeros(self.num_experts, dtype=torch.int64, device=c.device)
        if self._identity:
            self.expert_load += c
        else:
            self.expert_load.index_add_(0, torch.tensor(self.placement, device=c.device), c)

    def measured_load(self) -> Tensor:
        """Token-expert slots routed to each expert since construction, summed over
        all ranks (a collective: every rank calls it)."""
        load = self.expert_load.clone() if self.expert_load is not None else torch.zeros(
            self.num_experts, dtype=torch.int64, device=self.gate_weight.device)
        if self.world > 1:
            dist.all_reduce(load, group=self.group)
        return load

    def rows_permuted(self) -> bool:
        """Whether the local experts' GEMM takes rows in the tensor-memory GEMM's K order
        (the same answer on every rank: it depends on the layer's shapes alone)."""
        if self._rows_permuted is None:
            self._rows_permuted = bool(_lib.load().gemq_moe_experts_row_order(self.local.layer_handle()))
        return self._rows_permuted

    def _dispatch(self, idx: Tensor, w: Tensor, x: Tensor):
        T, k, E, D = x.shape[0], self.top_k, self.num_experts, self.hidden_dim
        P = T * k
        counts = torch.empty(E, dtype=torch.int32, device=x.device)
        slot_row = torch.empty(max(P, 1), dtype=torch.int32, device=x.device)
        w_rows = torch.empty(max(P, 1), dtype=torch.float16, device=x.device)
        x_rows = torch.empty((max(P, 1), D), dtype=torch.float16, device=x.device)
        lib = _lib.load()
        ws = torch.empty(lib.gemq_dispatch_workspace_size(T, k, E), dtype=torch.uint8, device=x.device)
        perm = None
        if self.rows_permuted():
            perm = self.w1_nbits_all.to(device=x.device, dtype=torch.int32).contiguous()
        check(lib.gemq_moe_dispatch(ptr(idx), ptr(w), ptr(x), T, k, E, D, ptr(perm), ptr(counts), ptr(slot_row),
                                    ptr(w_rows), ptr(x_rows), ptr(ws), ws.numel(), stream_ptr(x.device)))
        return counts, slot_row[:P], w_rows[:P], x_rows[:P]

    def _experts(self, rows: Tensor, group_counts: Tensor, weights: Tensor) -> Tensor:
        if rows.shape[0] == 0:
            return rows.clone()
        lib = _lib.load()
        handle = self.local.layer_handle()
        G = group_counts.shape[0]
        out = torch.empty_like(rows)
        gc = group_counts.to(device=rows.device, dtype=torch.int32).contiguous()
        ws = torch.empty(lib.gemq_moe_experts_workspace_size(handle, rows.shape[0], G), dtype=torch.uint8,
                         device=rows.device)
        flags = _lib.FWD_PERMUTED_ROWS if self.rows_permuted() else 0
        check(lib.gemq_moe_experts(handle, ptr(rows), rows.shape[0], ptr(gc), G, ptr(weights.contiguous()), ptr(out),
                                   self.sm_budget, flags, ptr(ws), ws.numel(), stream_ptr(rows.device)))
        return out

    def _combine(self, y: Tensor, slot_row: Tensor, topk_idx: Tensor, residual: Optional[Tensor]) -> Tensor:
        T = topk_idx.shape[0]
        out = torch.empty((T, self.hidden_dim), dtype=torch.float16, device=topk_idx.device)
        if y.shape[0] == 0:  # no slot: a zero-row tensor has no device address to pass
            y = torch.zeros((1, self.hidden_dim), dtype=torch.float16, device=topk_idx.device)
        check(_lib.load().gemq_moe_combine(ptr(y), ptr(slot_row), ptr(topk_idx), T, self.top_k, self.hidden_dim, 0,
                                           ptr(residual), ptr(out), stream_ptr(topk_idx.device)))
        return out

    # ------------------------------------------------------------------ exchange
    def _a2a(self, send: Tensor, send_counts, recv_counts, step: str) -> Tensor:
        recv = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
        if self.world == 1:
            recv.copy_(send)
            return recv
        try:
            dist.all_to_all_single(recv, send.contiguous(), [int(c) for c in recv_counts],
                                   [int(c) for c in send_counts], group=self.group)
        except Exception as exc:  # a peer is gone, timed out or aborted
            self._broken = f"exchange of {step} failed on rank {self.rank} of {self.world}: {exc}"
            raise ExpertParallelError(self._broken) from exc
        return recv

    def _mark(self, i: int, device) -> None:
        if not self.time_stages or device.type != "cuda":
            return
        if self._events is None:
            self._events = [torch.cuda.Event(enable_timing=True) for _ in range(len(STAGES) + 1)]
        self._events[i].record()

    def stage_times(self) -> dict:
        """Durations (ms) of the last forward's steps (``time_stages=True``, CUDA only)."""
        if self._events is None:
            return {}
        self._events[-1].synchronize()
        return {name: self._events[i].elapsed_time(self._events[i + 1]) for i, name in enumerate(STAGES)}

    def forward_tokens(self, x: Tensor) -> Tuple[Tensor, Tensor]:
        """``x [T, D]`` fp16 on this rank -> ``(out [T, D], router_logits [T, E])``."""
        if self._broken is not None:
            raise ExpertParallelError(f"an earlier exchange failed ({self._broken}); rebuild the process group")
        x = x.contiguous()
        dev = x.device
        epr, W = self.experts_per_rank, self.world
        self._mark(0, dev)
        logits, idx, w = self.route_fn(x)
        self._mark(1, dev)
        bad, didx = self._placed_ids(idx)
        counts, slot_row, w_rows, x_rows = self.dispatch_fn(didx, w, x)
        self._count_load(counts)
        self._mark(2, dev)
        # counts first, each destination's block with this rank's routing status, so
        # every rank can size its receives; the only host synchronisation
        msg = torch.cat([counts.to(torch.int32).reshape(W, epr), bad.to(counts.device).expand(W, 1)], dim=1)
        rmsg = self._a2a(msg.reshape(-1), [epr + 1] * W, [epr + 1] * W, "counts").reshape(W, epr + 1)
        both = torch.stack([msg, rmsg]).cpu()
        self._mark(3, dev)
        bad_ranks = [r for r in range(W) if int(both[1, r, epr]) != 0]
        if bad_ranks:
            raise ExpertParallelError(
                f"invalid routing table (expert id outside [0, {self.num_experts})) on rank(s) {bad_ranks}; "
                "no rows were exchanged")
        send_counts = both[0, :, :epr].sum(dim=1).tolist()
        recv_counts = both[1, :, :epr].sum(dim=1).tolist()
        rows = self._a2a(x_rows, send_counts, recv_counts, "activation rows")
        wts = self._a2a(w_rows, send_counts, recv_counts, "routing weights")
        self._mark(4, dev)
        y = self.experts_fn(rows, rmsg[:, :epr], wts)
        self._mark(5, dev)
        back = self._a2a(y, recv_counts, send_counts, "expert outputs")
        self._mark(6, dev)
        residual = None
        if self.shared is not None:
            residual = self.shared.forward_shared(x)
        out = self.combine_fn(back, slot_row, idx.to(torch.int32).contiguous(), residual)
        self._mark(7, dev)
        return out, logits

    def _placed_ids(self, idx: Tensor) -> Tuple[Tensor, Tensor]:
        """``(bad [1] int32, ids to dispatch by)``: whether any routed id lies outside
        ``[0, E)``, and each id's position in the placement (invalid ids pass through,
        for the dispatch to record and skip)."""
        flat = idx.reshape(-1)
        valid = (flat >= 0) & (flat < self.num_experts)
        bad = (~valid).any().to(torch.int32).reshape(1)
        if self._identity:
            return bad, idx
        if self._slot_of is None or self._slot_of.device != idx.device:
            slot = torch.empty(self.num_experts, dtype=torch.int32)
            slot[torch.tensor(self.placement)] = torch.arange(self.num_experts, dtype=torch.int32)
            self._slot_of = slot.to(idx.device)
        didx = torch.where(valid, self._slot_of[flat.clamp(0, self.num_experts - 1).long()], flat.to(torch.int32))
        return bad, didx.reshape(idx.shape).to(idx.dtype)

    def _a2a_start(self, send: Tensor, send_counts, recv_counts, step: str):
        """Starts an all-to-all; returns ``(recv, wait)``, ``wait()`` completing it (on
        NCCL the current stream then waits for it; the exchange itself runs on the
        process group's own stream, beside the GEMMs enqueued meanwhile)."""
        recv = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
        if self.world == 1:
            recv.copy_(send)
            return recv, lambda: None
        try:
            work = dist.all_to_all_single(recv, send.contiguous(), [int(c) for c in recv_counts],
                                          [int(c) for c in send_counts], group=self.group, async_op=True)
        except Exception as exc:
            self._broken = f"exchange of {step} failed on rank {self.rank} of {self.world}: {exc}"
            raise ExpertParallelError(self._broken) from exc

        def wait():
            try:
                work.wait()
            except Exception as exc:  # a peer is gone, timed out or aborted
                self._broken = f"exchange of {step} failed on rank {self.rank} of {self.world}: {exc}"
                raise ExpertParallelError(self._broken) from exc

        return recv, wait

    def forward_tokens_chunked(self, x: Tensor, chunks: int) -> Tuple[Tensor, Tensor]:
        """``forward_tokens`` over ``chunks`` contiguous token chunks whose exchanges
        overlap the expert GEMMs: chunk c + 1's activation rows and weights travel
        while chunk c's experts run, and chunk c's outputs travel back while later
        chunks compute. The whole batch is routed at once and one counts exchange
        (the one host synchronisation) covers every chunk. The output equals
        ``forward_tokens``' bit for bit: each row is computed alone and the combine
        visits a token's experts in ascending id. Every rank must pass the same
        ``chunks``. Stage timing is not recorded here."""
        T = x.shape[0]
        if chunks <= 1:
            return self.forward_tokens(x)
        if self._broken is not None:
            raise ExpertParallelError(f"an earlier exchange failed ({self._broken}); rebuild the process group")
        x = x.contiguous()
        epr, W = self.experts_per_rank, self.world
        bounds = [T * c // chunks for c in range(chunks + 1)]
        logits, idx, w = self.route_fn(x)
        bad, didx = self._placed_ids(idx)
        parts = []
        for c in range(chunks):
            a, b = bounds[c], bounds[c + 1]
            counts, slot_row, w_rows, x_rows = self.dispatch_fn(didx[a:b].contiguous(), w[a:b].contiguous(),
                                                                x[a:b].contiguous())
            self._count_load(counts)
            parts.append((counts, slot_row, w_rows, x_rows))
        # one message per destination: every chunk's counts of its experts, then this
        # rank's routing status
        cnt = torch.stack([p[0].to(torch.int32).reshape(W, epr) for p in parts], dim=1).reshape(W, chunks * epr)
        msg = torch.cat([cnt, bad.to(cnt.device).expand(W, 1)], dim=1)
        n = chunks * epr + 1
        rmsg = self._a2a(msg.reshape(-1), [n] * W, [n] * W, "counts").reshape(W, n)
        both = torch.stack([msg, rmsg]).cpu()
        bad_ranks = [r for r in range(W) if int(both[1, r, n - 1]) != 0]
        if bad_ranks:
            raise ExpertParallelError(
                f"invalid routing table (expert id outside [0, {self.num_experts})) on rank(s) {bad_ranks}; "
                "no rows were exchanged")
        sent = both[0, :, :n - 1].reshape(W, chunks, epr).sum(dim=2)  # [destination, chunk]
        got = both[1, :, :n - 1].reshape(W, chunks, epr).sum(dim=2)   # [source, chunk]

        def start_rows(c):
            sc, rc = sent[:, c].tolist(), got[:, c].tolist()
            rows = self._a2a_start(parts[c][3], sc, rc, f"activation rows of chunk {c}")
            wts = self._a2a_start(parts[c][2], sc, rc, f"routing weights of chunk {c}")
            return rows, wts

        backs = []
        nxt = start_rows(0)
        for c in range(chunks):
            (rows, wait_rows), (wts, wait_wts) = nxt
            wait_rows()
            wait_wts()
            if c + 1 < chunks:
                nxt = start_rows(c + 1)
            y = self.experts_fn(rows, rmsg[:, c * epr:(c + 1) * epr], wts)
            backs.append(self._a2a_start(y, got[:, c].tolist(), sent[:, c].tolist(), f"expert outputs of chunk {c}"))
        outs = []
        for c in range(chunks):
            back, wait_back = backs[c]
            wait_back()
            a, b = bounds[c], bounds[c + 1]
            residual = self.shared.forward_shared(x[a:b]) if self.shared is not None else None
            outs.append(self.combine_fn(back, parts[c][1], idx[a:b].to(torch.int32).contiguous(), residual))
        return torch.cat(outs), logits

    def forward(self, hidden_states: Tensor):
        shape = hidden_states.shape
        out, logits = self.forward_tokens(hidden_states.reshape(-1, self.hidden_dim))
        out = out.reshape(shape)
        return (out, logits) if self.returns_logits else out
