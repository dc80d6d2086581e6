"""Expert parallelism for the quantized MoE block over ``torch.distributed``.

Rank ``r`` of ``P`` holds experts ``[r * E / P, (r + 1) * E / P)`` of every
projection (the stacked packed layout of ``from_hf``, sliced by expert with its
strides rebased). A forward on a rank's own tokens:

1. routes them over all ``E`` experts (``gemq_route``; the gate is replicated);
2. orders the ``T * k`` token-expert slots by the rank owning the expert and sends
   each slot's activation row, local expert id and routing weight there with
   ``all_to_all_single`` (counts first);
3. the owner runs its local experts on the rows it received, one expert per row
   (``gemq_moe_forward`` with given routing and ``top_k = 1``, whose output row is
   exactly ``fp16(fp16(y) * w)``: the down projection's route-weight epilogue);
4. sends the rows back with the reverse ``all_to_all_single``;
5. combines each token's ``k`` rows in ascending expert id with fp16 rounding after
   every add (``gemq_moe_combine``): the fp16 ``index_add_`` order of
   ``forward_n_tokens`` (moe_block.py:799-812), so a rank's output equals the 1-GPU
   block's on the same tokens whenever the per-row GEMM results do.

DeepSeek's shared experts are replicated and run on the token's own rank; their
output is added in fp16 after the combine (moe_block.py:575).

Failures end in ``ExpertParallelError`` on every rank, never in a hang:

* an invalid routing table on one rank (an expert id outside ``[0, E)``) travels
  with the counts of step 2 as a per-peer status, so every rank learns of it in
  the same exchange and raises before any row is sent; all ranks took the same
  collective steps, so the group stays usable for the next forward;
* a rank that is gone or never joins ends the others' pending exchange through
  the process group's timeout (or the closed connection); the error names the
  step, and the wrapper refuses further forwards, since the group's state is no
  longer known (rebuild the group and the wrapper).

With NCCL the exchange runs over NVLink; with gloo (CPU tests) the local expert
compute, the router and the combine can be replaced by callables (``route_fn``,
``experts_fn``, ``combine_fn``) so the dispatch / combine bookkeeping is tested
without a GPU. The defaults are the CUDA kernels; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor, nn

from .. import _lib
from .._lib import check, ptr, stream_ptr
from .moe_block import _QuantFusedMoEBlock


class ExpertParallelError(RuntimeError):
    """An expert-parallel forward failed: invalid routing on some rank, or a failed exchange."""


def plan_dispatch(topk_idx: Tensor, experts_per_rank: int, world: int) -> Tuple[Tensor, Tensor, Tensor]:
    """Send order of the ``T * k`` slots (stable, grouped by destination rank), the
    per-rank slot counts, and each sent slot's expert id local to its destination."""
    flat = topk_idx.reshape(-1).to(torch.int64)
    dest = torch.div(flat, experts_per_rank, rounding_mode="floor")
    if bool(((dest < 0) | (dest >= world)).any()):
        raise ValueError("expert id out of range for the expert-parallel layout")
    order = torch.argsort(dest, stable=True)
    counts = torch.bincount(dest, minlength=world)
    local = (flat - dest * experts_per_rank)[order]
    return order, counts, local


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


class _LocalExperts(_QuantFusedMoEBlock):
    """A rank's slice of the routed experts, run with given routing and ``top_k = 1``."""

    def __init__(self, hidden: int, ffn: int, num_experts: int):
        nn.Module.__init__(self)
        self._init_common(hidden, ffn, num_experts, 1, False)


class ExpertParallelMoE(nn.Module):
    """Expert-parallel wrapper of a ``QuantFused*MoEBlock`` (see the module docstring)."""

    def __init__(self, block: _QuantFusedMoEBlock, group=None, route_fn: Optional[Callable] = None,
                 experts_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        E = block.num_experts
        if E % self.world != 0:
            raise ValueError(f"{E} experts do not split evenly over {self.world} ranks")
        self.num_experts, self.top_k = E, block.top_k
        self.hidden_dim, self.ffn_dim = block.hidden_dim, block.ffn_dim
        self.experts_per_rank = E // self.world
        self.e0 = self.rank * self.experts_per_rank
        self.router_fp32 = block.router_fp32
        self.norm = bool(block.norm_topk_prob or block.always_normalize)
        self.returns_logits = block.returns_logits
        self.gate_weight = block.gate.weight.detach().to(torch.float16).contiguous()
        self.shared = block if getattr(block, "has_shared", False) else None
        self.local = _LocalExperts(block.hidden_dim, block.ffn_dim, self.experts_per_rank)
        if block.w1_wq is not None:
            self._load_local(block)
        self.route_fn = route_fn or self._route
        self.experts_fn = experts_fn or self._experts
        self.combine_fn = combine_fn or self._combine
        self._broken: Optional[str] = None  # set when an exchange failed

    def _load_local(self, block: _QuantFusedMoEBlock):
        e1 = self.e0 + self.experts_per_rank
        for name, k in (("w1", block.hidden_dim), ("w3", block.hidden_dim), ("w2", block.ffn_dim)):
            for key, t in slice_projection(block, name, self.e0, e1, k).items():
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
        check(_lib.load().gemq_route(ptr(x), T, self.hidden_dim, ptr(gw), self.num_experts, self.top_k, router,
                                     int(self.norm), 0, ptr(logits), ptr(idx), ptr(w), ptr(ws), ws.numel(),
                                     stream_ptr(x.device)))
        return logits, idx, w

    def _experts(self, rows: Tensor, local_ids: Tensor, weights: Tensor) -> Tensor:
        if rows.shape[0] == 0:
            return rows.clone()
        return self.local.forward_routed(rows, local_ids.reshape(-1, 1), weights.reshape(-1, 1))

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

    def forward_tokens(self, x: Tensor) -> Tuple[Tensor, Tensor]:
        """``x [T, D]`` fp16 on this rank -> ``(out [T, D], router_logits [T, E])``."""
        if self._broken is not None:
            raise ExpertParallelError(f"an earlier exchange failed ({self._broken}); rebuild the process group")
        x = x.contiguous()
        T, k = x.shape[0], self.top_k
        logits, idx, w = self.route_fn(x)
        flat = idx.reshape(-1)
        valid = not bool(((flat < 0) | (flat >= self.num_experts)).any())
        if valid:
            order, send_counts, local_ids = plan_dispatch(idx, self.experts_per_rank, self.world)
        else:  # send no rows; the status below tells every peer
            order = torch.arange(T * k, device=x.device)
            send_counts = torch.zeros(self.world, dtype=torch.int64)
            local_ids = torch.zeros(T * k, dtype=torch.int64)
        order = order.to(x.device)
        # counts first, so every rank can size its receive buffers, each sent with
        # this rank's routing status
        sc = send_counts.to(device=x.device, dtype=torch.int64)
        msg = torch.stack([sc, torch.full_like(sc, 0 if valid else 1)], dim=1).reshape(-1)
        rmsg = self._a2a(msg, [2] * self.world, [2] * self.world, "counts").reshape(self.world, 2)
        bad = [r for r in range(self.world) if int(rmsg[r, 1]) != 0]
        if bad:
            raise ExpertParallelError(
                f"invalid routing table (expert id outside [0, {self.num_experts})) on rank(s) {bad}; "
                "no rows were exchanged")
        send_counts, recv_counts = sc.tolist(), rmsg[:, 0].tolist()
        tok = torch.div(order, k, rounding_mode="floor")
        rows = self._a2a(x.index_select(0, tok), send_counts, recv_counts, "activation rows")
        ids = self._a2a(local_ids.to(device=x.device, dtype=torch.int32), send_counts, recv_counts, "expert ids")
        wts = self._a2a(w.reshape(-1).index_select(0, order), send_counts, recv_counts, "routing weights")
        y = self.experts_fn(rows, ids, wts)
        back = self._a2a(y, recv_counts, send_counts, "expert outputs")
        slot_row = torch.empty(T * k, dtype=torch.int32, device=x.device)
        slot_row[order] = torch.arange(T * k, dtype=torch.int32, device=x.device)
        residual = None
        if self.shared is not None:
            residual = self.shared.forward_shared(x)
        out = self.combine_fn(back, slot_row, idx.to(torch.int32).contiguous(), residual)
        return out, logits

    def forward(self, hidden_states: Tensor):
        shape = hidden_states.shape
        out, logits = self.forward_tokens(hidden_states.reshape(-1, self.hidden_dim))
        out = out.reshape(shape)
        return (out, logits) if self.returns_logits else out
