"""Quantized MoE blocks: drop-in for gemq/inference/moe_block.py's QuantFused* classes.

Same constructors (``cls(config)``), ``from_hf(config, hf_block)``, attribute names
(``w{1,2,3}_{wq,scales,zeros,nbits,group_sizes,wq_strides,zs_strides}``,
``block_group_size``; DeepSeek ``shared_w{1,2,3}_*``, ``shared_nbits``,
``shared_group_size``), guards and return conventions (OLMoE/Qwen3/Mixtral return
``(out, router_logits)`` from the n-token path and ``(out, None)`` from the
one-token path; DeepSeek returns ``out``). The forward passes run entirely in
``libgemq_b200.so``:

* ``forward_n_tokens`` (moe_block.py:781-815): device router -> histogram/scan
  dispatch -> tcgen05 grouped GEMM with fused gate/up + SiLU*mul -> grouped
  down-projection with the routing weight -> ascending-expert fp16 combine. No host
  synchronisation, no Python loop over experts.
* ``forward_one_token`` (moe_block.py:817-853): device router -> deterministic
  split-K dequant GEMVs -> fp32 combine; graph-capturable (no host sync, no
  allocation after the first call with a given shape).

Expert linears are read by attribute (``W_q``, ``scales``, ``zeros``, ``W_nbits``,
``group_size``) as the reference reads GemLite layers; ``quant.PackedLinear`` is the
in-tree producer of that layout.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch
import torch.nn as nn
from torch import Tensor

from .. import _lib
from .._lib import LayerDescT, check, ptr, stream_ptr
from ..ops import dequant_gemm, dequant_group_gemm, make_proj


# --------------------------------------------------------------------------- guards
def check_deepseek_routing_supported(config):
    """Expert-selection features the fused DeepSeek forward does not implement
    (moe_block.py:18-28). The reference accepts only ``topk_method='greedy'``; this
    block also runs DeepSeek-V2's ``group_limited_greedy`` (``n_group`` groups of
    experts, ``topk_group`` kept per token, as transformers'
    ``DeepseekV2Moe.route_tokens_to_experts`` selects them). Scoring stays softmax."""
    scoring_func = getattr(config, "scoring_func", "softmax")
    assert scoring_func == "softmax", (
        f"fused block always uses softmax scoring, config asks for '{scoring_func}'"
    )
    method = getattr(config, "topk_method", "greedy")
    assert method in ("greedy", "group_limited_greedy"), (
        f"fused block implements topk_method 'greedy' and 'group_limited_greedy', got '{method}'"
    )
    if method == "group_limited_greedy":
        n_group, topk_group = int(config.n_group), int(config.topk_group)
        assert 1 <= n_group <= 32 and config.n_routed_experts % n_group == 0, (
            f"n_group ({n_group}) must be in [1, 32] and divide n_routed_experts ({config.n_routed_experts})"
        )
        assert 1 <= topk_group <= n_group, f"topk_group ({topk_group}) must be in [1, n_group]"
        assert topk_group * (config.n_routed_experts // n_group) >= config.num_experts_per_tok, (
            "the kept groups must hold at least num_experts_per_tok experts"
        )


def deepseek_group_routing(config):
    """``(n_group, topk_group)`` of the config's expert selection; (1, 1) for greedy."""
    if getattr(config, "topk_method", "greedy") == "group_limited_greedy":
        return int(config.n_group), int(config.topk_group)
    return 1, 1


def check_deepseek_gate_matches(config, hf_block):
    """How the replaced block combines its routing weights, as ``(normalize, scale)``:
    the fused block computes ``w / w.sum()`` when ``normalize``, else
    ``w * scale`` (moe_block.py:31-66 lists the two gates):

        official modeling_deepseek.py:  w /= w.sum()  if top_k > 1 and norm_topk_prob
                                        else  w *= routed_scaling_factor
        HF built-in:                    w *= routed_scaling_factor  (norm_topk_prob unused)

    The reference's fused block never scales, so it asserts that the replaced gate
    does not either; this block applies the scale and accepts every combination."""
    is_builtin = type(hf_block).__module__.startswith("transformers.models.deepseek_v2")
    scaling = float(getattr(config, "routed_scaling_factor", 1.0))
    if is_builtin:
        return False, scaling
    if bool(config.norm_topk_prob) and config.num_experts_per_tok > 1:
        return True, 1.0
    return False, scaling


def check_w1_w3_aligned(fused_block):
    """``forward_one_token`` reads w3 with w1's nbits/strides (moe_block.py:69-80)."""
    assert torch.equal(fused_block.w1_nbits, fused_block.w3_nbits), (
        "w1 and w3 must share bit-widths: forward_one_token indexes w3 with w1's nbits"
    )
    assert torch.equal(fused_block.w1_wq_strides, fused_block.w3_wq_strides), (
        "w1 and w3 must share packed strides: forward_one_token reads w3 at w1's offsets"
    )


def _exclusive_cumsum(sizes: Sequence[int], device) -> Tensor:
    out = [0]
    for s in sizes[:-1]:
        out.append(out[-1] + int(s))
    return torch.tensor(out, dtype=torch.int32, device=device)


def _is_packed(linear) -> bool:
    return all(hasattr(linear, a) for a in ("W_q", "scales", "zeros", "W_nbits", "group_size"))


# --------------------------------------------------------------------------- base
class _QuantFusedMoEBlock(nn.Module):
    """Shared machinery; subclasses fix the family's config names and conventions."""

    expert_names = ("gate_proj", "up_proj", "down_proj")  # -> w1, w3, w2
    router_fp32 = False        # DeepSeek forms logits in fp32 (moe_block.py:549)
    always_normalize = False   # Mixtral renormalises unconditionally (moe_block.py:247)
    fp16_softmax_one_token = False  # Mixtral one-token router on fp16 tensors (moe_block.py:280-283)
    returns_logits = True
    has_shared = False

    def _init_common(self, hidden, ffn, num_experts, top_k, norm_topk_prob):
        self.hidden_dim = hidden
        self.ffn_dim = ffn
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = bool(norm_topk_prob)
        self.gate = nn.Linear(self.hidden_dim, self.num_experts, bias=False)
        self.w1_wq, self.w1_scales, self.w1_zeros = None, None, None
        self.w2_wq, self.w2_scales, self.w2_zeros = None, None, None
        self.w3_wq, self.w3_scales, self.w3_zeros = None, None, None
        self.w1_nbits, self.w1_group_sizes = None, None
        self.w2_nbits, self.w2_group_sizes = None, None
        self.w3_nbits, self.w3_group_sizes = None, None
        self.block_group_size = None
        self.w1_wq_strides, self.w1_zs_strides = None, None
        self.w2_wq_strides, self.w2_zs_strides = None, None
        self.w3_wq_strides, self.w3_zs_strides = None, None
        self.n_group, self.topk_group = 1, 1
        self.routed_scaling_factor = 1.0
        self._handle = None
        self._workspaces = {}
        self._fwd_flags = 0

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_hf(cls, config, hf_block):
        """Stack the repacked expert linears of an HF block (moe_block.py:715-761)."""
        fused_block = cls(config)
        fused_block.gate.weight.data = hf_block.gate.weight.data.clone()
        n1, n3, n2 = cls.expert_names
        if not _is_packed(getattr(hf_block.experts[0], n1)):
            raise ValueError(f"Expected linears in {type(hf_block).__name__}. Please patch and replace them first.")
        lin = lambda name: [getattr(ex, name) for ex in hf_block.experts]  # noqa: E731
        fused_block.load_packed(lin(n1), lin(n3), lin(n2))
        return fused_block

    @classmethod
    def from_packed(cls, config, gate_weight: Tensor, w1: List, w3: List, w2: List, shared: Optional[tuple] = None):
        """Build from per-expert packed linears directly (no HF block)."""
        fused_block = cls(config)
        fused_block.gate.weight.data = gate_weight.detach().clone()
        fused_block.load_packed(w1, w3, w2)
        if shared is not None:
            fused_block.load_shared(*shared)
        return fused_block

    def load_packed(self, w1: List, w3: List, w2: List):
        for name, linears in (("w1", w1), ("w2", w2), ("w3", w3)):
            setattr(self, f"{name}_wq", torch.cat([l.W_q.data for l in linears]).contiguous())
            setattr(self, f"{name}_scales", torch.cat([l.scales.data for l in linears]).contiguous())
            setattr(self, f"{name}_zeros", torch.cat([l.zeros.data for l in linears]).contiguous())
            device = getattr(self, f"{name}_wq").device
            setattr(self, f"{name}_nbits", torch.tensor([l.W_nbits for l in linears], dtype=torch.int32, device=device))
            setattr(self, f"{name}_group_sizes",
                    torch.tensor([l.group_size for l in linears], dtype=torch.int32, device=device))
            setattr(self, f"{name}_wq_strides", _exclusive_cumsum([l.W_q.numel() for l in linears], device))
            setattr(self, f"{name}_zs_strides", _exclusive_cumsum([l.scales.numel() for l in linears], device))
        block_group_size = torch.unique(torch.cat([self.w1_group_sizes, self.w2_group_sizes, self.w3_group_sizes]))
        assert len(block_group_size) == 1, "Group sizes must be the same across all experts."
        self.block_group_size = int(block_group_size.item())
        check_w1_w3_aligned(self)
        self.invalidate()

    def set_routing(self, norm_topk_prob: Optional[bool] = None, routed_scaling_factor: Optional[float] = None,
                    n_group: Optional[int] = None, topk_group: Optional[int] = None):
        """Change the router's weight rule (``w / sum`` when ``norm_topk_prob``, else
        ``w * routed_scaling_factor``) or its group-limited selection."""
        if norm_topk_prob is not None:
            self.norm_topk_prob = bool(norm_topk_prob)
        if routed_scaling_factor is not None:
            self.routed_scaling_factor = float(routed_scaling_factor)
        if n_group is not None:
            self.n_group = int(n_group)
        if topk_group is not None:
            self.topk_group = int(topk_group)
        if self._handle is not None:
            self._apply_routing(self._handle)

    def routing_options(self) -> "_lib.RoutingT":
        return _lib.RoutingT(int(self.norm_topk_prob or self.always_normalize), self.n_group, self.topk_group,
                             self.routed_scaling_factor)

    def _apply_routing(self, handle):
        r = self.routing_options()
        check(_lib.load().gemq_layer_set_routing(handle, ctypes.byref(r)))

    def invalidate(self):
        """Drop the native layer handle (call after replacing weight tensors)."""
        if self._handle is not None:
            _lib.load().gemq_layer_destroy(self._handle)
        self._handle = None
        self._workspaces = {}

    def __del__(self):
        try:
            if getattr(self, "_handle", None) is not None:
                _lib.load().gemq_layer_destroy(self._handle)
        except Exception:
            pass

    # ------------------------------------------------------------------ native handle
    def _proj(self, name: str, k: int):
        return make_proj(getattr(self, f"{name}_wq"), getattr(self, f"{name}_scales"), getattr(self, f"{name}_zeros"),
                         getattr(self, f"{name}_nbits"), getattr(self, f"{name}_wq_strides"),
                         getattr(self, f"{name}_zs_strides"), k, self.block_group_size)

    def _fill_shared(self, d: LayerDescT):
        return None

    def layer_handle(self):
        if self._handle is None:
            if self.w1_wq is None:
                raise ValueError("block has no packed weights; build it with from_hf or from_packed")
            gw = self.gate.weight
            if gw.dtype != torch.float16 or gw.device != self.w1_wq.device:
                self.gate.to(device=self.w1_wq.device, dtype=torch.float16)
            self._gate_w = self.gate.weight.data.contiguous()
            d = LayerDescT()
            d.hidden, d.inter, d.num_experts, d.top_k = self.hidden_dim, self.ffn_dim, self.num_experts, self.top_k
            d.group_size = self.block_group_size
            d.norm_topk_prob = int(self.norm_topk_prob or self.always_normalize)
            d.router = _lib.GEMQ_ROUTER_FP32 if self.router_fp32 else _lib.GEMQ_ROUTER_FP16
            d.gate_weight = self._gate_w.data_ptr()
            d.w1 = self._proj("w1", self.hidden_dim)
            d.w3 = self._proj("w3", self.hidden_dim)
            d.w2 = self._proj("w2", self.ffn_dim)
            d.has_shared = 0
            self._fill_shared(d)
            handle = ctypes.c_void_p()
            check(_lib.load().gemq_layer_create(ctypes.byref(d), ctypes.byref(handle)))
            try:
                self._apply_routing(handle)
            except Exception:
                _lib.load().gemq_layer_destroy(handle)
                raise
            self._handle = handle
        return self._handle

    def _workspace(self, T: int, flags: int, device) -> Tensor:
        key = (T, flags)
        ws = self._workspaces.get(key)
        if ws is None:
            n = _lib.load().gemq_moe_workspace_size(self.layer_handle(), T, flags)
            ws = torch.empty(n, dtype=torch.uint8, device=device)
            self._workspaces[key] = ws
        return ws

    def _run(self, x: Tensor, flags: int, want_logits: bool, topk_idx: Optional[Tensor] = None,
             topk_w: Optional[Tensor] = None, logits_in: Optional[Tensor] = None):
        if not x.is_cuda:
            raise ValueError("QuantFused blocks run on CUDA only (no CPU path)")
        if x.dtype != torch.float16:
            raise ValueError("hidden_states must be float16 (the reference computes in fp16)")
        if _lib.off_current_device(x):
            with torch.cuda.device(x.device):
                return self._run(x, flags, want_logits, topk_idx, topk_w, logits_in)
        x = x.contiguous()
        T = x.shape[0]
        handle = self.layer_handle()
        out = torch.empty_like(x)
        logits = None
        if logits_in is not None:
            flags |= _lib.FWD_GIVEN_LOGITS
            logits = logits_in.float().contiguous()
        elif want_logits:
            logits = torch.empty((T, self.num_experts), device=x.device,
                                 dtype=torch.float32 if self.router_fp32 else torch.float16)
        if topk_idx is not None:
            flags |= _lib.FWD_GIVEN_ROUTING
            topk_idx = topk_idx.to(device=x.device, dtype=torch.int32).contiguous()
            topk_w = topk_w.to(device=x.device, dtype=torch.float16).contiguous()
        flags |= self._fwd_flags
        ws = self._workspace(T, flags, x.device)
        check(_lib.load().gemq_moe_forward(handle, ptr(x), T, ptr(out), ptr(logits), ptr(topk_idx), ptr(topk_w),
                                           flags, ptr(ws), ws.numel(), stream_ptr(x.device)))
        return out, logits

    # ------------------------------------------------------------------ reference API
    def forward_single_expert(self, expert_idx: Tensor, hidden_states: Tensor) -> Tensor:
        """One expert's SwiGLU through three grouped GEMMs (moe_block.py:763-779)."""
        x = hidden_states
        x1 = dequant_group_gemm(x, expert_idx, self.w1_wq, self.w1_scales, self.w1_zeros, self.w1_nbits,
                                self.w1_group_sizes, self.w1_wq_strides, self.w1_zs_strides)[0]
        x3 = dequant_group_gemm(x, expert_idx, self.w3_wq, self.w3_scales, self.w3_zeros, self.w3_nbits,
                                self.w3_group_sizes, self.w3_wq_strides, self.w3_zs_strides)[0]
        h = torch.nn.functional.silu(x1) * x3
        return dequant_group_gemm(h, expert_idx, self.w2_wq, self.w2_scales, self.w2_zeros, self.w2_nbits,
                                  self.w2_group_sizes, self.w2_wq_strides, self.w2_zs_strides)[0]

    def forward_n_tokens(self, hidden_states: Tensor):
        batch_size, sequence_length, hidden_dim = hidden_states.shape
        out, logits = self._run(hidden_states.view(-1, hidden_dim), 0, want_logits=self.returns_logits)
        out = out.reshape(batch_size, sequence_length, hidden_dim)
        return (out, logits) if self.returns_logits else out

    def forward_one_token(self, hidden_states: Tensor):
        batch_size, sequence_length, hidden_dim = hidden_states.shape
        x = hidden_states.view(-1, self.hidden_dim)
        assert x.shape[0] == 1, f"This function only supports single token forward. But got {x.shape[0]} tokens."
        flags = _lib.FWD_ONE_TOKEN | (_lib.FWD_FP16_SOFTMAX if self.fp16_softmax_one_token else 0)
        out, _ = self._run(x, flags, want_logits=False)
        out = out.reshape(batch_size, sequence_length, hidden_dim)
        return (out, None) if self.returns_logits else out

    def forward(self, hidden_states: Tensor):
        if hidden_states.shape[0] == hidden_states.shape[1] == 1:
            return self.forward_one_token(hidden_states)
        return self.forward_n_tokens(hidden_states)

    # ------------------------------------------------------------------ extensions
    def forward_routed(self, hidden_states: Tensor, topk_idx: Tensor, topk_w: Tensor, one_token: bool = False,
                       fp32_combine: bool = False) -> Tensor:
        """Block forward with a given routing (``[T, k]`` expert ids and fp16 weights)."""
        x = hidden_states.reshape(-1, self.hidden_dim)
        flags = (_lib.FWD_ONE_TOKEN if one_token else 0) | (_lib.FWD_FP32_COMBINE if fp32_combine else 0)
        out, _ = self._run(x, flags, want_logits=False, topk_idx=topk_idx, topk_w=topk_w)
        return out.reshape(hidden_states.shape)

    def forward_logits(self, hidden_states: Tensor, router_logits: Tensor) -> Tensor:
        """Block forward routed from given fp32 logits (skips the gate GEMM)."""
        x = hidden_states.reshape(-1, self.hidden_dim)
        out, _ = self._run(x, 0, want_logits=False, logits_in=router_logits)
        return out.reshape(hidden_states.shape)

    def route(self, hidden_states: Tensor):
        """Router only: ``(logits, topk_idx int32, topk_w fp16)``."""
        if _lib.off_current_device(hidden_states):
            with torch.cuda.device(hidden_states.device):
                return self.route(hidden_states)
        x = hidden_states.reshape(-1, self.hidden_dim).contiguous()
        T = x.shape[0]
        logits = torch.empty((T, self.num_experts), device=x.device,
                             dtype=torch.float32 if self.router_fp32 else torch.float16)
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.top_k), dtype=torch.float16, device=x.device)
        ws = torch.empty(4096, dtype=torch.uint8, device=x.device)
        check(_lib.load().gemq_moe_route(self.layer_handle(), ptr(x), T, ptr(logits), ptr(idx), ptr(w), 0, ptr(ws),
                                         ws.numel(), stream_ptr(x.device)))
        return logits, idx, w


# --------------------------------------------------------------------------- families
class QuantFusedMixtralMoEBlock(_QuantFusedMoEBlock):
    """moe_block.py:140-309: always renormalises; fp16 softmax at decode."""

    expert_names = ("w1", "w3", "w2")
    always_normalize = True
    fp16_softmax_one_token = True

    def __init__(self, config) -> None:
        super().__init__()
        self._init_common(config.hidden_size, config.intermediate_size, config.num_local_experts,
                          config.num_experts_per_tok, True)


class QuantFusedOlmoeMoEBlock(_QuantFusedMoEBlock):
    """moe_block.py:688-858."""

    def __init__(self, config) -> None:
        super().__init__()
        self._init_common(config.hidden_size, config.intermediate_size, config.num_experts,
                          config.num_experts_per_tok, config.norm_topk_prob)


class QuantFusedQwen3MoeMoEBlock(_QuantFusedMoEBlock):
    """moe_block.py:918-1088."""

    def __init__(self, config) -> None:
        super().__init__()
        self._init_common(config.hidden_size, config.moe_intermediate_size, config.num_experts,
                          config.num_experts_per_tok, config.norm_topk_prob)


class QuantFusedDeepseekV2MoEBlock(_QuantFusedMoEBlock):
    """moe_block.py:394-628: fp32 router, two always-on shared experts, returns a tensor."""

    router_fp32 = True
    returns_logits = False
    has_shared = True

    def __init__(self, config) -> None:
        super().__init__()
        check_deepseek_routing_supported(config)
        self._init_common(config.hidden_size, config.moe_intermediate_size, config.n_routed_experts,
                          config.num_experts_per_tok, config.norm_topk_prob)
        self.n_group, self.topk_group = deepseek_group_routing(config)
        self.num_shared_experts = config.n_shared_experts
        for name in ("shared_w1", "shared_w2", "shared_w3"):
            setattr(self, f"{name}_wq", None)
            setattr(self, f"{name}_scales", None)
            setattr(self, f"{name}_zeros", None)
        self.shared_nbits, self.shared_group_size = None, None

    @classmethod
    def from_hf(cls, config, hf_block):
        normalize, scale = check_deepseek_gate_matches(config, hf_block)
        fused_block = super().from_hf(config, hf_block)
        fused_block.set_routing(norm_topk_prob=normalize, routed_scaling_factor=scale)
        se = hf_block.shared_experts
        fused_block.load_shared(se.gate_proj, se.up_proj, se.down_proj)
        return fused_block

    def load_shared(self, gate_proj, up_proj, down_proj):
        """Shared experts (moe_block.py:477-504): one bit-width and group size for all three."""
        self.shared_w1_wq, self.shared_w1_scales, self.shared_w1_zeros = (
            gate_proj.W_q.data.clone().contiguous(), gate_proj.scales.data.clone(), gate_proj.zeros.data.clone())
        self.shared_w2_wq, self.shared_w2_scales, self.shared_w2_zeros = (
            down_proj.W_q.data.clone().contiguous(), down_proj.scales.data.clone(), down_proj.zeros.data.clone())
        self.shared_w3_wq, self.shared_w3_scales, self.shared_w3_zeros = (
            up_proj.W_q.data.clone().contiguous(), up_proj.scales.data.clone(), up_proj.zeros.data.clone())
        self.shared_nbits = gate_proj.W_nbits
        self.shared_group_size = gate_proj.group_size
        for name, lin in (("up_proj", up_proj), ("down_proj", down_proj)):
            assert lin.W_nbits == self.shared_nbits, (
                f"shared expert {name} uses {lin.W_nbits} bits but gate_proj uses {self.shared_nbits}; "
                "the shared-expert kernels assume one bit-width")
            assert lin.group_size == self.shared_group_size, (
                f"shared expert {name} uses group_size {lin.group_size} but gate_proj uses {self.shared_group_size}; "
                "the shared-expert kernels assume one group size")
        self.invalidate()

    def _fill_shared(self, d: LayerDescT):
        if self.shared_w1_wq is None:
            raise ValueError("DeepSeek block needs its shared experts (load_shared / from_hf)")
        dev = self.shared_w1_wq.device
        nb = torch.tensor([self.shared_nbits], dtype=torch.int32, device=dev)
        zero = torch.zeros(1, dtype=torch.int32, device=dev)
        self._shared_meta = (nb, zero)
        g = self.shared_group_size
        fs = self.shared_w1_wq.shape[1]
        d.has_shared = 1
        d.shared_w1 = make_proj(self.shared_w1_wq, self.shared_w1_scales, self.shared_w1_zeros, nb, zero, zero,
                                self.hidden_dim, g)
        d.shared_w3 = make_proj(self.shared_w3_wq, self.shared_w3_scales, self.shared_w3_zeros, nb, zero, zero,
                                self.hidden_dim, g)
        d.shared_w2 = make_proj(self.shared_w2_wq, self.shared_w2_scales, self.shared_w2_zeros, nb, zero, zero, fs, g)

    def forward_single_expert(self, expert_idx: Tensor, hidden_states: Tensor, is_shared: bool = False) -> Tensor:
        """Routed expert ``expert_idx``, or the shared experts when ``is_shared``
        (moe_block.py:508-538)."""
        if is_shared:
            return self.forward_shared(hidden_states)
        return super().forward_single_expert(expert_idx, hidden_states)

    def forward_shared(self, hidden_states: Tensor) -> Tensor:
        """Shared experts alone through dequant_gemm (moe_block.py:511-522)."""
        x = hidden_states
        x1 = dequant_gemm(x, self.shared_w1_wq, self.shared_w1_scales, self.shared_w1_zeros, self.shared_nbits,
                          self.shared_group_size)
        x3 = dequant_gemm(x, self.shared_w3_wq, self.shared_w3_scales, self.shared_w3_zeros, self.shared_nbits,
                          self.shared_group_size)
        return dequant_gemm(torch.nn.functional.silu(x1) * x3, self.shared_w2_wq, self.shared_w2_scales,
                            self.shared_w2_zeros, self.shared_nbits, self.shared_group_size)
