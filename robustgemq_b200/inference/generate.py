"""Whole-model decode on this library's blocks: the generate loop of
gemq/benchmark_generate.py:113-156 with a static KV cache and the decode step
captured once in a CUDA graph (the reference compiles ``decode_one_token`` with
``torch.compile(mode="reduce-overhead", fullgraph=True)``, benchmark_generate.py:180-182,
which replays CUDA graphs the same way).

``synthetic_olmoe`` builds an OLMoE-1B-7B-shaped ``OlmoeForCausalLM`` (transformers'
own modelling code) with seeded random weights. No checkpoint is available here. Its MoE
blocks are ``QuantFusedOlmoeMoEBlock`` with packed experts (the config's bit mix),
and its attention projections are 4-bit ``QuantLinear`` layers (the reference's
GemLite 4-bit attention). Embeddings and the LM head stay fp16; the RMSNorms run in
one launch each (``RMSNormF16``, this library's ``gemq_rms_norm``).
``StaticDecoder`` prefills a prompt eagerly and then decodes greedily, one CUDA graph
replay per token.
"""

from __future__ import annotations

import time
from typing import Optional

import torch
from torch import Tensor, nn

from .. import _lib, synth
from ..quant import rtn_quantize
from .linear import QuantLinear
from .moe_block import QuantFusedOlmoeMoEBlock


class MoEAdapter(nn.Module):
    """A fused block as a decoder layer's ``mlp``: returns the hidden states alone.
    transformers 5.x decoder layers expect a tensor; the reference's blocks return
    ``(out, router_logits)`` for the 4.x layers (moe_block.py:815, 853)."""

    def __init__(self, block: nn.Module):
        super().__init__()
        self.block = block

    def forward(self, hidden_states: Tensor) -> Tensor:
        out = self.block(hidden_states)
        return out[0] if isinstance(out, tuple) else out


class RMSNormF16(nn.Module):
    """transformers' OlmoeRMSNorm on fp16 rows in one launch (``gemq_rms_norm``):
    ``weight * fp16(x * rsqrt(mean(x^2) + eps))`` with x in fp32, where the eager module
    runs six element-wise and reduction kernels. The sum of squares is reduced in
    another order than torch's, so a result can differ from the eager module's by one
    fp16 ulp."""

    def __init__(self, weight: Tensor, eps: float):
        super().__init__()
        self.weight = nn.Parameter(weight.detach().to(torch.float16).contiguous(), requires_grad=False)
        self.variance_epsilon = float(eps)

    def forward(self, hidden_states: Tensor) -> Tensor:
        n = hidden_states.shape[-1]
        x = hidden_states.reshape(-1, n).contiguous()
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("RMSNormF16 takes fp16 CUDA tensors")
        out = torch.empty_like(x)
        _lib.check(_lib.load().gemq_rms_norm(_lib.ptr(x), _lib.ptr(self.weight), x.shape[0], n, self.variance_epsilon,
                                             _lib.ptr(out), _lib.stream_ptr(x.device)))
        return out.reshape(hidden_states.shape)


def _fused_norm(norm: nn.Module) -> RMSNormF16:
    return RMSNormF16(norm.weight, norm.variance_epsilon)


def _rand_w(out_f: int, in_f: int, gen: torch.Generator, device) -> Tensor:
    return (torch.randn((out_f, in_f), generator=gen, device=device) * 0.02).half()


def _quant_from_w(W: Tensor, nbits: int, group_size: int) -> QuantLinear:
    # RTN groups run along the input dim of each output row, so quantising stacked
    # weights row-wise equals quantising each part alone
    Q, s, z = rtn_quantize(W, nbits, group_size)
    return QuantLinear(nbits, group_size, W.shape[1], W.shape[0]).pack(Q, s, z)


class FusedOlmoeAttention(nn.Module):
    """transformers' OlmoeAttention (``modeling_olmoe.OlmoeAttention.forward``) with
    q, k and v from one 4-bit projection (one GEMV) and its prologue, q_norm / k_norm
    and the rotary embedding, in one launch (``gemq_qk_norm_rope``). For one token of
    one sequence it also writes k and v into a transformers static cache, advancing
    its length, and the attention over the cache's written positions runs in one more
    launch (``gemq_decode_attention``; the causal mask of such a step hides exactly the
    unwritten positions, so no padding mask is taken). Otherwise the cache's update and
    the model's ``_attn_implementation`` run. o_proj is the module's own. ``attn`` is the replaced module, kept for its configuration."""

    def __init__(self, attn: nn.Module, qkv_proj: QuantLinear):
        super().__init__()
        if getattr(attn.config, "clip_qkv", None) is not None:
            raise ValueError("clip_qkv is not supported by the fused attention prologue")
        self.config = attn.config
        self.layer_idx = attn.layer_idx
        self.head_dim = attn.head_dim
        self.scaling = attn.scaling
        self.is_causal = True
        self.num_key_value_groups = attn.num_key_value_groups
        self.attention_dropout = attn.attention_dropout
        self.qkv_proj = qkv_proj
        self.o_proj = attn.o_proj
        self.q_norm_weight = nn.Parameter(attn.q_norm.weight.detach().half().contiguous(), requires_grad=False)
        self.k_norm_weight = nn.Parameter(attn.k_norm.weight.detach().half().contiguous(), requires_grad=False)
        self.eps = float(attn.q_norm.variance_epsilon)
        if float(attn.k_norm.variance_epsilon) != self.eps:
            raise ValueError("q_norm and k_norm must share eps")

    def _static_layer(self, cache, rows: int, qkv: Tensor):
        """The cache layer to write directly: one token, batch 1, an initialised
        transformers ``StaticLayer`` with contiguous fp16 keys / values and an int64
        device length; else None (the cache's own update runs)."""
        if cache is None or rows != 1 or qkv.shape[0] != 1:
            return None
        layers = getattr(cache, "layers", None)
        if layers is None or self.layer_idx >= len(layers):
            return None
        layer = layers[self.layer_idx]
        if type(layer).__name__ != "StaticLayer" or not getattr(layer, "is_initialized", False):
            return None
        keys, values, length = layer.keys, layer.values, getattr(layer, "cumulative_length", None)
        if not (isinstance(length, Tensor) and length.dtype == torch.int64 and length.is_cuda and length.numel() == 1):
            return None
        ok = all(t.dtype == torch.float16 and t.is_contiguous() and t.dim() == 4 and t.shape[0] == 1 and
                 t.shape[-1] == self.head_dim for t in (keys, values))
        return layer if ok else None

    def forward(self, hidden_states: Tensor, position_embeddings, attention_mask, past_key_values=None, **kwargs):
        from transformers.models.olmoe.modeling_olmoe import ALL_ATTENTION_FUNCTIONS, eager_attention_forward

        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        qkv = self.qkv_proj(hidden_states)  # [..., 3 D]
        n = qkv.shape[-1] // 3
        rows = qkv.numel() // qkv.shape[-1]
        cos, sin = position_embeddings
        cos = cos.to(torch.float16).contiguous()
        sin = sin.to(torch.float16).contiguous()
        if cos.numel() != rows * self.head_dim:
            raise ValueError("rotary tables must have one row per token")
        q = torch.empty((*input_shape, n), dtype=torch.float16, device=qkv.device)
        ld = qkv.stride(-2) if qkv.dim() > 1 else 3 * n
        layer = self._static_layer(past_key_values, rows, qkv)
        if layer is not None:
            # one token: k and v straight into the static cache at its device-side
            # length, which the kernel advances (the cache's own update, in this launch)
            _lib.check(_lib.load().gemq_qk_norm_rope(
                _lib.ptr(qkv), ld, rows, n, self.head_dim, _lib.ptr(self.q_norm_weight), _lib.ptr(self.k_norm_weight),
                self.eps, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(q), None, _lib.ptr(layer.keys),
                _lib.ptr(layer.values), layer.keys.shape[2], _lib.ptr(layer.cumulative_length),
                _lib.stream_ptr(qkv.device)))
            if self.num_key_value_groups == 1:
                # one query token over the cache's written positions (the causal mask
                # of a one-token step of one sequence), in one launch
                attn = torch.empty_like(q)
                _lib.check(_lib.load().gemq_decode_attention(
                    _lib.ptr(q), _lib.ptr(layer.keys), _lib.ptr(layer.values), n // self.head_dim,
                    layer.keys.shape[2], self.head_dim, _lib.ptr(layer.cumulative_length), float(self.scaling),
                    _lib.ptr(attn), _lib.stream_ptr(qkv.device)))
                return self.o_proj(attn), None
            key_states, value_states = layer.keys, layer.values
        else:
            k = torch.empty_like(q)
            _lib.check(_lib.load().gemq_qk_norm_rope(
                _lib.ptr(qkv), ld, rows, n, self.head_dim, _lib.ptr(self.q_norm_weight), _lib.ptr(self.k_norm_weight),
                self.eps, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(q), _lib.ptr(k), None, None, 0, None,
                _lib.stream_ptr(qkv.device)))
            key_states = k.view(hidden_shape).transpose(1, 2)
            value_states = qkv[..., 2 * n:].view(hidden_shape).transpose(1, 2)
            if past_key_values is not None:
                key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx)
        query_states = q.view(hidden_shape).transpose(1, 2)
        attention_interface = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation,
                                                                    eager_attention_forward)
        attn_output, attn_weights = attention_interface(
            self, query_states, key_states, value_states, attention_mask, dropout=0.0, scaling=self.scaling,
            sliding_window=getattr(self.config, "sliding_window", None), **kwargs)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return self.o_proj(attn_output), attn_weights


def synthetic_olmoe(num_layers: int = 16, device="cuda", seed: int = 0, attn_bits: int = 4,
                    attn_group: int = 64, max_position_embeddings: int = 4096, blocks=None,
                    fused_norms: bool = True, fused_attention: bool = True):
    """OLMoE-1B-7B-shaped causal LM (hidden 2048, 16 heads, 64 experts top-8,
    intermediate 1024, vocab 50304) with seeded random weights, MoE blocks of this
    library (``blocks``: already built ``QuantFusedOlmoeMoEBlock`` layers to use, one
    per decoder layer), ``attn_bits``-bit attention projections, (``fused_norms``) the
    RMSNorms in one launch each (``RMSNormF16``) and (``fused_attention``) the attention
    as ``FusedOlmoeAttention``. The random weights do not depend on the two flags."""
    from transformers import OlmoeConfig, OlmoeForCausalLM
    from transformers.models.olmoe.modeling_olmoe import OlmoeRotaryEmbedding

    device = torch.device(device)
    cfg = OlmoeConfig(hidden_size=2048, intermediate_size=1024, num_hidden_layers=num_layers, num_attention_heads=16,
                      num_key_value_heads=16, num_experts=64, num_experts_per_tok=8, norm_topk_prob=False,
                      vocab_size=50304, max_position_embeddings=max_position_embeddings)
    cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = OlmoeForCausalLM(cfg)
    for layer in model.model.layers:  # experts are never materialised in fp16
        layer.mlp = nn.Module()
    model.to_empty(device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=gen, device=device) * 0.02)
    model.half()
    model.model.rotary_emb = OlmoeRotaryEmbedding(config=cfg, device=device)  # fp32 inverse frequencies
    moe_cfg, shp = synth.olmoe_config()
    D = cfg.hidden_size
    for l, layer in enumerate(model.model.layers):
        if blocks is not None:
            blk = blocks[l]
        else:
            blk = synth.random_block(QuantFusedOlmoeMoEBlock, moe_cfg, shp["hidden"], shp["inter"],
                                     shp["num_experts"], shp["mean_bits"], shp["group_size"], seed * 1000 + l, device)
        layer.mlp = MoEAdapter(blk)
        att = layer.self_attn
        wq, wk, wv, wo = (_rand_w(D, D, gen, device) for _ in range(4))
        att.o_proj = _quant_from_w(wo, attn_bits, attn_group)
        if fused_attention:
            layer.self_attn = FusedOlmoeAttention(att, _quant_from_w(torch.cat([wq, wk, wv]), attn_bits, attn_group))
        else:
            att.q_proj = _quant_from_w(wq, attn_bits, attn_group)
            att.k_proj = _quant_from_w(wk, attn_bits, attn_group)
            att.v_proj = _quant_from_w(wv, attn_bits, attn_group)
        if fused_norms:
            layer.input_layernorm = _fused_norm(layer.input_layernorm)
            layer.post_attention_layernorm = _fused_norm(layer.post_attention_layernorm)
            if not fused_attention:
                att.q_norm = _fused_norm(att.q_norm)
                att.k_norm = _fused_norm(att.k_norm)
    if fused_norms:
        model.model.norm = _fused_norm(model.model.norm)
    model.eval()
    return model


class StaticDecoder:
    """Greedy generation with a static KV cache; the decode step is one CUDA graph."""

    def __init__(self, model, max_cache_len: int):
        from transformers import StaticCache

        self.model = model
        self.device = next(model.parameters()).device
        self.cache = StaticCache(config=model.config, max_cache_len=max_cache_len)
        self.max_cache_len = max_cache_len
        self.static_ids = torch.zeros((1, 1), dtype=torch.long, device=self.device)
        self.static_pos = torch.zeros((1,), dtype=torch.long, device=self.device)
        self.static_next = None
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    @torch.no_grad()
    def _step(self):
        out = self.model(input_ids=self.static_ids, past_key_values=self.cache, cache_position=self.static_pos,
                         use_cache=True)
        return out.logits[:, -1].argmax(dim=-1, keepdim=True)

    @torch.no_grad()
    def prefill(self, prompt: Tensor) -> Tensor:
        T = prompt.shape[-1]
        pos = torch.arange(T, device=self.device)
        out = self.model(input_ids=prompt.view(1, -1), past_key_values=self.cache, cache_position=pos, use_cache=True)
        return out.logits[:, -1].argmax(dim=-1, keepdim=True)

    @torch.no_grad()
    def capture(self, prompt_len: int):
        """Capture the decode step (after a prefill, so the cache is allocated)."""
        self.static_pos.fill_(prompt_len)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up: workspaces, cuBLAS handles
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.static_next = self._step()
        self.graph = g

    @torch.no_grad()
    def generate(self, prompt: Tensor, max_new_tokens: int):
        """Greedy tokens after ``prompt`` ([T] int64) and timing stats (prefill and
        decode tokens/s, as benchmark_generate.py reports them)."""
        T = prompt.shape[-1]
        if T + max_new_tokens > self.max_cache_len:
            raise ValueError("prompt + new tokens exceed the cache length")
        self.cache.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        nxt = self.prefill(prompt)
        torch.cuda.synchronize()
        t_prefill = time.perf_counter() - t0
        if self.graph is None:
            self.capture(T)
            self.cache.reset()
            nxt = self.prefill(prompt)
        tokens = [nxt.view(-1)]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(max_new_tokens - 1):
            self.static_ids.copy_(tokens[-1].view(1, 1))
            self.static_pos.fill_(T + i)
            self.graph.replay()
            tokens.append(self.static_next.view(-1).clone())
        torch.cuda.synchronize()
        t_decode = time.perf_counter() - t0
        seq = torch.cat([prompt.view(-1), torch.cat(tokens)])
        stats = {"prefill_latency_s": t_prefill, "prefill_tokens_per_s": T / t_prefill,
                 "decode_latency_s": t_decode, "decode_tokens_per_s": (max_new_tokens - 1) / t_decode}
        return seq, stats
