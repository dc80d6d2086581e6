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


def _quant_linear(out_f: int, in_f: int, nbits: int, group_size: int, gen: torch.Generator, device) -> QuantLinear:
    W = (torch.randn((out_f, in_f), generator=gen, device=device) * 0.02).half()
    Q, s, z = rtn_quantize(W, nbits, group_size)
    return QuantLinear(nbits, group_size, in_f, out_f).pack(Q, s, z)


def synthetic_olmoe(num_layers: int = 16, device="cuda", seed: int = 0, attn_bits: int = 4,
                    attn_group: int = 64, max_position_embeddings: int = 4096, blocks=None,
                    fused_norms: bool = True):
    """OLMoE-1B-7B-shaped causal LM (hidden 2048, 16 heads, 64 experts top-8,
    intermediate 1024, vocab 50304) with seeded random weights, MoE blocks of this
    library (``blocks``: already built ``QuantFusedOlmoeMoEBlock`` layers to use, one
    per decoder layer), ``attn_bits``-bit attention projections, and (``fused_norms``)
    the RMSNorms in one launch each (``RMSNormF16``)."""
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
        for pname in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(att, pname, _quant_linear(D, D, attn_bits, attn_group, gen, device))
        if fused_norms:
            layer.input_layernorm = _fused_norm(layer.input_layernorm)
            layer.post_attention_layernorm = _fused_norm(layer.post_attention_layernorm)
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
