"""Whole-model decode (``inference/generate.py``): an OLMoE-shaped transformers model
on this library's MoE blocks and 4-bit attention linears, decoded from a static KV
cache with the step captured in a CUDA graph (gemq/benchmark_generate.py:113-156,
180-182). The graph replays must give the tokens an eager step-by-step decode gives."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graph_decode_matches_eager_decode(cuda_device):
    from robustgemq_b200 import _lib
    from robustgemq_b200.inference.generate import StaticDecoder, synthetic_olmoe

    model = synthetic_olmoe(num_layers=2, seed=3, max_position_embeddings=64)
    prompt = torch.randint(0, model.config.vocab_size, (9,), generator=torch.Generator().manual_seed(0)).cuda()
    new = 12
    dec = StaticDecoder(model, max_cache_len=32)
    seq, stats = dec.generate(prompt, new)
    assert seq.shape == (9 + new,)
    assert stats["decode_tokens_per_s"] > 0
    # eager: the same greedy steps without the graph
    eager = StaticDecoder(model, max_cache_len=32)
    with torch.no_grad():
        nxt = eager.prefill(prompt)
        toks = [nxt.view(-1)]
        for i in range(new - 1):
            eager.static_ids.copy_(toks[-1].view(1, 1))
            eager.static_pos.fill_(9 + i)
            toks.append(eager._step().view(-1).clone())
    assert torch.equal(seq[9:], torch.cat(toks))
    # a second generate replays the captured graph from a reset cache
    seq2, _ = dec.generate(prompt, new)
    assert torch.equal(seq2, seq)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("rows", [1, 9, 64])
def test_fused_rms_norm_matches_transformers(cuda_device, rows):
    """``RMSNormF16`` (one launch) against transformers' OlmoeRMSNorm on the same
    fp16 rows and random weights. The sums of squares are reduced in different
    orders, so the normalised value fp16(x * rsqrt(.)) may differ by one fp16 ulp;
    after the multiply by the weight and its rounding that is at most |w| times that
    ulp plus one ulp of the output, about two output ulps."""
    from transformers.models.olmoe.modeling_olmoe import OlmoeRMSNorm

    from robustgemq_b200.inference.generate import RMSNormF16

    g = torch.Generator(device="cuda").manual_seed(rows)
    x = (torch.randn((rows, 2048), generator=g, device="cuda") * 3).half()
    ref = OlmoeRMSNorm(2048, eps=1e-5).cuda().half()
    with torch.no_grad():
        ref.weight.copy_(torch.rand((2048,), generator=g, device="cuda") * 2 - 0.5)
        y_ref = ref(x)
    y = RMSNormF16(ref.weight, ref.variance_epsilon)(x)
    torch.cuda.synchronize()
    assert y.shape == y_ref.shape and y.dtype == torch.float16
    ulp = torch.finfo(torch.float16).eps * y_ref.float().abs().clamp_min(2.0 ** -14)
    assert ((y.float() - y_ref.float()).abs() <= 2 * ulp).all()
    mismatched = (y != y_ref).float().mean().item()
    assert mismatched < 0.01


@pytest.mark.parametrize("rows", [1, 9])
def test_fused_qk_norm_rope_matches_transformers(cuda_device, rows):
    """``gemq_qk_norm_rope`` against transformers' q_norm / k_norm (OlmoeRMSNorm) and
    apply_rotary_pos_emb on the same fp16 rows, random norm weights and the model's
    own rotary tables. The norm may differ by about two fp16 ulps (see above); the
    rotation adds and rounds two such values, which may nearly cancel, so the bound is
    four ulps of the result plus a small absolute term (a quarter ulp of the largest
    value)."""
    from transformers import OlmoeConfig
    from transformers.models.olmoe.modeling_olmoe import OlmoeRMSNorm, OlmoeRotaryEmbedding, apply_rotary_pos_emb

    from robustgemq_b200 import _lib

    D, H, hd = 2048, 16, 128
    g = torch.Generator(device="cuda").manual_seed(10 + rows)
    qkv = (torch.randn((1, rows, 3 * D), generator=g, device="cuda") * 2).half()
    qn, kn = OlmoeRMSNorm(D).cuda().half(), OlmoeRMSNorm(D).cuda().half()
    with torch.no_grad():
        qn.weight.copy_(torch.rand((D,), generator=g, device="cuda") + 0.5)
        kn.weight.copy_(torch.rand((D,), generator=g, device="cuda") + 0.5)
        cfg = OlmoeConfig(hidden_size=D, num_attention_heads=H, num_key_value_heads=H, max_position_embeddings=64)
        rope = OlmoeRotaryEmbedding(config=cfg, device="cuda")
        pos = torch.arange(5, 5 + rows, device="cuda").view(1, -1)
        cos, sin = rope(qkv, pos)
        q_ref = qn(qkv[..., :D]).view(1, rows, H, hd).transpose(1, 2)
        k_ref = kn(qkv[..., D:2 * D]).view(1, rows, H, hd).transpose(1, 2)
        q_ref, k_ref = apply_rotary_pos_emb(q_ref, k_ref, cos, sin)
    q = torch.empty((rows, D), dtype=torch.float16, device="cuda")
    k = torch.empty_like(q)
    cos16, sin16 = cos.half().contiguous(), sin.half().contiguous()
    _lib.check(_lib.load().gemq_qk_norm_rope(_lib.ptr(qkv), 3 * D, rows, D, hd, _lib.ptr(qn.weight.data),
                                             _lib.ptr(kn.weight.data), qn.variance_epsilon, _lib.ptr(cos16),
                                             _lib.ptr(sin16), _lib.ptr(q), _lib.ptr(k), None, None, 0, None,
                                             _lib.stream_ptr(q.device)))
    torch.cuda.synchronize()
    for got, ref in ((q, q_ref), (k, k_ref)):
        ref = ref.transpose(1, 2).reshape(rows, D).float()
        ulp = torch.finfo(torch.float16).eps * ref.abs().clamp_min(2.0 ** -14)
        err = (got.float() - ref).abs()
        assert (err <= 4 * ulp + 4 * torch.finfo(torch.float16).eps * ref.abs().max() * 2.0 ** -4).all()
        assert (got != ref.half()).float().mean().item() < 0.02


def test_fused_attention_model_matches_unfused(cuda_device):
    """The same synthetic weights with transformers' attention (separate 4-bit q / k /
    v projections, norms, rotary and static-cache update) and with
    ``FusedOlmoeAttention``: the last-token logits of a prompt, and of one decode step
    after it (the fused kernel writing the cache), agree to rounding (the projections'
    split-K sums and the norms' reductions run in another order)."""
    from conftest import rel_l2

    from robustgemq_b200.inference.generate import synthetic_olmoe

    from transformers import StaticCache

    prompt = torch.randint(0, 50304, (1, 9), generator=torch.Generator().manual_seed(1)).cuda()
    nxt = torch.tensor([[123]], device="cuda")
    outs, steps = [], []
    for fused in (False, True):
        model = synthetic_olmoe(num_layers=2, seed=5, max_position_embeddings=64, fused_norms=fused,
                                fused_attention=fused)
        with torch.no_grad():
            outs.append(model(input_ids=prompt).logits[0, -1].float().cpu().numpy())
            # prefill into a static cache (its own update), then one token, whose k / v
            # the fused kernel writes into the cache itself
            cache = StaticCache(config=model.config, max_cache_len=32)
            model(input_ids=prompt, past_key_values=cache, cache_position=torch.arange(9, device="cuda"),
                  use_cache=True)
            step = model(input_ids=nxt, past_key_values=cache, cache_position=torch.tensor([9], device="cuda"),
                         use_cache=True)
            steps.append(step.logits[0, -1].float().cpu().numpy())
            assert int(cache.layers[0].cumulative_length.item()) == 10
        del model, cache
    assert rel_l2(outs[1], outs[0]) <= 5e-3
    assert rel_l2(steps[1], steps[0]) <= 5e-3


@pytest.mark.parametrize("length", [1, 9, 73])
def test_decode_attention_matches_fp32_reference(cuda_device, length):
    """``gemq_decode_attention`` against softmax(scale q K^T) V in fp32 over the first
    ``length`` cache positions; the positions after them hold garbage that must not be
    read. One fp16 rounding of an fp32 result: within 2e-3 relative."""
    from conftest import rel_l2

    from robustgemq_b200 import _lib

    H, hd, max_len = 16, 128, 73
    g = torch.Generator(device="cuda").manual_seed(length)
    q = torch.randn((H, hd), generator=g, device="cuda").half()
    kc = torch.randn((H, max_len, hd), generator=g, device="cuda").half()
    vc = torch.randn((H, max_len, hd), generator=g, device="cuda").half()
    kc[:, length:] = 1e4  # unwritten positions
    vc[:, length:] = float("nan")
    cache_len = torch.tensor([length], dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    scale = hd ** -0.5
    _lib.check(_lib.load().gemq_decode_attention(_lib.ptr(q), _lib.ptr(kc), _lib.ptr(vc), H, max_len, hd,
                                                 _lib.ptr(cache_len), scale, _lib.ptr(out), _lib.stream_ptr(q.device)))
    k, v = kc[:, :length].float(), vc[:, :length].float()
    p = torch.softmax(torch.einsum("hd,hjd->hj", q.float(), k) * scale, dim=-1)
    ref = torch.einsum("hj,hjd->hd", p, v)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) <= 2e-3
