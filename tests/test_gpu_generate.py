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
