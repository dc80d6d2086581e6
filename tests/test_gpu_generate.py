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
