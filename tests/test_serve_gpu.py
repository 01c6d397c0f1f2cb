"""Continuous batching on the real model: requests admitted into 4 slots, prompts
prefilled in 48-token varlen chunks across steps, decode batches of 1..4 sequences,
against running each request alone through ``generate`` (greedy)."""

from __future__ import annotations

import pytest
import torch

from rwkv_tl_b200 import ContinuousBatcher, Request, RWKV7Weight, State, make_rwkv7
from rwkv_tl_b200.synth import ModelConfig, synth_checkpoint

pytestmark = pytest.mark.gpu


def test_continuous_batching_matches_sequential_generate():
    cfg = ModelConfig(n_layer=2, n_embd=768, vocab=4096)
    dev = torch.device("cuda")
    w = RWKV7Weight(synth_checkpoint(cfg, seed=5, device=dev), device=dev)
    m = make_rwkv7(dev, backend="b200", use_graph=False)(w)
    g = torch.Generator().manual_seed(7)
    lens = [1, 2, 5, 17, 40, 3, 64, 9, 130, 7]
    reqs = [Request(i, torch.randint(0, cfg.vocab, (L,), generator=g), 3 + (i * 5) % 11)
            for i, L in enumerate(lens)]
    b = ContinuousBatcher(m, max_batch=4, prefill_tokens=48)
    for r in reqs:
        b.submit(r)
    done = b.run()
    assert sorted(r.rid for r in done) == list(range(len(reqs)))
    agree = total = 0
    for r in reqs:
        ref, _ = m.generate(r.prompt.to(dev), State(w.L, w.C, 64, device=dev), r.max_new_tokens)
        assert len(r.output) == r.max_new_tokens
        if r.output[0] != ref[0]:
            # same state -> same first greedy token, up to a near-tie: small-batch decode sums
            # with float atomics, so its last fp32 bits vary from run to run
            lg, _ = m.forward(r.prompt.to(dev), State(w.L, w.C, 64, device=dev))
            lg = lg.float()
            gap = abs(float(lg[ref[0]] - lg[r.output[0]]))
            assert gap <= 2e-3 * float(lg.abs().max()), (r.rid, gap)
        agree += sum(a == c for a, c in zip(r.output, ref))
        total += len(ref)
    # prefill split at other chunk boundaries rounds differently in fp32; a near-tie
    # can flip one greedy id, after which the two continuations differ
    assert agree >= 0.9 * total, (agree, total)
    from rwkv_tl_b200 import _lib

    assert _lib.load().rwkv_b200_device_error() == 0
