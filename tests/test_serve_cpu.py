"""Continuous-batching scheduler (host logic) against a deterministic fake model on CPU:
admission into a few slots, prompts prefilled across several steps, slot reuse, stop
tokens. The fake model's state is a hash chain over the tokens it has seen, so any
scheduling mistake (wrong slot, token dropped or repeated, state not reset) changes
the generated ids."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from rwkv_tl_b200.serve import ContinuousBatcher, Request

V = 97
MOD = 1000003


def _h(h: float, t: int) -> float:
    return float((int(h) * 31 + t + 1) % MOD)


class FakeModel:
    L, C = 1, 64

    def __init__(self):
        self.w = SimpleNamespace(device=torch.device("cpu"))
        self.prefill_rows = []

    def prefill_batch(self, seqs, state, slots):
        self.prefill_rows.append(sum(len(s) for s in seqs))
        for s, slot in zip(seqs, slots):
            h = state.rnn[0, int(slot), 0, 0, 0].item()
            for t in torch.as_tensor(s).tolist():
                h = _h(h, t)
            state.rnn[0, int(slot), 0, 0, 0] = h
        return state

    def decode_batch(self, tok, state, slots):
        logits = torch.zeros(tok.numel(), V)
        for i, (t, slot) in enumerate(zip(tok.tolist(), slots.tolist())):
            h = _h(state.rnn[0, slot, 0, 0, 0].item(), t)
            state.rnn[0, slot, 0, 0, 0] = h
            logits[i, int(h) % V] = 1.0
        return logits.half()


def _expected(prompt, n, stop=None):
    h = 0.0
    for t in prompt[:-1]:
        h = _h(h, t)
    tok, out = prompt[-1], []
    for _ in range(n):
        h = _h(h, tok)
        tok = int(h) % V
        out.append(tok)
        if tok == stop:
            break
    return out


def _requests(seed=0, n=11):
    g = torch.Generator().manual_seed(seed)
    lens = [1, 2, 5, 17, 40, 3, 64, 9, 130, 7, 1][:n]
    return [Request(i, torch.randint(0, V, (L,), generator=g), 3 + (i * 5) % 11)
            for i, L in enumerate(lens)]


@pytest.mark.parametrize("max_batch,budget", [(3, 7), (4, 64), (16, 4096)])
def test_scheduler_matches_per_request_reference(max_batch, budget):
    model = FakeModel()
    b = ContinuousBatcher(model, max_batch=max_batch, prefill_tokens=budget)
    reqs = _requests()
    for r in reqs:
        b.submit(r)
    done = b.run()
    assert sorted(r.rid for r in done) == list(range(len(reqs)))
    for r in reqs:
        assert r.output == _expected(r.prompt.tolist(), r.max_new_tokens), r.rid
    assert max(model.prefill_rows) <= budget
    assert len(b.free) == max_batch and b.idle()


def test_stop_token_ends_sequences_early():
    reqs = _requests(seed=3)
    stop = _expected(reqs[4].prompt.tolist(), reqs[4].max_new_tokens)[1]
    b = ContinuousBatcher(FakeModel(), max_batch=4, prefill_tokens=32, stop_token=stop)
    for r in reqs:
        b.submit(r)
    b.run()
    for r in reqs:
        assert r.output == _expected(r.prompt.tolist(), r.max_new_tokens, stop)
    assert len(reqs[4].output) == 2


def test_rejects_bad_requests():
    b = ContinuousBatcher(FakeModel(), max_batch=2)
    with pytest.raises(RuntimeError):
        b.submit(Request(0, torch.tensor([], dtype=torch.int64), 4))
    with pytest.raises(ValueError):
        b.submit(Request(1, torch.tensor([1, 2]), 0))
    with pytest.raises(TypeError):
        ContinuousBatcher(object())
