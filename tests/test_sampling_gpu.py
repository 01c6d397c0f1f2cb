"""The fused sampling kernel (``rwkv7_sample``) against the reference's rules.

``demo/sampling.py:13-70`` is restated with torch ops in ``sample_logits``'s CPU
branch; the kernel must pick the same id where the rules leave no choice (greedy,
with and without the repetition penalty; top-k = 1), never draw outside the kept
set (top-k, then nucleus), draw with the kept set's softmax probabilities, and be
bit-reproducible for fixed uniforms.
"""

from __future__ import annotations

import pytest
import torch

from rwkv_tl_b200 import _lib
from rwkv_tl_b200.sampling import sample_logits

pytestmark = pytest.mark.gpu


def _logits(B, V, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(B, V, generator=g)).half()


@pytest.mark.parametrize("V", [1024, 65536, 50000])
def test_greedy_matches_argmax_with_penalty(V):
    lg = _logits(6, V, V)
    lg[2, 100:200] = lg[2].max()  # ties: lowest id wins, like torch.argmax
    seen = torch.tensor([5, 7, 7, 150, V - 1, 3])
    for pen in (1.0, 1.3, 0.7):
        want = sample_logits(lg, repetition_penalty=pen, seen=seen)
        got = sample_logits(lg.cuda(), repetition_penalty=pen, seen=seen.cuda())
        assert torch.equal(got.cpu(), want)
    assert int(sample_logits(lg[2].cuda())) == int(lg[2].float().argmax())


def test_top_k_one_is_greedy():
    lg = _logits(8, 65536, 1)
    got = sample_logits(lg.cuda(), temperature=0.7, top_k=1)
    assert torch.equal(got.cpu(), lg.float().argmax(-1))


def _kept(row, temperature, top_k, top_p):
    """Kept ids and their probabilities under the reference's rules (float64)."""
    x = row.double() / temperature
    V = x.numel()
    if 0 < top_k < V:
        kth = torch.topk(x, top_k).values[-1]
        x = torch.where(x >= kth, x, torch.full_like(x, float("-inf")))
    if top_p < 1.0:
        p = torch.softmax(x, -1)
        ps, idx = torch.sort(p, descending=True)
        drop = (ps.cumsum(0) - ps) > top_p
        x[idx[drop]] = float("-inf")
    p = torch.softmax(x, -1)
    return p


@pytest.mark.parametrize("T,k,p", [(1.0, 0, 0.9), (0.8, 50, 1.0), (1.3, 200, 0.7), (1.0, 0, 1.0)])
def test_draws_stay_in_the_kept_set_with_its_probabilities(T, k, p):
    V, N = 4096, 20000
    row = _logits(1, V, 3, scale=2.0)[0]
    want = _kept(row, T, k, p)
    g = torch.Generator(device="cuda").manual_seed(11)
    ids = sample_logits(row.cuda().expand(N, V).contiguous(), temperature=T, top_k=k, top_p=p,
                        generator=g).cpu()
    assert bool((want[ids] > 0).all()), "a draw fell outside the kept set"
    freq = torch.bincount(ids, minlength=V).double() / N
    sigma = (want * (1 - want) / N).sqrt()
    assert float(((freq - want).abs() - 5 * sigma).max()) <= 1.0 / N
    # the same uniforms give the same ids
    g2 = torch.Generator(device="cuda").manual_seed(11)
    again = sample_logits(row.cuda().expand(N, V).contiguous(), temperature=T, top_k=k,
                          top_p=p, generator=g2).cpu()
    assert torch.equal(ids, again)


def test_per_row_seen_lists_and_bad_arguments():
    lg = _logits(3, 1024, 9)
    seen = [torch.tensor([int(lg[0].float().argmax())]), torch.tensor([], dtype=torch.long),
            torch.tensor([1, 2])]
    got = sample_logits(lg.cuda(), repetition_penalty=50.0, seen=seen).cpu()
    for b in range(3):
        assert int(got[b]) == int(sample_logits(lg[b], repetition_penalty=50.0, seen=seen[b]))
    lib = _lib.load()
    assert lib.rwkv7_sample(None, 1, 1024, 0.0, 0, 1.0, 1.0, None, None, None, None,
                            None) == _lib.RWKV_ERR_ARG
    x = torch.zeros(1, 65544, dtype=torch.float16, device="cuda")
    out = torch.empty(1, dtype=torch.int64, device="cuda")
    assert lib.rwkv7_sample(x.data_ptr(), 1, 65544, 0.0, 0, 1.0, 1.0, None, None, None,
                            out.data_ptr(), None) == _lib.RWKV_ERR_ARG
