"""Token sampling for ``generate`` (behaviour of ``demo/sampling.py:13-70``).

Greedy argmax when ``temperature`` is None or <= 0; otherwise temperature,
top-k, nucleus (top-p) filtering and multinomial sampling. A repetition
penalty divides positive / multiplies negative logits of already-seen ids.
Works on ``[V]`` or ``[B, V]`` logits (one row per sequence).
"""

from __future__ import annotations

import torch
from torch import Tensor


def sample_logits(logits: Tensor, *, temperature: float | None = None, top_k: int = 0,
                  top_p: float = 1.0, repetition_penalty: float = 1.0,
                  seen: Tensor | None = None) -> Tensor:
    x = logits.float()
    if repetition_penalty != 1.0 and seen is not None and seen.numel():
        picked = x[..., seen]
        x[..., seen] = torch.where(picked > 0, picked / repetition_penalty,
                                   picked * repetition_penalty)
    if temperature is None or temperature <= 0:
        return x.argmax(dim=-1)
    x = x / temperature
    V = x.shape[-1]
    if 0 < top_k < V:
        kth = torch.topk(x, top_k, dim=-1).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    if top_p < 1.0:
        p_sorted, idx = torch.sort(torch.softmax(x, dim=-1), descending=True, dim=-1)
        drop_sorted = (p_sorted.cumsum(-1) - p_sorted) > top_p
        drop = torch.zeros_like(drop_sorted).scatter(-1, idx, drop_sorted)
        x = x.masked_fill(drop, float("-inf"))
    return torch.multinomial(torch.softmax(x, dim=-1).reshape(-1, V), 1).reshape(x.shape[:-1])
