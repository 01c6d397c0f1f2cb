"""Token sampling for ``generate`` (behaviour of ``demo/sampling.py:13-70``).

Greedy argmax when ``temperature`` is None or <= 0; otherwise temperature,
top-k, nucleus (top-p) filtering and multinomial sampling. A repetition
penalty divides positive / multiplies negative logits of already-seen ids.
Works on ``[V]`` or ``[B, V]`` logits (one row per sequence).

CUDA logits go through one fused kernel of the CUDA library (``rwkv7_sample``:
penalty, temperature, top-k and top-p by radix selection, and the draw, with no
sort and no host synchronisation); it draws from the same distribution as the
reference, with uniforms from ``torch.rand`` (pass ``generator`` to seed them).
Logits on the CPU (the pure-torch reference's own use) are sampled with torch ops.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


def _seen_csr(seen, B: int, device) -> tuple[Tensor | None, Tensor | None]:
    """Per-row seen ids as CSR (ids int64, offsets int32). ``seen`` is one 1-D tensor
    shared by every row (the reference's form) or a list of B per-row tensors."""
    if seen is None:
        return None, None
    rows = [torch.as_tensor(s).reshape(-1) for s in seen] if isinstance(seen, (list, tuple)) \
        else [torch.as_tensor(seen).reshape(-1)] * B
    if len(rows) != B:
        raise ValueError(f"seen has {len(rows)} rows for {B} logits rows")
    lens = torch.tensor([0] + [r.numel() for r in rows], dtype=torch.int64).cumsum(0)
    ids = torch.cat([r.to(device=device, dtype=torch.int64) for r in rows]) if lens[-1] else \
        torch.zeros(1, dtype=torch.int64, device=device)
    return ids.contiguous(), lens.to(device=device, dtype=torch.int32)


def sample_logits(logits: Tensor, *, temperature: float | None = None, top_k: int = 0,
                  top_p: float = 1.0, repetition_penalty: float = 1.0,
                  seen=None, generator: torch.Generator | None = None) -> Tensor:
    if logits.is_cuda:
        return _sample_cuda(logits, temperature, top_k, top_p, repetition_penalty, seen,
                            generator)
    x = logits.float()
    if repetition_penalty != 1.0 and seen is not None and torch.as_tensor(seen).numel():
        seen = torch.as_tensor(seen)
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
    return torch.multinomial(torch.softmax(x, dim=-1).reshape(-1, V), 1,
                             generator=generator).reshape(x.shape[:-1])


def _sample_cuda(logits, temperature, top_k, top_p, repetition_penalty, seen, generator):
    lib = _lib.load()
    V = logits.shape[-1]
    x = logits.reshape(-1, V)
    if x.dtype != torch.float16 or not x.is_contiguous():
        x = x.to(torch.float16).contiguous()
    B = x.shape[0]
    t = 0.0 if temperature is None else float(temperature)
    pen = float(repetition_penalty)
    ids, cu = _seen_csr(seen, B, x.device) if pen != 1.0 else (None, None)
    u = torch.rand(B, device=x.device, generator=generator) if t > 0 else None
    out = torch.empty(B, dtype=torch.int64, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check(lib.rwkv7_sample(x.data_ptr(), B, V, t, int(top_k), float(top_p), pen,
                                _lib.ptr(ids), _lib.ptr(cu), _lib.ptr(u), out.data_ptr(), stream))
    return out.reshape(logits.shape[:-1])
