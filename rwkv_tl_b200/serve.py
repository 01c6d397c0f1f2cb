"""Continuous batching over the B200 model: a scheduler that admits new sequences
into free state slots, prefills their prompts in varlen chunks and advances every
active sequence by one token per step.

The reference has no batched engine (its ``RWKV7Model`` serves one sequence per call,
``demo/_rwkv7_abc.py:21-89``); this mixes the reference's two per-sequence calls the
way ``forward`` does (``demo/_rwkv7_abc.py:74-89``): a prompt's tokens except the last
go through ``prefill`` (prefill rounding), the last prompt token and every generated
token through ``decode`` (decode rounding). One scheduler step is

1. admit waiting requests into free slots (their state rows are zeroed);
2. one varlen prefill call over the admitted prompts, at most ``prefill_tokens`` rows
   (long prompts continue in later steps);
3. one batched decode call over every sequence whose prompt is done, greedy (or
   sampled) next tokens written on the device.

Generated tokens stay on the device until a sequence finishes; the host only keeps
counts, so a step needs no device->host synchronisation unless ``stop_token`` is set.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import torch
from torch import Tensor

from .model import RWKV7B200
from .sampling import sample_logits
from .state import BatchedState

__all__ = ["Request", "ContinuousBatcher"]


@dataclass
class Request:
    """A prompt (1-D token ids, at least one) and how many tokens to generate."""

    rid: int
    prompt: Tensor
    max_new_tokens: int
    output: list[int] = field(default_factory=list)


class ContinuousBatcher:
    """Runs ``Request``s to completion, ``max_batch`` at a time.

    ``model`` is an eager ``RWKV7B200`` (a CUDA-graph wrapper is unwrapped: batch
    shapes change from step to step) or any object with the same ``L``, ``C``, ``w``,
    ``prefill_batch`` and ``decode_batch``. ``sampling`` is passed to
    ``sample_logits`` (default greedy).
    """

    def __init__(self, model: RWKV7B200, max_batch: int = 256, prefill_tokens: int = 4096,
                 stop_token: int | None = None, **sampling) -> None:
        if not isinstance(model, RWKV7B200) and isinstance(getattr(model, "model", None), RWKV7B200):
            model = model.model  # unwrap a CUDAGraph wrapper
        if not all(hasattr(model, a) for a in ("L", "C", "w", "prefill_batch", "decode_batch")):
            raise TypeError("ContinuousBatcher needs an RWKV7B200-like model")
        self.model = model
        self.dev = model.w.device
        self.max_batch = max_batch
        self.prefill_tokens = prefill_tokens
        self.stop_token = stop_token
        self.sampling = sampling
        t = sampling.get("temperature")
        # greedy decoding goes through the fused greedy head when the model has one
        self._greedy = ((t is None or t <= 0) and sampling.get("repetition_penalty", 1.0) == 1.0
                        and hasattr(model, "decode_batch_greedy"))
        self.state = BatchedState(model.L, model.C, max_batch, device=self.dev)
        self.free = deque(range(max_batch))
        self.waiting: deque[Request] = deque()
        self.prefilling: dict[int, tuple[Request, int]] = {}  # slot -> (request, tokens done)
        self.decoding: dict[int, Request] = {}                 # slot -> request
        self.next_tok = torch.zeros(max_batch, dtype=torch.int64, device=self.dev)
        self.gen = torch.zeros(max_batch, dtype=torch.int64, device=self.dev)  # counts
        self.out = torch.zeros(max_batch, 1, dtype=torch.int64, device=self.dev)  # ids
        self.n_gen: dict[int, int] = {}
        self.done: list[Request] = []
        self.steps = 0

    # ------------------------------------------------------------------ #
    def submit(self, req: Request) -> None:
        p = torch.as_tensor(req.prompt).reshape(-1)
        if p.numel() == 0:
            raise RuntimeError("prefill received an empty token sequence")
        if req.max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        req.prompt = p.to(torch.int64)
        if req.max_new_tokens > self.out.shape[1]:  # widen the on-device output rows
            wider = torch.zeros(self.max_batch, req.max_new_tokens, dtype=torch.int64,
                                device=self.dev)
            wider[:, : self.out.shape[1]] = self.out
            self.out = wider
        self.waiting.append(req)

    def idle(self) -> bool:
        return not (self.waiting or self.prefilling or self.decoding)

    def run(self) -> list[Request]:
        while not self.idle():
            self.step()
        return self.done

    # ------------------------------------------------------------------ #
    def _admit(self) -> None:
        st = self.state
        while self.waiting and self.free:
            req = self.waiting.popleft()
            slot = self.free.popleft()
            st.rnn[:, slot].zero_()
            st.tmix_x[:, slot].zero_()
            st.cmix_x[:, slot].zero_()
            self.gen[slot] = 0
            self.n_gen[slot] = 0
            if req.prompt.numel() == 1:  # nothing to prefill: the token is decoded directly
                self.next_tok[slot] = int(req.prompt[0])
                self.decoding[slot] = req
            else:
                self.prefilling[slot] = (req, 0)

    def _prefill(self) -> None:
        budget = self.prefill_tokens
        seqs, slots, finished = [], [], []
        for slot, (req, off) in list(self.prefilling.items()):
            if budget <= 0:
                break
            total = req.prompt.numel() - 1  # the last prompt token is decoded
            take = min(total - off, budget)
            seqs.append(req.prompt[off:off + take])
            slots.append(slot)
            budget -= take
            if off + take == total:
                finished.append(slot)
            else:
                self.prefilling[slot] = (req, off + take)
        if seqs:
            self.model.prefill_batch(seqs, self.state, slots)
        for slot in finished:
            req, _ = self.prefilling.pop(slot)
            self.next_tok[slot] = int(req.prompt[-1])
            self.decoding[slot] = req

    def _decode(self) -> None:
        if not self.decoding:
            return
        slots = list(self.decoding)
        sl = torch.tensor(slots, dtype=torch.int64).to(self.dev, non_blocking=True)
        tok = self.next_tok.index_select(0, sl)
        if self._greedy:
            nxt = self.model.decode_batch_greedy(tok, self.state, sl.to(torch.int32))
        else:
            logits = self.model.decode_batch(tok, self.state, sl.to(torch.int32))
            nxt = sample_logits(logits, **self.sampling).to(torch.int64)
        self.next_tok.index_copy_(0, sl, nxt)
        self.out.index_put_((sl, self.gen.index_select(0, sl)), nxt)
        self.gen.index_add_(0, sl, torch.ones_like(sl))
        stopped = set()
        if self.stop_token is not None:  # the one per-step device -> host read
            stopped = {slots[i] for i in torch.nonzero(nxt == self.stop_token).flatten().tolist()}
        finished = []
        for slot in slots:
            self.n_gen[slot] += 1
            if self.n_gen[slot] == self.decoding[slot].max_new_tokens or slot in stopped:
                finished.append(slot)
        if finished:
            rows = self.out[torch.tensor(finished, device=self.dev)].cpu()
            for slot, row in zip(finished, rows):
                req = self.decoding.pop(slot)
                req.output = row[: self.n_gen.pop(slot)].tolist()
                self.free.append(slot)
                self.done.append(req)

    def step(self) -> None:
        """One scheduler step: admit, prefill (bounded), decode every ready sequence."""
        self._admit()
        self._prefill()
        self._decode()
        self.steps += 1
