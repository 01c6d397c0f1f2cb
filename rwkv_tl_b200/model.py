"""RWKV-7 model classes: the reference's ``RWKV7Model`` contract on B200 kernels.

``RWKV7Model`` restates the reference ABC (``demo/_rwkv7_abc.py:21-89``):
``decode(token, S) -> (logits, S)``, ``prefill(tokens, S) -> S``,
``forward(tokens, S) -> (logits, S)`` (= prefill of all but the last token, then
decode of the last) and ``generate``. ``RWKV7B200`` implements it by calling the
CUDA library (``librwkv_b200.so``) once per call; it adds batched entry points
over many sequences (``decode_batch``, ``prefill_batch``, ``forward_batch``) on a
``BatchedState``.
"""

from __future__ import annotations

import os
from abc import ABC, abstractmethod

import torch
from torch import Tensor

from . import _lib
from ._lib import SEM_DECODE, SEM_PREFILL, check, ptr
from .sampling import sample_logits
from .state import BatchedState, State
from .weight import RWKV7Weight

__all__ = ["RWKV7Model", "RWKV7B200"]


class RWKV7Model(ABC):
    """Common inference interface (``demo/_rwkv7_abc.py:21-89``)."""

    def __init__(self, w: RWKV7Weight, *args, **kwargs) -> None:
        self.w = w
        self.L = w.L
        self.C = w.C
        self.N = 64
        self.H = self.C // self.N

    @abstractmethod
    def decode(self, token: Tensor, S: State) -> tuple[Tensor, State]:
        """Advance one token; returns ``(logits, state)``."""

    @abstractmethod
    def prefill(self, tokens: Tensor, S: State) -> State:
        """Feed a token sequence, updating ``S`` in place; returns ``S``."""

    def generate(self, tokens, S: State, max_tokens: int = 32, *, temperature=None, top_k: int = 0,
                 top_p: float = 1.0, repetition_penalty: float = 1.0) -> tuple[list[int], State]:
        """Autoregressive generation (``demo/_rwkv7_abc.py:41-72``)."""
        if isinstance(tokens, Tensor) and tokens.ndim != 1:
            raise ValueError(f"Expected 1D token sequence, got {tokens.shape}")
        if isinstance(tokens, list):
            tokens = torch.as_tensor(tokens, device=self.w.device)
        tokens = tokens.to(self.w.device)
        out = torch.tensor([], dtype=torch.long, device=self.w.device)
        if tokens.numel() > 1:
            S = self.prefill(tokens[:-1], S)
        token = tokens[-1]
        for _ in range(max_tokens):
            logits, S = self.decode(token, S)
            token = sample_logits(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                  repetition_penalty=repetition_penalty, seen=out)
            out = torch.cat([out, token.reshape(1)])
        return out.tolist(), S

    def forward(self, tokens: Tensor, S: State) -> tuple[Tensor, State]:
        """``demo/_rwkv7_abc.py:74-89``: prefill(tokens[:-1]) then decode(tokens[-1])."""
        if tokens.ndim == 0 and tokens.numel() == 1:
            return self.decode(tokens, S)
        if tokens.ndim != 1:
            raise ValueError(f"Expected 1D token sequence, got {tokens.shape}")
        if tokens.numel() == 1:
            return self.decode(tokens[0], S)
        S = self.prefill(tokens[:-1], S)
        return self.decode(tokens[-1], S)


class RWKV7B200(RWKV7Model):
    """fp16 RWKV-7 on B200 CUDA kernels (drop-in for the reference's ``RWKV7FP16``).

    Args:
        w: ``RWKV7Weight`` on a CUDA device.
        is_torch_compile: accepted for signature compatibility with the
            reference (``demo/rwkv7_fp16.py:17-25``); the CUDA library is the
            compute path either way.
        max_rows: token rows per library call; longer prefills are split
            into consecutive chunks (the state carries across chunks).
    """

    def __init__(self, w: RWKV7Weight, *, is_torch_compile: bool = False, max_rows: int = 4096):
        super().__init__(w)
        if w.device.type != "cuda":
            raise RuntimeError("RWKV7B200 needs weights on a CUDA device (no CPU fallback)")
        self._lib = _lib.load()
        self._cm = w.cmodel()
        self.max_rows = max_rows
        self._ws: Tensor | None = None
        self._ws_dec: Tensor | None = None
        self._meta: dict = {}
        self.V = w.V

    # ------------------------------------------------------------------ #
    # plumbing
    # ------------------------------------------------------------------ #
    def _workspace(self, M: int, S: int, n_logits: int) -> tuple[int, int]:
        need = self._lib.rwkv7_forward_workspace_bytes(self._cm, M, S, n_logits)
        if need == 0:
            raise _lib.RWKVError("invalid model/batch for workspace sizing")
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.w.device)
        return self._ws.data_ptr(), self._ws.numel()

    def _use_gemv(self, B: int) -> bool:
        """Small batches take the fused GEMV decode path (RWKV_B200_DECODE=token forces
        the token-batch path, =gemv the GEMV path)."""
        mode = os.environ.get("RWKV_B200_DECODE", "")
        if mode == "token":
            return False
        if mode == "gemv":
            return B <= 8 and self.C in (768, 1024)
        return B <= 4 and self.C in (768, 1024)

    def run_decode_gemv(self, tokens: Tensor, slots: Tensor | None, sdesc, logits: Tensor) -> None:
        """One ``rwkv7_decode_gemv`` call (B <= 8 sequences, one token each)."""
        B = tokens.numel()
        need = self._lib.rwkv7_decode_gemv_workspace_bytes(self._cm, B)
        if need == 0:
            raise _lib.RWKVError("invalid model/batch for the decode GEMV path")
        if self._ws_dec is None or self._ws_dec.numel() < need:
            self._ws_dec = torch.empty(need, dtype=torch.uint8, device=self.w.device)
        stream = torch.cuda.current_stream(self.w.device).cuda_stream
        check(self._lib.rwkv7_decode_gemv(self._cm, ptr(tokens), B, ptr(slots), sdesc,
                                          ptr(logits), self._ws_dec.data_ptr(),
                                          self._ws_dec.numel(), stream))

    def _arange(self, n: int) -> Tensor:
        key = ("arange", n)
        t = self._meta.get(key)
        if t is None:
            t = self._meta[key] = torch.arange(n, dtype=torch.int32, device=self.w.device)
        return t

    def _zeros(self, n: int) -> Tensor:
        key = ("zeros", n)
        t = self._meta.get(key)
        if t is None:
            t = self._meta[key] = torch.zeros(n, dtype=torch.int32, device=self.w.device)
        return t

    def _const(self, vals: tuple[int, ...]) -> Tensor:
        key = ("const", vals)
        t = self._meta.get(key)
        if t is None:
            t = self._meta[key] = torch.tensor(vals, dtype=torch.int32, device=self.w.device)
        return t

    def _tokens(self, tokens) -> Tensor:
        if isinstance(tokens, Tensor):
            t = tokens.reshape(-1)
            if t.device != self.w.device:
                t = t.to(self.w.device, non_blocking=True)
            if t.dtype != torch.int64:
                t = t.to(torch.int64)
            return t.contiguous()
        return torch.as_tensor(tokens, dtype=torch.int64, device=self.w.device).reshape(-1)

    def run_batch(self, tokens: Tensor, cu: Tensor, row_seq: Tensor, slots: Tensor | None,
                  sdesc: _lib.StateDesc, logit_rows: Tensor | None, logits: Tensor | None,
                  semantics: int, next_ids: Tensor | None = None) -> None:
        """One ``rwkv7_forward`` call on the current stream (all args on device)."""
        M, S = tokens.numel(), cu.numel() - 1
        n_log = 0 if logit_rows is None else logit_rows.numel()
        ws, nbytes = self._workspace(M, S, n_log)
        b = _lib.Batch(M, S, ptr(tokens), ptr(cu), ptr(row_seq), ptr(slots), n_log,
                       ptr(logit_rows), ptr(logits), semantics, ptr(next_ids))
        stream = torch.cuda.current_stream(self.w.device).cuda_stream
        check(self._lib.rwkv7_forward(self._cm, b, sdesc, ws, nbytes, stream))

    def _state_desc(self, S: State):
        """(descriptor, slot tensor, copy-back) for a reference-layout State."""
        if isinstance(S, State) and S._rnn.device == self.w.device and S.bound():
            d, slot = S.desc()
            return d, self._const((slot,)), None
        # foreign or rebound State: stage through a private one and copy back
        tmp = State(self.L, self.C, 64, device=self.w.device)
        for dst, src in zip(tmp.tmix + tmp.cmix, S[0] + S[1]):
            for k in dst:
                dst[k].copy_(src[k])
        d, slot = tmp.desc()

        def back():
            for dst, src in zip(S[0] + S[1], tmp.tmix + tmp.cmix):
                for k in dst:
                    dst[k].copy_(src[k])

        return d, self._const((slot,)), back

    # ------------------------------------------------------------------ #
    # reference API
    # ------------------------------------------------------------------ #
    def decode(self, token, S: State) -> tuple[Tensor, State]:
        """One token of one sequence (``demo/_rwkv7_base.py:74-87``)."""
        tok = self._tokens(token)
        if tok.numel() != 1:
            raise ValueError(f"decode expects one token, got {tok.numel()}")
        d, slot, back = self._state_desc(S)
        logits = torch.empty(1, self.V, dtype=torch.float16, device=self.w.device)
        if self._use_gemv(1):
            self.run_decode_gemv(tok, slot, d, logits)
        else:
            self.run_batch(tok, self._const((0, 1)), self._zeros(1), slot, d, self._zeros(1),
                           logits, SEM_DECODE)
        if back:
            back()
        return logits[0], S

    def prefill(self, tokens, S: State) -> State:
        """Feed tokens, state only (``demo/_rwkv7_base.py:89-98``)."""
        if isinstance(tokens, Tensor) and tokens.ndim != 1:
            raise ValueError(f"Expected 1D token sequence, got {tokens.shape}")
        tok = self._tokens(tokens)
        if tok.numel() == 0:
            raise RuntimeError("prefill received an empty token sequence")
        d, slot, back = self._state_desc(S)
        for s in range(0, tok.numel(), self.max_rows):
            chunk = tok[s:s + self.max_rows]
            T = chunk.numel()
            self.run_batch(chunk, self._const((0, T)), self._zeros(T), slot, d, None, None,
                           SEM_PREFILL)
        if back:
            back()
        return S

    # ------------------------------------------------------------------ #
    # batched extensions
    # ------------------------------------------------------------------ #
    def decode_batch(self, tokens: Tensor, state: BatchedState, slots: Tensor | None = None,
                     logits: Tensor | None = None) -> Tensor:
        """One decode step of B sequences: ``tokens [B]`` -> logits ``[B, V]``.

        Sequence b uses state slot ``slots[b]`` (default b). Numerics are those
        of ``decode`` on each sequence.
        """
        tok = self._tokens(tokens)
        B = tok.numel()
        if slots is None and B > state.n_slots:
            raise ValueError(f"{B} tokens but only {state.n_slots} state slots")
        if logits is None:
            logits = torch.empty(B, self.V, dtype=torch.float16, device=self.w.device)
        if self._use_gemv(B):
            self.run_decode_gemv(tok, slots, state.desc(), logits)
            return logits
        rows = self._arange(B + 1)
        for s in range(0, B, self.max_rows):
            n = min(self.max_rows, B - s)
            sl = slots[s:s + n] if slots is not None else (
                None if s == 0 else self._arange(B)[s:s + n])
            self.run_batch(tok[s:s + n], rows[: n + 1], rows[:n], sl, state.desc(), rows[:n],
                           logits[s:s + n], SEM_DECODE)
        return logits

    def decode_batch_greedy(self, tokens: Tensor, state: BatchedState,
                            slots: Tensor | None = None, out: Tensor | None = None) -> Tensor:
        """One decode step of B sequences returning greedy next ids ``[B]`` int64.

        Same state update as ``decode_batch``; the ids equal
        ``decode_batch(...).argmax(-1)`` (lowest id among equal fp16 logits). On the
        token-batch path the lm head reduces each row to its argmax inside the GEMM
        epilogue, so the ``[B, V]`` logits are never written; the fused GEMV path
        (B <= 4) produces logits and takes their argmax on the device.
        """
        tok = self._tokens(tokens)
        B = tok.numel()
        if slots is None and B > state.n_slots:
            raise ValueError(f"{B} tokens but only {state.n_slots} state slots")
        if out is None:
            out = torch.empty(B, dtype=torch.int64, device=self.w.device)
        if self._use_gemv(B):
            return torch.argmax(self.decode_batch(tok, state, slots), dim=-1, out=out)
        rows = self._arange(B + 1)
        for s in range(0, B, self.max_rows):
            n = min(self.max_rows, B - s)
            sl = slots[s:s + n] if slots is not None else (
                None if s == 0 else self._arange(B)[s:s + n])
            self.run_batch(tok[s:s + n], rows[: n + 1], rows[:n], sl, state.desc(), rows[:n],
                           None, SEM_DECODE, next_ids=out[s:s + n])
        return out

    def prefill_batch(self, seqs: list, state: BatchedState, slots=None) -> BatchedState:
        """Prefill several sequences in one varlen batch (state only).

        ``seqs[i]`` (1-D tokens) goes to slot ``slots[i]`` (default i).
        """
        lens = [int(torch.as_tensor(s).numel()) for s in seqs]
        if any(n == 0 for n in lens):
            raise RuntimeError("prefill received an empty token sequence")
        slot_list = list(range(len(seqs))) if slots is None else [int(x) for x in slots]
        # group sequences into calls of at most max_rows rows; split longer ones
        pending = [(i, 0) for i in range(len(seqs))]
        toks = [self._tokens(s) for s in seqs]
        while pending:
            batch, rows = [], 0
            nxt = []
            for i, off in pending:
                take = min(lens[i] - off, self.max_rows - rows)
                if take <= 0:
                    nxt.append((i, off))
                    continue
                batch.append((i, off, take))
                rows += take
                if off + take < lens[i]:
                    nxt.append((i, off + take))
            cu = [0]
            for _, _, n in batch:
                cu.append(cu[-1] + n)
            tok = torch.cat([toks[i][o:o + n] for i, o, n in batch])
            cu_t = torch.tensor(cu, dtype=torch.int32).to(self.w.device, non_blocking=True)
            row_seq = torch.repeat_interleave(
                torch.arange(len(batch), dtype=torch.int32),
                torch.tensor([n for _, _, n in batch])).to(self.w.device, non_blocking=True)
            sl = torch.tensor([slot_list[i] for i, _, _ in batch],
                              dtype=torch.int32).to(self.w.device, non_blocking=True)
            self.run_batch(tok, cu_t, row_seq, sl, state.desc(), None, None, SEM_PREFILL)
            pending = nxt
        return state

    def forward_batch(self, seqs: list, state: BatchedState, slots=None) -> Tensor:
        """``forward`` of several sequences: logits ``[B, V]`` of each last token."""
        heads = [torch.as_tensor(s).reshape(-1) for s in seqs]
        pre = [(i, h[:-1]) for i, h in enumerate(heads) if h.numel() > 1]
        slot_list = list(range(len(seqs))) if slots is None else [int(x) for x in slots]
        if pre:
            self.prefill_batch([p for _, p in pre], state, [slot_list[i] for i, _ in pre])
        last = torch.stack([h[-1] for h in heads]).to(self.w.device)
        sl = torch.tensor(slot_list, dtype=torch.int32, device=self.w.device)
        return self.decode_batch(last, state, sl)
