"""CUDA-Graph wrapper for ``RWKV7B200`` (role of ``demo/cuda_graph.py``).

Like the reference's ``CUDAGraph`` it captures the wrapped model's own
``decode`` and per-length ``prefill`` (T in [2, ``prefill_graph_max_t``]) lazily
and replays them. Differences, B200-side:

* the token goes through a device buffer filled by an on-stream copy, so a
  CUDA-tensor token never forces a host sync (the reference calls
  ``token.item()``, ``demo/cuda_graph.py:123``);
* graphs are captured against the caller's own state blocks (keyed by their
  addresses, a small LRU), so there is no copy of the whole state into and out
  of a shadow state around every replay (``demo/cuda_graph.py:124-126``);
  a ``State`` that is not bound to library-addressable blocks runs eagerly;
* ``decode_batch`` is captured per (batch size, state, slots, output buffer); given
  an output buffer it writes the logits there with no extra copy.

Capture failures fall back to eager, with a warning, as in the reference.
"""

from __future__ import annotations

import warnings
from collections import OrderedDict

import torch
from torch import Tensor

from .model import RWKV7B200, RWKV7Model
from .state import BatchedState, State
from .weight import RWKV7Weight

__all__ = ["CUDAGraph", "make_graph_cls"]


class _Entry:
    __slots__ = ("graph", "tok", "logits", "extra")

    def __init__(self, graph, tok, logits, extra=None):
        self.graph, self.tok, self.logits, self.extra = graph, tok, logits, extra


class CUDAGraph(RWKV7Model):
    def __init__(self, model: RWKV7B200, *, prefill_graph_max_t: int = 64, warmup: int = 3,
                 max_graphs: int = 16):
        super().__init__(model.w)
        self.model = model
        self.prefill_graph_max_t = prefill_graph_max_t
        self._warmup = warmup
        self._max = max_graphs
        self._graphs: OrderedDict = OrderedDict()
        self._failed: set = set()
        self._keep: dict = {}

    def __getattr__(self, name):
        model = self.__dict__.get("model")
        if model is not None:
            return getattr(model, name)
        raise AttributeError(name)

    # ------------------------------------------------------------------ #
    def _get(self, key):
        e = self._graphs.get(key)
        if e is not None:
            self._graphs.move_to_end(key)
        return e

    def _put(self, key, e):
        e.extra = self._keep.pop(key, None)
        self._graphs[key] = e
        while len(self._graphs) > self._max:
            self._graphs.popitem(last=False)

    def _capture(self, key, run_on, scratch_state, live_state, name):
        """Warm up ``run_on(scratch)`` on a side stream, then capture ``run_on(live)``."""
        try:
            s = torch.cuda.Stream(device=self.w.device)
            s.wait_stream(torch.cuda.current_stream(self.w.device))
            with torch.cuda.stream(s):
                for _ in range(self._warmup):
                    run_on(scratch_state)
            torch.cuda.current_stream(self.w.device).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                run_on(live_state)
            torch.cuda.current_stream(self.w.device).wait_stream(s)
            # The graph holds the addresses of the model's scratch buffers as they
            # were during capture. The model replaces a buffer when a later call needs
            # more bytes; keeping the captured ones referenced here means they are
            # never returned to the allocator while this graph can still replay.
            self._keep[key] = (self.model._ws, self.model._ws_dec)
            return g
        except Exception as e:  # noqa: BLE001 - capture problem -> eager
            warnings.warn(f"CUDA-Graph {name} capture failed ({e}); running eager.", stacklevel=3)
            self._failed.add(key)
            return None

    # ------------------------------------------------------------------ #
    def decode(self, token, S: State) -> tuple[Tensor, State]:
        if not (isinstance(S, State) and S._rnn.device == self.w.device and S.bound()):
            return self.model.decode(token, S)
        key = ("dec", S._rnn.data_ptr(), S._slot)
        e = self._get(key)
        if e is None and key not in self._failed:
            tok = torch.zeros(1, dtype=torch.long, device=self.w.device)
            out = {}

            def run(st):
                out["logits"], _ = self.model.decode(tok, st)

            scratch = State(self.L, self.C, 64, device=self.w.device)
            self.model._const((S._slot,))  # built outside the capture
            g = self._capture(key, run, scratch, S, "decode")
            if g is not None:
                e = _Entry(g, tok, out["logits"])
                self._put(key, e)
        if e is None:
            return self.model.decode(token, S)
        if isinstance(token, Tensor):
            e.tok.copy_(token.reshape(1), non_blocking=True)
        else:
            e.tok.fill_(int(token))
        e.graph.replay()
        return e.logits.clone(), S

    def prefill(self, tokens, S: State) -> State:
        tok = self.model._tokens(tokens)
        T = tok.numel()
        if (T < 2 or T > self.prefill_graph_max_t or not isinstance(S, State)
                or S._rnn.device != self.w.device or not S.bound()):
            return self.model.prefill(tok, S)
        key = ("pre", T, S._rnn.data_ptr(), S._slot)
        e = self._get(key)
        if e is None and key not in self._failed:
            buf = torch.zeros(T, dtype=torch.long, device=self.w.device)
            scratch = State(self.L, self.C, 64, device=self.w.device)
            self.model._const((S._slot,))
            self.model._const((0, T))
            g = self._capture(key, lambda st: self.model.prefill(buf, st), scratch, S,
                              f"prefill(T={T})")
            if g is not None:
                e = _Entry(g, buf, None)
                self._put(key, e)
        if e is None:
            return self.model.prefill(tok, S)
        e.tok.copy_(tok, non_blocking=True)
        e.graph.replay()
        return S

    def decode_batch(self, tokens: Tensor, state: BatchedState, slots: Tensor | None = None,
                     logits: Tensor | None = None) -> Tensor:
        tok = self.model._tokens(tokens)
        B = tok.numel()
        # A caller-provided `logits` buffer is captured as the graph's output (keyed by its
        # address), so replays write straight into it; without one, the graph owns its
        # buffer and the caller gets a copy, as with the reference's wrapper.
        key = ("decb", B, state.rnn.data_ptr(), None if slots is None else slots.data_ptr(),
               None if logits is None else logits.data_ptr())
        e = self._get(key)
        if e is None and key not in self._failed:
            buf = torch.zeros(B, dtype=torch.long, device=self.w.device)
            lg = logits if logits is not None else torch.empty(
                B, self.model.V, dtype=torch.float16, device=self.w.device)
            scratch = BatchedState(self.L, self.C, state.n_slots, device=self.w.device)
            g = self._capture(key, lambda st: self.model.decode_batch(buf, st, slots, lg), scratch,
                              state, f"decode_batch(B={B})")
            if g is not None:
                e = _Entry(g, buf, lg)
                self._put(key, e)
        if e is None:
            return self.model.decode_batch(tok, state, slots, logits)
        e.tok.copy_(tok, non_blocking=True)
        e.graph.replay()
        if logits is not None:
            return logits
        return e.logits.clone()

    def decode_batch_greedy(self, tokens: Tensor, state: BatchedState,
                            slots: Tensor | None = None, out: Tensor | None = None) -> Tensor:
        """Graph-replayed ``decode_batch_greedy``: one decode step, greedy next ids ``[B]``.

        A caller-provided ``out`` is captured as the graph's output (keyed by its
        address); without one the graph owns its id buffer and the caller gets a copy.

        Serving loops that keep token ids on the host can pass ``tokens`` (int64) and
        ``out`` as pinned CPU tensors: the graph then also holds the host -> device copy of
        the ids and the device -> host copy of the next ids, so a step is one replay. The
        call returns as soon as the step is queued; ``out`` holds the next ids once the
        current stream has been synchronised.
        """
        if (isinstance(tokens, Tensor) and not tokens.is_cuda and tokens.is_pinned()
                and tokens.dtype == torch.int64 and out is not None and not out.is_cuda
                and out.is_pinned() and out.dtype == torch.int64):
            return self._decode_batch_greedy_host(tokens, state, slots, out)
        tok = self.model._tokens(tokens)
        B = tok.numel()
        key = ("decg", B, state.rnn.data_ptr(), None if slots is None else slots.data_ptr(),
               None if out is None else out.data_ptr())
        e = self._get(key)
        if e is None and key not in self._failed:
            buf = torch.zeros(B, dtype=torch.long, device=self.w.device)
            ids = out if out is not None else torch.empty(B, dtype=torch.long,
                                                          device=self.w.device)
            scratch = BatchedState(self.L, self.C, state.n_slots, device=self.w.device)
            g = self._capture(key, lambda st: self.model.decode_batch_greedy(buf, st, slots, ids),
                              scratch, state, f"decode_batch_greedy(B={B})")
            if g is not None:
                e = _Entry(g, buf, ids)
                self._put(key, e)
        if e is None:
            return self.model.decode_batch_greedy(tok, state, slots, out)
        e.tok.copy_(tok, non_blocking=True)
        e.graph.replay()
        if out is not None:
            return out
        return e.logits.clone()

    def _decode_batch_greedy_host(self, tokens: Tensor, state: BatchedState,
                                  slots: Tensor | None, out: Tensor) -> Tensor:
        """``decode_batch_greedy`` with pinned host token ids in and next ids out, the two
        copies captured into the graph with the step (keyed by both host addresses)."""
        B = tokens.numel()
        key = ("decgh", B, state.rnn.data_ptr(), None if slots is None else slots.data_ptr(),
               tokens.data_ptr(), out.data_ptr())
        e = self._get(key)
        if e is None and key not in self._failed:
            buf = torch.zeros(B, dtype=torch.long, device=self.w.device)
            ids = torch.empty(B, dtype=torch.long, device=self.w.device)

            def run(st):
                buf.copy_(tokens.reshape(-1), non_blocking=True)
                self.model.decode_batch_greedy(buf, st, slots, ids)
                out.reshape(-1).copy_(ids, non_blocking=True)

            scratch = BatchedState(self.L, self.C, state.n_slots, device=self.w.device)
            g = self._capture(key, run, scratch, state, f"decode_batch_greedy_host(B={B})")
            if g is not None:
                e = _Entry(g, buf, ids)
                self._put(key, e)
        if e is None:
            ids = self.model.decode_batch_greedy(self.model._tokens(tokens), state, slots)
            out.reshape(-1).copy_(ids, non_blocking=True)
            return out
        e.graph.replay()
        return out

    def prefill_batch(self, seqs, state, slots=None):
        return self.model.prefill_batch(seqs, state, slots)

    def forward_batch(self, seqs, state, slots=None):
        return self.model.forward_batch(seqs, state, slots)


def make_graph_cls(base_cls: type[RWKV7B200], *, prefill_graph_max_t: int = 64,
                   warmup: int = 3) -> type[CUDAGraph]:
    """Class whose constructor ``cls(w, **kw)`` builds ``base_cls(w, **kw)`` and wraps it."""

    def _init(self, w: RWKV7Weight, **kwargs) -> None:
        CUDAGraph.__init__(self, base_cls(w, **kwargs), prefill_graph_max_t=prefill_graph_max_t,
                           warmup=warmup)

    return type(f"CUDAGraph{base_cls.__name__}", (CUDAGraph,), {"__init__": _init})
