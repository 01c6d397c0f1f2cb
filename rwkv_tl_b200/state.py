"""Recurrent state with the reference's per-sequence layout, over batched storage.

``State`` keeps the reference's interface exactly (``src/rwkv_tl/state.py:9-61``):
a 2-tuple ``(tmix, cmix)`` of per-layer dicts, ``tmix[i] = {"x": [C] fp16,
"rnn": [H, 64, 64] fp32}``, ``cmix[i] = {"x": [C] fp16}``, updated in place,
with ``reset()``. Here every per-layer tensor is a view into three contiguous
blocks (``rnn [L, 1, H, 64, 64]``, ``tmix_x [L, 1, C]``, ``cmix_x [L, 1, C]``) so
the CUDA library can address the whole state with three pointers.

``BatchedState`` holds the same blocks for ``n_slots`` sequences and hands out
per-sequence ``State`` views (``state[b]``) whose tensors alias its storage.
"""

from __future__ import annotations

from typing import Self

import torch
from torch import Tensor

from . import _lib

__all__ = ["State", "BatchedState"]


def _alloc(L: int, C: int, slots: int, device, dtype) -> tuple[Tensor, Tensor, Tensor]:
    H = C // 64
    rnn = torch.zeros((L, slots, H, 64, 64), dtype=torch.float32, device=device)
    tx = torch.zeros((L, slots, C), dtype=dtype, device=device)
    cx = torch.zeros((L, slots, C), dtype=dtype, device=device)
    return rnn, tx, cx


class State(tuple[list[dict[str, Tensor]], list[dict[str, Tensor]]]):
    """Runtime state of one sequence (reference-compatible layout)."""

    _rnn: Tensor
    _tx: Tensor
    _cx: Tensor
    _slot: int

    def __new__(
        cls,
        n_layer: int,
        n_embd: int,
        head_dim: int = 64,
        *,
        device: torch.device | str | None = None,
        dtype: torch.dtype = torch.float16,
    ) -> Self:
        if head_dim != 64:
            raise ValueError(f"RWKV-7 head_dim is 64 (got {head_dim})")
        rnn, tx, cx = _alloc(n_layer, n_embd, 1, device, dtype)
        return cls._from_blocks(rnn, tx, cx, 0)

    @classmethod
    def _from_blocks(cls, rnn: Tensor, tx: Tensor, cx: Tensor, slot: int) -> Self:
        L = rnn.shape[0]
        tmix = [{"x": tx[i, slot], "rnn": rnn[i, slot]} for i in range(L)]
        cmix = [{"x": cx[i, slot]} for i in range(L)]
        obj = super().__new__(cls, (tmix, cmix))
        obj._rnn, obj._tx, obj._cx, obj._slot = rnn, tx, cx, slot
        return obj

    @property
    def tmix(self) -> list[dict[str, Tensor]]:
        return self[0]

    @property
    def cmix(self) -> list[dict[str, Tensor]]:
        return self[1]

    def reset(self) -> None:
        """Zero all state tensors in place."""
        for s in self.tmix + self.cmix:
            for t in s.values():
                t.zero_()

    # ---- library plumbing ------------------------------------------------
    def bound(self) -> bool:
        """True while every dict entry still aliases the backing blocks."""
        s = self._slot
        for i, (t, c) in enumerate(zip(self[0], self[1])):
            if (
                t["x"].data_ptr() != self._tx[i, s].data_ptr()
                or t["rnn"].data_ptr() != self._rnn[i, s].data_ptr()
                or c["x"].data_ptr() != self._cx[i, s].data_ptr()
            ):
                return False
        return True

    def desc(self) -> tuple[_lib.StateDesc, int]:
        """(state descriptor over the backing blocks, this sequence's slot)."""
        d = _lib.StateDesc(self._rnn.data_ptr(), self._tx.data_ptr(), self._cx.data_ptr(),
                           self._rnn.shape[1])
        return d, self._slot


class BatchedState:
    """State of ``n_slots`` independent sequences in contiguous blocks.

    ``rnn [L, n_slots, H, 64, 64]`` fp32, ``tmix_x`` / ``cmix_x [L, n_slots, C]``.
    ``state[b]`` is a reference-layout ``State`` view of slot ``b``.
    """

    def __init__(self, n_layer: int, n_embd: int, n_slots: int, *, device=None,
                 dtype: torch.dtype = torch.float16):
        self.L, self.C, self.n_slots = n_layer, n_embd, n_slots
        self.rnn, self.tmix_x, self.cmix_x = _alloc(n_layer, n_embd, n_slots, device, dtype)

    def __getitem__(self, b: int) -> State:
        if not 0 <= b < self.n_slots:
            raise IndexError(b)
        return State._from_blocks(self.rnn, self.tmix_x, self.cmix_x, b)

    def __len__(self) -> int:
        return self.n_slots

    def reset(self, slots=None) -> None:
        if slots is None:
            self.rnn.zero_(); self.tmix_x.zero_(); self.cmix_x.zero_()
        else:
            for t in (self.rnn, self.tmix_x, self.cmix_x):
                t[:, slots] = 0

    def desc(self) -> _lib.StateDesc:
        return _lib.StateDesc(self.rnn.data_ptr(), self.tmix_x.data_ptr(),
                              self.cmix_x.data_ptr(), self.n_slots)
