"""The fp16 noise floor of the reference's rounding schedule (CPU, oracle only).

Evaluates the same fp16 rounding schedule with fp32 and with fp64 accumulation
on seeded random-init models. The difference is what any fp16 implementation
(the reference's TileLang path included) can be expected to show against any
other; it grows with depth and on 12 layers exceeds the north star's
relative-L2 1e-3 logits bar, which is why the GPU parity tests compare
against the fp64 evaluation with a floor-relative tolerance (tests/_util.py).
"""

from __future__ import annotations

import torch

from rwkv_tl_b200.synth import ModelConfig, synth_checkpoint
from tests._util import OraclePair, max_abs, rel_l2


def _floor(L: int) -> tuple[float, float]:
    sd = synth_checkpoint(ModelConfig(n_layer=L, n_embd=768, vocab=4096), seed=0)
    op = OraclePair(sd)
    S2 = op.state()
    worst_r = worst_a = 0.0
    for t in (5, 77, 1234):
        r64, r32 = op.decode(t, S2)
        worst_r, worst_a = max(worst_r, rel_l2(r32, r64)), max(worst_a, max_abs(r32, r64))
    return worst_r, worst_a


def test_floor_one_layer_is_below_north_star_bar():
    r, a = _floor(1)
    assert r < 1e-3 and a < 2e-2


def test_floor_twelve_layers_exceeds_north_star_rel_bar():
    r, a = _floor(12)
    assert 1e-3 < r < 5e-2, r
    assert a < 2e-1
