"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py`` (the reference's own
``RWKV7Torch`` and ``RWKV7FP16`` classes run on CPU on a synthetic checkpoint).
"""

from __future__ import annotations

import torch

from oracle.rwkv7_oracle import OracleState, OracleWeights, RWKV7Oracle
from rwkv_tl_b200.synth import CONFIG_0_1B, CONFIG_TINY, synth_checkpoint


def _run(oracle: RWKV7Oracle, tokens: list[int]):
    w = oracle.w
    S = OracleState(w.L, w.C)
    per_step = [oracle.decode(t, S) for t in tokens]
    S2 = OracleState(w.L, w.C)
    fwd = oracle.forward(tokens, S2)
    return torch.stack(per_step), S, fwd, S2


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def test_oracle_fp32_matches_reference_torch_tiny(golden_dir):
    g = torch.load(golden_dir / "tiny_torch_fp32.pt")
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_TINY, seed=1), mode="fp32"))
    dec, S, fwd, S2 = _run(o, g["tokens"].tolist())
    assert (dec - g["decode_logits"]).abs().max() < 1e-4
    assert (fwd - g["forward_logits"]).abs().max() < 1e-4
    assert _rel(torch.stack(S.rnn), g["decode_state"]["rnn"]) < 1e-5
    assert _rel(torch.stack(S2.rnn), g["forward_state"]["rnn"]) < 1e-5
    assert (torch.stack(S2.tmix_x) - g["forward_state"]["tmix_x"]).abs().max() < 1e-5
    assert (torch.stack(S2.cmix_x) - g["forward_state"]["cmix_x"]).abs().max() < 1e-5


def test_oracle_fp16_close_to_reference_fp16_tiny(golden_dir):
    """fp16 oracle (GPU-kernel rounding points) vs the reference fp16 model's CPU
    fallbacks (per-op rounding): the two differ only in fp16 rounding placement."""
    g = torch.load(golden_dir / "tiny_fp16_cpu.pt")
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_TINY, seed=1), mode="fp16"))
    dec, S, fwd, S2 = _run(o, g["tokens"].tolist())
    assert (dec - g["decode_logits"]).abs().max() < 5e-2
    assert _rel(dec, g["decode_logits"]) < 1e-2
    # prefill rounding points are the per-op torch ones in both: tighter
    assert (fwd - g["forward_logits"]).abs().max() < 3e-2
    assert _rel(torch.stack(S2.rnn), g["forward_state"]["rnn"]) < 1e-2
    assert (dec.argmax(-1) == g["decode_logits"].argmax(-1)).all()


def test_oracle_fp16_close_to_fp32_tiny(golden_dir):
    g = torch.load(golden_dir / "tiny_torch_fp32.pt")
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_TINY, seed=1), mode="fp16"))
    dec, S, fwd, S2 = _run(o, g["tokens"].tolist())
    assert _rel(dec, g["decode_logits"]) < 2e-2
    assert _rel(fwd, g["forward_logits"]) < 2e-2


def test_oracle_fp32_config0_greedy(golden_dir):
    """BASELINE config 0 (0.1B fp32, 8-token prompt, 16 greedy steps)."""
    g = torch.load(golden_dir / "cfg0_torch_fp32.pt")
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_0_1B, seed=0), mode="fp32"))
    S = OracleState(o.w.L, o.w.C)
    prompt_logits = o.forward(g["prompt"].tolist(), S)
    assert (prompt_logits - g["prompt_logits"]).abs().max() < 1e-3
    S = OracleState(o.w.L, o.w.C)
    gen, last = o.generate_greedy(g["prompt"].tolist(), 16, S)
    assert gen == g["generated"].tolist()
    assert (last - g["last_logits"]).abs().max() < 1e-3
    assert torch.allclose(S.rnn[0][0], g["state_rnn_layer0_head0"], atol=1e-4, rtol=1e-4)
