"""Seeded inputs of the reference-GPU parity cases (2, 3).

Shared by ``make_golden_gpu.py`` (which runs the reference's own fp16 TileLang
model on them and stores its outputs) and by ``tests/test_ref_gpu_parity.py``
(which runs this library on the same inputs and compares). Everything is drawn
on the CPU from ``torch.Generator`` seeds, so the two sides see bit-identical
inputs on any machine.
"""

from __future__ import annotations

import torch

from rwkv_tl_b200.synth import CONFIG_0_1B, CONFIG_0_4B

# 0.1B, 8-token prompt, 16 greedy steps from a zero state.
CFG0 = dict(cfg=CONFIG_0_1B, weight_seed=0, prompt_len=8, prompt_seed=0, steps=16)
# 0.1B decode (T=1) of 256 sequences from random states.
CFG2 = dict(cfg=CONFIG_0_1B, weight_seed=0, batch=256, state_seed=2, token_seed=2)
# 0.4B prefill at these T, then 32 greedy decode steps.
CFG3 = dict(cfg=CONFIG_0_4B, weight_seed=0, lengths=(8, 64, 128, 1024, 4096), steps=32)

# sequences of config 2 whose full logits / states are stored
CFG2_LOGIT_SEQS = (0, 1, 2, 3, 4, 5, 7, 31, 63, 64, 127, 200, 255)
CFG2_STATE_SEQS = (0, 3, 7, 63, 255)
# top-k (values, ids) stored for every logits position
TOPK = 64

# Short prompts, many seeds: the distance of one short-prompt forward to the exact
# value is one draw from a wide distribution (fp32-vs-fp64 noise after an 8-token
# prefill ranges 3e-3..2e-2 in logits relative-L2 over seeds), so these cases are
# compared as means over seeds.
SHORT = {
    "short_0p1b": dict(cfg=CONFIG_0_1B, weight_seed=0, prompt_len=8, seeds=tuple(range(100, 124))),
    "short_0p4b": dict(cfg=CONFIG_0_4B, weight_seed=0, prompt_len=8, seeds=tuple(range(200, 216))),
}
SHORT_STATE_HEADS = 2  # heads 0..1 of the last layer's wkv state are stored


def prompt(n: int, seed: int, vocab: int = 65536) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def cfg3_prompt(T: int) -> list[int]:
    return prompt(T, 1000 + T)


def state_layers(L: int) -> tuple[int, ...]:
    """Layers whose full wkv state a fixture stores (first, middle, last)."""
    return (0, L // 2, L - 1)


def random_states(cfg, B: int, seed: int):
    """Config 2 start states: rnn ~ N(0, 0.1) fp32, token-shift x ~ N(0, 1) fp16.

    Returns ``(rnn [L, B, H, 64, 64] fp32, tmix_x [L, B, C] fp16, cmix_x [L, B, C] fp16)``.
    """
    g = torch.Generator().manual_seed(seed)
    L, C, H = cfg.n_layer, cfg.n_embd, cfg.n_head
    rnn = 0.1 * torch.randn(L, B, H, 64, 64, generator=g)
    tx = torch.randn(L, B, C, generator=g).half()
    cx = torch.randn(L, B, C, generator=g).half()
    return rnn, tx, cx


def cfg2_tokens() -> list[int]:
    return prompt(CFG2["batch"], CFG2["token_seed"])


def cfg3_steps_full(steps: int) -> tuple[int, ...]:
    """Positions (0 = the forward's logits, i = after greedy step i) stored in full."""
    return (0, steps // 2, steps)
