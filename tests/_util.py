"""Helpers shared by the parity tests."""

from __future__ import annotations

import torch

# Parity bar (north star): logits max-abs 2e-2 and relative-L2 1e-3 against the
# reference fp16 path; wkv state relative 1e-3; greedy argmax >= 99% of steps.
LOGIT_MAX_ABS = 2e-2
LOGIT_REL_L2 = 1e-3
STATE_REL = 1e-3


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.double().cpu() - b.double().cpu()).abs().max())


def assert_logits_close(got, ref, label=""):
    ma, rl = max_abs(got, ref), rel_l2(got, ref)
    assert ma <= LOGIT_MAX_ABS and rl <= LOGIT_REL_L2, f"{label}: max_abs={ma:.4g} rel_l2={rl:.4g}"


def gpu_state_to_oracle(S, oracle_state):
    """Copy a reference-layout State (GPU) into an OracleState (CPU)."""
    for i in range(len(S.tmix)):
        oracle_state.tmix_x[i] = S.tmix[i]["x"].float().cpu().clone()
        oracle_state.rnn[i] = S.tmix[i]["rnn"].float().cpu().clone()
        oracle_state.cmix_x[i] = S.cmix[i]["x"].float().cpu().clone()


def assert_state_close(S, So, label=""):
    rnn = torch.stack([d["rnn"].float().cpu() for d in S.tmix])
    r = rel_l2(rnn, torch.stack(So.rnn))
    assert r <= STATE_REL, f"{label}: state rel={r:.4g}"
    tx = torch.stack([d["x"].float().cpu() for d in S.tmix])
    cx = torch.stack([d["x"].float().cpu() for d in S.cmix])
    assert max_abs(tx, torch.stack(So.tmix_x)) <= 2e-2, f"{label}: tmix x"
    assert max_abs(cx, torch.stack(So.cmix_x)) <= 2e-2, f"{label}: cmix x"
