"""Seeded random-init RWKV-7 checkpoints in the reference's key format.

The reference only loads real ``rwkv7-g1d`` checkpoints with ``torch.load``
(``src/rwkv_tl/weight.py:155-184``); none exist on the build or GPU machines,
so every test and benchmark here runs on a synthetic checkpoint with the same
keys and shapes (``src/rwkv_tl/weight.py:11-12,68-106,124-126,171-184``).

Init scheme (fixed so that the oracle and the CUDA path see identical weights):

* every Linear / LoRA matrix ~ N(0, 1/fan_in) (std = 1/sqrt(fan_in));
* LayerNorm / GroupNorm weight = 1, bias = 0;
* decay bias ``w0`` ~ U(-6, -1);
* token-shift mixes ``x_*`` ~ U(0, 1);
* ``k_k`` ~ N(1, 0.1), ``k_a`` = 1, ``a0`` = 0, ``v0`` = 0, ``r_k`` ~ N(0, 0.1);
* ``emb`` ~ N(0, 1) (LN0 renormalises it at load anyway).

Tensors are drawn in fp32 from one ``torch.Generator`` in a fixed key order and
stored in ``dtype`` (the reference casts to fp16 at load anyway).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["ModelConfig", "CONFIG_0_1B", "CONFIG_0_4B", "CONFIG_TINY", "synth_checkpoint"]


@dataclass(frozen=True)
class ModelConfig:
    n_layer: int
    n_embd: int
    vocab: int = 65536
    rank_w: int = 64
    rank_a: int = 64
    rank_v: int = 32
    rank_g: int = 128
    head_size: int = 64

    @property
    def n_head(self) -> int:
        return self.n_embd // self.head_size

    @property
    def ffn(self) -> int:
        return 4 * self.n_embd


CONFIG_0_1B = ModelConfig(n_layer=12, n_embd=768)
CONFIG_0_4B = ModelConfig(n_layer=24, n_embd=1024)
# Small model used for golden fixtures and fast parity tests.
CONFIG_TINY = ModelConfig(n_layer=2, n_embd=128, vocab=1024)


def synth_checkpoint(
    cfg: ModelConfig,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: str | torch.device = "cpu",
) -> dict[str, torch.Tensor]:
    """Return a state dict with the reference checkpoint's keys and shapes.

    Drawing happens on ``device`` with a generator seeded by ``seed``; the
    CPU stream is the canonical one (bit-identical on every x86 host with the
    same torch build), a CUDA stream is only used for large benchmark models.
    """
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    C, V, H, N = cfg.n_embd, cfg.vocab, cfg.n_head, cfg.head_size
    W: dict[str, torch.Tensor] = {}

    def normal(shape, std, mean=0.0):
        t = torch.randn(shape, generator=g, device=dev, dtype=torch.float32)
        return (t * std + mean).to(dtype)

    def uniform(shape, lo, hi):
        t = torch.rand(shape, generator=g, device=dev, dtype=torch.float32)
        return (t * (hi - lo) + lo).to(dtype)

    def const(shape, val):
        return torch.full(shape, float(val), device=dev, dtype=dtype)

    def linear(out_f, in_f):
        # checkpoint orientation is [out, in]; fan_in = in_f
        return normal((out_f, in_f), in_f ** -0.5)

    W["emb.weight"] = normal((V, C), 1.0)
    W["blocks.0.ln0.weight"] = const((C,), 1.0)
    W["blocks.0.ln0.bias"] = const((C,), 0.0)
    for i in range(cfg.n_layer):
        p = f"blocks.{i}"
        for ln in ("ln1", "ln2"):
            W[f"{p}.{ln}.weight"] = const((C,), 1.0)
            W[f"{p}.{ln}.bias"] = const((C,), 0.0)
        a = f"{p}.att"
        for name in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
            W[f"{a}.{name}"] = uniform((1, 1, C), 0.0, 1.0)
        W[f"{a}.w0"] = uniform((1, 1, C), -6.0, -1.0)
        W[f"{a}.a0"] = const((1, 1, C), 0.0)
        W[f"{a}.v0"] = const((1, 1, C), 0.0)
        for name, r in (("w", cfg.rank_w), ("a", cfg.rank_a), ("v", cfg.rank_v), ("g", cfg.rank_g)):
            W[f"{a}.{name}1"] = normal((C, r), C ** -0.5)  # x @ w1: fan_in = C
            W[f"{a}.{name}2"] = normal((r, C), r ** -0.5)  # h @ w2: fan_in = r
        W[f"{a}.k_k"] = normal((1, 1, C), 0.1, mean=1.0)
        W[f"{a}.k_a"] = const((1, 1, C), 1.0)
        W[f"{a}.r_k"] = normal((H, N), 0.1)
        for name in ("receptance", "key", "value", "output"):
            W[f"{a}.{name}.weight"] = linear(C, C)
        W[f"{a}.ln_x.weight"] = const((C,), 1.0)
        W[f"{a}.ln_x.bias"] = const((C,), 0.0)
        f = f"{p}.ffn"
        W[f"{f}.x_k"] = uniform((1, 1, C), 0.0, 1.0)
        W[f"{f}.key.weight"] = linear(4 * C, C)
        W[f"{f}.value.weight"] = linear(C, 4 * C)
    W["ln_out.weight"] = const((C,), 1.0)
    W["ln_out.bias"] = const((C,), 0.0)
    W["head.weight"] = linear(V, C)
    return W
