"""``make_rwkv7`` (``demo/__init__.py:43-120``) for the B200 path.

Returns a model *class* (instantiate with ``cls(w, ...)``), pre-wrapped in the
CUDA-Graph wrapper unless ``use_graph=False``. Every fp16 backend name of the
reference resolves to the B200 kernels on a CUDA device; there is no CPU or
bf16 variant and no fallback: other requests raise ``ValueError``.
"""

from __future__ import annotations

import torch

from .cuda_graph import make_graph_cls
from .model import RWKV7B200, RWKV7Model

_FP16_BACKENDS = ("b200", "fp16", "tuned", "auto", "rtx3060")
_UNSUPPORTED = ("bf16", "mx450", "torch")


def make_rwkv7(device: torch.device | str, *, backend: str = "tuned", use_graph: bool = True,
               device_name: str | None = None) -> type[RWKV7Model]:
    device = torch.device(device)
    if backend in _UNSUPPORTED:
        raise ValueError(f"backend {backend!r} is not provided by rwkv_tl_b200 (fp16 B200 path only)")
    if backend not in _FP16_BACKENDS:
        raise ValueError(f"unknown backend {backend!r} (expected one of {', '.join(_FP16_BACKENDS)})")
    if device.type != "cuda":
        raise ValueError(f"rwkv_tl_b200 runs on CUDA devices only (got {device})")
    return make_graph_cls(RWKV7B200) if use_graph else RWKV7B200
