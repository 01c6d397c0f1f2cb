"""B200-native RWKV-7 forward hot path (drop-in for rwkv-tl's fp16 model class).

Public API (mirrors yuyi2439/rwkv-tl's ``demo`` + ``rwkv_tl`` names):
``make_rwkv7``, ``RWKV7Model``, ``RWKV7B200``, ``CUDAGraph``, ``State``,
``BatchedState``, ``RWKV7Weight``, ``sample_logits``.
"""

from . import ops  # registers torch.ops.rwkv_b200::*
from .cuda_graph import CUDAGraph, make_graph_cls
from .factory import make_rwkv7
from .model import RWKV7B200, RWKV7Model
from .sampling import sample_logits
from .serve import ContinuousBatcher, Request
from .state import BatchedState, State
from .weight import RWKV7Weight

__all__ = [
    "BatchedState", "ContinuousBatcher", "CUDAGraph", "RWKV7B200", "RWKV7Model", "RWKV7Weight",
    "Request", "State", "make_graph_cls", "make_rwkv7", "ops", "sample_logits",
]
