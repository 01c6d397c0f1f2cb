"""ctypes binding of ``librwkv_b200.so`` (declared in ``include/rwkv_b200.h``).

The library is the only compute path: importing this module without the built
library, or calling it without a CUDA device, raises instead of falling back.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("RWKV_B200_LIB", _PKG / "librwkv_b200.so"))

# Every symbol the header declares (checked by tests/test_capi_symbols.py).
EXPORTED = (
    "rwkv_b200_last_error",
    "rwkv_b200_abi_version",
    "rwkv_b200_launch_count",
    "rwkv_b200_device_error",
    "rwkv_b200_wait_selftest",
    "rwkv7_dplr_step",
    "rwkv7_dplr_seq",
    "rwkv7_wkv_gn_step",
    "rwkv7_dplr_chunked_workspace_bytes",
    "rwkv7_dplr_chunked",
    "rwkv7_dplr_chunked_noalloc",
    "rwkv7_gemm_f16",
    "rwkv7_sample",
    "rwkv7_forward_workspace_bytes",
    "rwkv7_forward",
    "rwkv7_decode_gemv_workspace_bytes",
    "rwkv7_decode_gemv",
)

RWKV_OK, RWKV_ERR_ARG, RWKV_ERR_CUDA, RWKV_ERR_SPACE = 0, 1, 2, 3
SEM_DECODE, SEM_PREFILL = 0, 1
EPI_STORE, EPI_RESID, EPI_RELUSQ = 0, 1, 2


class RWKVError(RuntimeError):
    """A nonzero status from the CUDA library."""


vp = C.c_void_p


class Layer(C.Structure):
    _fields_ = [
        (n, vp)
        for n in (
            "ln1_w", "ln1_b", "ln2_w", "ln2_b", "mix6", "w_rkv", "w_lora_dn", "w_lora_up",
            "w0", "a0", "v0", "k_k", "k_a", "r_k", "lnx_w", "lnx_b", "w_o", "ffn_x_k",
            "w_fk", "w_fv", "w_lora_up_t",
        )
    ]


class Model(C.Structure):
    _fields_ = [
        ("n_layer", C.c_int), ("n_embd", C.c_int), ("vocab", C.c_int),
        ("rank_v", C.c_int), ("rank_w", C.c_int), ("rank_a", C.c_int), ("rank_g", C.c_int),
        ("emb", vp), ("head", vp), ("lnout_w", vp), ("lnout_b", vp),
        ("layers", C.POINTER(Layer)),
    ]


class StateDesc(C.Structure):
    _fields_ = [("rnn", vp), ("tmix_x", vp), ("cmix_x", vp), ("n_slots", C.c_int)]


class Batch(C.Structure):
    _fields_ = [
        ("n_rows", C.c_int), ("n_seqs", C.c_int),
        ("tokens", vp), ("cu_seqlens", vp), ("row_seq", vp), ("slots", vp),
        ("n_logits", C.c_int), ("logit_rows", vp), ("logits", vp),
        ("semantics", C.c_int), ("next_ids", vp),
    ]


class GemmProblem(C.Structure):
    _fields_ = [
        ("A", vp), ("B", vp), ("C", vp), ("R", vp),
        ("M", C.c_int), ("N", C.c_int), ("K", C.c_int),
        ("lda", C.c_int), ("ldb", C.c_int), ("ldc", C.c_int),
    ]


_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load the CUDA library (once); raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RWKVError(
            f"{LIB_PATH} not found: build it with `python -m rwkv_tl_b200.build` "
            "(there is no CPU fallback)"
        )
    lib = C.CDLL(str(LIB_PATH))
    lib.rwkv_b200_last_error.restype = C.c_char_p
    lib.rwkv_b200_abi_version.restype = C.c_int
    lib.rwkv_b200_launch_count.restype = C.c_ulonglong
    lib.rwkv_b200_device_error.restype = C.c_int
    lib.rwkv_b200_wait_selftest.restype = C.c_int
    lib.rwkv_b200_wait_selftest.argtypes = [C.c_int, vp, vp]
    for name in ("rwkv7_dplr_step", "rwkv7_dplr_seq"):
        f = getattr(lib, name)
        f.restype = C.c_int
        f.argtypes = [vp] * 8 + [C.c_int, C.c_int, vp]
    lib.rwkv7_dplr_chunked_workspace_bytes.restype = C.c_size_t
    lib.rwkv7_dplr_chunked_workspace_bytes.argtypes = [C.c_int, C.c_int, C.c_int]
    lib.rwkv7_dplr_chunked.restype = C.c_int
    lib.rwkv7_dplr_chunked.argtypes = [vp] * 8 + [C.c_int] * 3 + [vp, C.c_size_t, vp]
    lib.rwkv7_dplr_chunked_noalloc.restype = C.c_int
    lib.rwkv7_dplr_chunked_noalloc.argtypes = [vp] * 8 + [C.c_int] * 3 + [vp]
    lib.rwkv7_wkv_gn_step.restype = C.c_int
    lib.rwkv7_wkv_gn_step.argtypes = [vp] * 13 + [C.c_int, C.c_int, C.c_int, vp]
    lib.rwkv7_sample.restype = C.c_int
    lib.rwkv7_sample.argtypes = [vp, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float,
                                 vp, vp, vp, vp, vp]
    lib.rwkv7_gemm_f16.restype = C.c_int
    lib.rwkv7_gemm_f16.argtypes = [C.POINTER(GemmProblem), C.c_int, C.c_int, vp]
    lib.rwkv7_forward_workspace_bytes.restype = C.c_size_t
    lib.rwkv7_forward_workspace_bytes.argtypes = [C.POINTER(Model), C.c_int, C.c_int, C.c_int]
    lib.rwkv7_forward.restype = C.c_int
    lib.rwkv7_forward.argtypes = [C.POINTER(Model), C.POINTER(Batch), C.POINTER(StateDesc), vp,
                                  C.c_size_t, vp]
    lib.rwkv7_decode_gemv_workspace_bytes.restype = C.c_size_t
    lib.rwkv7_decode_gemv_workspace_bytes.argtypes = [C.POINTER(Model), C.c_int]
    lib.rwkv7_decode_gemv.restype = C.c_int
    lib.rwkv7_decode_gemv.argtypes = [C.POINTER(Model), vp, C.c_int, vp, C.POINTER(StateDesc),
                                      vp, vp, C.c_size_t, vp]
    if lib.rwkv_b200_abi_version() != 2:
        raise RWKVError("librwkv_b200.so ABI version mismatch")
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != RWKV_OK:
        msg = load().rwkv_b200_last_error().decode(errors="replace")
        raise RWKVError(f"librwkv_b200 error {rc}: {msg}")


def ptr(t) -> int:
    """Device address of a torch tensor (0 for None)."""
    return 0 if t is None else t.data_ptr()
