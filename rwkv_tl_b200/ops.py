"""``torch.ops.rwkv_b200::*``: the library's kernels as PyTorch operators.

Mirrors the reference's operator layer (``src/rwkv_tl/operators/__init__.py:39-68``,
``torch.library.define`` + ``torch.library.impl``, the low-dispatch-overhead form) so
that the B200 kernels can be called from code that goes through ``torch.ops`` and
traced by ``torch.compile``:

* ``fused_dplr(Tensor(a!) S, R, W, K, V, A, B) -> Tensor``   one wkv7 step
  (``operators/__init__.py:304-322``, ``kernels/dplr.py:256-270``);
* ``fused_dplr_T(Tensor(a!) S, R, W, K, V, A, B) -> Tensor`` the recurrence over T
  tokens (``kernels/dplr.py:272-285``), chunk-parallel;
* ``wkv_gn_step(Tensor(a!) S, r, w, k, v, a, b, g, r_k, ln_xW, ln_xB, int semantics)
  -> Tensor``  the decode attention tail: wkv step, GroupNorm + bonus
  (``fused_gn_rkrk``, ``operators/__init__.py:278-300``) and the g gate;
* ``gemm_f16(Tensor A, Tensor B, Tensor? R, int epilogue) -> Tensor``
  ``epi(A @ B^T)``, the projections (``kernels/gemm.py:215-305``).

Each op has a CUDA implementation (the C-ABI library on the current stream) and a
Meta implementation (shapes only, for ``torch.compile`` / fake-tensor tracing).
There is deliberately no CPU implementation: the B200 path has no CPU fallback, so a
CPU call fails in the dispatcher. In-place state updates are declared with the
``Tensor(a!)`` alias annotation; outputs are fresh tensors, as in the reference.
"""

from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from . import _lib

__all__ = ["NAMESPACE", "EPI_STORE", "EPI_RESID", "EPI_RELUSQ", "EPI_STORE_F32"]

NAMESPACE = "rwkv_b200"
EPI_STORE, EPI_RESID, EPI_RELUSQ, EPI_STORE_F32 = 0, 1, 2, 3
_HD = 64

_LIB = torch.library.Library(NAMESPACE, "DEF")


def _define(name: str, schema: str, cuda, meta) -> None:
    _LIB.define(name + schema)
    _LIB.impl(name, cuda, "CUDA")
    _LIB.impl(name, meta, "Meta")


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(f"rwkv_b200: {msg}")


def _stream(t: Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _p(t: Tensor | None) -> C.c_void_p | None:
    return None if t is None else C.c_void_p(t.data_ptr())


def _inputs(S: Tensor, vecs: list[Tensor], what: str) -> None:
    _check(S.is_cuda and S.dtype == torch.float32 and S.is_contiguous(),
           f"{what}: S must be a contiguous fp32 CUDA tensor")
    for t in vecs:
        _check(t.is_cuda and t.dtype == torch.float16 and t.is_contiguous(),
               f"{what}: activations must be contiguous fp16 CUDA tensors")
        _check(t.device == S.device, f"{what}: all tensors must be on one device")


# ---- fused_dplr: one token per sequence -------------------------------------------
def _dplr_cuda(S: Tensor, R: Tensor, W: Tensor, K: Tensor, V: Tensor, A: Tensor, B: Tensor) -> Tensor:
    vecs = [R, W, K, V, A, B]
    _inputs(S, vecs, "fused_dplr")
    _check(S.dim() in (3, 4) and S.shape[-2:] == (_HD, _HD), "fused_dplr: S must be [(n,) H, 64, 64]")
    H = S.shape[-3]
    n = S.shape[0] if S.dim() == 4 else 1
    for t in vecs:
        _check(t.numel() == n * H * _HD, "fused_dplr: R..B must hold n * H * 64 elements")
    y = torch.empty_like(R)
    _lib.check(_lib.load().rwkv7_dplr_step(_p(S), *[_p(t) for t in vecs], _p(y), n, H, _stream(S)))
    return y


def _dplr_meta(S, R, *_args) -> Tensor:
    return torch.empty_like(R)


# ---- fused_dplr_T: T tokens per sequence, chunk-parallel ---------------------------
def _dplr_T_cuda(S: Tensor, R: Tensor, W: Tensor, K: Tensor, V: Tensor, A: Tensor, B: Tensor) -> Tensor:
    vecs = [R, W, K, V, A, B]
    _inputs(S, vecs, "fused_dplr_T")
    _check(S.dim() in (3, 4) and S.shape[-2:] == (_HD, _HD),
           "fused_dplr_T: S must be [(n,) H, 64, 64]")
    H = S.shape[-3]
    n = S.shape[0] if S.dim() == 4 else 1
    _check(R.numel() % (n * H * _HD) == 0 and R.numel() > 0,
           "fused_dplr_T: R..B must be [(n,) T, H, 64]")
    T = R.numel() // (n * H * _HD)
    for t in vecs:
        _check(t.numel() == R.numel(), "fused_dplr_T: R..B must have one shape")
    lib = _lib.load()
    ws_bytes = lib.rwkv7_dplr_chunked_workspace_bytes(n, T, H)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=S.device)
    y = torch.empty_like(R)
    _lib.check(lib.rwkv7_dplr_chunked(_p(S), *[_p(t) for t in vecs], _p(y), n, T, H, _p(ws),
                                      ws_bytes, _stream(S)))
    return y


# ---- wkv_gn_step: decode attention tail --------------------------------------------
def _wkv_gn_cuda(S: Tensor, r: Tensor, w: Tensor, k: Tensor, v: Tensor, a: Tensor, b: Tensor,
                 g: Tensor, r_k: Tensor, ln_xW: Tensor, ln_xB: Tensor, semantics: int) -> Tensor:
    vecs = [r, w, k, v, a, b, g]
    _inputs(S, vecs + [r_k, ln_xW, ln_xB], "wkv_gn_step")
    _check(S.dim() == 4 and S.shape[-2:] == (_HD, _HD), "wkv_gn_step: S must be [n, H, 64, 64]")
    n, H = S.shape[0], S.shape[1]
    for t in vecs:
        _check(t.numel() == n * H * _HD, "wkv_gn_step: r..g must be [n, H * 64]")
    for t in (r_k, ln_xW, ln_xB):
        _check(t.numel() == H * _HD, "wkv_gn_step: r_k, ln_xW, ln_xB must hold H * 64 elements")
    _check(semantics in (0, 1), "wkv_gn_step: semantics must be 0 (decode) or 1 (prefill)")
    out = torch.empty_like(r)
    _lib.check(_lib.load().rwkv7_wkv_gn_step(
        _p(S), None, *[_p(t) for t in vecs], _p(r_k), _p(ln_xW), _p(ln_xB), _p(out), n, H,
        semantics, _stream(S)))
    return out


def _wkv_gn_meta(S, r, *_args) -> Tensor:
    return torch.empty_like(r)


# ---- gemm_f16: epi(A @ B^T) ----------------------------------------------------------
def _gemm_cuda(A: Tensor, B: Tensor, R: Tensor | None, epilogue: int) -> Tensor:
    _check(epilogue in (EPI_STORE, EPI_RESID, EPI_RELUSQ, EPI_STORE_F32),
           "gemm_f16: epilogue must be STORE, RESID, RELUSQ or STORE_F32")
    for t in (A, B) + ((R,) if R is not None else ()):
        _check(t.is_cuda and t.dtype == torch.float16 and t.is_contiguous() and t.dim() == 2,
               "gemm_f16: A, B (and R) must be contiguous 2-D fp16 CUDA tensors")
        _check(t.device == A.device, "gemm_f16: all tensors must be on one device")
    M, K = A.shape
    N, K2 = B.shape
    _check(K == K2, f"gemm_f16: A is [{M}, {K}] but B is [{N}, {K2}]")
    _check((R is not None) == (epilogue == EPI_RESID), "gemm_f16: R is required by RESID only")
    if R is not None:
        _check(R.shape == (M, N), "gemm_f16: R must be [M, N]")
    out = torch.empty(M, N, dtype=torch.float32 if epilogue == EPI_STORE_F32 else torch.float16,
                      device=A.device)
    if M == 0 or N == 0:
        return out
    prob = _lib.GemmProblem(A.data_ptr(), B.data_ptr(), out.data_ptr(),
                            None if R is None else R.data_ptr(), M, N, K, K, K, N)
    _lib.check(_lib.load().rwkv7_gemm_f16(C.byref(prob), 1, epilogue, _stream(A)))
    return out


def _gemm_meta(A: Tensor, B: Tensor, R: Tensor | None, epilogue: int) -> Tensor:
    dt = torch.float32 if epilogue == EPI_STORE_F32 else torch.float16
    return A.new_empty((A.shape[0], B.shape[0]), dtype=dt)


_define("fused_dplr", "(Tensor(a!) S, Tensor R, Tensor W, Tensor K, Tensor V, Tensor A, Tensor B)"
        " -> Tensor", _dplr_cuda, _dplr_meta)
_define("fused_dplr_T", "(Tensor(a!) S, Tensor R, Tensor W, Tensor K, Tensor V, Tensor A,"
        " Tensor B) -> Tensor", _dplr_T_cuda, _dplr_meta)
_define("wkv_gn_step", "(Tensor(a!) S, Tensor r, Tensor w, Tensor k, Tensor v, Tensor a,"
        " Tensor b, Tensor g, Tensor r_k, Tensor ln_xW, Tensor ln_xB, int semantics) -> Tensor",
        _wkv_gn_cuda, _wkv_gn_meta)
_define("gemm_f16", "(Tensor A, Tensor B, Tensor? R, int epilogue) -> Tensor", _gemm_cuda,
        _gemm_meta)
