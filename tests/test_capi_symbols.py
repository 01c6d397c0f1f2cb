"""The C-ABI library loads without a GPU and exports every symbol of include/rwkv_b200.h."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from rwkv_tl_b200 import _lib

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from rwkv_tl_b200.build import build

        build()
    return _lib.load()


def _declared():
    hdr = (REPO / "include" / "rwkv_b200.h").read_text()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(rwkv\w*)\s*\(", hdr)))


def test_header_matches_binding_list():
    assert _declared() == sorted(_lib.EXPORTED)


def test_all_symbols_exported(lib):
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared():
        assert hasattr(raw, name), name


def test_abi_and_argument_errors_without_gpu(lib):
    assert lib.rwkv_b200_abi_version() == 2
    assert lib.rwkv7_dplr_step(None, None, None, None, None, None, None, None, 1, 16, None) == 1
    assert b"null pointer" in lib.rwkv_b200_last_error()
    assert lib.rwkv7_gemm_f16(None, 0, 0, None) == 1
    m = _lib.Model()
    assert lib.rwkv7_forward_workspace_bytes(m, 1, 1, 0) == 0  # invalid model -> 0
    assert lib.rwkv7_forward(m, None, None, None, 0, None) == 1
