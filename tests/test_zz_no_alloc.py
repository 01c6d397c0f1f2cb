"""The allocation-free chunked wkv7 entry point against the workspace one.

``rwkv7_dplr_chunked_noalloc`` exists for callers that cannot allocate device
memory when they run the recurrence; it keeps its scratch in a fixed array
inside the library. This file is collected last so that a run stopping at the
first failure has already run every other test; it also passes alone.
"""

from __future__ import annotations

import pytest
import torch

from tests._util import rel_l2
from tests.test_wkv_gpu import _inputs

pytestmark = pytest.mark.gpu


def _run(lib, fn_name, B, T, H, seed):
    from rwkv_tl_b200 import _lib

    r, w, k, v, A, Bv, S0 = _inputs(B, T, H, seed=seed)
    dev = [t.contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    S = S0.cuda().contiguous()
    y = torch.empty(B, T, H, 64, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if fn_name == "noalloc":
        rc = lib.rwkv7_dplr_chunked_noalloc(S.data_ptr(), *[t.data_ptr() for t in dev],
                                            y.data_ptr(), B, T, H, stream)
    else:
        nbytes = lib.rwkv7_dplr_chunked_workspace_bytes(B, T, H)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.rwkv7_dplr_chunked(S.data_ptr(), *[t.data_ptr() for t in dev], y.data_ptr(),
                                    B, T, H, ws.data_ptr(), nbytes, stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    return S.cpu(), y.float().cpu()


def test_noalloc_matches_workspace_entry_two_calls_in_a_row():
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    # two different problems back to back: the second must not see the first's scratch
    for B, T, seed in ((4, 100, 1), (2, 257, 2)):
        S_ref, y_ref = _run(lib, "workspace", B, T, 16, seed)
        S_na, y_na = _run(lib, "noalloc", B, T, 16, seed)
        assert rel_l2(S_na, S_ref) < 1e-4
        assert rel_l2(y_na, y_ref) < 1e-3


def test_noalloc_rejects_problems_beyond_its_scratch():
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    x = torch.zeros(1, device="cuda")
    p = x.data_ptr()
    rc = lib.rwkv7_dplr_chunked_noalloc(p, p, p, p, p, p, p, p, 64, 4096, 16,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.RWKV_ERR_SPACE
    assert b"33554432" in lib.rwkv_b200_last_error()
