"""Failure detection fires: each kind of bounded device wait is made to run out.

Every spin in the library's kernels is bounded; on expiry the kernel sets a bit of
the device error word (``rwkv_b200_device_error``) and returns instead of hanging.
``rwkv_b200_wait_selftest`` runs the very wait functions the GEMM pipeline, the
persistent decode kernel and the chunk scan use, on a barrier that nothing signals.
The test checks the wait gave up, the right bit is reported (and cleared on read),
and the next ordinary call on the same context is correct. Nothing faults, traps or
hangs the GPU: the waits end by their own time limits (1 s, 0.4 s, 0.2 s).
"""

from __future__ import annotations

import pytest
import torch

from rwkv_tl_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which,bit", [(0, 1), (1, 2), (2, 4)], ids=["gemm", "persist", "scan"])
def test_bounded_wait_expires_and_is_reported(which, bit):
    lib = _lib.load()
    assert lib.rwkv_b200_device_error() == 0
    scratch = torch.zeros(8, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.rwkv_b200_wait_selftest(which, scratch.data_ptr(), stream))
    torch.cuda.synchronize()
    out = int(scratch[4])
    assert out != 0, "the bounded wait did not give up"
    if which == 1:
        assert out == 3, "both the grid barrier and the mbarrier wait must give up"
    assert lib.rwkv_b200_device_error() == bit
    assert lib.rwkv_b200_device_error() == 0  # cleared on read
    # the context is still usable: an ordinary GEMM call right after is correct
    g = torch.Generator(device="cuda").manual_seed(which)
    a = torch.randn(128, 256, generator=g, device="cuda").half()
    b = torch.randn(192, 256, generator=g, device="cuda").half()
    c = torch.empty(128, 192, dtype=torch.float16, device="cuda")
    prob = (_lib.GemmProblem * 1)()
    prob[0] = _lib.GemmProblem(a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 128, 192, 256,
                               256, 256, 192)
    _lib.check(lib.rwkv7_gemm_f16(prob, 1, _lib.EPI_STORE, stream))
    torch.cuda.synchronize()
    ref = a.float() @ b.float().T
    # fp32 accumulation, one fp16 rounding of results of magnitude ~16
    assert ((c.float() - ref).abs() <= 2e-3 * ref.abs() + 2e-2).all()
    assert lib.rwkv_b200_device_error() == 0


def test_wait_selftest_rejects_bad_arguments():
    lib = _lib.load()
    scratch = torch.zeros(8, dtype=torch.int32, device="cuda")
    assert lib.rwkv_b200_wait_selftest(7, scratch.data_ptr(), None) == _lib.RWKV_ERR_ARG
    assert lib.rwkv_b200_wait_selftest(0, None, None) == _lib.RWKV_ERR_ARG
