"""Grouped fp16 GEMM + epilogues vs a plain torch fp32 reference."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def gemm_kernel():
    """Every case runs on the tcgen05 kernels; afterwards no bounded wait may have expired."""
    yield "tc"
    from rwkv_tl_b200 import _lib

    torch.cuda.synchronize()
    assert _lib.load().rwkv_b200_device_error() == 0


def _run(problems, epi):
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    arr = (_lib.GemmProblem * len(problems))()
    for i, (A, B, C, R) in enumerate(problems):
        M, K = A.shape
        N = B.shape[0]
        arr[i] = _lib.GemmProblem(A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                  0 if R is None else R.data_ptr(), M, N, K, A.stride(0),
                                  B.stride(0), C.stride(0))
    _lib.check(lib.rwkv7_gemm_f16(arr, len(problems), epi, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,N,K", [(1, 3072, 1024), (7, 288, 1024), (130, 1024, 4096),
                                   (256, 65536, 1024), (4096, 4096, 1024), (33, 32, 64), (300, 1000, 128),
                                   (256, 3072, 1024), (64, 1024, 4096), (256, 160, 1024),
                                   (130, 256, 96), (5, 64, 32), (1000, 1280, 160), (256, 520, 1056)])
def test_gemm_store(M, N, K):
    """K % 64 == 32 included (96, 32, 160, 1056): the last K-block reads zeros past K."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    C = torch.empty(M, N, device="cuda", dtype=torch.float16)
    _run([(A, B, C, None)], 0)
    ref = A.float() @ B.float().t()
    assert (C.float() - ref).abs().max() <= 2e-3 * ref.abs().max() + 1e-3


def test_gemm_grouped_epilogues():
    g = torch.Generator(device="cuda").manual_seed(3)
    M, K = 100, 1024
    As = [torch.randn(M, K, device="cuda", generator=g).half() for _ in range(3)]
    Bs = [(torch.randn(n, K, device="cuda", generator=g) / 32).half() for n in (32, 64, 128)]
    out = torch.zeros(M, 288, device="cuda", dtype=torch.float16)
    probs = [(As[0], Bs[0], out[:, 0:32], None), (As[1], Bs[1], out[:, 32:96], None),
             (As[2], Bs[2], out[:, 96:224], None)]
    _run(probs, 0)
    for (A, B, C, _) in probs:
        ref = A.float() @ B.float().t()
        assert (C.float() - ref).abs().max() < 1e-2
    # residual and relu^2 epilogues
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = (torch.randn(256, K, device="cuda", generator=g) / 32).half()
    R = torch.randn(M, 256, device="cuda", generator=g).half()
    C = torch.empty(M, 256, device="cuda", dtype=torch.float16)
    _run([(A, B, C, R)], 1)
    acc = (A.float() @ B.float().t()).half().float()
    assert (C.float() - (R.float() + acc)).abs().max() < 1e-2
    _run([(A, B, C, None)], 2)
    assert (C.float() - torch.relu(acc) ** 2).abs().max() < 2e-2 * (acc.abs().max() ** 2)


@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_gemm_large_grouped_ragged_epilogues(epi, gemm_kernel):
    """Large grouped problems (the persistent 128 x 256-tile kernel on the tcgen05 path):
    ragged M and N edges, every epilogue, two problems of different N in one launch."""
    g = torch.Generator(device="cuda").manual_seed(40 + epi)
    M, K = 1000, 1024
    A = [torch.randn(M, K, device="cuda", generator=g).half() for _ in range(2)]
    B = [(torch.randn(n, K, device="cuda", generator=g) / 32).half() for n in (1280, 1100)]
    R = [torch.randn(M, n, device="cuda", generator=g).half() if epi == 1 else None
         for n in (1280, 1100)]
    dt = torch.float32 if epi == 3 else torch.float16
    C = [torch.full((M, n), 7.0, device="cuda", dtype=dt) for n in (1280, 1100)]
    _run([(A[i], B[i], C[i], R[i]) for i in range(2)], epi)
    for i in range(2):
        acc = A[i].float() @ B[i].float().t()
        if epi == 0:
            ref = acc.half().float()
        elif epi == 1:
            ref = (R[i].float() + acc.half().float()).half().float()
        elif epi == 2:
            ref = (torch.relu(acc.half().float()) ** 2).half().float()
        else:
            ref = acc
        err = (C[i].float() - ref).abs().max()
        assert err <= 2e-3 * ref.abs().max() + 1e-3, (i, float(err))
