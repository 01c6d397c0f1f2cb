"""torch.ops.rwkv_b200 on the GPU: each op against the CPU oracle recurrence / torch,
and under torch.compile (fullgraph, aot_eager: dynamo + fake-tensor tracing through
the Meta implementations, the CUDA kernels at run time)."""

from __future__ import annotations

import pytest
import torch

import rwkv_tl_b200.ops as ops
from tests._util import rel_l2
from tests.test_wkv_gpu import _inputs, _ref

pytestmark = pytest.mark.gpu


def test_fused_dplr_op_matches_oracle():
    B, H = 8, 16
    r, w, k, v, A, Bv, S0 = _inputs(B, 1, H, seed=71)
    yref, Sref = _ref(S0, r, w, k, v, A, Bv)
    S = S0.cuda().contiguous()
    y = torch.ops.rwkv_b200.fused_dplr(S, *[t[:, 0].contiguous().cuda() for t in (r, w, k, v, A, Bv)])
    torch.cuda.synchronize()
    assert y.shape == (B, H, 64) and y.dtype == torch.float16
    assert rel_l2(S, Sref) < 1e-5
    assert (y.float().cpu() - yref[:, 0]).abs().max() <= 2e-3 * max(1.0, yref.abs().max())


def test_fused_dplr_T_op_matches_oracle():
    B, T, H = 2, 100, 16
    r, w, k, v, A, Bv, S0 = _inputs(B, T, H, seed=72)
    yref, Sref = _ref(S0, r, w, k, v, A, Bv)
    S = S0.cuda().contiguous()
    y = torch.ops.rwkv_b200.fused_dplr_T(S, *[t.contiguous().cuda() for t in (r, w, k, v, A, Bv)])
    torch.cuda.synchronize()
    assert y.shape == (B, T, H, 64)
    assert rel_l2(S, Sref) < 1e-4
    assert rel_l2(y.float(), yref) < 1e-3


@pytest.mark.parametrize("epi", [ops.EPI_STORE, ops.EPI_RESID, ops.EPI_RELUSQ, ops.EPI_STORE_F32])
def test_gemm_f16_op_matches_torch(epi):
    g = torch.Generator().manual_seed(epi)
    M, N, K = 96, 320, 512
    A = (torch.randn(M, K, generator=g) / K ** 0.5).half().cuda()
    Bm = torch.randn(N, K, generator=g).half().cuda()
    R = torch.randn(M, N, generator=g).half().cuda() if epi == ops.EPI_RESID else None
    out = torch.ops.rwkv_b200.gemm_f16(A, Bm, R, epi)
    acc = A.float() @ Bm.float().t()
    if epi == ops.EPI_STORE_F32:
        ref = acc
    elif epi == ops.EPI_RESID:
        ref = (R.float() + acc.half().float()).half().float()
    elif epi == ops.EPI_RELUSQ:
        ref = (torch.relu(acc.half().float()) ** 2).half().float()
    else:
        ref = acc.half().float()
    assert rel_l2(out.float(), ref) < 2e-3


def test_wkv_gn_step_op_matches_c_abi():
    from rwkv_tl_b200 import _lib

    B, H, C = 16, 16, 1024
    r, w, k, v, A, Bv, S0 = _inputs(B, 1, H, seed=73)
    g = torch.Generator().manual_seed(73)
    vecs = [t[:, 0].reshape(B, C).contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    gate = torch.randn(B, C, generator=g).half().cuda()
    r_k, lnw, lnb = ((0.1 * torch.randn(C, generator=g)).half().cuda() for _ in range(3))
    S1, S2 = S0.cuda().contiguous(), S0.cuda().contiguous()
    out = torch.ops.rwkv_b200.wkv_gn_step(S1, *vecs, gate, r_k, lnw, lnb, 0)
    ref = torch.empty_like(out)
    lib = _lib.load()
    _lib.check(lib.rwkv7_wkv_gn_step(S2.data_ptr(), None, *[t.data_ptr() for t in vecs],
                                     gate.data_ptr(), r_k.data_ptr(), lnw.data_ptr(),
                                     lnb.data_ptr(), ref.data_ptr(), B, H, 0,
                                     torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(S1, S2)


def test_ops_under_torch_compile():
    B, H = 4, 16
    r, w, k, v, A, Bv, S0 = _inputs(B, 1, H, seed=74)
    xs = [t[:, 0].contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    Wo = (torch.randn(256, H * 64) / 32).half().cuda()

    def step(S, r, w, k, v, a, b):
        y = torch.ops.rwkv_b200.fused_dplr(S, r, w, k, v, a, b)
        return torch.ops.rwkv_b200.gemm_f16(y.reshape(B, H * 64), Wo, None, ops.EPI_STORE) * 2

    S_eager, S_comp = S0.cuda().contiguous(), S0.cuda().contiguous()
    ref = step(S_eager, *xs)
    out = torch.compile(step, backend="aot_eager", fullgraph=True)(S_comp, *xs)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.equal(S_comp, S_eager)  # the in-place state update survives compilation


def test_ops_reject_bad_inputs():
    S = torch.zeros(1, 16, 64, 64, device="cuda")
    R = torch.zeros(1, 16, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="fp32"):
        torch.ops.rwkv_b200.fused_dplr(S.half(), R, R, R, R, R, R)
    with pytest.raises(RuntimeError, match="n \\* H \\* 64"):
        torch.ops.rwkv_b200.fused_dplr(S, R[:, :8], R, R, R, R, R)
    with pytest.raises(RuntimeError, match="gemm_f16"):
        torch.ops.rwkv_b200.gemm_f16(R.reshape(16, 64), R.reshape(16, 64)[:, :32].contiguous(),
                                     None, 0)
