"""torch.ops.rwkv_b200 registration: schemas, Meta (shape) implementations used by
torch.compile / fake-tensor tracing, and no CPU fallback (the dispatcher refuses)."""

from __future__ import annotations

import pytest
import torch

import rwkv_tl_b200.ops as ops

OPS = ("fused_dplr", "fused_dplr_T", "wkv_gn_step", "gemm_f16")


def test_ops_registered_with_reference_style_schemas():
    ns = getattr(torch.ops, ops.NAMESPACE)
    for name in OPS:
        schema = str(getattr(ns, name).default._schema)
        assert schema.startswith(f"{ops.NAMESPACE}::{name}(")
    # in-place state declared like the reference's rwkv_tl::fused_dplr
    assert "Tensor(a!) S" in str(torch.ops.rwkv_b200.fused_dplr.default._schema)
    assert "Tensor(a!) S" in str(torch.ops.rwkv_b200.fused_dplr_T.default._schema)


def _vec(*shape, dtype=torch.float16, device="meta"):
    return torch.empty(*shape, dtype=dtype, device=device)


def test_meta_shapes():
    H = 16
    S = _vec(4, H, 64, 64, dtype=torch.float32)
    R = _vec(4, H, 64)
    y = torch.ops.rwkv_b200.fused_dplr(S, R, R, R, R, R, R)
    assert y.shape == R.shape and y.dtype == torch.float16 and y.device.type == "meta"
    RT = _vec(4, 100, H, 64)
    assert torch.ops.rwkv_b200.fused_dplr_T(S, RT, RT, RT, RT, RT, RT).shape == RT.shape
    r = _vec(4, H * 64)
    c = _vec(H * 64)
    assert torch.ops.rwkv_b200.wkv_gn_step(S, r, r, r, r, r, r, r, c, c, c, 0).shape == r.shape
    A, B = _vec(256, 1024), _vec(3072, 1024)
    out = torch.ops.rwkv_b200.gemm_f16(A, B, None, ops.EPI_STORE)
    assert out.shape == (256, 3072) and out.dtype == torch.float16
    assert torch.ops.rwkv_b200.gemm_f16(A, B, None, ops.EPI_STORE_F32).dtype == torch.float32


def test_fake_tensor_tracing_records_the_ops():
    from torch.fx.experimental.proxy_tensor import make_fx

    def step(S, r, w, k, v, a, b, Wo):
        y = torch.ops.rwkv_b200.fused_dplr(S, r, w, k, v, a, b)
        return torch.ops.rwkv_b200.gemm_f16(y.reshape(1, -1), Wo, None, ops.EPI_STORE)

    H = 2
    S = _vec(1, H, 64, 64, dtype=torch.float32)
    vs = [_vec(1, H, 64) for _ in range(6)]
    gm = make_fx(step, tracing_mode="fake")(S, *vs, _vec(32, H * 64))
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert any("rwkv_b200.fused_dplr" in t for t in targets)
    assert any("rwkv_b200.gemm_f16" in t for t in targets)


def test_no_cpu_fallback():
    S = torch.zeros(1, 1, 64, 64)
    R = torch.zeros(1, 1, 64, dtype=torch.float16)
    with pytest.raises(NotImplementedError):
        torch.ops.rwkv_b200.fused_dplr(S, R, R, R, R, R, R)
    with pytest.raises(NotImplementedError):
        torch.ops.rwkv_b200.gemm_f16(torch.zeros(2, 64, dtype=torch.float16),
                                     torch.zeros(4, 64, dtype=torch.float16), None, 0)
