"""wkv7 DPLR kernels vs the CPU oracle recurrence (BASELINE config 1 shapes/inits)."""

from __future__ import annotations

import pytest
import torch

from oracle.rwkv7_oracle import RWKV7Oracle

from tests._util import rel_l2

pytestmark = pytest.mark.gpu


def _inputs(B, T, H, seed):
    """Config-1 inits: r,k,v ~ N(0,1); k_hat = k/|k|; a = sigmoid(N); w = exp(-0.606531 sigmoid(N));
    A = k_hat, B = -k_hat * a; S0 = 0.1 N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    r = torch.randn(B, T, H, 64, generator=g)
    k = torch.randn(B, T, H, 64, generator=g)
    v = torch.randn(B, T, H, 64, generator=g)
    a = torch.sigmoid(torch.randn(B, T, H, 64, generator=g))
    w = torch.exp(-0.606531 * torch.sigmoid(torch.randn(B, T, H, 64, generator=g)))
    kh = k / k.norm(dim=-1, keepdim=True)
    S0 = 0.1 * torch.randn(B, H, 64, 64, generator=g)
    h = lambda t: t.half()  # noqa: E731
    return h(r), h(w), h(k), h(v), h(kh), h(-kh * a), S0


def _ref(S0, r, w, k, v, A, B):
    """Serial recurrence in fp32 on the fp16-rounded inputs."""
    S = S0.clone()
    T = r.shape[1]
    ys = []
    for t in range(T):
        y, S = zip(*[RWKV7Oracle._wkv_step(S[b], r[b, t].float(), w[b, t].float(), k[b, t].float(),
                                           v[b, t].float(), A[b, t].float(), B[b, t].float())
                     for b in range(S.shape[0])])
        S = torch.stack(S)
        ys.append(torch.stack(y))
    return torch.stack(ys, 1), S


@pytest.mark.parametrize("B", [1, 8, 64])
def test_dplr_step_batched(B):
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    H = 16
    r, w, k, v, A, Bv, S0 = _inputs(B, 1, H, seed=B)
    yref, Sref = _ref(S0, r, w, k, v, A, Bv)
    dev = [t[:, 0].contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    S = S0.cuda().contiguous()
    y = torch.empty(B, H, 64, dtype=torch.float16, device="cuda")
    _lib.check(lib.rwkv7_dplr_step(S.data_ptr(), *[t.data_ptr() for t in dev], y.data_ptr(), B, H,
                                   torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rel_l2(S, Sref) < 1e-5
    assert (y.float().cpu() - yref[:, 0]).abs().max() <= 2e-3 * max(1.0, yref.abs().max())


@pytest.mark.parametrize("T", [1, 64, 1024])
def test_dplr_seq(T):
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    H = 16
    r, w, k, v, A, Bv, S0 = _inputs(1, T, H, seed=T)
    yref, Sref = _ref(S0, r, w, k, v, A, Bv)
    dev = [t[0].contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    S = S0[0].cuda().contiguous()
    y = torch.empty(T, H, 64, dtype=torch.float16, device="cuda")
    _lib.check(lib.rwkv7_dplr_seq(S.data_ptr(), *[t.data_ptr() for t in dev], y.data_ptr(), T, H,
                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rel_l2(S, Sref[0]) < 1e-4
    assert rel_l2(y.float(), yref[0]) < 2e-3


def test_dplr_rejects_bad_args():
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    rc = lib.rwkv7_dplr_step(None, None, None, None, None, None, None, None, 1, 16, None)
    assert rc == _lib.RWKV_ERR_ARG
    assert b"rwkv7_dplr_step" in lib.rwkv_b200_last_error()


def _batched_ref(S0, r, w, k, v, A, Bv):
    """Serial fp32 recurrence, batched over sequences: inputs [B, T, H, 64]."""
    S = S0.clone()
    ys = torch.empty(r.shape, dtype=torch.float32, device=S0.device)
    f = lambda t: t.float()  # noqa: E731
    r, w, k, v, A, Bv = map(f, (r, w, k, v, A, Bv))
    for t in range(r.shape[1]):
        sa = torch.einsum("bhvk,bhk->bhv", S, A[:, t])
        S = S * w[:, t, :, None, :] + sa[..., None] * Bv[:, t, :, None, :] + v[:, t, :, :, None] * k[:, t, :, None, :]
        ys[:, t] = torch.einsum("bhvk,bhk->bhv", S, r[:, t])
    return ys, S


@pytest.mark.parametrize("B,T", [(b, t) for b in (1, 8, 64) for t in (64, 1024, 4096)] + [(3, 37)])
def test_dplr_chunked_config1(B, T):
    """BASELINE config 1 sweep (H=16, B in {1, 8, 64}, T in {64, 1024, 4096}) through the
    chunk-parallel kernel; T=1 is the step kernel's test above. The serial fp32
    reference runs in torch, on the GPU for the large cases."""
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    H = 16
    r, w, k, v, A, Bv, S0 = _inputs(B, T, H, seed=B * 10000 + T)
    on = "cuda" if B * T > 8192 else "cpu"
    yref, Sref = _batched_ref(*(t.to(on) for t in (S0, r, w, k, v, A, Bv)))
    yref, Sref = yref.cpu(), Sref.cpu()
    dev = [t.contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    S = S0.cuda().contiguous()
    y = torch.empty(B, T, H, 64, dtype=torch.float16, device="cuda")
    nbytes = lib.rwkv7_dplr_chunked_workspace_bytes(B, T, H)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.rwkv7_dplr_chunked(S.data_ptr(), *[t.data_ptr() for t in dev], y.data_ptr(),
                                      B, T, H, ws.data_ptr(), nbytes,
                                      torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rel_l2(S, Sref) < 1e-4
    assert rel_l2(y.float(), yref) < 1e-3


@pytest.mark.parametrize("B", [1, 37, 256])
def test_wkv_gn_step_decode(B):
    """wkv7 step + GroupNorm + bonus + g gate (fused_dplr + fused_gn_rkrk + (y*g)),
    decode rounding points, against an fp64 torch restatement."""
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    H, C = 16, 1024
    r, w, k, v, A, Bv, S0 = _inputs(B, 1, H, seed=500 + B)
    g = torch.Generator().manual_seed(B)
    gate = torch.randn(B, C, generator=g).half()
    r_k = (0.1 * torch.randn(C, generator=g)).half()
    lnw = (1 + 0.1 * torch.randn(C, generator=g)).half()
    lnb = (0.1 * torch.randn(C, generator=g)).half()
    slots = torch.randperm(B, generator=g).to(torch.int32)
    S_slot = torch.empty_like(S0)
    S_slot[slots.long()] = S0  # sequence i lives in slot slots[i]
    vecs = [t[:, 0].reshape(B, C) for t in (r, w, k, v, A, Bv)]
    # reference (fp64, fp16 stores where the decode kernels store)
    d = lambda t: t.double()  # noqa: E731
    S = d(S0)
    rr, ww, kk, vv, aa, bb = (d(t).reshape(B, H, 64) for t in vecs)
    sa = torch.einsum("bhvk,bhk->bhv", S, aa)
    S = S * ww[:, :, None, :] + sa[..., None] * bb[:, :, None, :] + vv[..., None] * kk[:, :, None, :]
    y = torch.einsum("bhvk,bhk->bhv", S, rr).half().double()
    mean = y.mean(-1, keepdim=True)
    var = ((y - mean) ** 2).mean(-1, keepdim=True)
    yn = ((y - mean) / torch.sqrt(var + 64e-5)).reshape(B, C) * d(lnw) + d(lnb)
    rkrk = (rr * kk * d(r_k).reshape(H, 64)).sum(-1, keepdim=True)
    out = (yn + (rkrk * vv).reshape(B, C)).half().double() * d(gate)
    dev = [t.contiguous().cuda() for t in vecs]
    Sd = S_slot.cuda().contiguous()
    o = torch.empty(B, C, dtype=torch.float16, device="cuda")
    # keep every device tensor referenced until the kernel has run
    sl_d, g_d, rk_d, lw_d, lb_d = (t.cuda() for t in (slots, gate, r_k, lnw, lnb))
    _lib.check(lib.rwkv7_wkv_gn_step(Sd.data_ptr(), sl_d.data_ptr(), *[t.data_ptr() for t in dev],
                                     g_d.data_ptr(), rk_d.data_ptr(), lw_d.data_ptr(),
                                     lb_d.data_ptr(), o.data_ptr(), B, H, 0,
                                     torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rel_l2(Sd.cpu()[slots.long()], S.float()) < 1e-5
    assert rel_l2(o.float(), out) < 2e-3


@pytest.mark.parametrize("B,T", [(1, 4096), (8, 1024), (2, 257)])
def test_dplr_chunked_is_bit_reproducible(B, T):
    """The chunk-parallel wkv (tensor-core segment scan, segment pass, output correction)
    gives bit-identical outputs and states on repeated calls with the same inputs."""
    from rwkv_tl_b200 import _lib

    lib = _lib.load()
    H = 16
    r, w, k, v, A, Bv, S0 = _inputs(B, T, H, seed=B * 10000 + T + 1)
    dev = [t.contiguous().cuda() for t in (r, w, k, v, A, Bv)]
    nbytes = lib.rwkv7_dplr_chunked_workspace_bytes(B, T, H)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(5):
        S = S0.cuda().contiguous()
        y = torch.empty(B, T, H, 64, dtype=torch.float16, device="cuda")
        _lib.check(lib.rwkv7_dplr_chunked(S.data_ptr(), *[t.data_ptr() for t in dev],
                                          y.data_ptr(), B, T, H, ws.data_ptr(), nbytes,
                                          torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        outs.append((y, S))
    for y, S in outs[1:]:
        assert torch.equal(y, outs[0][0]) and torch.equal(S, outs[0][1])
