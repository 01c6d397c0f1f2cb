"""CPU oracle for the RWKV-7 forward hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` arm may import this module, and only as the checker or as
the timed CPU baseline. The product path (``rwkv_tl_b200``) never calls it and
has no CPU fallback.

It restates, in plain torch-on-CPU code written for this project, two
reference numerics of yuyi2439/rwkv-tl (paths relative to that project):

``mode="fp32"``
    The pure-torch model ``demo/rwkv7_torch.py`` (``time_mix`` :67-120,
    ``channel_mix`` :123-128, ``_dplr_rwkv`` :49-64, batched prefill
    :192-257), evaluated in fp32. This is the reference's CPU baseline.

``mode="fp16"``
    The reference's fp16 GPU model ``demo/_rwkv7_base.py`` with the TileLang
    kernels of ``src/rwkv_tl/kernels/*.py``: every value is computed in fp32
    and rounded to fp16 (``_r16``) exactly where the reference stores an fp16
    tensor. Decode follows the fused-kernel rounding points
    (``_rwkv7_base.py:153-206``, ``lerp.py:79-138``, ``gates.py:125-285``,
    ``dplr.py:45-172``); prefill follows the per-op torch rounding points of
    ``_rwkv7_base.py:223-310`` (each torch fp16 op rounds its result once).
    The wkv state stays fp32 in both.

Parity pins (``tests/test_oracle_golden.py``): ``fp32`` mode against golden
vectors produced by running ``demo.rwkv7_torch.RWKV7Torch`` itself, and
``fp16`` mode against vectors produced by running the reference's own fp16
model (``tests/golden/make_golden.py`` records how each file was made).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

__all__ = ["OracleWeights", "OracleState", "RWKV7Oracle"]

_INV_SQRT_E = 1.0 / math.sqrt(math.e)  # w = exp(-sigmoid(.)/sqrt(e)), gates.py:27
_SQRT_E_PREFILL = 1.6487212707001282  # literal divisor, _rwkv7_base.py:247
GN_EPS = 64e-5  # dplr.py:103, _rwkv7_base.py:264
LN_EPS = 1e-5  # F.layer_norm default, weight.py:15


def _r16(x: Tensor) -> Tensor:
    """Round to fp16 precision and back to the compute dtype (one fp16 store)."""
    return x.to(torch.float16).to(x.dtype)


class OracleWeights:
    """Reference-format checkpoint -> per-layer fp32 tensors.

    Mirrors ``RWKV7Weight`` (``src/rwkv_tl/weight.py:140-184``): cast every
    tensor to the model dtype (fp16 for ``mode="fp16"``; kept as fp32 values
    after rounding), fold LN0 into the embedding (``weight.py:175``), and keep
    projections in ``[in, out]`` orientation (``weight.py:98-106,124-126``).
    """

    def __init__(self, sd: dict[str, Tensor], mode: str = "fp16",
                 compute_dtype: torch.dtype = torch.float32):
        if mode not in ("fp16", "fp32"):
            raise ValueError(mode)
        self.mode = mode
        self.compute_dtype = compute_dtype
        q = _r16 if mode == "fp16" else (lambda t: t)
        W = {k: q(v.detach().to("cpu", compute_dtype)) for k, v in sd.items()}
        self.C = W["emb.weight"].shape[1]
        self.V = W["emb.weight"].shape[0]
        self.L = 1 + max(int(k.split(".")[1]) for k in W if k.startswith("blocks."))
        self.H = self.C // 64
        ln = lambda x, p: F.layer_norm(x, (x.shape[-1],), W[p + ".weight"], W[p + ".bias"], LN_EPS)
        # weight.py:175 -- LN0 applied once to the (model-dtype) embedding.
        self.emb = q(ln(W["emb.weight"], "blocks.0.ln0"))
        self.head = W["head.weight"]  # [V, C]
        self.ln_out = (W["ln_out.weight"], W["ln_out.bias"])
        self.blocks = []
        for i in range(self.L):
            p = f"blocks.{i}"
            a = p + ".att"
            blk = {
                "ln1": (W[p + ".ln1.weight"], W[p + ".ln1.bias"]),
                "ln2": (W[p + ".ln2.weight"], W[p + ".ln2.bias"]),
                "ln_x": (W[a + ".ln_x.weight"], W[a + ".ln_x.bias"]),
                "r_k": W[a + ".r_k"],  # [H, 64]
                "Wr": W[a + ".receptance.weight"].t(),  # [in, out]
                "Wk": W[a + ".key.weight"].t(),
                "Wv": W[a + ".value.weight"].t(),
                "Wo": W[a + ".output.weight"].t(),
                "ffn_x_k": W[p + ".ffn.x_k"].reshape(-1),
                "Wfk": W[p + ".ffn.key.weight"].t(),  # [C, 4C]
                "Wfv": W[p + ".ffn.value.weight"].t(),  # [4C, C]
            }
            for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "w0", "a0", "v0", "k_k", "k_a"):
                blk[n] = W[f"{a}.{n}"].reshape(-1)
            for n in ("w1", "w2", "a1", "a2", "v1", "v2", "g1", "g2"):
                blk[n] = W[f"{a}.{n}"]
            self.blocks.append(blk)


class OracleState:
    """Per-sequence state with the layout of ``src/rwkv_tl/state.py:31-44``."""

    def __init__(self, L: int, C: int, *, dtype: torch.dtype = torch.float32):
        H = C // 64
        self.tmix_x = [torch.zeros(C, dtype=dtype) for _ in range(L)]
        self.rnn = [torch.zeros(H, 64, 64, dtype=dtype) for _ in range(L)]
        self.cmix_x = [torch.zeros(C, dtype=dtype) for _ in range(L)]

    def clone(self) -> "OracleState":
        s = OracleState.__new__(OracleState)
        s.tmix_x = [t.clone() for t in self.tmix_x]
        s.rnn = [t.clone() for t in self.rnn]
        s.cmix_x = [t.clone() for t in self.cmix_x]
        return s


class RWKV7Oracle:
    """CPU restatement of the reference forward, ``decode``/``prefill``/``forward``."""

    def __init__(self, w: OracleWeights):
        self.w = w
        self.mode = w.mode
        self.q = _r16 if self.mode == "fp16" else (lambda t: t)

    # ------------------------------------------------------------------ #
    # shared pieces
    # ------------------------------------------------------------------ #
    def _ln(self, x: Tensor, wb) -> Tensor:
        return self.q(F.layer_norm(x, (x.shape[-1],), wb[0], wb[1], LN_EPS))

    @staticmethod
    def _wkv_step(S: Tensor, r, w, k, v, A, B) -> tuple[Tensor, Tensor]:
        """One wkv7 DPLR step on [H,64,64] fp32 state (rows v, columns k).

        ``demo/rwkv7_torch.py:49-64`` / ``kernels/dplr.py:126-172``:
        sa[v] = sum_a S[v,a] A[a]; S'[v,k] = S[v,k] w[k] + sa[v] B[k] + v[v] k[k];
        y[v] = sum_k S'[v,k] r[k].
        """
        sa = torch.einsum("hva,ha->hv", S, A)
        S_new = S * w[:, None, :] + sa[:, :, None] * B[:, None, :] + v[:, :, None] * k[:, None, :]
        y = torch.einsum("hvk,hk->hv", S_new, r)
        return y, S_new

    # ------------------------------------------------------------------ #
    # decode (T = 1)
    # ------------------------------------------------------------------ #
    def decode(self, token: int, S: OracleState) -> Tensor:
        """``RWKV7Base.decode`` (``demo/_rwkv7_base.py:74-87``) / ``RWKV7Torch.decode``."""
        w, q = self.w, self.q
        x = w.emb[int(token)].clone()
        v_first = None
        for i, b in enumerate(w.blocks):
            x, v_first = self._tmix_decode(i, b, x, v_first, S)
            x = self._cmix_decode(i, b, x, S)
        x = self._ln(x, w.ln_out)
        return q(w.head @ x)

    def _tmix_decode(self, i, b, x0, v_first, S):
        q, H = self.q, self.w.H
        x = self._ln(x0, b["ln1"])
        prev = S.tmix_x[i]
        if self.mode == "fp16":
            # lerp.py:106-114: diff in fp16, x + mu*diff as one fused fp16 fma
            diff = q(prev - x)
            mix = {n: q(x + b[n] * diff) for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")}
        else:
            mix = {n: x + b[n] * (prev - x) for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")}
        S.tmix_x[i] = x.clone()
        xr, xw, xk, xv, xa, xg = (mix[n] for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"))
        r, k, v = q(xr @ b["Wr"]), q(xk @ b["Wk"]), q(xv @ b["Wv"])
        if self.mode == "fp16":
            # gates.py:215-285 (rank GEMV, fp16 store) then gates.py:125-213
            vr, wr, ar, gr = q(xv @ b["v1"]), q(xw @ b["w1"]), q(xa @ b["a1"]), q(xg @ b["g1"])
            vf = v if v_first is None else v_first
            if v_first is None:
                v_first = v
            v12 = vr @ b["v2"]
            w12 = torch.tanh(wr) @ b["w2"]
            a12 = ar @ b["a2"]
            g12 = torch.sigmoid(gr) @ b["g2"]
            v = q(v + torch.sigmoid(b["v0"] + v12) * (vf - v))
            wd = q(torch.exp(-torch.sigmoid(b["w0"] + w12) * _INV_SQRT_E))
            a32 = torch.sigmoid(b["a0"] + a12)
            a = q(a32)
            kk = q(k * b["k_k"])
            k = q(k + b["k_a"] * (k * a32 - k))
            g = q(g12)
            # dplr.py:45-71 l2norm + B = -kk_hat * a
            kk = kk.reshape(H, 64)
            den = torch.clamp(torch.sqrt((kk * kk).sum(-1, keepdim=True)), min=1e-12)
            kn32 = kk / den
            A = q(kn32)
            B = q(-(kn32 * a.reshape(H, 64)))
        else:
            if v_first is None:
                v_first = v
            else:
                v = v + torch.sigmoid(b["v0"] + xv @ b["v1"] @ b["v2"]) * (v_first - v)
            wd = torch.exp(-torch.sigmoid(b["w0"] + torch.tanh(xw @ b["w1"]) @ b["w2"]) / (math.e ** 0.5))
            a = torch.sigmoid(b["a0"] + xa @ b["a1"] @ b["a2"])
            kk = k * b["k_k"]
            k = k + b["k_a"] * (k * a - k)
            kk = kk.reshape(H, 64)
            kn = kk / torch.clamp(torch.sqrt((kk * kk).sum(-1, keepdim=True)), min=1e-12)
            A, B = kn, -kn * a.reshape(H, 64)
            g = torch.sigmoid(xg @ b["g1"]) @ b["g2"]
        rh, wh, kh, vh = (t.reshape(H, 64) for t in (r, wd, k, v))
        y, S.rnn[i] = self._wkv_step(S.rnn[i], rh, wh, kh, vh, A, B)
        y = q(y)
        # dplr.py:73-124 GroupNorm(eps 64e-5) + (sum r*k*r_k) * v
        mean = y.mean(-1, keepdim=True)
        var = ((y - mean) ** 2).mean(-1, keepdim=True)
        yn = (y - mean) / torch.sqrt(var + GN_EPS)
        yn = yn.reshape(-1) * b["ln_x"][0] + b["ln_x"][1]
        rkrk = (rh * kh * b["r_k"]).sum(-1, keepdim=True)
        y = q(yn + (rkrk * vh).reshape(-1))
        out = q(q(y * g) @ b["Wo"])
        return q(x0 + out), v_first

    def _cmix_decode(self, i, b, x0, S):
        q = self.q
        x = self._ln(x0, b["ln2"])
        prev = S.cmix_x[i]
        if self.mode == "fp16":
            xk = q(x + b["ffn_x_k"] * q(prev - x))  # lerp.py:118-138 (fma)
        else:
            xk = x + b["ffn_x_k"] * (prev - x)
        S.cmix_x[i] = x.clone()
        h = q(xk @ b["Wfk"])
        h = q(torch.relu(h) ** 2)
        return q(x0 + q(h @ b["Wfv"]))

    # ------------------------------------------------------------------ #
    # prefill (T > 1): per-op rounding of the torch fp16 prefill path
    # ------------------------------------------------------------------ #
    def prefill(self, tokens, S: OracleState) -> None:
        """``RWKV7Base.prefill`` (``demo/_rwkv7_base.py:89-98``); state only, no logits."""
        tokens = torch.as_tensor(tokens).reshape(-1)
        if tokens.numel() == 0:
            raise RuntimeError("prefill received an empty token sequence")
        w = self.w
        x = w.emb[tokens].clone()
        v_first = None
        for i, b in enumerate(w.blocks):
            x, v_first = self._tmix_prefill(i, b, x, v_first, S)
            x = self._cmix_prefill(i, b, x, S)

    def _tmix_prefill(self, i, b, x0, v_first, S):
        q, H = self.q, self.w.H
        T = x0.shape[0]
        x = self._ln(x0, b["ln1"])
        prev = torch.cat([S.tmix_x[i][None], x[:-1]], 0)
        diff = q(prev - x)
        mix = {n: q(x + q(b[n] * diff)) for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")}
        S.tmix_x[i] = x[-1].clone()
        xr, xw, xk, xv, xa, xg = (mix[n] for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"))
        r, k, v = q(xr @ b["Wr"]), q(xk @ b["Wk"]), q(xv @ b["Wv"])
        if v_first is None:
            v_first = v
        else:
            v12 = q(q(xv @ b["v1"]) @ b["v2"])
            v = q(v + q(q(torch.sigmoid(q(b["v0"] + v12))) * q(v_first - v)))
        w12 = q(q(torch.tanh(q(xw @ b["w1"]))) @ b["w2"])
        wd = q(torch.exp(q(-q(torch.sigmoid(q(b["w0"] + w12))) / _SQRT_E_PREFILL)))
        a = q(torch.sigmoid(q(b["a0"] + q(q(xa @ b["a1"]) @ b["a2"]))))
        kk = q(k * b["k_k"])
        k = q(k + q(b["k_a"] * q(q(k * a) - k)))
        r3, w3, k3, v3, kk3, a3 = (t.reshape(T, H, 64) for t in (r, wd, k, v, kk, a))
        den = q(torch.sqrt(q(q(kk3 * kk3).sum(-1, keepdim=True))))
        kn = q(kk3 / torch.clamp(den, min=1e-12))
        B = q(-kn * a3)
        y = torch.empty(T, H, 64, dtype=x0.dtype)
        St = S.rnn[i]
        for t in range(T):
            yt, St = self._wkv_step(St, r3[t], w3[t], k3[t], v3[t], kn[t], B[t])
            y[t] = q(yt)
        S.rnn[i] = St
        mean = y.mean(-1, keepdim=True)
        var = ((y - mean) ** 2).mean(-1, keepdim=True)
        yn = (y - mean) / torch.sqrt(var + GN_EPS)
        yn = q(yn.reshape(T, -1) * b["ln_x"][0] + b["ln_x"][1]).reshape(T, H, 64)
        rkrk = q(q(q(r3 * k3) * b["r_k"]).sum(-1, keepdim=True))
        yo = q(yn + q(rkrk * v3)).reshape(T, -1)
        g = q(q(torch.sigmoid(q(xg @ b["g1"]))) @ b["g2"])
        return q(x0 + q(q(yo * g) @ b["Wo"])), v_first

    def _cmix_prefill(self, i, b, x0, S):
        q = self.q
        x = self._ln(x0, b["ln2"])
        prev = torch.cat([S.cmix_x[i][None], x[:-1]], 0)
        xk = q(x + q(b["ffn_x_k"] * q(prev - x)))
        S.cmix_x[i] = x[-1].clone()
        h = q(xk @ b["Wfk"])
        h = q(torch.relu(h) ** 2)
        return q(x0 + q(h @ b["Wfv"]))

    # ------------------------------------------------------------------ #
    def forward(self, tokens, S: OracleState) -> Tensor:
        """``RWKV7Model.forward`` (``demo/_rwkv7_abc.py:74-89``)."""
        tokens = torch.as_tensor(tokens).reshape(-1)
        if tokens.numel() > 1:
            self.prefill(tokens[:-1], S)
        return self.decode(int(tokens[-1]), S)

    def generate_greedy(self, prompt, n: int, S: OracleState) -> tuple[list[int], Tensor]:
        """Prompt via ``forward`` then ``n-1`` more greedy decode steps (argmax)."""
        logits = self.forward(prompt, S)
        out = []
        for step in range(n):
            tok = int(torch.argmax(logits))
            out.append(tok)
            if step + 1 < n:
                logits = self.decode(tok, S)
        return out, logits
