"""RWKV-7 weights in the B200 kernels' layout.

``RWKV7Weight(model_path, device=None, dtype=torch.float16)`` keeps the
reference's constructor (``src/rwkv_tl/weight.py:155-184``): ``torch.load`` the
checkpoint, cast every tensor to fp16, fold LN0 into the embedding, infer L
and C from the keys. Instead of the reference's transposed ``[in, out]``
copies it keeps the checkpoint's ``[out, in]`` orientation (contiguous along
the reduction dim for both the GEMV and the K-major tensor-core GEMM) and
packs per layer:

* ``w_rkv [3C, C]`` = receptance | key | value;
* ``w_lora_dn [288, C]`` = v1^T | w1^T | a1^T | g1^T (LoRA down, ranks 32/64/64/128);
* ``w_lora_up [288, C]`` = v2 | w2 | a2 | g2 (LoRA up, ``[r, C]`` as stored) and its
  K-major copy ``w_lora_up_t [C, 512]`` (v padded to 64, w and g repeated for the
  hi + lo activation split) for the tensor-core GEMM;
* ``mix6 [6, C]`` = x_r | x_w | x_k | x_v | x_a | x_g.

Weight preparation runs once at load with plain torch ops; only the forward
path is the CUDA library.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib

__all__ = ["RWKV7Weight"]

_RANKS = {"v": 32, "w": 64, "a": 64, "g": 128}


class RWKV7Weight:
    dtype: torch.dtype
    device: torch.device
    L: int
    C: int
    V: int

    def __init__(self, model_path: str | dict, device: str | torch.device | None = None,
                 dtype: torch.dtype = torch.float16):
        if dtype != torch.float16:
            raise ValueError("the B200 path computes in fp16 (dtype=torch.float16)")
        if isinstance(model_path, dict):
            W = model_path
        else:
            W = torch.load(model_path, map_location=device, weights_only=True)
        dev = torch.device(device) if device is not None else next(iter(W.values())).device
        W = {k: v.to(device=dev, dtype=dtype) for k, v in W.items() if isinstance(v, Tensor)}
        self.dtype, self.device = dtype, dev
        emb = W["emb.weight"]
        self.V, self.C = emb.shape
        self.L = 1 + max(int(k.split(".")[1]) for k in W if k.startswith("blocks."))
        C = self.C
        if C % 128:
            raise ValueError(f"n_embd must be a multiple of 128 (got {C})")
        # weight.py:175: LN0 folded into the embedding once (fp32 math, fp16 store)
        self.emb = F.layer_norm(emb.float(), (C,), W["blocks.0.ln0.weight"].float(),
                                W["blocks.0.ln0.bias"].float()).to(dtype).contiguous()
        self.head = W["head.weight"].contiguous()
        self.lnout_w = W["ln_out.weight"].contiguous()
        self.lnout_b = W["ln_out.bias"].contiguous()
        self.layers: list[dict[str, Tensor]] = []
        for i in range(self.L):
            p, a = f"blocks.{i}", f"blocks.{i}.att"
            for g, r in _RANKS.items():
                if W[f"{a}.{g}1"].shape != (C, r):
                    raise ValueError(f"{a}.{g}1 must be [{C}, {r}] (LoRA ranks v32 w64 a64 g128)")
            vec = lambda k: W[k].reshape(-1).contiguous()  # noqa: E731
            lay = {
                "ln1_w": vec(f"{p}.ln1.weight"), "ln1_b": vec(f"{p}.ln1.bias"),
                "ln2_w": vec(f"{p}.ln2.weight"), "ln2_b": vec(f"{p}.ln2.bias"),
                "mix6": torch.stack([vec(f"{a}.{n}") for n in
                                     ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")]).contiguous(),
                "w_rkv": torch.cat([W[f"{a}.receptance.weight"], W[f"{a}.key.weight"],
                                    W[f"{a}.value.weight"]], 0).contiguous(),
                "w_lora_dn": torch.cat([W[f"{a}.{g}1"].t() for g in "vwag"], 0).contiguous(),
                "w_lora_up": torch.cat([W[f"{a}.{g}2"] for g in "vwag"], 0).contiguous(),
                "w0": vec(f"{a}.w0"), "a0": vec(f"{a}.a0"), "v0": vec(f"{a}.v0"),
                "k_k": vec(f"{a}.k_k"), "k_a": vec(f"{a}.k_a"), "r_k": vec(f"{a}.r_k"),
                "lnx_w": vec(f"{a}.ln_x.weight"), "lnx_b": vec(f"{a}.ln_x.bias"),
                "w_o": W[f"{a}.output.weight"].contiguous(),
                "ffn_x_k": vec(f"{p}.ffn.x_k"),
                "w_fk": W[f"{p}.ffn.key.weight"].contiguous(),
                "w_fv": W[f"{p}.ffn.value.weight"].contiguous(),
            }
            # K-major LoRA up for the tensor-core GEMM: v padded from rank 32 to 64, w and g
            # repeated so that an activation carried as fp16 hi + lo is applied exactly
            zeros = torch.zeros(C, 32, dtype=dtype, device=dev)
            w2t, g2t = W[f"{a}.w2"].t(), W[f"{a}.g2"].t()
            lay["w_lora_up_t"] = torch.cat(
                [W[f"{a}.v2"].t(), zeros, w2t, w2t, W[f"{a}.a2"].t(), g2t, g2t], 1).contiguous()
            self.layers.append(lay)
        self._cmodel: _lib.Model | None = None

    @classmethod
    def from_state_dict(cls, sd: dict[str, Tensor], device=None) -> "RWKV7Weight":
        return cls(sd, device=device)

    @property
    def H(self) -> int:
        return self.C // 64

    def nbytes(self) -> int:
        n = self.emb.numel() + self.head.numel() + 2 * self.C
        n += sum(t.numel() for lay in self.layers for t in lay.values())
        return 2 * n

    def cmodel(self) -> _lib.Model:
        """ctypes ``rwkv7_model`` over these tensors (built once, cached)."""
        if self._cmodel is None:
            arr = (_lib.Layer * self.L)()
            for i, lay in enumerate(self.layers):
                for name, _ in _lib.Layer._fields_:
                    setattr(arr[i], name, lay[name].data_ptr())
            m = _lib.Model(self.L, self.C, self.V, 32, 64, 64, 128, self.emb.data_ptr(),
                           self.head.data_ptr(), self.lnout_w.data_ptr(), self.lnout_b.data_ptr(),
                           ctypes.cast(arr, ctypes.POINTER(_lib.Layer)))
            self._layer_arr = arr  # keep alive
            self._cmodel = m
        return self._cmodel
