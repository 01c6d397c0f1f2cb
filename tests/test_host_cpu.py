"""Host-side logic that needs no GPU: state layout, weight packing, factory errors."""

from __future__ import annotations

import pytest
import torch

from rwkv_tl_b200 import BatchedState, RWKV7Weight, State, make_rwkv7
from rwkv_tl_b200.synth import CONFIG_TINY, synth_checkpoint


def test_state_layout_matches_reference():
    S = State(3, 128, 64, device="cpu")
    assert len(S) == 2 and len(S.tmix) == 3 and len(S.cmix) == 3
    assert S.tmix[0]["x"].shape == (128,) and S.tmix[0]["x"].dtype == torch.float16
    assert S.tmix[0]["rnn"].shape == (2, 64, 64) and S.tmix[0]["rnn"].dtype == torch.float32
    assert S.cmix[2]["x"].shape == (128,)
    S.tmix[1]["rnn"].fill_(3.0)
    assert S._rnn[1, 0].eq(3.0).all() and S.bound()
    S.reset()
    assert S._rnn.abs().sum() == 0
    S.tmix[0]["x"] = torch.zeros(128, dtype=torch.float16)
    assert not S.bound()


def test_batched_state_views_alias_storage():
    bs = BatchedState(2, 128, 4, device="cpu")
    v = bs[2]
    v.tmix[1]["rnn"][0, 0, 0] = 7.0
    v.cmix[0]["x"][5] = 1.5
    assert bs.rnn[1, 2, 0, 0, 0] == 7.0 and bs.cmix_x[0, 2, 5] == 1.5
    bs.reset([2])
    assert bs.rnn.abs().sum() == 0
    with pytest.raises(IndexError):
        bs[4]


def test_weight_packing_orientation():
    sd = synth_checkpoint(CONFIG_TINY, seed=3)
    w = RWKV7Weight(sd, device="cpu")
    C = CONFIG_TINY.n_embd
    lay = w.layers[1]
    a = "blocks.1.att"
    assert torch.equal(lay["w_rkv"][C:2 * C], sd[f"{a}.key.weight"].half())
    assert torch.equal(lay["w_lora_dn"][32:96], sd[f"{a}.w1"].t().half())
    assert torch.equal(lay["w_lora_up"][160:288], sd[f"{a}.g2"].half())
    assert torch.equal(lay["mix6"][4], sd[f"{a}.x_a"].reshape(-1).half())
    assert torch.equal(lay["r_k"], sd[f"{a}.r_k"].reshape(-1).half())
    ref = torch.nn.functional.layer_norm(sd["emb.weight"].half().float(), (C,))
    assert torch.equal(w.emb, ref.half())
    assert w.L == 2 and w.C == C and w.V == CONFIG_TINY.vocab


def test_weight_rejects_other_dtype_and_ranks():
    sd = synth_checkpoint(CONFIG_TINY, seed=3)
    with pytest.raises(ValueError):
        RWKV7Weight(sd, device="cpu", dtype=torch.bfloat16)
    sd["blocks.0.att.w1"] = torch.zeros(CONFIG_TINY.n_embd, 32)
    with pytest.raises(ValueError):
        RWKV7Weight(sd, device="cpu")


def test_factory_errors():
    with pytest.raises(ValueError):
        make_rwkv7(torch.device("cpu"), backend="b200")
    with pytest.raises(ValueError):
        make_rwkv7(torch.device("cuda"), backend="bogus")
    with pytest.raises(ValueError):
        make_rwkv7(torch.device("cuda"), backend="torch")


def test_synth_checkpoint_keys_and_init():
    sd = synth_checkpoint(CONFIG_TINY, seed=0)
    assert sd["blocks.1.att.r_k"].shape == (2, 64)
    assert sd["blocks.0.ffn.key.weight"].shape == (512, 128)
    w0 = sd["blocks.0.att.w0"]
    assert w0.min() >= -6 and w0.max() <= -1
    assert torch.equal(sd["blocks.0.att.k_a"], torch.ones(1, 1, 128))
    assert torch.equal(synth_checkpoint(CONFIG_TINY, seed=0)["head.weight"], sd["head.weight"])
