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


def test_loader_bf16_pth_matches_reference_loader(tmp_path):
    """A bf16 ``.pth`` file through ``RWKV7Weight`` gives the tensors the reference's own
    loader gives (``src/rwkv_tl/weight.py:155-184``, fixture ``loader_bf16.pt`` made by
    running it): every cast and re-layout bit-exact, the LN0-folded embedding to within
    one fp16 rounding (fp32 reduction order of the LayerNorm)."""
    import torch

    from rwkv_tl_b200.synth import CONFIG_TINY, synth_checkpoint
    from rwkv_tl_b200.weight import RWKV7Weight
    from tests.conftest import GOLDEN

    ref = torch.load(GOLDEN / "loader_bf16.pt", weights_only=False)
    p = tmp_path / "tiny_bf16.pth"
    torch.save(synth_checkpoint(CONFIG_TINY, seed=3, dtype=torch.bfloat16), p)
    w = RWKV7Weight(str(p), device="cpu")
    assert w.emb.dtype == torch.float16 and w.L == len(ref["blocks"])
    d = (w.emb.float() - ref["emb"].float()).abs()
    ulp = torch.finfo(torch.float16).eps * ref["emb"].float().abs().clamp(min=2 ** -14)
    assert bool((d <= ulp).all()) and float((d > 0).float().mean()) < 0.01
    assert torch.equal(w.head, ref["head"])
    assert torch.equal(w.lnout_w, ref["ln_out"][0]) and torch.equal(w.lnout_b, ref["ln_out"][1])
    for lay, rb in zip(w.layers, ref["blocks"]):
        eq = lambda a, b: torch.equal(a, b.reshape(a.shape))  # noqa: E731
        assert eq(lay["w_rkv"], torch.cat([rb["rkvWt"][i].t() for i in range(3)], 0))
        assert eq(lay["w_o"], rb["oWt"].t()) and eq(lay["w_fk"], rb["kWt"].t())
        assert eq(lay["w_fv"], rb["vWt"].t())
        assert eq(lay["w_lora_dn"], torch.cat([rb[g + "1"].t() for g in "vwag"], 0))
        assert eq(lay["w_lora_up"], torch.cat([rb[g + "2"] for g in "vwag"], 0))
        assert eq(lay["mix6"], torch.stack([rb[n].reshape(-1) for n in
                                            ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")]))
        for ours, theirs in (("w0", "w0"), ("a0", "a0"), ("v0", "v0"), ("k_k", "k_k"),
                             ("k_a", "k_a"), ("r_k", "r_k"), ("ffn_x_k", "ffn_x_k")):
            assert eq(lay[ours], rb[theirs])
        for ours, theirs in (("ln1_w", ("ln1", 0)), ("ln1_b", ("ln1", 1)), ("ln2_w", ("ln2", 0)),
                             ("ln2_b", ("ln2", 1)), ("lnx_w", ("ln_x", 0)), ("lnx_b", ("ln_x", 1))):
            assert eq(lay[ours], rb[theirs[0]][theirs[1]])
