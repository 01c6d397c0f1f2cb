"""End-to-end parity of the B200 model against the fp16 CPU oracle.

Mirrors the reference's ``test/test_forward.py`` cases (decode per token,
prefill + last-token decode) on seeded synthetic checkpoints, at the north
star's tolerance (logits max-abs 2e-2, relative-L2 1e-3; wkv state relative
1e-3; greedy argmax), plus the batched (many-sequence) entry points.
"""

from __future__ import annotations

import pytest
import torch

from rwkv_tl_b200 import BatchedState, RWKV7B200, RWKV7Weight, State, make_rwkv7
from rwkv_tl_b200.synth import CONFIG_0_1B, CONFIG_0_4B, CONFIG_TINY, ModelConfig, synth_checkpoint
from tests._util import OraclePair, assert_logits_close, assert_state_close, gpu_state_to_oracle

pytestmark = pytest.mark.gpu

_CACHE: dict = {}


def _pair(cfg, seed):
    key = (cfg, seed)
    if key not in _CACHE:
        sd = synth_checkpoint(cfg, seed=seed)
        w = RWKV7Weight(sd, device="cuda")
        _CACHE.clear()
        _CACHE[key] = (RWKV7B200(w), OraclePair(sd))
    return _CACHE[key]


def _tokens(n, V, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (n,), generator=g).tolist()


def test_one_layer_strict_north_star_bar():
    """A 1-layer 0.1B-width model sits above the fp16 noise floor: hold it to the
    north star's absolute bar (max-abs 2e-2, rel-L2 1e-3, state rel 1e-3)."""
    m, o = _pair(ModelConfig(n_layer=1, n_embd=768, vocab=4096), 2)
    S, So = State(m.L, m.C, 64, device="cuda"), o.state()
    toks = _tokens(24, 4096, 9)
    lg, S = m.forward(torch.tensor(toks[:16], device="cuda"), S)
    assert_logits_close(lg.float(), o.forward(toks[:16], So), "1-layer forward", strict=True)
    for i, t in enumerate(toks[16:]):
        lg, S = m.decode(torch.tensor([t], device="cuda"), S)
        assert_logits_close(lg.float(), o.decode(t, So), f"1-layer decode {i}", strict=True)
    assert_state_close(S, So, "1-layer", strict=True)


def test_tiny_decode_per_token():
    m, o = _pair(CONFIG_TINY, 1)
    S, So = State(m.L, m.C, 64, device="cuda"), o.state()
    for i, t in enumerate(_tokens(12, CONFIG_TINY.vocab, 0)):
        lg, S = m.decode(torch.tensor([t], device="cuda"), S)
        assert_logits_close(lg.float(), o.decode(t, So), f"step {i}")
    assert_state_close(S, So, "tiny decode")


def test_tiny_forward_prefill_then_decode():
    m, o = _pair(CONFIG_TINY, 1)
    toks = _tokens(33, CONFIG_TINY.vocab, 1)
    S, So = State(m.L, m.C, 64, device="cuda"), o.state()
    lg, S = m.forward(torch.tensor(toks, device="cuda"), S)
    assert_logits_close(lg.float(), o.forward(toks, So), "forward")
    assert_state_close(S, So, "tiny forward")


def test_prefill_chunking_matches_single_call():
    m, _ = _pair(CONFIG_TINY, 1)
    toks = torch.tensor(_tokens(50, CONFIG_TINY.vocab, 2), device="cuda")
    S1 = State(m.L, m.C, 64, device="cuda")
    m.prefill(toks, S1)
    m2 = RWKV7B200(m.w, max_rows=16)
    S2 = State(m.L, m.C, 64, device="cuda")
    m2.prefill(toks, S2)
    # chunks of 16 rows take the per-token wkv, the single call the chunked one
    for a, b in zip(S1.tmix, S2.tmix):
        assert ((a["rnn"] - b["rnn"]).norm() / a["rnn"].norm()) < 1e-3
        assert (a["x"].float() - b["x"].float()).abs().max() < 1e-2


def test_cfg0_greedy_0p1b():
    """BASELINE config 0 workload on the GPU path: 0.1B, 8-token prompt, 16 greedy steps."""
    m, o = _pair(CONFIG_0_1B, 0)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 65536, (8,), generator=g).tolist()
    S, So = State(m.L, m.C, 64, device="cuda"), o.state()
    lg, S = m.forward(torch.tensor(prompt, device="cuda"), S)
    olg = o.forward(prompt, So)
    assert_logits_close(lg.float(), olg, "prompt")
    agree = 0
    for step in range(16):
        tok = int(olg[0].argmax())
        agree += int(lg.float().argmax()) == tok
        if step == 15:
            break
        lg, S = m.decode(torch.tensor([tok], device="cuda"), S)
        olg = o.decode(tok, So)
        assert_logits_close(lg.float(), olg, f"greedy step {step}")
    assert agree >= 16  # >= 99% of 16 steps
    assert_state_close(S, So, "cfg0 state")


def test_0p4b_prefill64_and_decode():
    m, o = _pair(CONFIG_0_4B, 0)
    toks = _tokens(64, 65536, 3)
    S, So = State(m.L, m.C, 64, device="cuda"), o.state()
    lg, S = m.forward(torch.tensor(toks, device="cuda"), S)
    assert_logits_close(lg.float(), o.forward(toks, So), "0.4B forward")
    for i, t in enumerate(_tokens(3, 65536, 4)):
        lg, S = m.decode(torch.tensor([t], device="cuda"), S)
        assert_logits_close(lg.float(), o.decode(t, So), f"0.4B decode {i}")
    assert_state_close(S, So, "0.4B state")


def test_decode_batch_random_states():
    """Config 2 style: one decode step of B sequences from random states."""
    m, o = _pair(CONFIG_TINY, 1)
    B = 5
    bs = BatchedState(m.L, m.C, B, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    bs.rnn.copy_(0.1 * torch.randn(bs.rnn.shape, generator=g, device="cuda"))
    bs.tmix_x.copy_(torch.randn(bs.tmix_x.shape, generator=g, device="cuda").half())
    bs.cmix_x.copy_(torch.randn(bs.cmix_x.shape, generator=g, device="cuda").half())
    toks = _tokens(B, CONFIG_TINY.vocab, 6)
    oracle_states = []
    for b in range(B):
        So = o.state()
        gpu_state_to_oracle(bs[b], So)
        oracle_states.append(So)
    lg = m.decode_batch(torch.tensor(toks, device="cuda"), bs)
    for b in range(B):
        assert_logits_close(lg[b].float(), o.decode(toks[b], oracle_states[b]), f"seq {b}")
        assert_state_close(bs[b], oracle_states[b], f"seq {b}")


def test_prefill_batch_varlen_and_slots():
    m, o = _pair(CONFIG_TINY, 1)
    lens = [1, 7, 20, 3]
    seqs = [_tokens(n, CONFIG_TINY.vocab, 10 + i) for i, n in enumerate(lens)]
    bs = BatchedState(m.L, m.C, 6, device="cuda")
    slots = [5, 0, 3, 1]
    lg = m.forward_batch([torch.tensor(s) for s in seqs], bs, slots)
    for i, s in enumerate(seqs):
        So = o.state()
        assert_logits_close(lg[i].float(), o.forward(s, So), f"seq {i}")
        assert_state_close(bs[slots[i]], So, f"seq {i}")
    # untouched slots stay zero
    assert bs.rnn[:, 2].abs().max() == 0 and bs.rnn[:, 4].abs().max() == 0


def test_graph_wrapper_matches_eager():
    m, _ = _pair(CONFIG_TINY, 1)
    cls = make_rwkv7(torch.device("cuda"), backend="b200")
    gm = cls(m.w)
    toks = _tokens(40, CONFIG_TINY.vocab, 7)
    S1, S2 = State(m.L, m.C, 64, device="cuda"), State(m.L, m.C, 64, device="cuda")
    for chunk in (toks[:9], toks[9:30]):
        m.prefill(torch.tensor(chunk, device="cuda"), S1)
        gm.prefill(torch.tensor(chunk, device="cuda"), S2)
    for t in toks[30:]:
        a, _ = m.decode(torch.tensor([t], device="cuda"), S1)
        b, _ = gm.decode(torch.tensor(t, device="cuda"), S2)
        assert torch.equal(a, b)
    for x, y in zip(S1.tmix, S2.tmix):
        assert torch.equal(x["rnn"], y["rnn"])


@pytest.mark.parametrize("B", [2, 64])
def test_graph_greedy_matches_eager_greedy(B):
    """The graph wrapper's decode_batch_greedy replays the eager greedy step exactly:
    same ids every step (with and without a caller-provided id buffer) and same states."""
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 5)
    gm = make_rwkv7(torch.device("cuda"), backend="b200")(m.w)
    g = torch.Generator(device="cuda").manual_seed(11)
    states = [BatchedState(m.L, m.C, B, device="cuda") for _ in range(2)]
    for t in ("rnn", "tmix_x", "cmix_x"):
        src = torch.randn(getattr(states[0], t).shape, generator=g, device="cuda")
        src = 0.1 * src if t == "rnn" else src.half()
        for bs in states:
            getattr(bs, t).copy_(src)
    toks = torch.randint(0, 4096, (B,), generator=g, device="cuda")
    out = torch.empty(B, dtype=torch.int64, device="cuda")
    a_ids, b_ids = toks.clone(), toks.clone()
    for step in range(4):
        a_ids = m.decode_batch_greedy(a_ids, states[0])
        b_ids = gm.decode_batch_greedy(b_ids, states[1], out=out if step % 2 else None).clone()
        assert torch.equal(a_ids, b_ids), step
    for t in ("rnn", "tmix_x", "cmix_x"):
        assert torch.equal(getattr(states[0], t), getattr(states[1], t))


def test_graph_replay_after_workspace_growth():
    """A captured graph keeps working after later calls grew the model's scratch.

    Capture a short prefill, then a longer one and an eager prefill longer than any
    graph, then replay the first graph: it must still match eager. Same for a graphed
    B=1 decode (persistent kernel, C=768) replayed after a B=4 decode_batch and a
    B=64 token-batch decode have grown both scratch buffers.
    """
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 5)
    gm = make_rwkv7(torch.device("cuda"), backend="b200")(m.w)
    toks = _tokens(400, 4096, 17)
    Sg, Se = State(m.L, m.C, 64, device="cuda"), State(m.L, m.C, 64, device="cuda")
    gm.prefill(torch.tensor(toks[:9], device="cuda"), Sg)        # capture T=9
    m.prefill(torch.tensor(toks[:9], device="cuda"), Se)
    big = State(m.L, m.C, 64, device="cuda")
    gm.prefill(torch.tensor(toks[:60], device="cuda"), big)      # capture T=60 (more scratch)
    gm.prefill(torch.tensor(toks[:400], device="cuda"), big)     # eager, larger still
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    junk = torch.full((64 << 20,), 7, dtype=torch.uint8, device="cuda")  # reuse freed blocks
    gm.prefill(torch.tensor(toks[9:18], device="cuda"), Sg)      # replay T=9
    m.prefill(torch.tensor(toks[9:18], device="cuda"), Se)
    del junk
    for x, y in zip(Sg.tmix, Se.tmix):
        assert torch.equal(x["rnn"], y["rnn"])
    a, _ = gm.decode(torch.tensor(5, device="cuda"), Sg)        # capture decode B=1
    b, _ = m.decode(torch.tensor(5, device="cuda"), Se)
    bs = BatchedState(m.L, m.C, 64, device="cuda")
    gm.decode_batch(torch.arange(4, device="cuda"), bs)          # B=4: larger GEMV scratch
    gm.decode_batch(torch.arange(64, device="cuda"), bs)         # token batch scratch
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    junk = torch.full((64 << 20,), 7, dtype=torch.uint8, device="cuda")
    a, _ = gm.decode(torch.tensor(11, device="cuda"), Sg)       # replay
    b, _ = m.decode(torch.tensor(11, device="cuda"), Se)
    del junk
    assert torch.equal(a, b)
    for x, y in zip(Sg.tmix, Se.tmix):
        assert torch.equal(x["rnn"], y["rnn"])


def test_foreign_state_layout_roundtrip():
    """A State whose dict entries were rebound still works (staged copy in/out)."""
    m, o = _pair(CONFIG_TINY, 1)
    S = State(m.L, m.C, 64, device="cuda")
    for d in S.tmix:
        d["rnn"] = d["rnn"].clone()  # rebind: no longer aliases the blocks
    So = o.state()
    for t in _tokens(4, CONFIG_TINY.vocab, 8):
        lg, S = m.decode(t, S)
        assert_logits_close(lg.float(), o.decode(t, So), "foreign")
    assert_state_close(S, So, "foreign")


def test_errors():
    m, _ = _pair(CONFIG_TINY, 1)
    S = State(m.L, m.C, 64, device="cuda")
    with pytest.raises(RuntimeError):
        m.prefill(torch.tensor([], dtype=torch.long, device="cuda"), S)
    with pytest.raises(ValueError):
        m.forward(torch.zeros(2, 2, dtype=torch.long, device="cuda"), S)
    with pytest.raises(ValueError):
        make_rwkv7(torch.device("cuda"), backend="nope")


@pytest.mark.parametrize("lens", [[70], [1, 33, 16, 100], [17, 5], [300, 700, 17, 257]])
def test_chunked_wkv_matches_serial(monkeypatch, lens):
    """The chunk-parallel wkv and the per-token wkv give the same model state (to the
    fp32 noise that fp16 rounding amplifies through the layers: state rel 1e-3)."""
    m, _ = _pair(CONFIG_TINY, 1)
    seqs = [torch.tensor(_tokens(n, CONFIG_TINY.vocab, 20 + i)) for i, n in enumerate(lens)]
    out = {}
    for mode in ("serial", "chunked"):
        monkeypatch.setenv("RWKV_B200_WKV", mode)
        bs = BatchedState(m.L, m.C, len(lens), device="cuda")
        m.prefill_batch(seqs, bs)
        torch.cuda.synchronize()
        out[mode] = bs
    a, b = out["serial"], out["chunked"]
    assert ((a.rnn - b.rnn).norm() / a.rnn.norm()) < 1e-3
    assert (a.tmix_x.float() - b.tmix_x.float()).abs().max() < 1e-2
    assert (a.cmix_x.float() - b.cmix_x.float()).abs().max() < 1e-2


@pytest.mark.parametrize("B", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("mode", ["persist", "gemv", "token"])
def test_small_batch_decode_paths(monkeypatch, B, mode):
    """Small-batch decode from random states vs the oracle, at a width the GEMV paths
    take (C=768): the persistent single-kernel step (B <= 4), the three-kernel PDL
    chain, and the token-batch kernels."""
    monkeypatch.setenv("RWKV_B200_DECODE", "token" if mode == "token" else "gemv")
    monkeypatch.setenv("RWKV_B200_DECODE_PERSIST", "1" if mode == "persist" else "0")
    m, o = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 4)
    bs = BatchedState(m.L, m.C, B + 2, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(11 + B)
    bs.rnn.copy_(0.1 * torch.randn(bs.rnn.shape, generator=g, device="cuda"))
    bs.tmix_x.copy_(torch.randn(bs.tmix_x.shape, generator=g, device="cuda").half())
    bs.cmix_x.copy_(torch.randn(bs.cmix_x.shape, generator=g, device="cuda").half())
    slots = torch.tensor(list(range(B + 1, 0, -1))[:B], dtype=torch.int32, device="cuda")
    refs = []
    for b in range(B):
        So = o.state()
        gpu_state_to_oracle(bs[int(slots[b])], So)
        refs.append(So)
    for step in range(2):
        toks = _tokens(B, 4096, 30 + step)
        lg = m.decode_batch(torch.tensor(toks, device="cuda"), bs, slots)
        for b in range(B):
            assert_logits_close(lg[b].float(), o.decode(toks[b], refs[b]), f"{mode} B={B} seq {b}")
    for b in range(B):
        assert_state_close(bs[int(slots[b])], refs[b], f"{mode} state {b}")
    # the spare slot 0 (never used) stays as it was
    from rwkv_tl_b200 import _lib

    assert _lib.load().rwkv_b200_device_error() == 0


@pytest.mark.parametrize("B,V", [(1, 4096), (16, 4096), (200, 4096), (200, 65536)])
def test_decode_batch_greedy_matches_argmax_of_logits(B, V):
    """The greedy head (argmax inside the lm-head GEMM epilogue, no logits stored)
    returns exactly argmax(decode_batch logits), and updates the state identically.
    V = 65536 puts the head on the persistent 128 x 256-tile GEMM."""
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=V), 3)
    g = torch.Generator(device="cuda").manual_seed(B)
    states = []
    for _ in range(2):
        bs = BatchedState(m.L, m.C, B, device="cuda")
        states.append(bs)
    for t in ("rnn", "tmix_x", "cmix_x"):
        src = torch.randn(getattr(states[0], t).shape, generator=g, device="cuda")
        src = 0.1 * src if t == "rnn" else src.half()
        for bs in states:
            getattr(bs, t).copy_(src)
    toks = torch.randint(0, V, (B,), generator=g, device="cuda")
    slots = torch.randperm(B, generator=g, device="cuda").to(torch.int32)
    lg = m.decode_batch(toks, states[0], slots)
    ids = m.decode_batch_greedy(toks, states[1], slots)
    torch.cuda.synchronize()
    assert ids.dtype == torch.int64 and ids.shape == (B,)
    # every path is deterministic (split-K slices summed in order on the token path,
    # fixed-point atomics in the small-batch kernels), so the two runs agree exactly
    assert torch.equal(ids, lg.argmax(-1))
    for t in ("rnn", "tmix_x", "cmix_x"):
        assert torch.equal(getattr(states[0], t), getattr(states[1], t))


def test_greedy_head_ties_pick_the_lowest_id():
    """Rows of the head that are identical give equal fp16 logits; like torch.argmax
    the greedy head must return the first of them."""
    sd = synth_checkpoint(ModelConfig(n_layer=1, n_embd=768, vocab=4096), seed=4)
    head = sd["head.weight"]
    head[:] = 0.01 * head
    head[100:4096:97] = 5.0 * head[7]  # ids 100, 197, 294, ... have equal, large logits
    w = RWKV7Weight(sd, device="cuda")
    m = RWKV7B200(w)
    B = 32
    bs = BatchedState(m.L, m.C, B, device="cuda")
    toks = torch.arange(B, device="cuda")
    lg = m.decode_batch(toks, BatchedState(m.L, m.C, B, device="cuda"))
    ids = m.decode_batch_greedy(toks, bs)
    torch.cuda.synchronize()
    ref = lg.argmax(-1)
    assert torch.equal(ids, ref)
    # the tied rows really are tied and the winner is the lowest of them when they win
    tied = torch.arange(100, 4096, 97, device="cuda")
    wins = torch.isin(ref, tied)
    assert wins.any()
    assert torch.all(ref[wins] == 100)


@pytest.mark.parametrize("B,mode", [(1, "persist"), (2, "persist"), (4, "persist"), (8, "gemv")])
def test_small_batch_decode_is_bit_reproducible(monkeypatch, B, mode):
    """The small-batch decode kernels sum their cross-CTA partials with order-independent
    fixed-point atomics: the same step from the same state gives bit-identical logits and
    states on every run (0.4B width, 2 layers)."""
    monkeypatch.setenv("RWKV_B200_DECODE", "gemv")
    monkeypatch.setenv("RWKV_B200_DECODE_PERSIST", "1" if mode == "persist" else "0")
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=1024, vocab=8192), 6)
    g = torch.Generator(device="cuda").manual_seed(40 + B)
    src = BatchedState(m.L, m.C, B, device="cuda")
    src.rnn.copy_(0.1 * torch.randn(src.rnn.shape, generator=g, device="cuda"))
    src.tmix_x.copy_(torch.randn(src.tmix_x.shape, generator=g, device="cuda").half())
    src.cmix_x.copy_(torch.randn(src.cmix_x.shape, generator=g, device="cuda").half())
    toks = torch.randint(0, 8192, (B,), generator=g, device="cuda")
    outs = []
    for _ in range(3):
        st = BatchedState(m.L, m.C, B, device="cuda")
        for t in ("rnn", "tmix_x", "cmix_x"):
            getattr(st, t).copy_(getattr(src, t))
        lg = m.decode_batch(toks, st)
        lg2 = m.decode_batch(toks, st)
        torch.cuda.synchronize()
        outs.append((lg.clone(), lg2.clone(), st.rnn.clone(), st.tmix_x.clone(), st.cmix_x.clone()))
    for o in outs[1:]:
        for a, b in zip(outs[0], o):
            assert torch.equal(a, b)


def test_wide_and_narrow_row_layouts_are_bit_identical(monkeypatch):
    """Token batches of >= 1024 rows run the row / gate / GroupNorm kernels 8 channels
    per thread; their sums replay the narrow layouts' summation trees, so forcing the
    narrow layouts (RWKV_B200_NARROW=1) changes no bit of the states or the logits."""
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 7)
    seqs = [torch.tensor(_tokens(n, 4096, 60 + i)) for i, n in enumerate((900, 700, 400))]
    toks = torch.tensor(_tokens(1100, 4096, 70), device="cuda")
    out = {}
    for mode in ("wide", "narrow"):
        monkeypatch.setenv("RWKV_B200_NARROW", "1" if mode == "narrow" else "0")
        bs = BatchedState(m.L, m.C, 1100, device="cuda")
        m.prefill_batch(seqs, bs)
        lg = m.decode_batch(toks, bs)
        torch.cuda.synchronize()
        out[mode] = (bs.rnn.clone(), bs.tmix_x.clone(), bs.cmix_x.clone(), lg.clone())
    for a, b in zip(out["wide"], out["narrow"]):
        assert torch.equal(a, b)


def test_side_stream_rkv_is_bit_identical(monkeypatch):
    """Decode batches (<= 512 rows) run the r/k/v projections on a side stream beside the
    LoRA chain; the same kernels compute the same values, so turning the side stream off
    (RWKV_B200_FORK=0) changes no bit of the states or the logits, eager or replayed from
    a CUDA graph."""
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 9)
    g = make_rwkv7("cuda", backend="b200", use_graph=True)(m.w)
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("RWKV_B200_FORK", mode)
        for B in (64, 256):
            bs = BatchedState(m.L, m.C, B, device="cuda")
            gen = torch.Generator(device="cuda").manual_seed(B)
            bs.rnn.normal_(0.0, 0.1, generator=gen)
            toks = torch.tensor(_tokens(B, 4096, 80 + B), device="cuda")
            lg = m.decode_batch(toks, bs)
            bs2 = BatchedState(m.L, m.C, B, device="cuda")
            bs2.rnn.copy_(bs.rnn)
            for _ in range(2):
                lg2 = g.decode_batch(toks, bs2)
            torch.cuda.synchronize()
            out[(mode, B)] = (bs.rnn.clone(), bs.cmix_x.clone(), lg.clone(), lg2.clone())
        g = make_rwkv7("cuda", backend="b200", use_graph=True)(m.w)  # fresh captures
    for B in (64, 256):
        for a, b in zip(out[("1", B)], out[("0", B)]):
            assert torch.equal(a, b)


def test_first_call_under_capture_runs_on_one_stream():
    """The side stream is never created inside a stream capture: a process whose very
    first decode-batch call is captured into a CUDA graph gets a one-stream graph whose
    replay equals the eager step (fresh process, so nothing was created before)."""
    import subprocess
    import sys
    import textwrap

    code = textwrap.dedent("""
        import torch
        from rwkv_tl_b200 import BatchedState
        from rwkv_tl_b200.synth import ModelConfig
        from tests.test_model_gpu import _pair, _tokens
        m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 9)
        B = 64
        toks = torch.tensor(_tokens(B, 4096, 5), device="cuda")
        a = BatchedState(m.L, m.C, B, device="cuda")
        b = BatchedState(m.L, m.C, B, device="cuda")
        a.rnn.normal_(0.0, 0.1, generator=torch.Generator(device="cuda").manual_seed(1))
        b.rnn.copy_(a.rnn)
        lg = torch.empty(B, 4096, dtype=torch.float16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            m.decode_batch(toks, a, logits=lg)
        a.rnn.copy_(b.rnn)
        a.tmix_x.zero_(); a.cmix_x.zero_()
        g.replay()
        ref = m.decode_batch(toks, b)
        torch.cuda.synchronize()
        assert torch.equal(lg, ref) and torch.equal(a.rnn, b.rnn), "graph != eager"
        print("OK")
    """)
    import os
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, PYTHONPATH=str(root))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_graphed_greedy_on_pinned_host_buffers():
    """decode_batch_greedy with pinned host ids in and out (the copies captured into the
    graph) gives the same next ids and states as the device-buffer call, step after step,
    including when the host buffers' contents change between replays."""
    m, _ = _pair(ModelConfig(n_layer=2, n_embd=768, vocab=4096), 11)
    g = make_rwkv7("cuda", backend="b200", use_graph=True)(m.w)
    B = 64
    a = BatchedState(m.L, m.C, B, device="cuda")
    b = BatchedState(m.L, m.C, B, device="cuda")
    a.rnn.normal_(0.0, 0.1, generator=torch.Generator(device="cuda").manual_seed(3))
    b.rnn.copy_(a.rnn)
    host_tok = torch.tensor(_tokens(B, 4096, 12), dtype=torch.int64).pin_memory()
    host_out = torch.empty(B, dtype=torch.int64).pin_memory()
    dev_ids = torch.empty(B, dtype=torch.int64, device="cuda")
    for step in range(4):
        g.decode_batch_greedy(host_tok, a, out=host_out)
        g.decode_batch_greedy(host_tok.cuda(), b, out=dev_ids)
        torch.cuda.synchronize()
        assert torch.equal(host_out, dev_ids.cpu()), step
        host_tok.copy_(host_out)  # feed the step's ids back, as a serving loop does
    assert torch.equal(a.rnn, b.rnn) and torch.equal(a.cmix_x, b.cmix_x)
