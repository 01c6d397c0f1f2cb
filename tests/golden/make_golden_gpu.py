"""Generate ``ref_gpu_*.pt``: the reference's own fp16 GPU model on configs 0, 2, 3.

Two steps, run by hand (the fixtures are committed; tests never run this):

1. On a CUDA machine that has a yuyi2439/rwkv-tl checkout (its ``src/rwkv_tl``
   and ``demo`` packages) and TileLang::

       python tests/golden/make_golden_gpu.py reference --reference <checkout>

   runs ``make_rwkv7(dev, backend="fp16", use_graph=False)(w, is_torch_compile=False)``
   (reference ``demo/__init__.py:43-78``, ``demo/rwkv7_fp16.py:16-25``: the eager
   fp16 TileLang path) on the seeded synthetic checkpoints and inputs of
   ``cases.py`` and writes its outputs.

2. On any machine (CPU)::

       python tests/golden/make_golden_gpu.py oracle

   adds the fp64-accumulated oracle (``oracle/rwkv7_oracle.py``, fp16 rounding
   schedule) on the same inputs, teacher-forced with the reference's greedy
   tokens, so each fixture also holds "reference vs fp64" for the same values.

Each greedy case stores, per logits position, the top-``TOPK`` (values, ids) and
the greedy id, full logits at a few positions, and the fp32 wkv state of three
layers plus all token-shift states, keeping the files small.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from rwkv_tl_b200.synth import synth_checkpoint  # noqa: E402
from tests.golden import cases  # noqa: E402


def _logit_record(logits_list, full_pos):
    lg = torch.stack([x.float().cpu() for x in logits_list])  # [P, V]
    top = torch.topk(lg, cases.TOPK, dim=-1)
    return {
        "gen": lg.argmax(-1),
        "topv": top.values.half(),
        "topi": top.indices.int(),
        "full": {int(p): lg[p].half() for p in full_pos if p < lg.shape[0]},
    }


def _state_record(rnn_layers, tx, cx, layers):
    return {
        "layers": torch.tensor(layers),
        "rnn": torch.stack([rnn_layers[i].float().cpu() for i in layers]),
        "tmix_x": torch.stack([t.float().cpu() for t in tx]).half(),
        "cmix_x": torch.stack([t.float().cpu() for t in cx]).half(),
    }


# --------------------------------------------------------------------------- #
# step 1: the reference on the GPU
# --------------------------------------------------------------------------- #
def run_reference(ref_root: str, out_dir: Path, which: list[str]) -> None:
    src = os.path.join(ref_root, "src")
    sys.path[:0] = [src if os.path.isdir(src) else ref_root, ref_root]
    from demo import make_rwkv7
    from rwkv_tl.state import State
    from rwkv_tl.weight import RWKV7Weight

    dev = torch.device("cuda")
    cls = make_rwkv7(dev, backend="fp16", use_graph=False)
    meta = {"torch": str(torch.__version__), "gpu": torch.cuda.get_device_name(0)}
    try:
        import tilelang

        meta["tilelang"] = str(tilelang.__version__)
    except Exception as e:  # noqa: BLE001
        meta["tilelang"] = f"import failed: {e}"

    def load(cfg, seed, td):
        p = os.path.join(td, f"w_{cfg.n_layer}_{cfg.n_embd}_{seed}.pth")
        if not os.path.exists(p):
            torch.save(synth_checkpoint(cfg, seed=seed), p)
        w = RWKV7Weight(p, device=dev, dtype=torch.float16)
        return w, cls(w, is_torch_compile=False)

    def st_rec(S, L):
        return _state_record([d["rnn"] for d in S.tmix], [d["x"] for d in S.tmix],
                             [d["x"] for d in S.cmix], cases.state_layers(L))

    def greedy(m, w, toks, n_decode):
        S = State(w.L, w.C, 64, device=dev, dtype=torch.float16)
        logits, S = m.forward(torch.tensor(toks, device=dev), S)
        outs = [logits.clone()]
        st_fwd = st_rec(S, w.L)
        for _ in range(n_decode):
            tok = int(torch.argmax(logits.float()))
            logits, S = m.decode(torch.tensor([tok], device=dev), S)
            outs.append(logits.clone())
        return outs, st_fwd, st_rec(S, w.L)

    with tempfile.TemporaryDirectory() as td:
        if "cfg0" in which:
            c = cases.CFG0
            w, m = load(c["cfg"], c["weight_seed"], td)
            toks = cases.prompt(c["prompt_len"], c["prompt_seed"])
            outs, st_fwd, st_end = greedy(m, w, toks, c["steps"] - 1)
            rec = {"prompt": torch.tensor(toks), "ref": _logit_record(outs, range(len(outs))),
                   "ref_state_fwd": st_fwd, "ref_state_end": st_end, "meta": meta}
            torch.save(rec, out_dir / "ref_gpu_cfg0.pt")
            print("cfg0 done", rec["ref"]["gen"].tolist())
        if "cfg2" in which:
            c = cases.CFG2
            cfg = c["cfg"]
            w, m = load(cfg, c["weight_seed"], td)
            rnn, tx, cx = cases.random_states(cfg, c["batch"], c["state_seed"])
            toks = cases.cfg2_tokens()
            logits_all, states = [], {}
            for b in range(c["batch"]):
                S = State(w.L, w.C, 64, device=dev, dtype=torch.float16)
                for i in range(w.L):
                    S.tmix[i]["rnn"].copy_(rnn[i, b])
                    S.tmix[i]["x"].copy_(tx[i, b])
                    S.cmix[i]["x"].copy_(cx[i, b])
                logits, S = m.decode(torch.tensor([toks[b]], device=dev), S)
                logits_all.append(logits.clone())
                if b in cases.CFG2_STATE_SEQS:
                    states[b] = st_rec(S, w.L)
            rec = {"tokens": torch.tensor(toks),
                   "ref": _logit_record(logits_all, cases.CFG2_LOGIT_SEQS),
                   "ref_states": states, "meta": meta}
            torch.save(rec, out_dir / "ref_gpu_cfg2.pt")
            print("cfg2 done")
        for name, c in cases.SHORT.items():
            if name not in which:
                continue
            w, m = load(c["cfg"], c["weight_seed"], td)
            lg, st = [], []
            for seed in c["seeds"]:
                S = State(w.L, w.C, 64, device=dev, dtype=torch.float16)
                toks = cases.prompt(c["prompt_len"], seed)
                logits, S = m.forward(torch.tensor(toks, device=dev), S)
                lg.append(logits.float().cpu().half())
                st.append(S.tmix[w.L - 1]["rnn"][: cases.SHORT_STATE_HEADS].float().cpu())
            torch.save({"ref_logits": torch.stack(lg), "ref_state": torch.stack(st),
                        "meta": meta}, out_dir / f"ref_gpu_{name}.pt")
            print(name, "done")
        for T in cases.CFG3["lengths"]:
            if f"cfg3_T{T}" not in which:
                continue
            c = cases.CFG3
            w, m = load(c["cfg"], c["weight_seed"], td)
            toks = cases.cfg3_prompt(T)
            outs, st_fwd, st_end = greedy(m, w, toks, c["steps"])
            rec = {"prompt": torch.tensor(toks),
                   "ref": _logit_record(outs, cases.cfg3_steps_full(c["steps"])),
                   "ref_state_fwd": st_fwd, "ref_state_end": st_end, "meta": meta}
            torch.save(rec, out_dir / f"ref_gpu_cfg3_T{T}.pt")
            print(f"cfg3 T={T} done", rec["ref"]["gen"][:8].tolist())


# --------------------------------------------------------------------------- #
# step 2: the fp64 oracle on the same inputs (CPU)
# --------------------------------------------------------------------------- #
def run_oracle(out_dir: Path, which: list[str]) -> None:
    from oracle.rwkv7_oracle import OracleState, OracleWeights, RWKV7Oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cache: dict = {}

    def oracle(cfg, seed):
        key = (cfg, seed)
        if key not in cache:
            cache.clear()
            cache[key] = RWKV7Oracle(OracleWeights(synth_checkpoint(cfg, seed=seed), "fp16",
                                                   torch.float64))
        return cache[key]

    def forced(o, L, C, toks, gen, n_decode):
        S = OracleState(L, C, dtype=torch.float64)
        outs = [o.forward(toks, S)]
        st_fwd = _state_record(S.rnn, S.tmix_x, S.cmix_x, cases.state_layers(L))
        for i in range(n_decode):
            outs.append(o.decode(int(gen[i]), S))
        return outs, st_fwd, _state_record(S.rnn, S.tmix_x, S.cmix_x, cases.state_layers(L))

    for name in which:
        p = out_dir / f"ref_gpu_{name}.pt"
        if not p.exists():
            continue
        rec = torch.load(p, weights_only=False)
        if name in cases.SHORT:
            c = cases.SHORT[name]
            cfg = c["cfg"]
            o = oracle(cfg, c["weight_seed"])
            lg, st = [], []
            for seed in c["seeds"]:
                S = OracleState(cfg.n_layer, cfg.n_embd, dtype=torch.float64)
                lg.append(o.forward(cases.prompt(c["prompt_len"], seed), S).float())
                st.append(S.rnn[cfg.n_layer - 1][: cases.SHORT_STATE_HEADS].float())
            rec["o64_logits"], rec["o64_state"] = torch.stack(lg), torch.stack(st)
            torch.save(rec, p)
            print(name, "oracle added")
            continue
        if name == "cfg2":
            c = cases.CFG2
            cfg = c["cfg"]
            o = oracle(cfg, c["weight_seed"])
            rnn, tx, cx = cases.random_states(cfg, c["batch"], c["state_seed"])
            toks = rec["tokens"].tolist()
            outs, states = [], {}
            for b in range(c["batch"]):
                S = OracleState(cfg.n_layer, cfg.n_embd, dtype=torch.float64)
                for i in range(cfg.n_layer):
                    S.rnn[i] = rnn[i, b].double().clone()
                    S.tmix_x[i] = tx[i, b].double().clone()
                    S.cmix_x[i] = cx[i, b].double().clone()
                outs.append(o.decode(toks[b], S))
                if b in cases.CFG2_STATE_SEQS:
                    states[b] = _state_record(S.rnn, S.tmix_x, S.cmix_x,
                                              cases.state_layers(cfg.n_layer))
            rec["o64"] = _logit_record(outs, cases.CFG2_LOGIT_SEQS)
            rec["o64_states"] = states
        else:
            if name == "cfg0":
                c, n_dec, full = cases.CFG0, cases.CFG0["steps"] - 1, range(cases.CFG0["steps"])
            else:
                c = cases.CFG3
                n_dec, full = c["steps"], cases.cfg3_steps_full(c["steps"])
            cfg = c["cfg"]
            o = oracle(cfg, c["weight_seed"])
            outs, st_fwd, st_end = forced(o, cfg.n_layer, cfg.n_embd, rec["prompt"].tolist(),
                                          rec["ref"]["gen"], n_dec)
            rec["o64"] = _logit_record(outs, full)
            rec["o64_state_fwd"], rec["o64_state_end"] = st_fwd, st_end
        # the oracle's logits at the reference's top-k ids, for every position
        lg = torch.stack([x.double() for x in outs])
        rec["o64_at_ref_topi"] = lg.gather(1, rec["ref"]["topi"].long()).float()
        torch.save(rec, p)
        print(name, "oracle added")


ALL = ["cfg0", "cfg2", *cases.SHORT] + [f"cfg3_T{T}" for T in cases.CFG3["lengths"]]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("step", choices=["reference", "oracle"])
    ap.add_argument("--reference", default=os.environ.get("RWKV_TL_REFERENCE"),
                    help="path of a yuyi2439/rwkv-tl checkout (or RWKV_TL_REFERENCE)")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--cases", default=",".join(ALL))
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    which = args.cases.split(",")
    if args.step == "reference":
        if not args.reference:
            ap.error("--reference (or RWKV_TL_REFERENCE) is required")
        run_reference(args.reference, out, which)
    else:
        run_oracle(out, which)


if __name__ == "__main__":
    main()
