"""Generate the golden fixtures in this folder by running the reference itself.

Run on a machine that has the yuyi2439/rwkv-tl sources (not needed at test
time; the fixtures are committed)::

    python tests/golden/make_golden.py --reference <path to rwkv-tl checkout>

Every fixture is produced by the reference's own classes on CPU, on a seeded
synthetic checkpoint from ``rwkv_tl_b200.synth`` written in the reference's key
format and loaded through the reference's ``RWKV7Weight``:

* ``tiny_torch_fp32.pt`` -- ``demo.rwkv7_torch.RWKV7Torch`` (fp32), tiny model
  (L=2, C=128, V=1024, seed 1): per-step decode logits over 8 tokens from a zero
  state, prefill(7)+decode(1) logits, and the final state of both runs.
* ``tiny_fp16_cpu.pt`` -- ``demo.rwkv7_fp16.RWKV7FP16`` (fp16 weights) on CPU,
  same cases. On CPU the reference's fp16 kernels run their torch fallbacks
  (``src/rwkv_tl/kernels/*.py``, ``device.type != "cuda"`` branches), which round
  after every torch op, so this pins the fp16 oracle only loosely.
* ``loader_bf16.pt`` -- the reference loader ``RWKV7Weight(path, device="cpu",
  dtype=torch.float16)`` (``src/rwkv_tl/weight.py:155-184``) on a bf16 ``.pth`` file of
  the tiny config (seed 3): the fp16 embedding with LN0 folded in, the head, ln_out and
  every per-layer tensor in the reference's own orientation.
* ``cfg0_torch_fp32.pt``: 0.1B (L=12, C=768, V=65536,
  seed 0), 8-token prompt of seeded uniform ids, ``forward`` then 16 greedy
  decode steps with ``RWKV7Torch`` in fp32. Stores the generated tokens, the
  logits of the prompt and of the last step (fp32), and state checksums.
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

from rwkv_tl_b200.synth import CONFIG_0_1B, CONFIG_TINY, synth_checkpoint  # noqa: E402

TINY_TOKENS = [(i * 1103515245 + 12345) % 1024 for i in range(8)]


def cfg0_prompt() -> list[int]:
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, 65536, (8,), generator=g).tolist()


def state_to_dict(S) -> dict:
    return {
        "tmix_x": torch.stack([d["x"].float() for d in S.tmix]),
        "rnn": torch.stack([d["rnn"].float() for d in S.tmix]),
        "cmix_x": torch.stack([d["x"].float() for d in S.cmix]),
    }


def run_cases(model, w, dtype, tokens) -> dict:
    from rwkv_tl.state import State

    S = State(w.L, w.C, 64, device="cpu", dtype=dtype)
    per_step = []
    for t in tokens:
        logits, S = model.decode(torch.tensor([t]), S)
        per_step.append(logits.float().clone())
    out = {"decode_logits": torch.stack(per_step), "decode_state": state_to_dict(S)}
    S2 = State(w.L, w.C, 64, device="cpu", dtype=dtype)
    logits, S2 = model.forward(torch.tensor(tokens), S2)
    out["forward_logits"] = logits.float().clone()
    out["forward_state"] = state_to_dict(S2)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RWKV_TL_REFERENCE"), required="RWKV_TL_REFERENCE" not in os.environ,
                    help="path of a yuyi2439/rwkv-tl checkout (or set RWKV_TL_REFERENCE)")
    args = ap.parse_args()
    sys.path[:0] = [os.path.join(args.reference, "src"), args.reference]
    torch.set_num_threads(os.cpu_count() or 1)

    from demo.rwkv7_fp16 import RWKV7FP16
    from demo.rwkv7_torch import RWKV7Torch
    from rwkv_tl.weight import RWKV7Weight

    with tempfile.TemporaryDirectory() as td:
        # ---- tiny model ----
        p = os.path.join(td, "tiny.pth")
        torch.save(synth_checkpoint(CONFIG_TINY, seed=1), p)
        w32 = RWKV7Weight(p, device="cpu", dtype=torch.float32)
        m32 = RWKV7Torch(w32, is_torch_compile=False)
        out = run_cases(m32, w32, torch.float32, TINY_TOKENS)
        out["tokens"] = torch.tensor(TINY_TOKENS)
        out["how"] = "RWKV7Torch fp32 CPU, CONFIG_TINY seed 1"
        torch.save(out, HERE / "tiny_torch_fp32.pt")

        w16 = RWKV7Weight(p, device="cpu", dtype=torch.float16)
        m16 = RWKV7FP16(w16, is_torch_compile=False)
        out = run_cases(m16, w16, torch.float16, TINY_TOKENS)
        out["tokens"] = torch.tensor(TINY_TOKENS)
        out["how"] = "RWKV7FP16 (CPU torch fallbacks), CONFIG_TINY seed 1"
        torch.save(out, HERE / "tiny_fp16_cpu.pt")

        # ---- loader: a bf16 checkpoint file through the reference's RWKV7Weight ----
        p = os.path.join(td, "tiny_bf16.pth")
        torch.save(synth_checkpoint(CONFIG_TINY, seed=3, dtype=torch.bfloat16), p)
        wr = RWKV7Weight(p, device="cpu", dtype=torch.float16)
        blocks = []
        for b in wr.blocks:
            a, f = b.att, b.ffn
            blocks.append({
                "ln1": (b.att.ln_pre.w, b.att.ln_pre.b), "ln2": (f.ln_pre.w, f.ln_pre.b),
                "ln_x": (a.ln_x.w, a.ln_x.b),
                **{n: getattr(a, n) for n in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "w0",
                                              "w1", "w2", "a0", "a1", "a2", "v0", "v1", "v2",
                                              "g1", "g2", "r_k", "k_k", "k_a", "rkvWt", "oWt")},
                "ffn_x_k": f.x_k, "kWt": f.kWt, "vWt": f.vWt,
            })
        torch.save({"emb": wr.emb, "head": wr.head, "ln_out": (wr.ln_out.w, wr.ln_out.b),
                    "blocks": blocks,
                    "how": "reference RWKV7Weight(tiny bf16 .pth, cpu, fp16), CONFIG_TINY seed 3"},
                   HERE / "loader_bf16.pt")

        # ---- config 0: 0.1B fp32 pure torch, 8-token prompt + 16 greedy steps ----
        p = os.path.join(td, "cfg0.pth")
        torch.save(synth_checkpoint(CONFIG_0_1B, seed=0), p)
        w = RWKV7Weight(p, device="cpu", dtype=torch.float32)
        m = RWKV7Torch(w, is_torch_compile=False)
        from rwkv_tl.state import State

        prompt = cfg0_prompt()
        S = State(w.L, w.C, 64, device="cpu", dtype=torch.float32)
        logits, S = m.forward(torch.tensor(prompt), S)
        prompt_logits = logits.float().clone()
        gen = []
        for step in range(16):
            tok = int(torch.argmax(logits))
            gen.append(tok)
            if step + 1 < 16:
                logits, S = m.decode(torch.tensor([tok]), S)
        sd = state_to_dict(S)
        torch.save(
            {
                "prompt": torch.tensor(prompt),
                "generated": torch.tensor(gen),
                "prompt_logits": prompt_logits,
                "last_logits": logits.float().clone(),
                "state_rnn_layer0_head0": sd["rnn"][0, 0].clone(),
                "state_rnn_sum": sd["rnn"].double().sum(dim=(1, 2, 3)),
                "state_tmix_x": sd["tmix_x"],
                "state_cmix_x": sd["cmix_x"],
                "how": "RWKV7Torch fp32 CPU, CONFIG_0_1B seed 0, forward(prompt) + 16 greedy",
            },
            HERE / "cfg0_torch_fp32.pt",
        )
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
