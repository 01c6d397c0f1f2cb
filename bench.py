"""Benchmark: RWKV-7 0.4B fp16 batched decode on B200 (one process per GPU).

``python bench.py --gpus N --steps K --warmup W [--impl b200|reference]``

Workload (BASELINE metric "decode tokens/s (0.4B, B=1..256, 1/2/4/8 GPU);
prefill tokens/s at T=4096"): one step = one decode token for each of B=256
independent sequences per GPU (config 4's per-GPU decode batch, config 2's
random states), random-init 0.4B weights (L=24, C=1024, V=65536), seeded
uniform token ids. Sequences are sharded across ranks (each rank owns its own
256 sequences and their states): no collective on the hot path, weak scaling.
Inputs (weights 0.77 GB + states 3.3 GB per GPU) are far larger than the
126 MB L2, so every step streams from HBM without an explicit flush.

* ``value``: tokens/s with inputs resident in HBM, K replays of the captured
  decode step, CUDA events on the launching stream, max over ranks.
* ``e2e``: the same step through the public API with host buffers: each step
  copies the B token ids from pinned host memory, runs ``decode_batch`` (CUDA
  graph), takes the greedy argmax on the device and reads the B next-token ids
  back into pinned host memory (synchronised).
* ``roofline``: the dominant kernel of the step (the one-token wkv7 + GroupNorm +
  gate kernel, 22% of the step in the ncu launch list) timed alone with CUDA events
  on the launching stream; ``step_roofline``: the whole step against HBM.
* ``cpu_baseline``: the CPU oracle port of the reference's pure-torch model
  (``oracle/``) decoding a bounded sample on the host cores (rank 0, N=1).
* ``--impl reference``: only the CPU port, on all host threads (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tokens/s (0.4B, B=1..256, 1/2/4/8 GPU); prefill tokens/s at T=4096"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


class Clocks:
    """Sample nvidia-smi clocks / throttle reasons while the timed region runs.

    The sampler is started, and its first sample awaited (up to 5 s), before the
    caller's timed region begins; ``mark()`` brackets the timed region, and the summary
    uses the samples taken inside it (the closest ones when the region is shorter
    than the 50 ms sampling period)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list = []
        self.window = [None, None]

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append((time.time(), ln))

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        threading.Thread(target=self._read, daemon=True).start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0:
            time.sleep(0.01)
        return self

    def mark(self, which: int) -> None:
        self.window[which] = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0, t1 = self.window
        lines = list(self.lines)
        if t0 is not None and t1 is not None:
            inside = [x for x in lines if t0 <= x[0] <= t1 + 0.05]
            if not inside and lines:  # region shorter than one sampling period
                inside = [min(lines, key=lambda x: abs(x[0] - (t0 + t1) / 2))]
            lines = inside
        for _, ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = max(smax, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    from rwkv_tl_b200.shard import max_over_ranks as _max

    return _max(x, device="cuda") if world > 1 else x


# --------------------------------------------------------------------------- #
# CPU port of the reference (oracle) -- the baseline, never the product path
# --------------------------------------------------------------------------- #
def cpu_decode_rate(n_tokens: int, threads: int) -> dict:
    from oracle.rwkv7_oracle import OracleState, OracleWeights, RWKV7Oracle
    from rwkv_tl_b200.synth import CONFIG_0_4B, synth_checkpoint

    torch.set_num_threads(threads)
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_0_4B, seed=0), mode="fp32"))
    S = OracleState(o.w.L, o.w.C)
    o.decode(1, S)  # warm-up
    times = []
    for i in range(n_tokens):
        t0 = time.perf_counter()
        o.decode(1000 + i, S)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    cfg0 = cpu_config0(threads)
    return {"value": 1.0 / med, "unit": "tokens/s", "cores": threads, "kind": "port",
            "config0": cfg0,
            "sample": f"0.4B fp32 decode (oracle port of demo/rwkv7_torch.py), 1 sequence, "
                      f"{n_tokens} tokens after 1 warm-up, median {med * 1e3:.1f} ms/token; "
                      "batched CPU decode loops over sequences, so tokens/s is per token"}


def cpu_config0(threads: int) -> dict:
    """BASELINE config 0 on the CPU port: 0.1B fp32, an 8-token prompt (forward), then
    16 greedy tokens (``demo/rwkv7_torch.py:149-171``)."""
    from oracle.rwkv7_oracle import OracleState, OracleWeights, RWKV7Oracle
    from rwkv_tl_b200.synth import CONFIG_0_1B, synth_checkpoint

    torch.set_num_threads(threads)
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_0_1B, seed=0), mode="fp32"))
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 65536, (8,), generator=g).tolist()
    S = OracleState(o.w.L, o.w.C)
    t0 = time.perf_counter()
    _, _ = o.generate_greedy(prompt, 16, S)
    dt = time.perf_counter() - t0
    return {"workload": "0.1B fp32, forward(8-token prompt) + 16 greedy tokens, 1 sequence",
            "seconds": dt, "tokens_per_s": (8 + 15) / dt, "cores": threads}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle.rwkv7_oracle import OracleState, OracleWeights, RWKV7Oracle
    from rwkv_tl_b200.synth import CONFIG_0_4B, synth_checkpoint

    torch.set_num_threads(threads)
    o = RWKV7Oracle(OracleWeights(synth_checkpoint(CONFIG_0_4B, seed=0), mode="fp32"))
    S = OracleState(o.w.L, o.w.C)
    for i in range(args.warmup):
        o.decode(i, S)
    t0 = time.perf_counter()
    for i in range(args.steps):
        o.decode(100 + i, S)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "0.4B decode, one token of one sequence per step (CPU port; "
                               "the B=256 batch is a loop over sequences)",
                   "global_batch": 1, "seq_len": 1, "parallelism": "none"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} decode tokens of one sequence"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- #
def timed(fn, steps: int, stream) -> float:
    """Average ms per call over `steps` calls, CUDA events on `stream`."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def run_b200(args, world, rank, local):
    from rwkv_tl_b200 import BatchedState, RWKV7Weight, State, _lib, make_rwkv7
    from rwkv_tl_b200.synth import CONFIG_0_4B, synth_checkpoint

    cfg = CONFIG_0_4B
    dev = torch.device("cuda", local)
    B = args.batch
    sd = synth_checkpoint(cfg, seed=0, device=dev)
    w = RWKV7Weight(sd, device=dev)
    del sd
    torch.cuda.empty_cache()
    model = make_rwkv7(dev, backend="b200")(w)
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    state = BatchedState(w.L, w.C, B, device=dev)
    state.rnn.normal_(0.0, 0.1, generator=g)
    state.tmix_x.copy_(torch.randn(state.tmix_x.shape, generator=g, device=dev).half())
    state.cmix_x.copy_(torch.randn(state.cmix_x.shape, generator=g, device=dev).half())
    tokens = torch.randint(0, cfg.vocab, (B,), generator=g, device=dev)
    stream = torch.cuda.current_stream(dev)

    # launches per step (eager call through the library)
    c0 = lib.rwkv_b200_launch_count()
    model.model.decode_batch(tokens, state)
    launches_per_step = int(lib.rwkv_b200_launch_count() - c0)

    logits_buf = torch.empty(B, cfg.vocab, dtype=torch.float16, device=dev)
    # graph replay writing into the caller's buffer (no copy of the [B, V] logits)
    step = lambda: model.decode_batch(tokens, state, logits=logits_buf)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    with Clocks(local) as clk:
        barrier(world)
        clk.mark(0)
        ms = timed(step, args.steps, stream)
        clk.mark(1)
        barrier(world)
    ms = max_over_ranks(ms, world)
    value = world * B / (ms * 1e-3)

    # ---- e2e through the public API with host buffers ----
    # (the greedy step a serving loop makes: token ids in from pinned host memory, the
    # graph-replayed step with the argmax fused into the lm head, next ids back to the host)
    host_tok = torch.randint(0, cfg.vocab, (B,), dtype=torch.int64).pin_memory()
    host_out = torch.empty(B, dtype=torch.int64).pin_memory()

    def e2e_step():
        # pinned host ids in, next ids out: the graph holds both copies with the step
        model.decode_batch_greedy(host_tok, state, out=host_out)
        torch.cuda.current_stream(dev).synchronize()

    for _ in range(3):
        e2e_step()
    barrier(world)
    e2e_ms = timed(e2e_step, args.steps, stream)
    e2e_ms = max_over_ranks(e2e_ms, world)
    e2e_val = world * B / (e2e_ms * 1e-3)

    # ---- roofline: the whole step, and its dominant kernel timed alone ----
    pk, pk_kind = peaks()
    wbytes = w.nbytes() - 2 * w.emb.numel()  # weights streamed per step (emb: rows only)

    def step_bytes_of(nb: int) -> int:  # weights once + per-sequence state r/w + io
        return wbytes + nb * w.L * (w.H * 64 * 64 * 4 * 2 + 2 * w.C * 2 * 2) + \
            nb * (w.C * 2 + cfg.vocab * 2)

    step_bytes = step_bytes_of(B)
    kern = wkv_kernel_roofline(lib, B, w.H, dev, stream, pk["hbm_gbs"])
    extra = {}
    if rank == 0 and world == 1 and not args.quick:
        extra = side_measurements(model, w, dev, stream, step_bytes_of, pk["hbm_gbs"])

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init 0.4B weights, random states, uniform token ids)",
            "config": {"workload": f"RWKV-7 0.4B fp16 decode, B={B} sequences per GPU, one "
                                   "token each per step (CUDA graph)",
                       "model": "rwkv7-0.4B (L24 C1024 V65536)", "global_batch": world * B,
                       "seq_len": 1, "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs > L2 (weights 0.77 GB + state 3.3 GB per GPU), no flush"},
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": B * 8,
                    "d2h_bytes_per_step": B * 8,
                    "api": "decode_batch_greedy (CUDA graph) on pinned host buffers: the graph "
                           "copies the ids in and the next ids out every step; synchronised "
                           "every step"},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": dict(kern, peak_kind=pk_kind),
            "step_roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes,
                              "achieved": step_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
                              "frac": step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]},
            "clocks": clocks,
        }
        line.update(extra)
        if world == 1 and not args.quick:
            line["cpu_baseline"] = cpu_decode_rate(args.cpu_tokens, os.cpu_count() or 1)
        print(json.dumps(line), flush=True)


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch recorded from an ncu capture (profiles/<name>.txt)."""
    p = REPO / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


def wkv_kernel_roofline(lib, B: int, H: int, dev, stream, peak: float) -> dict:
    """Dominant kernel of the batched decode step: the one-token wkv7 + GroupNorm + gate
    kernel (rwkv7_wkv_gn_step), timed alone with CUDA events on the launching stream
    over the same shapes as one layer of the step (B sequences, H heads)."""
    from rwkv_tl_b200 import _lib

    C = H * 64
    g = torch.Generator(device=dev).manual_seed(7)
    # one state block per layer, as in the step: 24 x 67 MB, far beyond the 126 MB L2
    states = [0.1 * torch.randn(B, H, 64, 64, generator=g, device=dev) for _ in range(24)]
    vec = [torch.randn(B, C, generator=g, device=dev).half() for _ in range(7)]
    cst = [torch.randn(C, generator=g, device=dev).half() for _ in range(3)]
    out = torch.empty(B, C, dtype=torch.float16, device=dev)
    def launch(S, h):
        _lib.check(lib.rwkv7_wkv_gn_step(S.data_ptr(), None, *[t.data_ptr() for t in vec],
                                         *[t.data_ptr() for t in cst], out.data_ptr(), B, H, 0, h))

    for i in range(5):
        launch(states[i], stream.cuda_stream)
    # the 24 launches (one per state block) captured in a CUDA graph, so that the timed
    # replays measure the kernel back to back rather than the host's launch rate
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        for S in states:
            launch(S, cap.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):  # replays go to the stream the events are recorded on
        graph.replay()
        n = 10  # ten passes over the 24 state blocks
        ms = timed(graph.replay, n, stream) / len(states)
    # per launch: fp32 state read + write, 7 fp16 input vectors, 1 fp16 output vector
    algo = B * H * 64 * 64 * 4 * 2 + 8 * B * C * 2
    achieved = algo / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": "k_wkv_decode (rwkv7_wkv_gn_step), one layer of the step",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": profile_traffic("wkv_decode_b256"), "algorithmic_bytes_per_launch": algo,
            "avg_launch_us": ms * 1e3}


def side_measurements(model, w, dev, stream, step_bytes_of, hbm_gbs) -> dict:
    """Decode at B = 1 .. 64 and prefill at T = 4096 (reported beside the headline); the
    B = 1 step (the persistent single-kernel path) also against the HBM roofline."""
    from rwkv_tl_b200 import BatchedState, State

    out = {"decode_tokens_per_s_by_batch": {}}
    for B in (1, 2, 4, 8, 64):
        st = BatchedState(w.L, w.C, B, device=dev)
        tok = torch.randint(0, w.V, (B,), device=dev)
        lg = torch.empty(B, w.V, dtype=torch.float16, device=dev)
        # the graph writes into the caller's logits buffer, as in the headline step
        f = lambda: model.decode_batch(tok, st, logits=lg)  # noqa: E731
        for _ in range(3):
            f()
        ms = timed(f, 50 if B <= 8 else 10, stream)
        out["decode_tokens_per_s_by_batch"][str(B)] = B / (ms * 1e-3)
        if B == 1:
            gbs = step_bytes_of(1) / (ms * 1e-3) / 1e9
            out["decode_b1_roofline"] = {"bound": "hbm", "us_per_token": ms * 1e3,
                                         "algorithmic_bytes_per_step": step_bytes_of(1),
                                         "achieved": gbs, "unit": "GB/s", "frac": gbs / hbm_gbs}
    # B = 256 eager (no graph): logits written vs the greedy head (argmax in the GEMM epilogue)
    eng = model.model if hasattr(model, "model") else model
    st = BatchedState(w.L, w.C, 256, device=dev)
    tok = torch.randint(0, w.V, (256,), device=dev)
    for name, f in (("logits", lambda: eng.decode_batch(tok, st)),
                    ("greedy_ids", lambda: eng.decode_batch_greedy(tok, st))):
        for _ in range(3):
            f()
        ms = timed(f, 20, stream)
        out.setdefault("decode_b256_eager", {})[name] = {"ms": ms, "tokens_per_s": 256 / (ms * 1e-3)}
    del st
    S = State(w.L, w.C, 64, device=dev)
    toks = torch.randint(0, w.V, (4096,), device=dev)
    f = lambda: model.prefill(toks, S)  # noqa: E731
    f()
    ms = timed(f, 3, stream)
    out["prefill_T4096"] = {"tokens_per_s": 4096 / (ms * 1e-3), "ms": ms}
    # prefill against the tensor roofline: the projections' GEMM flops (2 x parameters
    # of r/k/v, LoRA down + up, W_o, FFN key + value, per token; prefill runs no head)
    # plus the wkv recurrence's (~5 x 64 x 64 multiply-adds per head per token)
    C, L = w.C, w.L
    gemm_flop = 2 * L * (12 * C * C + 2 * 288 * C) * 4096
    wkv_flop = 2 * L * (C // 64) * 5 * 64 * 64 * 4096
    pk, pk_kind = peaks()
    tf = (gemm_flop + wkv_flop) / (ms * 1e-3) / 1e12
    out["prefill_roofline"] = {"bound": "tensor", "flop_per_call": gemm_flop + wkv_flop,
                               "achieved": tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                               "frac": tf / pk["bf16_tflops"], "peak_kind": pk_kind,
                               "T": 4096, "ms": ms}
    out.update(config_sweeps(model, w, dev, stream, pk["hbm_gbs"]))
    out["continuous_batching"] = continuous_batching(model, w, dev, stream, n_seqs=256,
                                                     max_new=128, max_batch=256)
    return out


def config_sweeps(model, w, dev, stream, hbm_gbs) -> dict:
    """The other BASELINE configs, timed beside the headline (rank 0, N=1):

    * config 1: the isolated wkv7 kernels, H=16, B in {1, 8, 64}, T in {1, 64, 1024,
      4096} (T=1: the one-token step kernel; T>1: the chunk-parallel kernel), against
      HBM (fp16 r/w/k/v/a/b in + y out, fp32 state read + write);
    * config 2: 0.1B decode at B in {1, 8, 64, 256} from random states (CUDA graph);
    * config 3: 0.4B forward at T in {8, 64, 128, 1024, 4096} then 32 greedy decode
      steps, one sequence.
    """
    from rwkv_tl_b200 import BatchedState, RWKV7Weight, State, _lib, make_rwkv7
    from rwkv_tl_b200.synth import CONFIG_0_1B, synth_checkpoint

    lib = _lib.load()
    out: dict = {"config1_wkv_sweep": {}, "config2_0p1b_decode": {}, "config3_0p4b_prefill": {}}
    H, h = 16, stream.cuda_stream
    g = torch.Generator(device=dev).manual_seed(11)
    for B in (1, 8, 64):
        for T in (1, 64, 1024, 4096):
            vec = [torch.randn(B, T, H, 64, generator=g, device=dev).half() for _ in range(7)]
            S = 0.1 * torch.randn(B, H, 64, 64, generator=g, device=dev)
            if T == 1:
                f = lambda: _lib.check(lib.rwkv7_dplr_step(  # noqa: E731
                    S.data_ptr(), *[t.data_ptr() for t in vec], B, H, h))
            else:
                nb = lib.rwkv7_dplr_chunked_workspace_bytes(B, T, H)
                ws = torch.empty(nb, dtype=torch.uint8, device=dev)
                f = lambda: _lib.check(lib.rwkv7_dplr_chunked(  # noqa: E731
                    S.data_ptr(), *[t.data_ptr() for t in vec], B, T, H, ws.data_ptr(), nb, h))
            for _ in range(3):
                f()
            ms = timed(f, 20 if B * T <= 65536 else 5, stream)
            algo = B * T * H * 64 * 2 * 7 + B * H * 64 * 64 * 4 * 2
            out["config1_wkv_sweep"][f"B{B}_T{T}"] = {
                "us": ms * 1e3, "tokens_per_s": B * T / (ms * 1e-3),
                "hbm_frac": algo / (ms * 1e-3) / 1e9 / hbm_gbs}
            del vec, S
    # config 2: 0.1B
    w1 = RWKV7Weight(synth_checkpoint(CONFIG_0_1B, seed=0, device=dev), device=dev)
    m1 = make_rwkv7(dev, backend="b200")(w1)
    gg = torch.Generator(device=dev).manual_seed(2)
    for B in (1, 8, 64, 256):
        st = BatchedState(w1.L, w1.C, B, device=dev)
        st.rnn.normal_(0.0, 0.1, generator=gg)
        tok = torch.randint(0, w1.V, (B,), generator=gg, device=dev)
        lg = torch.empty(B, w1.V, dtype=torch.float16, device=dev)
        f = lambda: m1.decode_batch(tok, st, logits=lg)  # noqa: E731
        for _ in range(3):
            f()
        ms = timed(f, 50, stream)
        out["config2_0p1b_decode"][f"B{B}"] = {"ms": ms, "tokens_per_s": B / (ms * 1e-3)}
    del m1, w1
    torch.cuda.empty_cache()
    # config 3: 0.4B forward(T) + 32 greedy steps
    for T in (8, 64, 128, 1024, 4096):
        toks = torch.randint(0, w.V, (T,), generator=gg, device=dev)
        S = State(w.L, w.C, 64, device=dev)

        def run():
            S.reset()
            logits, _ = model.forward(toks, S)
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            for _ in range(32):
                logits, _ = model.decode(logits.argmax(), S)
            return e

        run()
        s0 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s0.record(stream)
        mid = run()
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        torch.cuda.synchronize()
        fwd_ms, dec_ms = s0.elapsed_time(mid), mid.elapsed_time(e1)
        out["config3_0p4b_prefill"][f"T{T}"] = {
            "forward_ms": fwd_ms, "prefill_tokens_per_s": T / (fwd_ms * 1e-3),
            "decode32_ms": dec_ms, "decode_tokens_per_s": 32 / (dec_ms * 1e-3)}
    return out


def continuous_batching(model, w, dev, stream, n_seqs: int, max_new: int, max_batch: int,
                        world: int = 1, rank: int = 0, seed: int = 4,
                        prefill_tokens: int = 16384) -> dict:
    """Config 4: n_seqs requests, prompt lengths ~U[16, 2048] and token ids uniform
    (seeded), max_new greedy tokens each, through ``ContinuousBatcher`` with decode
    batches of up to max_batch; sequences sharded over ranks by prompt length. Timed
    with CUDA events around the whole run (the host scheduler included)."""
    from rwkv_tl_b200 import ContinuousBatcher, Request
    from rwkv_tl_b200.shard import shard_by_length

    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(16, 2049, (n_seqs,), generator=g).tolist()
    prompts = [torch.randint(0, w.V, (n,), generator=g) for n in lens]
    mine = shard_by_length(lens, world)[rank]
    eng = model.model if hasattr(model, "model") else model
    warm = ContinuousBatcher(eng, max_batch=max_batch, prefill_tokens=4096)
    for i in mine[:8]:
        warm.submit(Request(i, prompts[i][:64], 4))
    warm.run()
    del warm
    b = ContinuousBatcher(eng, max_batch=max_batch, prefill_tokens=prefill_tokens)
    for i in mine:
        b.submit(Request(i, prompts[i], max_new))
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    b.run()
    e.record(stream)
    torch.cuda.synchronize()
    sec = max_over_ranks(s.elapsed_time(e) * 1e-3, world)
    prompt_tok = sum(lens) if world > 1 else sum(lens[i] for i in mine)
    gen_tok = (n_seqs if world > 1 else len(mine)) * max_new
    return {"workload": f"{n_seqs} requests, prompts U[16,2048], {max_new} greedy tokens each, "
                        f"decode batch <= {max_batch} per GPU, prefill budget {prefill_tokens} tokens "
                        f"per scheduler step", "seconds": sec,
            "tokens_per_s": (prompt_tok + gen_tok) / sec, "generated_tokens_per_s": gen_tok / sec,
            "prompt_tokens": prompt_tok, "generated_tokens": gen_tok, "scheduler_steps": b.steps}


def run_profile(args):
    """Small driver for ncu: the same weights/kernels as the bench, one kind of call."""
    from rwkv_tl_b200 import BatchedState, RWKV7Weight, State, make_rwkv7
    from rwkv_tl_b200.synth import CONFIG_0_4B, synth_checkpoint

    dev = torch.device("cuda", 0)
    sd = synth_checkpoint(CONFIG_0_4B, seed=0, device=dev)
    w = RWKV7Weight(sd, device=dev)
    del sd
    model = make_rwkv7(dev, backend="b200", use_graph=False)(w)
    stream = torch.cuda.current_stream(dev)
    if args.profile == "decode":
        st = BatchedState(w.L, w.C, args.batch, device=dev)
        tok = torch.randint(0, w.V, (args.batch,), device=dev)
        f = lambda: model.decode_batch(tok, st)  # noqa: E731
    else:
        S = State(w.L, w.C, 64, device=dev)
        toks = torch.randint(0, w.V, (args.seq_len,), device=dev)
        f = lambda: model.prefill(toks, S)  # noqa: E731
    for _ in range(args.warmup):
        f()
    ms = timed(f, args.steps, stream)
    print(f"{args.profile}: {ms:.3f} ms per call", flush=True)


def run_continuous(args, world, rank, local):
    from rwkv_tl_b200 import RWKV7Weight, make_rwkv7
    from rwkv_tl_b200.synth import CONFIG_0_4B, synth_checkpoint

    dev = torch.device("cuda", local)
    w = RWKV7Weight(synth_checkpoint(CONFIG_0_4B, seed=0, device=dev), device=dev)
    model = make_rwkv7(dev, backend="b200", use_graph=False)(w)
    stream = torch.cuda.current_stream(dev)
    with Clocks(local) as clk:
        r = continuous_batching(model, w, dev, stream, n_seqs=args.continuous, max_new=128,
                                max_batch=args.batch, world=world, rank=rank)
    if rank == 0:
        print(json.dumps({"metric": "continuous batching tokens/s (prompt + generated), config 4",
                          "value": r["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
                          "higher_is_better": True, "scaling": "strong", "dtype": "f16",
                          "data": "synthetic", "config": r, "clocks": clk.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--cpu-tokens", type=int, default=16)
    ap.add_argument("--quick", action="store_true", help="skip side measurements / CPU baseline")
    ap.add_argument("--profile", choices=["decode", "prefill"], default=None,
                    help="profiling driver: run only K decode steps (--batch) or K prefills "
                         "(--seq-len) and print the per-call time, no JSON line")
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--continuous", type=int, default=0, metavar="N_SEQS",
                    help="run only config 4 (continuous batching of N_SEQS requests, 128 new "
                         "tokens each, sharded over the ranks) and print its JSON line")
    args = ap.parse_args()
    if args.impl == "b200":
        world, rank, local = dist_setup()
    else:  # the reference arm is CPU-only: rank 0 runs it, the other ranks exit
        world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")),
                              int(os.environ.get("RANK", "0")), 0)
    if args.profile:
        run_profile(args)
    elif args.continuous and args.impl == "b200":
        run_continuous(args, world, rank, local)
    elif args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_b200(args, world, rank, local)
    if world > 1 and args.impl == "b200":
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
