"""Decode throughput of the Llama-3.2-1B F16 hot path on B200.

Workload (one "step"): batch-1 greedy decode of the random-init
Llama-3.2-1B architecture -- 31 decode forwards at positions 16..46 after a
16-token prompt (the 32-token greedy run of the reference's headline config;
the prompt prefill and the first generated token happen once, untimed).
All 31 forwards run in ONE launch of the fused decode kernel.

  value  device time of the fused launch (CUDA events), inputs resident
  e2e    the public C-ABI call lc_decode per step: host token in, host token
         ids out (pinned copies inside the timed region)
  --impl reference   the oracle (C restatement of the reference's
                     PlainJavaKernelFactory path) on the host cores

Further workloads (one JSON line per case; the default run prints only the
headline line above):
  --suite serving    64 sequences x (128-token prompt + 256 greedy tokens)
                     through lc_batch_generate (tcgen05 batched products);
                     under torchrun the sequences are dealt over the ranks
  --suite kernels    the per-kernel sweeps: batched F16 products (GEMV
                     shapes of the 1B model, batch 1 / 8 / 64, weight copies
                     rotated past 4x L2), RMSNorm / SwiGLU / RoPE / softmax
                     rows, GQA decode attention (batch 1 / 64, 128..8192
                     cached positions); device time of back-to-back calls;
                     --only gemm,prefill,elementwise,attention picks sections
  --suite lmshard    (torchrun, N GPUs) lm_head rows sharded over the ranks:
                     logits slice on each GPU, then NCCL all-gather of the
                     slices or all-reduce of packed argmax keys

Multi-GPU (torchrun): one independent sequence per GPU (replicas, no
collective on the data path); value = sequences x tokens / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "llama3-java-hat_b200")]

import numpy as np  # noqa: E402

METRIC = "decode tok/s @1B F16 batch1"
PROMPT_LEN = 16
NEW_TOKENS = 32
DECODE_STEPS = NEW_TOKENS - 1  # forwards after the first generated token
SEED = 1234


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ------------------------------------------------------------- clocks ----

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------- roofline ----

def algorithmic_bytes(cfg, positions) -> int:
    """Bytes one decode launch must move at minimum (per position: every weight
    once, norm vectors, the embedding row, KV write + KV read of positions
    0..pos, the logits write)."""
    total = 0
    kv_row = cfg.n_layers * 2 * cfg.kv_dim * 4
    for pos in positions:
        total += cfg.weight_bytes()
        total += (2 * cfg.n_layers + 1) * cfg.dim * 4
        total += cfg.dim * 2
        total += kv_row + kv_row * (pos + 1)
        total += cfg.vocab * 4
    return total


def measured_peak():
    """(HBM GB/s, where the figure comes from): the measured copy bandwidth in
    MEASURED_PEAKS.json, or the profiling recipe's fallback when the file is
    absent."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6,650 GB/s (MEASURED_PEAKS.json absent)"


def committed_traffic():
    """DRAM bytes per launch of the fused decode kernel from the committed ncu
    summary (profiles/decode_kernel_traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d
    except (OSError, ValueError):
        return None


# -------------------------------------------------------- CPU baseline ----

class OracleDecode:
    """The oracle (C restatement of the reference's PlainJavaKernelFactory
    path) on the host, driven like the headline workload: the 16-token
    prompt is prefilled once (untimed, LlamaInference.java:186-193), then
    greedy decode forwards run at positions 16..46, wrapping back to 16 (the
    KV cache is rewritten in order, so every pass repeats the first)."""

    def __init__(self, cfg, w, prompt, threads: int):
        from oracle import oracle as O
        O.build()
        O.set_threads(threads)
        self.O = O
        self.threads = threads
        self.om = O.OracleModel(cfg, w)
        logits = None
        for pos, t in enumerate(prompt):
            logits = self.om.forward(int(t), pos)
        self.first = O.argmax(logits)
        self.tokens = {}  # position -> token fed there, recorded on the first pass
        self.pos = len(prompt)
        self.tok = self.first
        self.lo, self.hi = len(prompt), len(prompt) + DECODE_STEPS  # positions [lo, hi)

    def forward(self) -> None:
        logits = self.om.forward(int(self.tok), self.pos)
        self.tokens.setdefault(self.pos, int(self.tok))
        nxt = self.O.argmax(logits)
        self.pos += 1
        if self.pos >= self.hi:
            self.pos, nxt = self.lo, self.first
        self.tok = self.tokens.get(self.pos, nxt)


def cpu_sample(cfg, w, prompt, threads: int, budget_s: float):
    """Decode forwards of the oracle at the configured positions until
    `budget_s` is spent (at least 2); returns (forwards, seconds)."""
    od = OracleDecode(cfg, w, prompt, threads)
    n, t0 = 0, time.perf_counter()
    while True:
        od.forward()
        n += 1
        el = time.perf_counter() - t0
        if n >= 2 and el >= budget_s:
            break
    return n, el


# --------------------------------------------------------------- main ----

def run_reference(args):
    """The reference arm: the reference's CPU path for the headline workload.
    The reference cannot run here (Java 26 + Babylon HAT, no JDK), so its
    C restatement runs instead, on one host thread as the reference's plain
    path does (GEMV.java:76-91 is a single-threaded loop), at the configured
    decode positions 16..46 after a 16-token prefill.  Each step is a bounded
    sample of that workload: BENCH_REF_FORWARDS (default 2) consecutive
    decode forwards."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from llamahat.config import LLAMA_3_2_1B
    from llamahat.synth import synth_prompt, synth_weights
    cfg = LLAMA_3_2_1B
    w = synth_weights(cfg, seed=SEED)
    prompt = synth_prompt(PROMPT_LEN, seed=SEED)
    od = OracleDecode(cfg, w, prompt, threads=1)
    per_step = max(1, int(os.environ.get("BENCH_REF_FORWARDS", "2")))
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for _ in range(per_step):
            od.forward()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    tot = sum(times)
    value = per_step * len(times) / tot
    sample = (f"{per_step} oracle decode forwards per step at positions {od.lo}..{od.hi - 1} (cycled) after the "
              f"{PROMPT_LEN}-token prefill, 1 host thread of {os.cpu_count()} (the reference's plain path is "
              "single-threaded); C restatement of PlainJavaKernelFactory, not the Java reference (no JDK on this host)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * tot / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": 1, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config():
    return {"workload": "Llama-3.2-1B random-init F16 (seed 1234), 16-token prompt, greedy decode; one step = "
                        "31 decode forwards (positions 16..46) in one fused launch",
            "model": "llama-3.2-1b-arch", "batch": 1, "prompt_tokens": PROMPT_LEN, "decode_forwards": DECODE_STEPS,
            "global_batch": None, "seq_len": PROMPT_LEN + NEW_TOKENS - 1, "parallelism": "replicas",
            "l2": "weights 2.47 GB per forward > 126 MB L2: inputs larger than L2, no flush"}


def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    import llamahat
    from llamahat.config import LLAMA_3_2_1B
    from llamahat.synth import synth_prompt, synth_weights

    cfg = LLAMA_3_2_1B
    t0 = time.perf_counter()
    w = synth_weights(cfg, seed=SEED)
    log(f"[rank {rank}] weights generated in {time.perf_counter() - t0:.1f}s")
    acc = llamahat.Accelerator(local)
    model = llamahat.CudaModel(cfg, w, acc=acc)
    sess = llamahat.Session(model)
    prompt = synth_prompt(PROMPT_LEN, seed=SEED + rank)
    first = sess.generate(prompt, 1, stop=())  # prefill + first token (untimed)
    tok0 = int(first[0])
    out = np.zeros(DECODE_STEPS, np.int32)
    stream = torch.cuda.ExternalStream(acc.stream, device=torch.device("cuda", local))

    # warm-up
    for _ in range(args.warmup):
        sess.decode(tok0, PROMPT_LEN, DECODE_STEPS, out)
    ref_tokens = out.copy()

    # device-resident timing: CUDA events around each fused launch
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launch_ms = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            sess.decode(tok0, PROMPT_LEN, DECODE_STEPS, out)
            launch_ms.append(sess.last_ms())
        torch.cuda.synchronize()
        # e2e: events on the library stream bracketing the public calls
        # (pinned token H2D, launch, token ids D2H, host sync -- every step)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            sess.decode(tok0, PROMPT_LEN, DECODE_STEPS, out)
        e1.record(stream)
        e1.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    assert np.array_equal(out, ref_tokens), "decode is not deterministic"

    dev_ms = sum(launch_ms) / len(launch_ms)
    if dist:
        t = torch.tensor([dev_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, e2e_ms = float(t[0]), float(t[1])
    n = ws
    value = n * DECODE_STEPS / (dev_ms / 1000.0)
    e2e_value = n * DECODE_STEPS / (e2e_ms / 1000.0)

    line = None
    if rank == 0:
        positions = range(PROMPT_LEN, PROMPT_LEN + DECODE_STEPS)
        alg = algorithmic_bytes(cfg, positions)
        peak, peak_kind = measured_peak()
        achieved = alg / (dev_ms / 1000.0) / 1e9
        tr = committed_traffic()
        roof = {"bound": "hbm", "kernel": "decode_kernel<16>", "achieved": achieved, "peak": peak,
                "peak_source": peak_kind, "unit": "GB/s",
                "frac": achieved / peak, "algorithmic_bytes_per_launch": alg,
                "traffic": tr.get("dram_bytes_per_launch") if tr else None,
                "traffic_source": tr.get("source") if tr else None}
        cpu = None
        if not args.no_cpu_baseline:
            try:
                nf, el = cpu_sample(cfg, w, prompt, threads=1, budget_s=args.cpu_budget)
                cpu = {"value": nf / el, "unit": "tok/s", "cores": 1, "kind": "port",
                       "sample": f"{nf} oracle decode forwards at positions {PROMPT_LEN}..{PROMPT_LEN + DECODE_STEPS - 1}"
                                 f" (cycled) after the {PROMPT_LEN}-token prefill, 1 host thread, {el:.1f}s; C "
                                 "restatement of PlainJavaKernelFactory (no JDK on the host)"}
            except Exception as e:  # pragma: no cover - reported, not fatal
                cpu = {"error": str(e)}
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "weights": "f16", "data": "synthetic",
            "config": workload_config(), "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * DECODE_STEPS, "ms_per_step": e2e_ms},
            # one fused decode launch per step in each timed loop (device and e2e)
            "gpu_launches": 2 * args.steps, "clocks": clk.summary(),
            "per_forward_us": 1000.0 * dev_ms / DECODE_STEPS,
        }
    sess.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ suites ----

SERVE_SEQS, SERVE_PROMPT, SERVE_NEW = 64, 128, 256


def run_serving(args):
    """Multi-sequence serving: SERVE_SEQS sequences x (SERVE_PROMPT prompt +
    SERVE_NEW greedy tokens), dealt over the ranks (strong scaling)."""
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    import llamahat
    from llamahat.config import LLAMA_3_2_1B
    from llamahat.synth import synth_weights
    cfg = LLAMA_3_2_1B.with_(max_seq=SERVE_PROMPT + SERVE_NEW)
    w = synth_weights(cfg, seed=SEED)
    acc = llamahat.Accelerator(local)
    model = llamahat.CudaModel(cfg, w, acc=acc)
    rng = np.random.default_rng(SEED)
    prompts = [rng.integers(0, 128000, SERVE_PROMPT).astype(np.int32) for _ in range(SERVE_SEQS)]
    mine = prompts[rank::ws]
    b = llamahat.Batch(model, len(mine))
    for _ in range(args.warmup):
        ref = b.generate(mine, SERVE_NEW, stop=())
    if dist:
        dist.barrier()
    dev, dec, wall = [], [], []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            out = b.generate(mine, SERVE_NEW, stop=())
            wall.append(time.perf_counter() - t0)
            tot_ms, dec_ms, nsteps = b.last_ms()
            dev.append(tot_ms)
            dec.append(dec_ms)
    assert all(np.array_equal(x, y) for x, y in zip(out, ref)), "serving is not deterministic"
    dev_ms, dec_ms, wall_ms = statistics.median(dev), statistics.median(dec), 1000 * statistics.median(wall)
    if dist:
        t = torch.tensor([dev_ms, dec_ms, wall_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, dec_ms, wall_ms = float(t[0]), float(t[1]), float(t[2])
    tokens = SERVE_SEQS * SERVE_NEW
    line = None
    if rank == 0:
        # algorithmic bytes: every weight once per step per GPU, KV read of
        # positions 0..pos and write of pos for every sequence of the step
        per_gpu = len(mine)
        kv_row = cfg.n_layers * 2 * cfg.kv_dim * 4
        steps = SERVE_PROMPT + SERVE_NEW - 1
        alg = steps * (cfg.weight_bytes()) + sum(per_gpu * kv_row * (p + 2) for p in range(steps))
        peak, peak_kind = measured_peak()
        achieved = alg / (dev_ms / 1000) / 1e9
        cpu = None
        if not args.no_cpu_baseline:
            nf, el = cpu_sample(cfg, w, prompts[0][:PROMPT_LEN], threads=1, budget_s=args.cpu_budget)
            cpu = {"value": nf / el, "unit": "tok/s", "cores": 1, "kind": "port",
                   "sample": f"{nf} oracle decode forwards of one sequence after a {PROMPT_LEN}-token prefix on 1 "
                             f"host thread, {el:.1f}s (per-forward cost is the 2.47 GB weight stream; the reference "
                             "serves sequences one generate call after another)"}
        line = {
            "metric": "serving generated tok/s @1B F16 64 seqs x (128 prompt + 256 new)", "value": tokens / (dev_ms / 1000),
            "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "weights": "f16",
            "data": "synthetic",
            "config": {"workload": f"{SERVE_SEQS} sequences x ({SERVE_PROMPT}-token prompt, ids uniform [0,128000) "
                                   f"seed {SEED}, + {SERVE_NEW} greedy tokens), Llama-3.2-1B random-init F16; one step "
                                   "= one lc_batch_generate call (all prompt tokens as one prefill of row-tiled "
                                   "products, then one graph replay per decode position)",
                       "model": "llama-3.2-1b-arch", "batch": SERVE_SEQS, "seqs_per_gpu": per_gpu,
                       "parallelism": f"sequences dealt over {ws} GPU(s), no collective",
                       "l2": "weights 2.47 GB per step > L2: no flush"},
            # decode phase: the positions after each sequence's first token
            "decode_tok_s": SERVE_SEQS * (SERVE_NEW - 1) / (dec_ms / 1000), "decode_ms": dec_ms,
            "prefill_ms": dev_ms - dec_ms, "positions": steps,
            "roofline": {"bound": "hbm", "kernel": "whole step (all kernels)", "achieved": achieved, "peak": peak,
                         "peak_source": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak, "algorithmic_bytes_per_launch": alg, "traffic": None},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (wall_ms / 1000), "unit": "tok/s",
                    "h2d_bytes_per_step": SERVE_SEQS * SERVE_PROMPT * 4, "d2h_bytes_per_step": tokens * 4,
                    "ms_per_step": wall_ms},
            "clocks": clk.summary(),
        }
    b.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def device_us(calls, stream, reps=3):
    """Device microseconds per call of `calls` (enqueue-only library calls on
    `stream`), run back to back.  A bounded sleep kernel holds the stream
    while the host enqueues them, so the events around the calls measure GPU
    time only, not host launch overhead."""
    import torch
    for c in calls[:2]:
        c()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for c in calls:
        c()
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    cycles = int(max(2e6, 3 * host_s * 2.0e9))  # ~3x the enqueue time at 2 GHz
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for _ in range(reps):
        with torch.cuda.stream(stream):
            torch.cuda._sleep(cycles)
        e0.record(stream)
        for c in calls:
            c()
        e1.record(stream)
        e1.synchronize()
        t = e0.elapsed_time(e1) * 1000 / len(calls)
        best = t if best is None else min(best, t)
    return best


def run_kernels(args):
    import torch
    import llamahat
    from llamahat import CudaKernelFactory
    acc = llamahat.Accelerator(0)
    f = CudaKernelFactory()
    gemv, rms, rope, silu, soft, att = (f.createGEMV(acc), f.createRMSNorm(acc), f.createRoPE(acc),
                                         f.createSiLU(acc), f.createSoftmax(acc), f.createAttention(acc))
    st = torch.cuda.ExternalStream(acc.stream)
    L2 = 126 * 1024 * 1024
    peak, peak_kind = measured_peak()
    out = []
    only = set(args.only.split(",")) if args.only else None

    def want(section):
        return only is None or section in only

    def emit(kind, case, us, nbytes, extra=None):
        gbs = nbytes / (us * 1e-6) / 1e9
        d = {"suite": kind, "case": case, "us_per_call": us, "algorithmic_bytes": nbytes, "GB_s": gbs,
             "frac_of_hbm_peak": gbs / peak, "peak_source": peak_kind}
        if extra:
            d.update(extra)
        out.append(d)
        print(json.dumps(d), flush=True)

    # Batched F16 products on the model's GEMV shapes (out x in).
    shapes = [(2048, 2048, "q/o"), (512, 2048, "k/v"), (8192, 2048, "gate/up"), (2048, 8192, "down"),
              (3072, 2048, "fused qkv"), (16384, 2048, "fused gate|up"), (128256, 2048, "lm_head")]
    for rows, cols, name in (shapes if want("gemm") else []):
        wb = rows * cols * 2
        ncopy = max(1, min(256, -(-4 * L2 // wb)))
        Ws = []
        for _ in range(ncopy):
            W = (torch.randn(rows * cols, device="cuda") * 0.02).half()
            Wt = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
            gemv.tile(W.view(torch.int16), Wt, rows, cols)
            Ws.append(Wt)
        torch.cuda.synchronize()
        reps = max(ncopy, 8)
        for B in (1, 8, 64):
            X = torch.randn(B, cols, device="cuda")
            Y = torch.empty(B, rows, device="cuda")
            calls = [lambda i=i: gemv.apply_batched_tiled(Ws[i % ncopy], X, Y, rows, cols, B) for i in range(reps)]
            us = device_us(calls, st)
            emit("gemm_tcgen05", f"{name} {rows}x{cols} batch {B}", us, wb + B * (rows + cols) * 4,
                 {"weight_copies": ncopy, "launches_per_call": "split + product (+ reduce when K is split)"})
        if ncopy == 1 or rows * cols * 2 * ncopy <= 8 * L2:
            # the IGEMV path on row-major weights (CUDA-core streaming kernel), batch 1
            Wr = [(torch.randn(rows * cols, device="cuda") * 0.02).half() for _ in range(ncopy)]
            x = torch.randn(cols, device="cuda")
            y = torch.empty(rows, device="cuda")
            calls = [lambda i=i: gemv.apply(Wr[i % ncopy], x, y, rows, cols) for i in range(reps)]
            us = device_us(calls, st)
            emit("gemv_rowmajor", f"{name} {rows}x{cols} batch 1", us, wb + (rows + cols) * 4, {"weight_copies": ncopy})
            del Wr
        del Ws
        torch.cuda.empty_cache()

    # Prefill products: 8192 activation rows (64 sequences x 128 prompt
    # tokens) on the layer shapes; tensor-bound, reported as TFLOP/s of the
    # useful product (2 M N K) and of the tensor work (the hi / lo halves
    # double it) against the measured bf16 GEMM peak.
    tpeak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpeak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        tpeak = 1590.0
    prefill_shapes = [(3072, 2048, "fused qkv"), (2048, 2048, "o"), (16384, 2048, "fused gate|up"), (2048, 8192, "down")]
    for rows, cols, name in (prefill_shapes if want("prefill") else []):
        M = 8192
        W = (torch.randn(rows * cols, device="cuda") * 0.02).half()
        Wt = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
        gemv.tile(W.view(torch.int16), Wt, rows, cols)
        X = torch.randn(M, cols, device="cuda")
        Y = torch.empty(M, rows, device="cuda")
        us = device_us([lambda: gemv.apply_batched_tiled(Wt, X, Y, rows, cols, M)] * 4, st)
        useful = 2.0 * M * rows * cols / (us * 1e-6) / 1e12
        d = {"suite": "gemm_tcgen05_prefill", "case": f"{name} {rows}x{cols} rows {M}", "us_per_call": us,
             "useful_TFLOP_s": useful, "tensor_TFLOP_s": 2 * useful, "frac_of_bf16_peak": 2 * useful / tpeak,
             "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst)",
             "algorithmic_bytes": rows * cols * 2 + M * (rows + cols) * 4, "GB_s": (rows * cols * 2 + M * (rows + cols) * 4) / (us * 1e-6) / 1e9,
             "frac_of_hbm_peak": (rows * cols * 2 + M * (rows + cols) * 4) / (us * 1e-6) / 1e9 / peak}
        out.append(d)
        print(json.dumps(d), flush=True)
        del W, Wt, X, Y
        torch.cuda.empty_cache()

    # Elementwise rows (fp32 ~N(0,1)); copies rotated past 4x L2 where small.
    wn = torch.ones(2048, device="cuda")
    for rows in ((1, 64, 4096) if want("elementwise") else ()):
        nb = rows * 2048 * 4
        ncopy = max(1, min(64, -(-4 * L2 // nb)))
        xs = [torch.randn(rows, 2048, device="cuda") for _ in range(ncopy)]
        calls = [lambda i=i: rms.apply_rows(xs[i % ncopy], wn, rows, 2048) for i in range(max(ncopy, 8))]
        emit("rmsnorm", f"width 2048 rows {rows}", device_us(calls, st), 2 * nb + 2048 * 4)
        g = [torch.randn(rows, 8192, device="cuda") for _ in range(ncopy)]
        u = [torch.randn(rows, 8192, device="cuda") for _ in range(ncopy)]
        calls = [lambda i=i: silu.swiglu(g[i % ncopy], u[i % ncopy], rows * 8192) for i in range(max(ncopy, 8))]
        emit("swiglu", f"width 8192 rows {rows}", device_us(calls, st), 3 * rows * 8192 * 4)
        pos = torch.randint(0, 8192, (rows,), dtype=torch.int32, device="cuda")
        for heads, nm in ((32, "q 32x64"), (8, "k 8x64")):
            v = [torch.randn(rows, heads * 64, device="cuda") for _ in range(ncopy)]
            calls = [lambda i=i: rope.apply_rows(v[i % ncopy], pos, rows, heads, 64, 500000.0)
                     for i in range(max(ncopy, 8))]
            emit("rope", f"{nm} rows {rows} pos uniform [0,8192)", device_us(calls, st), 2 * rows * heads * 64 * 4 + rows * 4)
        for width in (128, 1024, 8192):
            nbs = rows * width * 4
            nc = max(1, min(64, -(-4 * L2 // nbs)))
            sx = [torch.randn(rows, width, device="cuda") * 2.0 for _ in range(nc)]
            calls = [lambda i=i: soft.apply_rows(sx[i % nc], rows, width) for i in range(max(nc, 8))]
            emit("softmax", f"width {width} rows {rows} values N(0,4)", device_us(calls, st), 2 * nbs)
        del xs, g, u
        torch.cuda.empty_cache()

    # GQA decode attention: 32 q heads / 8 kv heads, head_dim 64, fp32 KV,
    # one query per sequence; a call = one layer, 16 layers timed.
    for B in ((1, 64) if want("attention") else ()):
        for L in (128, 1024, 8192):
            per_layer = B * 8 * L * 64 * 4 * 2
            ncopy = 1 if per_layer >= 4 * L2 else min(16, -(-4 * L2 // per_layer))
            ks = [torch.randn(B * 8 * L * 64, device="cuda") for _ in range(ncopy)]
            vs = [torch.randn(B * 8 * L * 64, device="cuda") for _ in range(ncopy)]
            q = torch.randn(B * 32 * 64, device="cuda")
            o = torch.empty(B * 32 * 64, device="cuda")
            lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
            calls = [lambda i=i: att.decode_maxlen(q, ks[i % ncopy], vs[i % ncopy], o, lens, B, 32, 8, 64,
                                                   8 * L * 64, L * 64, 64, L) for i in range(16)]
            us = device_us(calls, st)
            emit("attention", f"batch {B} cached {L} per layer", us, per_layer + 2 * B * 32 * 64 * 4,
                 {"kv_copies": ncopy})
            del ks, vs
            torch.cuda.empty_cache()
    return 0


def run_lmshard(args):
    """lm_head row-shard study: rank r of N owns rows shard_rows(vocab, N, r)
    of the 128256 x 2048 lm_head, computes its logits slice on the tcgen05
    product, then the ranks either all-gather the slices (NCCL) or
    max-all-reduce one packed argmax key per sequence.  Device time of
    back-to-back steps, max over ranks; compute and exchange reported apart."""
    import datetime
    import torch
    import torch.distributed as dist
    import llamahat
    from llamahat import CudaKernelFactory
    from llamahat.shard import PeerKeyExchange, shard_rows
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    acc = llamahat.Accelerator(local)
    gemv = CudaKernelFactory().createGEMV(acc)
    st = torch.cuda.ExternalStream(acc.stream, device=torch.device("cuda", local))
    kx = PeerKeyExchange(acc, ws, rank, max_batch=64)  # mailbox handles gathered over the process group
    V, D, L2 = 128256, 2048, 126 * 1024 * 1024
    lo, hi = shard_rows(V, ws, rank)
    n = hi - lo
    wb = n * D * 2
    ncopy = max(1, min(16, -(-4 * L2 // wb)))
    torch.manual_seed(SEED + rank)
    Ws = []
    for _ in range(ncopy):
        W = (torch.randn(n * D, device="cuda") * 0.02).half()
        Wt = torch.empty(n * D, dtype=torch.int16, device="cuda")
        gemv.tile(W.view(torch.int16), Wt, n, D)
        Ws.append(Wt)
    torch.cuda.synchronize()
    sign = -(1 << 63)
    res = {}
    for B in (1, 64):
        torch.manual_seed(SEED)
        X = torch.randn(B, D, device="cuda")
        Y = torch.empty(B, n, device="cuda")
        G = torch.empty(ws * B * n, device="cuda")
        K = torch.empty(B, dtype=torch.int64, device="cuda")
        it = [0]

        def compute():
            gemv.apply_batched_tiled(Ws[it[0] % ncopy], X, Y, n, D, B)
            it[0] += 1

        def gather():
            with torch.cuda.stream(st):
                if ws > 1:
                    dist.all_gather_into_tensor(G, Y.view(-1))
                else:
                    G.copy_(Y.view(-1))

        def keyreduce():
            with torch.cuda.stream(st):
                K.bitwise_xor_(sign)  # unsigned key order -> signed order
                if ws > 1:
                    dist.all_reduce(K, op=dist.ReduceOp.MAX)

        def compute_key():
            # the product's logits epilogue writes the slice's packed argmax keys
            gemv.apply_batched_tiled_argmax(Ws[it[0] % ncopy], X, Y, n, D, B, lo, K)
            it[0] += 1

        def peerreduce():
            kx.allreduce(K, B)  # NVLink peer stores into every rank's mailbox, bounded waits

        cases = {"compute": [compute] * 16, "gather": [gather] * 16,
                 "compute+gather": [lambda: (compute(), gather())] * 16,
                 "compute_with_argmax_keys": [compute_key] * 16,
                 "compute_with_argmax_keys+key_allreduce": [lambda: (compute_key(), keyreduce())] * 16,
                 "compute_with_argmax_keys+peer_key_exchange": [lambda: (compute_key(), peerreduce())] * 16}
        for name, calls in cases.items():
            us = device_us(calls, st)
            t = torch.tensor([us], device="cuda")
            if ws > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[f"B{B} {name}"] = float(t)
        # consistency: the gathered argmax, the key all-reduce and the peer
        # key exchange agree (all on the same weight copy)
        it0 = it[0]
        compute_key()
        gather()
        keyreduce()
        torch.cuda.synchronize()
        full = G.view(ws, B, n).permute(1, 0, 2).reshape(B, ws * n)[:, :V]
        idx_full = full.argmax(dim=1)
        idx_key = (~(K & 0xFFFFFFFF)) & 0xFFFFFFFF
        assert torch.equal(idx_full.cpu(), idx_key.cpu()), "gathered argmax != key all-reduce"
        it[0] = it0
        compute_key()
        peerreduce()
        torch.cuda.synchronize()
        acc.synchronize()
        idx_peer = (~(K & 0xFFFFFFFF)) & 0xFFFFFFFF
        assert torch.equal(idx_full.cpu(), idx_peer.cpu()), "gathered argmax != peer key exchange"
    if rank == 0:
        peak, kind = measured_peak()
        line = {"suite": "lmshard", "metric": "lm_head row-shard step, us (max over ranks)", "n_gpus": ws,
                "rows_per_gpu": n, "bytes_per_gpu": wb, "weight_copies": ncopy, "us": res,
                "compute_GB_s_per_gpu": {f"B{B}": (wb + B * (n + D) * 4) / (res[f'B{B} compute'] * 1e-6) / 1e9
                                         for B in (1, 64)},
                "peak_GB_s": peak, "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})",
                "exchange": "NCCL all_gather_into_tensor of the fp32 slices; or all_reduce(MAX) of one int64 key "
                            "per sequence (NCCL); or lc_keyx_allreduce: the keys stored into every rank's "
                            "mailbox over NVLink peer memory, bounded flag waits", "scaling": "strong"}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
    kx.close()
    if ws > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--suite", choices=["headline", "serving", "kernels", "lmshard"], default="headline")
    ap.add_argument("--only", default="", help="kernels suite: comma-separated sections to run "
                    "(gemm, prefill, elementwise, attention); default all")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.suite == "serving":
        return run_serving(args)
    if args.suite == "kernels":
        return run_kernels(args)
    if args.suite == "lmshard":
        return run_lmshard(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
