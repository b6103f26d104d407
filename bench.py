"""Benchmark of the B200 decode and readout-validation path.

Headline: decode tok/s of a Qwen3-0.6B-architecture model (random-init bf16,
seed 7), batch 1, greedy 32 tokens from a 24-token prompt of seeded random ids.
One bench step is one such generation: 24 prompt tokens and 31 generated tokens
go through the model one at a time (the reference feeds prompts token by token,
src/diagnosis.rs:81-99), i.e. 55 decode steps; `value` counts decode steps (tokens
through the model) per second, device-timed with CUDA events on the library's
stream.  `e2e` is the same generation through the C ABI call lsx_model_generate
with host buffers (prompt upload, token and Frame downloads inside the timing).

Sub-objects of the same line, one per measured configuration:
  readout         fused readout-margin validation of 4096 RMSNorm'd bf16 hidden
                  states against lm_head [151936, 1024] with a rank-16 Givens edit
  gemv            the bf16 GEMV microbenchmark (five shapes)
  long4b_batch    Qwen3-4B, 16 sequences decoded together after 4096-token prompts
  score8b         Qwen3-8B teacher-forced scoring, 64 cases per GPU
  readout_vocab   (N > 1) the validation with the lm_head split by vocabulary rows
  triton_baseline (N = 1) the reference's own Triton kernels on this GPU, in its
                  runtime pattern and as a CUDA graph (baseline/triton_reference.py)
Each carries its roofline, and (N = 1) a CPU baseline from the oracle.

Multi-GPU (torchrun): decode runs as one independent replica per GPU (a batch-1
stream does not shard); readout validation is row-sharded with a fixed 4096 rows
per GPU and every step all-gathers the per-row results to every rank (NCCL);
scoring is case-sharded; the vocabulary-sharded validation merges its shards with
one NCCL all-reduce per step.  Timing is the maximum over ranks.

--impl reference times the reference's CPU path (the oracle restatement of
tests/qwen_reference.rs's CPU forward, KV-cached, f64 reductions) on the host
cores over the same 55-step generation, with inputs from the oracle's own
generator; the reference's Rust crate cannot be built here.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

PROMPT, GENERATE = 24, 32
STEPS_PER_GENERATION = PROMPT + GENERATE - 1
READOUT_ROWS, VOCAB, HIDDEN, RANK = 4096, 151936, 1024, 16
METRIC = "decode tok/s (Qwen3-0.6B bs1, % HBM roofline); readout-margin rows/s"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# dominant kernel of each leg on this workload, from ncu captures of this script
# (--profile): persistent_decode_kernel per 55-step generation, and
# readout_pair_kernel per 4096-row validation.
DECODE_TRAFFIC_PER_LAUNCH = 65_560_912_000 + 31_543_296
READOUT_TRAFFIC_PER_LAUNCH = 339_733_248 + 4_837_888


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def decode_bytes_per_step(prompt=PROMPT, generate=GENERATE):
    """Algorithmic bytes of one decode step averaged over the generation: every
    bf16 weight once (28 layers x 15,728,640 + lm_head 151936 x 1024) plus the f32
    KV cache read (positions 0..t) and the new K/V write."""
    weights = 2 * (28 * 15_728_640 + 151_936 * 1024)
    steps = prompt + generate - 1
    kv_read = sum(28 * (t + 1) * 8192 for t in range(steps)) / steps
    return weights + kv_read + 28 * 8192


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
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
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- workload ----
def build_checkpoint(rank: int = 0, layers: int = 28) -> Path:
    """The Qwen3-0.6B-architecture checkpoint of the decode workload (seed 7),
    written once per machine (every rank shares it)."""
    from laplacesscissors_b200 import synth
    return synth.cached_checkpoint("QWEN3_0_6B", layers=layers) if layers != 28 else \
        synth.cached_checkpoint("QWEN3_0_6B")


def decode_config(world: int) -> dict:
    """`config` of the headline line (both arms print the same)."""
    return {"workload": "Qwen3-0.6B bs1 greedy decode, 24-token prompt + 32 tokens",
            "decode_steps_per_step": STEPS_PER_GENERATION, "batch": 1, "kv_cache": "f32",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "weights 1.19 GB per token > 126 MB L2 (no flush needed)"}


def readout_inputs(rank: int = 0, world: int = 1):
    """This rank's row shard of the validation set: READOUT_ROWS rows per rank out
    of a seeded global set of READOUT_ROWS x world rows (weak scaling); the lm_head
    and the edit are shared."""
    from laplacesscissors_b200 import random_subspace_rotation, synth
    from laplacesscissors_b200.sharding import row_shard
    w = synth.normal_bf16(7, 0, VOCAB * HIDDEN, 0.02)
    lo, hi = row_shard(READOUT_ROWS * world, world, rank)
    hidden = synth.readout_hidden(7, hi - lo, HIDDEN, first=lo)
    targets = synth.readout_targets(7, hi - lo, VOCAB, first=lo)
    edit = random_subspace_rotation(HIDDEN, RANK, 3.0, seed=7)
    return w, hidden, targets, edit


# ------------------------------------------------------------ CPU legs -----
def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_decode_rate(ckpt: Path, generations: int = 1):
    """The oracle's decode of the same checkpoint and prompt on the host cores: the
    whole 55-step generation (prompt token by token, then greedy), `generations`
    times.  Inputs come from the oracle's own generator (no library code runs)."""
    from oracle import binding as oracle
    from oracle import synth as osynth
    threads = cpu_threads()
    m = oracle.OracleModel(ckpt, 64, threads=threads)
    prompt = osynth.prompt_tokens(7, PROMPT, VOCAB)
    m.cursor = 0
    m.advance(int(prompt[0]))  # warm-up: pages the weights in
    t0 = time.perf_counter()
    for _ in range(generations):
        m.cursor = 0
        m.generate(prompt, GENERATE)
    dt = time.perf_counter() - t0
    return generations * STEPS_PER_GENERATION / dt, threads, \
        f"{generations} whole generation(s) of 55 decode steps (oracle, f64 reductions, {threads} threads)"


def cpu_gemv_rates(seconds: float = 0.5) -> tuple[dict, int]:
    """The oracle's GEMV (f64 accumulation over bf16 W, f32 x) on the host cores for
    every microbenchmark shape, each repeated for about `seconds`: GB/s of the same
    2NK + 4K + 4N bytes per GEMV.  Inputs from the oracle's own generator."""
    from oracle import binding as oracle
    from oracle import synth as osynth
    threads = cpu_threads()
    out = {}
    for n, k in GEMV_SHAPES:
        w = osynth.normal_bf16(7, 100 + n, n * k, 0.02)
        x = osynth.normal_f32(7, 200 + k, k)
        oracle.matvec(w, oracle.BF16, x, None, n, k, threads)
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < seconds:
            oracle.matvec(w, oracle.BF16, x, None, n, k, threads)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        out[f"{n}x{k}"] = (2 * n * k + 4 * k + 4 * n) / dt / 1e9
    return out, threads


def cpu_readout_rate(w, hidden, targets, edit, seconds: float = 8.0):
    from laplacesscissors_b200 import synth
    from oracle import binding as oracle
    threads = cpu_threads()
    rows = 8
    h = synth.bf16_to_f32(hidden[:rows]).astype(np.float64)
    edited = np.stack([edit.apply(x) for x in h]).astype(np.float32)
    t0 = time.perf_counter()
    done = 0
    while done == 0 or (time.perf_counter() - t0 < seconds and done < 64):
        oracle.readout_rows(w, oracle.BF16, None, VOCAB, HIDDEN, edited, targets[:rows], threads)
        done += rows
    dt = time.perf_counter() - t0
    return done / dt, threads, f"{done} rows (oracle readout with the rank-16 edit, f64 accumulation)"


# ------------------------------------------------------------ GPU legs -----
def cuda_timer(gpu):
    import torch
    stream = torch.cuda.ExternalStream(gpu.stream())

    def make():
        e = torch.cuda.Event(enable_timing=True)
        return e
    return stream, make


def run_decode(gpu, ckpt: Path, steps: int, warmup: int, dist, e2e: bool = True):
    import ctypes as C
    import torch

    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    from laplacesscissors_b200._lib import check, lib
    from laplacesscissors_b200.model import _fp, _up
    model = lsx.Model.load(ckpt, gpu, 64)
    assert model.fused
    prompt = np.ascontiguousarray(synth.prompt_tokens(7, PROMPT, VOCAB), dtype=np.uint32)
    tokens = np.empty(GENERATE, np.uint32)
    n = C.c_size_t()
    stopped = C.c_int()

    def generate(frames_h=None, frames_z=None):
        check(lib.lsx_model_generate(model.handle, _up(prompt), PROMPT, GENERATE, None, 0, None, _up(tokens),
                                     C.byref(n), C.byref(stopped), frames_h, frames_z))

    stream, event = cuda_timer(gpu)
    # Device-timed: the same generation with no frame copies; the graph replays
    # enqueue back to back and CUDA events bracket K generations.
    for _ in range(warmup):
        generate()
    gpu.synchronize()
    dist.barrier()
    start, stop = event(), event()
    with ClockSampler(gpu.device) as clocks:
        start.record(stream)
        for _ in range(steps):
            generate()
        stop.record(stream)
        stop.synchronize()
    dev_ms = start.elapsed_time(stop)
    dist.barrier()
    info = model.info()
    # End to end through the C ABI with host buffers: prompt in, tokens and the
    # Frame (hidden + logits) of every generated token out.
    hid = np.empty((GENERATE, HIDDEN), np.float32)
    lg = np.empty((GENERATE, VOCAB), np.float32)
    e2e_s = float("nan")
    if e2e:
        for _ in range(max(1, warmup)):
            generate(_fp(hid), _fp(lg))
        gpu.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            generate(_fp(hid), _fp(lg))
        e2e_s = time.perf_counter() - t0
    first_tokens = [int(t) for t in tokens[:8]]
    return {"dev_ms": dev_ms, "e2e_s": e2e_s, "clocks": clocks.summary(), "tokens": first_tokens,
            "h2d": prompt.nbytes, "d2h": tokens.nbytes + hid.nbytes + lg.nbytes, "model": model,
            "graph": int(info.graph), "kernels_per_step": int(info.kernels_per_step),
            "persistent": int(info.persistent)}


GEMV_SHAPES = [(2048, 1024), (6144, 1024), (1024, 3072), (151936, 1024), (12288, 4096)]


def run_gemv(gpu, iters: int = 20, e2e_iters: int = 200):
    """The bf16 GEMV microbenchmark: y = W x through lsx_linear_into (the drop-in
    for Gpu::linear / kernels/ops.py matvec), W [N, K] bf16 N(0, 0.02), x f32 from
    bf16 N(0, 1), y f32.  Launches over enough weight copies to exceed L2 (>= 256 MB
    per pass) are captured once in a CUDA graph so launch gaps do not count;
    CUDA events time `iters` replays.  bytes = 2NK + 4K + 4N per GEMV.
    End to end, per GEMV as the reference's Model calls it: x uploaded from the
    host (lsx_upload_f32), Gpu::linear (lsx_linear, a fresh output), y read back
    to the host (lsx_read); W stays resident and rotates over the same copies;
    host clock over `e2e_iters` GEMVs."""
    import ctypes as C
    from cuda.bindings import runtime as rt

    from laplacesscissors_b200 import synth
    from laplacesscissors_b200._lib import BF16
    stream = gpu.stream()
    out = {}
    for n, k in GEMV_SHAPES:
        w_host = synth.normal_bf16(7, 100 + n, n * k, 0.02)
        copies = max(2, min(64, -(-256_000_000 // (2 * n * k))))
        ws = [gpu.upload_raw(w_host, BF16) for _ in range(copies)]
        x = gpu.upload_f32(synth.bf16_to_f32(synth.normal_bf16(7, 200 + k, k)))
        y = gpu.zeros(n)
        gpu.synchronize()

        def ok(r):
            err = r[0] if isinstance(r, tuple) else r
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cuda runtime: {err}")
            return r[1] if isinstance(r, tuple) and len(r) > 1 else None

        ok(rt.cudaStreamBeginCapture(stream, rt.cudaStreamCaptureMode.cudaStreamCaptureModeRelaxed))
        for w in ws:
            gpu.linear_into(x, w, None, n, k, y)
        graph = ok(rt.cudaStreamEndCapture(stream))
        exe = ok(rt.cudaGraphInstantiate(graph, 0))
        for _ in range(3):
            ok(rt.cudaGraphLaunch(exe, stream))
        start, stop = ok(rt.cudaEventCreate()), ok(rt.cudaEventCreate())
        ok(rt.cudaEventRecord(start, stream))
        for _ in range(iters):
            ok(rt.cudaGraphLaunch(exe, stream))
        ok(rt.cudaEventRecord(stop, stream))
        ok(rt.cudaEventSynchronize(stop))
        ms = ok(rt.cudaEventElapsedTime(start, stop)) / (iters * copies)
        nbytes = 2 * n * k + 4 * k + 4 * n
        out[f"{n}x{k}"] = {"us": ms * 1e3, "GB/s": nbytes / (ms * 1e-3) / 1e9, "weight_copies": copies}
        x_host = gpu.read(x)
        for r in range(3):
            gpu.read(gpu.linear(gpu.upload_f32(x_host), ws[r % copies], None, n, k))
        t0 = time.perf_counter()
        for r in range(e2e_iters):
            y_host = gpu.read(gpu.linear(gpu.upload_f32(x_host), ws[r % copies], None, n, k))
        dt = (time.perf_counter() - t0) / e2e_iters
        assert y_host.size == n
        out[f"{n}x{k}"]["e2e"] = {"us": dt * 1e6, "GB/s": nbytes / dt / 1e9, "h2d_bytes": 4 * k, "d2h_bytes": 4 * n}
        ok(rt.cudaGraphExecDestroy(exe))
        ok(rt.cudaGraphDestroy(graph))
        ok(rt.cudaEventDestroy(start))
        ok(rt.cudaEventDestroy(stop))
        del ws
    return out


def run_readout(gpu, inputs, steps: int, warmup: int, dist, e2e: bool = True):
    """The validation step on device-resident rows.  With several ranks each step
    ends with one NCCL all-gather of every rank's per-row results (margin f64,
    argmax u32, target logit f32: 16 B per row) on the library's stream, so every
    rank holds the whole validation's results, as verify_cached aggregates one
    Verification over all rows (src/diagnosis.rs:493-580); the gather alone is
    timed as well."""
    import ctypes as C
    import torch

    from laplacesscissors_b200 import DeviceRotation
    from laplacesscissors_b200._lib import BF16, check, lib
    w, hidden, targets, edit = inputs
    weight = gpu.upload_raw(w, BF16)
    rot = DeviceRotation.upload_edit(gpu, edit, HIDDEN)
    dev = f"cuda:{gpu.device}"
    # Device-resident inputs for the device-timed leg.
    d_hidden = gpu.upload_raw(hidden, BF16)
    d_targets = torch.from_numpy(targets.astype(np.int32)).cuda(gpu.device)
    d_out = torch.empty(READOUT_ROWS * 16, dtype=torch.uint8, device=dev)
    gathered = torch.empty(dist.world * READOUT_ROWS * 16, dtype=torch.uint8, device=dev) if dist.world > 1 else None
    ws_bytes = lib.lsx_readout_workspace_bytes(VOCAB, HIDDEN, READOUT_ROWS, rot.handle)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    base = d_out.data_ptr()
    torch.cuda.synchronize(gpu.device)
    stream, event = cuda_timer(gpu)

    def gather():
        with torch.cuda.stream(stream):
            dist.pg.all_gather_into_tensor(gathered, d_out)

    def step():
        check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, None, VOCAB, HIDDEN,
                                            C.c_void_p(d_hidden.data_ptr), BF16, READOUT_ROWS,
                                            C.c_void_p(d_targets.data_ptr()), rot.handle, C.c_void_p(base),
                                            C.c_void_p(base + READOUT_ROWS * 8), C.c_void_p(base + READOUT_ROWS * 12),
                                            C.c_void_p(ws.data_ptr()), ws_bytes))
        if gathered is not None:
            gather()

    for _ in range(warmup):
        step()
    check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
    gpu.synchronize()
    dist.barrier()
    start, stop = event(), event()
    with ClockSampler(gpu.device) as clocks:
        start.record(stream)
        for _ in range(steps):
            step()
        stop.record(stream)
        stop.synchronize()
    dev_ms = start.elapsed_time(stop)
    check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
    gather_ms = None
    if gathered is not None:
        # the collective alone, same message, same stream
        dist.barrier()
        g0, g1 = event(), event()
        g0.record(stream)
        for _ in range(steps):
            gather()
        g1.record(stream)
        g1.synchronize()
        gather_ms = g0.elapsed_time(g1) / steps
        # every rank's block of the gathered results is that rank's own output
        mine = gathered[dist.rank * READOUT_ROWS * 16:(dist.rank + 1) * READOUT_ROWS * 16]
        assert torch.equal(mine, d_out)
    dist.barrier()
    from laplacesscissors_b200 import diagnosis
    e2e_s = float("nan")
    if e2e:
        for _ in range(max(1, warmup)):
            diagnosis.readout_margin(gpu, weight, None, VOCAB, HIDDEN, hidden, targets, rot)
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            diagnosis.readout_margin(gpu, weight, None, VOCAB, HIDDEN, hidden, targets, rot)
        e2e_s = time.perf_counter() - t0
    return {"dev_ms": dev_ms, "e2e_s": e2e_s, "clocks": clocks.summary(), "h2d": hidden.nbytes + targets.nbytes,
            "d2h": READOUT_ROWS * 16, "gather_ms": gather_ms}


class Dist:
    def __init__(self, world: int, local: int):
        self.world = world
        self.rank = int(os.environ.get("RANK", 0))
        self.pg = None
        if world > 1:
            import torch
            import torch.distributed as td
            from datetime import timedelta
            torch.cuda.set_device(local)
            td.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
            self.pg = td

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def ensure_checkpoints(rank: int, shapes: list[str]) -> dict:
    """Builds the named checkpoints once per machine before any process group
    exists (writing the 8B model takes longer than a collective may wait): rank 0
    writes, the other ranks wait for the completed folders."""
    from laplacesscissors_b200 import synth
    out = {}
    for shape in shapes:
        if rank == 0:
            out[shape] = synth.cached_checkpoint(shape)
        else:
            root = Path(tempfile.gettempdir()) / f"lsx-bench-{shape.lower()}-seed7"
            t0 = time.monotonic()
            while not (root / "config.json").exists():
                if time.monotonic() - t0 > 1800:
                    raise RuntimeError(f"checkpoint {root} was not written")
                time.sleep(1.0)
            out[shape] = root
    return out


def long_batch_leg(gpu, ckpt: Path, steps: int, prompt: int = 4096, batch: int = 16, cpu: bool = True):
    """Config 4, bs16: Qwen3-4B, 16 sequences decoded together after a 4096-token
    prompt each (lsx_model_generate_batch, host buffers).  Decode throughput is
    batch x K / (t(1 + K steps) - t(1 step)): the two calls share the prefill, so
    the difference is K decode steps at context 4097..4096 + K.  `value` takes the
    two times from CUDA events on the library's stream, `e2e` from the host clock
    around the same calls (prompts in, tokens out)."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    cfg = synth.QWEN3_4B
    K = max(8, steps)
    model = lsx.Model.load(ckpt, gpu, 64)
    prompts = np.stack([synth.prompt_tokens(7 + b, prompt, cfg["vocab"]) for b in range(batch)])
    model.generate_batch(prompts, 1 + K)  # warm-up: caches at their largest, modules loaded
    stream, event = cuda_timer(gpu)
    times = {}
    with ClockSampler(gpu.device) as clocks:
        for n in (1, 1 + K):
            e0, e1 = event(), event()
            t0 = time.perf_counter()
            e0.record(stream)
            model.generate_batch(prompts, n)
            e1.record(stream)
            e1.synchronize()
            times[n] = (e0.elapsed_time(e1) / 1e3, time.perf_counter() - t0)
    step_dev = (times[1 + K][0] - times[1][0]) / K
    step_e2e = (times[1 + K][1] - times[1][1]) / K
    kv_layers = cfg["layers"] * 2 * cfg["kv_heads"] * cfg["head_dim"] * 4
    step_bytes = weight_bytes_per_step(cfg) + batch * kv_layers * (prompt + 1 + K / 2)
    peaks = measured_peaks()
    achieved = step_bytes / step_dev / 1e9
    out = {
        "metric": f"decode tok/s (Qwen3-4B bs{batch} after a {prompt}-token prompt)", "value": batch / step_dev,
        "unit": "tok/s", "ms_per_step": step_dev * 1e3, "steps": K,
        "config": {"workload": f"Qwen3-4B bs{batch} greedy decode at context {prompt + 1}..{prompt + K}",
                   "prompt": prompt, "batch": batch, "kv_cache": "f32",
                   "timing": "generate_batch(1 + K) minus generate_batch(1): K decode steps after a shared prefill",
                   "l2": f"weights {weight_bytes_per_step(cfg) / 1e9:.2f} GB per step > L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "scope": f"{step_bytes / 1e9:.2f} GB per step: bf16 weights once + {batch} sequences' f32 KV, "
                              f"{peaks['source']} peak"},
        "e2e": {"value": batch / step_e2e, "unit": "tok/s", "h2d_bytes_per_step": int(prompts.nbytes),
                "d2h_bytes_per_step": int(batch * (1 + K) * 4)},
        "prefill_and_first_step_seconds": times[1][1],
        "clocks": clocks.summary(),
    }
    if cpu:
        from oracle import binding as oracle
        threads = cpu_threads()
        m = oracle.OracleModel(ckpt, 16, threads=threads)
        ids = synth.prompt_tokens(7, 4, cfg["vocab"])
        m.advance(int(ids[0]))  # pages the weights in
        m.cursor = 0
        t0 = time.perf_counter()
        for t in ids:
            m.advance(int(t))
        rate = len(ids) / (time.perf_counter() - t0)
        out["cpu_baseline"] = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                               "sample": "4 oracle decode steps of the Qwen3-4B model, one sequence, at context 1-4 "
                                         "(the reference decodes one sequence at a time; its KV read at context "
                                         "4096 adds 2.4 GB per step, so this rate is an upper bound)"}
    return out


SCORE_P, SCORE_N, SCORE_EOS = 64, 9, 151645


def score_cases(first: int, count: int, vocab: int = 151936):
    """Cases first .. first + count - 1 of the scoring job: 64 random prompt ids,
    8 random answer ids + EOS (seeded per case)."""
    from laplacesscissors_b200 import synth
    prompts = np.stack([synth.uniform_u32(7, 1000 + i, SCORE_P, vocab) for i in range(first, first + count)])
    answers = np.stack([synth.uniform_u32(7, 5000 + i, SCORE_N - 1, vocab) for i in range(first, first + count)])
    return prompts, np.concatenate([answers, np.full((count, 1), SCORE_EOS, np.uint32)], axis=1)


def scoring_leg(gpu, ckpt: Path, dist, cases: int = 64, batch: int = 64, cpu: bool = True):
    """Config 5: Qwen3-8B teacher-forced scoring (lsx_model_score_batch, host
    arrays in, losses, argmaxes and margins out), `cases` cases per rank, case
    shards across ranks (weak scaling).  `value` from CUDA events on the library's
    stream around the calls, `e2e` from the host clock; max over ranks."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    cfg = synth.QWEN3_8B
    model = lsx.Model.load(ckpt, gpu, 80)
    rank = dist.rank
    model.score_batch(*score_cases(10_000, batch))  # warm-up
    inputs = [score_cases(100 + rank * cases + i, min(batch, cases - i)) for i in range(0, cases, batch)]
    stream, event = cuda_timer(gpu)
    gpu.synchronize()
    dist.barrier()
    with ClockSampler(gpu.device) as clocks:
        e0, e1 = event(), event()
        t0 = time.perf_counter()
        e0.record(stream)
        for pr, tg in inputs:
            model.score_batch(pr, tg)
        e1.record(stream)
        e1.synchronize()
        wall = time.perf_counter() - t0
    dev_s = dist.max(e0.elapsed_time(e1) / 1e3)
    wall = dist.max(wall)
    world = dist.world
    tokens = SCORE_P + SCORE_N - 1
    flops_case = decoder_flops_per_token(cfg) * tokens + 2 * SCORE_N * cfg["vocab"] * cfg["hidden"]
    tflops = world * cases * flops_case / dev_s / 1e12
    peaks = measured_peaks()
    out = {
        "metric": "teacher-forced scoring cases/s (Qwen3-8B, 64-token prompt + 9 scored targets)",
        "value": world * cases / dev_s, "unit": "cases/s", "ms_per_case": dev_s / cases * 1e3,
        "scaling": "weak (case shards)" if world > 1 else "single GPU",
        "config": {"workload": "Qwen3-8B teacher-forced scoring, 64 prompt + 8 answer + EOS per case",
                   "cases_per_gpu": cases, "cases_per_call": batch, "job_cases": 1024,
                   "fed_tokens_per_case": tokens,
                   "timing": "lsx_model_score_batch calls with host arrays, CUDA events on the library stream "
                             "(value) and the host clock (e2e)"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": world * peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": tflops / (world * peaks["bf16_tflops"]),
                     "scope": f"algorithmic {flops_case / 1e12:.3f} TFLOP per case (2 x decoder parameters x 72 fed "
                              "tokens + the lm_head on 9 rows); the f32 activations enter the tensor cores as two "
                              f"bf16 terms, so 0.5 is this path's ceiling; {peaks['source']} burst peak"},
        "e2e": {"value": world * cases / wall, "unit": "cases/s",
                "h2d_bytes_per_step": int(sum(pr.nbytes + tg.nbytes for pr, tg in inputs)),
                "d2h_bytes_per_step": int(cases * SCORE_N * (8 + 4 + 8))},
        "job_seconds_estimate": 1024 / (world * cases / wall),
        "clocks": clocks.summary(),
    }
    if cpu and dist.world == 1:
        from oracle import binding as oracle
        threads = cpu_threads()
        m = oracle.OracleModel(ckpt, 16, threads=threads)
        pr, _ = score_cases(100, 1)
        m.advance(int(pr[0, 0]))  # pages the weights in
        m.cursor = 0
        fed = 6
        t0 = time.perf_counter()
        for t in pr[0, :fed]:
            m.advance(int(t))
        per_token = (time.perf_counter() - t0) / fed
        out["cpu_baseline"] = {"value": 1.0 / (per_token * tokens), "unit": "cases/s", "cores": threads,
                               "kind": "port",
                               "sample": f"{fed} oracle decode steps of the Qwen3-8B model (one case's first fed "
                                         f"tokens), scaled to the case's {tokens} fed tokens"}
    return out


def vocab_leg(gpu, dist, steps: int, warmup: int):
    """The validation workload (4096 rows, rank-16 edit) with the lm_head split by
    rows over the ranks (strong scaling: one whole validation over N GPUs): each
    rank scores every row against its vocabulary block into packed int64
    partials, one NCCL all-reduce MAX merges them, one kernel finalises.  The
    collective alone is timed as well."""
    import torch

    from laplacesscissors_b200 import DeviceRotation
    from laplacesscissors_b200._lib import BF16, lib
    from laplacesscissors_b200.sharding import vocab_shard, vocab_sharded_margin
    rank, world = dist.rank, dist.world
    w, hidden, targets, edit = readout_inputs(0, 1)
    v0, v1 = vocab_shard(VOCAB, world, rank)
    shard = gpu.upload_raw(np.ascontiguousarray(w.reshape(VOCAB, HIDDEN)[v0:v1]), BF16)
    del w
    rot = DeviceRotation.upload_edit(gpu, edit, HIDDEN)
    dev = torch.device("cuda", gpu.device)
    d_hidden = torch.from_numpy(hidden.view(np.int16)).to(dev)
    d_targets = torch.from_numpy(targets.astype(np.uint32).view(np.int32)).to(dev)
    ws = torch.empty(lib.lsx_readout_workspace_bytes(v1 - v0, HIDDEN, READOUT_ROWS, rot.handle), dtype=torch.uint8,
                     device=dev)
    partials = torch.empty(2 * READOUT_ROWS, dtype=torch.int64, device=dev)
    outs = (torch.empty(READOUT_ROWS, dtype=torch.float64, device=dev),
            torch.empty(READOUT_ROWS, dtype=torch.int32, device=dev),
            torch.empty(READOUT_ROWS, dtype=torch.float32, device=dev))
    torch.cuda.synchronize(dev)

    def step():
        vocab_sharded_margin(gpu, shard, None, v0, v1 - v0, HIDDEN, d_hidden.data_ptr(), BF16, READOUT_ROWS,
                             d_targets.data_ptr(), rot, workspace=ws, partials=partials, outputs=outs)

    stream, event = cuda_timer(gpu)
    for _ in range(warmup):
        step()
    gpu.synchronize()
    dist.barrier()
    start, stop = event(), event()
    start.record(stream)
    for _ in range(steps):
        step()
    stop.record(stream)
    stop.synchronize()
    ms = dist.max(start.elapsed_time(stop)) / steps
    dist.barrier()
    c0, c1 = event(), event()
    with torch.cuda.stream(stream):
        c0.record(stream)
        for _ in range(steps):
            dist.pg.all_reduce(partials, op=dist.pg.ReduceOp.MAX)
        c1.record(stream)
    c1.synchronize()
    coll_ms = dist.max(c0.elapsed_time(c1)) / steps
    peaks = measured_peaks()
    tflops = 2.0 * READOUT_ROWS * VOCAB * HIDDEN / (ms / 1e3) / 1e12
    return {
        "metric": "readout-margin rows/s (lm_head split by vocabulary rows)", "value": READOUT_ROWS / (ms / 1e3),
        "unit": "rows/s", "ms_per_step": ms, "scaling": "strong",
        "config": {"workload": "4096 rows x lm_head [151936, 1024], rank-16 edit, vocabulary-sharded",
                   "vocab_rows_per_gpu": v1 - v0,
                   "collective": "1 NCCL all-reduce MAX of 64 KiB (int64 [2 x 4096] packed partials) per step"},
        "collective_ms": coll_ms,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": world * peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / (world * peaks["bf16_tflops"]),
                     "scope": f"whole validation over {world} GPUs, {peaks['source']} burst peak x GPUs"},
    }


def triton_baseline_leg(ckpt: Path, steps: int = 2) -> dict:
    """The reference's own Triton kernels on this GPU (baseline/triton_reference.py,
    two subprocesses: the reference's runtime pattern, and its kernels alone in a
    CUDA graph)."""
    out = {}
    script = ROOT / "baseline" / "triton_reference.py"
    for mode in ("runtime", "graph"):
        cmd = [sys.executable, str(script), "--mode", mode, "--checkpoint", str(ckpt), "--steps", str(steps),
               "--warmup", "1", "--readout-rows", "128"]
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
            line = r.stdout.strip().splitlines()[-1] if r.stdout.strip() else ""
            out[mode] = json.loads(line) if line else {"unavailable": f"exit {r.returncode}: {r.stderr[-300:]}"}
        except (subprocess.TimeoutExpired, json.JSONDecodeError) as e:
            out[mode] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-triton", action="store_true", help="skip the reference's Triton kernels on the GPU")
    ap.add_argument("--headline-only", action="store_true",
                    help="decode, readout and GEMV only (no Qwen3-4B / Qwen3-8B sub-objects)")
    ap.add_argument("--workload", choices=["all", "decode", "readout", "gemv", "long4b", "long4b_batch", "score8b",
                                           "readout_vocab",
                                           "plane", "attribution"],
                    default="all",
                    help="all: the headline line; decode/readout/gemv: one leg only (with --profile); "
                         "long4b: Qwen3-4B decode after a long prompt; score8b: Qwen3-8B teacher-forced scoring; "
                         "readout_vocab: the validation workload with the lm_head split by rows over the GPUs; "
                         "plane: the plane search's constraint loop (GPU-screened) against the oracle's host loop; "
                         "attribution: the integrated-softmax credits over the vocabulary")
    ap.add_argument("--prompt", type=int, default=4096, help="long4b: prompt length")
    ap.add_argument("--cases", type=int, default=64, help="score8b: cases timed (of the 1024-case job)")
    ap.add_argument("--batch", type=int, default=64, help="score8b: cases per lsx_model_score_batch call "
                                                          "(0: one lsx_model_score call per case)")
    ap.add_argument("--profile", action="store_true",
                    help="profiling aid: device legs only, no e2e or CPU legs, warm-up as given")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling aid: decoder layers of the checkpoint (decode profile: default 28; score8b: a "
                         "reduced Qwen3-8B-width model for ncu section captures, one rank)")
    args = ap.parse_args()
    rank, local, world = env_rank()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.workload == "long4b":
        return long_decode(args, local)
    if args.workload == "long4b_batch":
        return long_decode_batch(args, local)
    if args.workload == "score8b":
        return scoring(args, rank, local, world)
    if args.workload == "readout_vocab":
        return vocab_readout(args, rank, local, world)
    if args.workload == "plane":
        return plane_bench(args, local)
    if args.workload == "attribution":
        return attribution_bench(args, local)
    if args.profile:
        return profile_run(args, local)
    if args.warmup < 3:
        args.warmup = 3
    full = not args.headline_only
    shapes = ["QWEN3_0_6B"] + (["QWEN3_4B", "QWEN3_8B"] if full and world == 1 else ["QWEN3_8B"] if full else [])
    ckpts = ensure_checkpoints(rank, shapes)  # before the process group: the 8B file takes a while
    import laplacesscissors_b200 as lsx
    dist = Dist(world, local)
    gpu = lsx.Gpu(local)
    peaks = measured_peaks()
    ckpt = ckpts["QWEN3_0_6B"]
    cpu = not args.no_cpu_baseline and world == 1
    dec = run_decode(gpu, ckpt, args.steps, args.warmup, dist)
    inputs = readout_inputs(rank, world)
    ro = run_readout(gpu, inputs, args.steps, args.warmup, dist)
    gemv = run_gemv(gpu) if rank == 0 else None
    # sub-objects: config 4 (one GPU), config 5 (case shards), vocabulary shards (N > 1)
    long4b = long_batch_leg(gpu, ckpts["QWEN3_4B"], 32, cpu=cpu) if full and world == 1 else None
    del dec["model"]
    score8b = scoring_leg(gpu, ckpts["QWEN3_8B"], dist, cpu=cpu) if full else None
    vocab = vocab_leg(gpu, dist, args.steps, args.warmup) if world > 1 else None
    # Kernels of ours per timed generation: one cooperative launch (persistent
    # engine) or the graph's per-step chain; readout: init, edit image, edit
    # coefficients, tcgen05 margin, finalize.
    dec_launches = 1 if dec["persistent"] else dec["kernels_per_step"] * STEPS_PER_GENERATION
    dec_ms = dist.max(dec["dev_ms"]) / args.steps
    dec_e2e = dist.max(dec["e2e_s"]) / args.steps
    ro_ms = dist.max(ro["dev_ms"]) / args.steps
    ro_e2e = dist.max(ro["e2e_s"]) / args.steps
    gather_ms = dist.max(ro["gather_ms"]) if ro["gather_ms"] is not None else None
    if rank == 0:
        step_s = dec_ms / 1e3 / STEPS_PER_GENERATION
        bytes_step = decode_bytes_per_step()
        achieved = bytes_step / step_s / 1e9
        flops = 2.0 * READOUT_ROWS * VOCAB * HIDDEN
        tflops = flops / (ro_ms / 1e3) / 1e12
        line = {
            "metric": METRIC,
            "value": world * STEPS_PER_GENERATION / (dec_ms / 1e3),
            "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dec_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16 weights, f32 activations and KV (f32 accumulate)",
            "data": "synthetic: random-init Qwen3-0.6B architecture (seed 7), 24 random prompt ids",
            "config": decode_config(world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"],
                         "traffic": DECODE_TRAFFIC_PER_LAUNCH if dec["persistent"] else None,
                         "traffic_unit": "bytes per launch (one generation of 55 decode steps)",
                         "scope": ("one cooperative decode kernel per generation" if dec["persistent"] else
                                   f"{dec['kernels_per_step']} kernels per decode step") +
                                  f", algorithmic bytes {bytes_step / 1e9:.4f} GB per decode step, "
                                  f"{peaks['source']} peak"},
            "e2e": {"value": world * STEPS_PER_GENERATION / dec_e2e, "unit": "tok/s",
                    "h2d_bytes_per_step": dec["h2d"], "d2h_bytes_per_step": dec["d2h"]},
            "clocks": dec["clocks"],
            "decode_graph": dec["graph"],
            "gpu_launches": args.steps * dec_launches + args.steps * 5,
            "readout": {
                "metric": "readout-margin rows/s", "value": world * READOUT_ROWS / (ro_ms / 1e3), "unit": "rows/s",
                "ms_per_step": ro_ms,
                "config": {"workload": "4096 RMSNorm'd bf16 hidden x lm_head [151936, 1024] bf16, rank-16 "
                                       "Givens edit within 3 degrees, target margin + argmax",
                           "rows_per_gpu": READOUT_ROWS,
                           "scaling": "weak (row shards), results all-gathered every step" if world > 1
                           else "single GPU",
                           "l2": "lm_head 311 MB > L2"},
                "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"],
                             "unit": "TFLOP/s", "frac": tflops / peaks["bf16_tflops"],
                             "traffic": READOUT_TRAFFIC_PER_LAUNCH,
                             "traffic_unit": "bytes per launch of the margin GEMM (lm_head read once)",
                             "scope": "whole validation step (tcgen05 edit image + coefficients + tcgen05 "
                                      "CTA-pair margin GEMM + finalize), 2*4096*151936*1024 flops, "
                                      f"{peaks['source']} burst peak"},
                "e2e": {"value": world * READOUT_ROWS / ro_e2e, "unit": "rows/s", "h2d_bytes_per_step": ro["h2d"],
                        "d2h_bytes_per_step": ro["d2h"]},
                "clocks": ro["clocks"],
            },
        }
        if gather_ms is not None:
            line["readout"]["collective"] = {"op": "NCCL all-gather of 16 B per row (margin f64, argmax u32, "
                                                   "target logit f32) per step, every rank receives all rows",
                                             "ms": gather_ms}
        gemv_frac = {k: dict(v, frac=v["GB/s"] / peaks["hbm_gbs"]) for k, v in gemv.items()}
        line["gemv"] = {
            "metric": "bf16 GEMV y = W x achieved HBM GB/s (lsx_linear_into, the Gpu::linear drop-in)",
            "unit": "GB/s", "peak": peaks["hbm_gbs"],
            "config": {"shapes": [f"{n}x{k}" for n, k in GEMV_SHAPES], "x": "f32", "y": "f32",
                       "l2": "weight copies rotated so each pass reads >= 256 MB",
                       "timing": "CUDA graph of the launches, CUDA events, rank 0"},
            "roofline": {"bound": "hbm", "unit": "GB/s", "peak": peaks["hbm_gbs"],
                         "bytes": "2NK + 4K + 4N per launch",
                         "note": "shapes below 12 MB are launch- and latency-bound: their time per launch (us) "
                                 "is the figure to read"},
            "results": gemv_frac,
            "e2e": {"value": {k: v["e2e"]["GB/s"] for k, v in gemv.items()}, "unit": "GB/s",
                    "us": {k: v["e2e"]["us"] for k, v in gemv.items()},
                    "h2d_bytes_per_step": {k: v["e2e"]["h2d_bytes"] for k, v in gemv.items()},
                    "d2h_bytes_per_step": {k: v["e2e"]["d2h_bytes"] for k, v in gemv.items()},
                    "path": "per GEMV: lsx_upload_f32 (host x) -> lsx_linear -> lsx_read (host y), W resident; "
                            "host clock"},
        }
        if cpu:
            rates, threads = cpu_gemv_rates()
            line["gemv"]["cpu_baseline"] = {"value": rates, "unit": "GB/s", "cores": threads, "kind": "port",
                                            "sample": "the oracle's GEMV of every shape repeated for ~0.5 s "
                                                      f"(f64 accumulation, {threads} threads)"}
        if long4b is not None:
            line["long4b_batch"] = long4b
        if score8b is not None:
            line["score8b"] = score8b
        if vocab is not None:
            line["readout_vocab"] = vocab
        if cpu:
            v, cores, sample = cpu_decode_rate(ckpt)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}
            rv, rcores, rsample = cpu_readout_rate(*inputs)
            line["readout"]["cpu_baseline"] = {"value": rv, "unit": "rows/s", "cores": rcores, "kind": "port",
                                               "sample": rsample}
        if world == 1 and not args.no_triton:
            tb = triton_baseline_leg(ckpt)
            rt, gr = tb.get("runtime", {}), tb.get("graph", {})
            line["triton_baseline"] = tb
            ratios = {}
            if "decode" in rt:
                ratios["decode_e2e_vs_runtime"] = line["e2e"]["value"] / rt["decode"]["tok_s"]
            if "decode" in gr:
                ratios["decode_vs_graph"] = line["value"] / gr["decode"]["tok_s"]
            if "readout" in rt:
                ratios["readout_e2e_vs_runtime"] = line["readout"]["e2e"]["value"] / rt["readout"]["rows_s"]
            if "readout" in gr:
                ratios["readout_vs_graph"] = line["readout"]["value"] / gr["readout"]["rows_s"]
            if "gemv" in gr:
                ratios["gemv_vs_graph"] = {k: gemv[k]["GB/s"] / gr["gemv"][k]["GB/s"] for k in gemv if k in gr["gemv"]}
            tb["ratios"] = ratios
        print(json.dumps(line))
    dist.close()


def vocab_readout(args, rank, local, world):
    """The readout-validation workload (4096 rows, rank-16 edit) with the lm_head
    split by rows over the ranks: each GPU scores all rows against its vocabulary
    block (lsx_readout_shard_device), one NCCL all-reduce MAX of the packed keys and
    one of the target logits merge the blocks, and lsx_readout_merge_device gives
    the margins.  Total work is fixed (strong scaling); each step is one whole
    validation, timed with CUDA events on the library stream, max over ranks."""
    import torch

    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import DeviceRotation
    from laplacesscissors_b200._lib import BF16, check, lib
    from laplacesscissors_b200.sharding import vocab_shard, vocab_sharded_margin
    args.warmup = max(args.warmup, 3)
    dist = Dist(world, local)
    gpu = lsx.Gpu(local)
    peaks = measured_peaks()
    w, hidden, targets, edit = readout_inputs(0, 1)
    v0, v1 = vocab_shard(VOCAB, world, rank)
    shard = gpu.upload_raw(np.ascontiguousarray(w.reshape(VOCAB, HIDDEN)[v0:v1]), BF16)
    del w
    rot = DeviceRotation.upload_edit(gpu, edit, HIDDEN)
    dev = torch.device("cuda", local)
    d_hidden = torch.from_numpy(hidden.view(np.int16)).to(dev)
    d_targets = torch.from_numpy(targets.astype(np.uint32).view(np.int32)).to(dev)
    ws = torch.empty(lib.lsx_readout_workspace_bytes(v1 - v0, HIDDEN, READOUT_ROWS, rot.handle), dtype=torch.uint8,
                     device=dev)
    torch.cuda.synchronize(dev)

    def step():
        return vocab_sharded_margin(gpu, shard, None, v0, v1 - v0, HIDDEN, d_hidden.data_ptr(), BF16, READOUT_ROWS,
                                    d_targets.data_ptr(), rot, workspace=ws)

    stream, event = cuda_timer(gpu)
    for _ in range(args.warmup):
        step()
    gpu.synchronize()
    dist.barrier()
    start, stop = event(), event()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        stop.synchronize()
    ms = dist.max(start.elapsed_time(stop)) / args.steps
    # The shard's kernels alone (no collective, no merge), to separate compute from exchange.
    import ctypes as C
    keys = torch.empty(READOUT_ROWS, dtype=torch.int64, device=dev)
    tlog = torch.empty(READOUT_ROWS, dtype=torch.float32, device=dev)

    def shard_only():
        check(lib.lsx_readout_shard_device(gpu.handle, shard.handle, None, v0, v1 - v0, HIDDEN,
                                           C.c_void_p(d_hidden.data_ptr()), BF16, READOUT_ROWS,
                                           C.c_void_p(d_targets.data_ptr()), rot.handle,
                                           C.c_void_p(keys.data_ptr()), C.c_void_p(tlog.data_ptr()),
                                           C.c_void_p(ws.data_ptr()), ws.numel()))

    for _ in range(args.warmup):
        shard_only()
    gpu.synchronize()
    start2, stop2 = event(), event()
    start2.record(stream)
    for _ in range(args.steps):
        shard_only()
    stop2.record(stream)
    stop2.synchronize()
    shard_ms = dist.max(start2.elapsed_time(stop2)) / args.steps
    if rank == 0:
        tflops = 2.0 * READOUT_ROWS * VOCAB * HIDDEN / (ms / 1e3) / 1e12
        print(json.dumps({
            "metric": "readout-margin rows/s (lm_head split by vocabulary rows)",
            "value": READOUT_ROWS / (ms / 1e3), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 operands, f32 accumulate",
            "data": "synthetic: lm_head N(0, 0.02) seed 7, 4096 RMSNorm'd rows, rank-16 Givens edit",
            "config": {"workload": "4096 rows x lm_head [151936, 1024], rank-16 edit, vocab-sharded",
                       "vocab_rows_per_gpu": VOCAB // world, "collective": "1 NCCL all-reduce MAX per step",
                       "l2": "lm_head shard read once per step"},
            "shard_kernels_ms": shard_ms,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": world * peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": tflops / (world * peaks["bf16_tflops"]),
                         "scope": f"whole validation over {world} GPU(s), {peaks['source']} burst peak x GPUs"},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * 6,
        }))
    dist.close()


def plane_bench(args, local, points: int = 64):
    """The plane search's constraint loop (src/diagnosis.rs:1118-1143) for one plane
    over the Qwen3-0.6B vocabulary and `points` target points: seeded head images
    and frame logits with each target 0.2-1.0 above its best competitor, so a few
    constraints bind and the set stays non-empty (every constraint is evaluated).
    lsx_plane_feasible (GPU formation and screening, host merge) end to end with
    host arrays, against the oracle's sequential host loop on the same inputs;
    constraints per second."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200.feasible import FeasibleSet, plane_constraints
    from oracle import binding as oracle
    gpu = lsx.Gpu(local)
    rng = np.random.default_rng(7)
    V, P = VOCAB, points
    wu = rng.standard_normal(V).astype(np.float32)
    wv = rng.standard_normal(V).astype(np.float32)
    z = (rng.standard_normal((P, V)) * 3).astype(np.float32)
    t = rng.integers(0, V, P).astype(np.uint32)
    for p in range(P):
        z[p, t[p]] = np.float32(z[p].max() + rng.uniform(0.2, 1.0))
    hu, hv = rng.standard_normal(P) * 3, rng.standard_normal(P) * 3
    bound_deg, margin, guard = 30.0, 0.1, 0.01

    def ours():
        f = FeasibleSet.for_angle(bound_deg)
        plane_constraints(gpu, f, wu, wv, z, t, hu, hv, margin, guard)
        return f

    for _ in range(max(3, args.warmup)):
        f = ours()
    with ClockSampler(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            f = ours()
        dt = (time.perf_counter() - t0) / args.steps
    constraints = f.work()[0]
    ref = oracle.Feasible(math.tan(math.radians(bound_deg) / 2.0))
    t1 = time.perf_counter()
    ref.plane(wu, wv, z, t, hu, hv, margin, guard)
    cpu = time.perf_counter() - t1
    assert ref.work() == f.work() and ref.intervals() == f.intervals() and ref.nearest() == f.nearest()
    print(json.dumps({
        "metric": "plane constraints/s (src/diagnosis.rs:1118-1143 loop, one plane)",
        "value": constraints / dt, "unit": "constraints/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": dt * 1e3, "higher_is_better": True,
        "dtype": "f64 constraints from f32 head images and logits",
        "data": "synthetic: seeded head images and frame logits, targets 0.2-1.0 above the best competitor",
        "config": {"workload": f"{P} target points x {V} vocabulary entries, half-angle bound 15 degrees",
                   "constraints": constraints, "work": f.work(),
                   "timing": "wall clock around lsx_plane_feasible with host arrays (uploads, screening passes, "
                             "mask downloads and the host merge)"},
        "cpu_baseline": {"value": constraints / cpu, "unit": "constraints/s", "cores": 1, "kind": "port",
                         "sample": "the whole loop once (oracle restatement, sequential as the reference)"},
        "clocks": clocks.summary(),
    }))


def attribution_bench(args, local, points: int = 64, panels: int = 64):
    """integrated_probabilities (src/attribution.rs:79-123) over the Qwen3-0.6B
    vocabulary: `points` points with seeded before/after logits, `panels` Simpson
    panels, through lsx_integrated_credits with host arrays (uploads and the credit
    download inside the timing).  Unit: softmax evaluations (points x (panels + 1) x
    vocabulary exponentials) per second; the oracle's sequential f64 loop on one
    point is the CPU baseline."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import attribution
    from oracle import binding as oracle
    gpu = lsx.Gpu(local)
    rng = np.random.default_rng(7)
    V, P = VOCAB, points
    before = (rng.standard_normal((P, V)) * 3).astype(np.float32)
    after = (before + rng.standard_normal((P, V)).astype(np.float32) * 0.5).astype(np.float32)
    targets = rng.integers(0, V, P).astype(np.uint32)
    weights = np.full(P, 1.0 / P)
    for _ in range(max(3, args.warmup)):
        attribution.integrated_credits(gpu, before, after, targets, weights, panels)
    with ClockSampler(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            credits, _, _ = attribution.integrated_credits(gpu, before, after, targets, weights, panels)
        dt = (time.perf_counter() - t0) / args.steps
    evals = P * (panels + 1) * V
    t1 = time.perf_counter()
    ref, _ = oracle.integrated_credits(before[:1], after[:1], targets[:1], weights[:1], panels)
    cpu = time.perf_counter() - t1
    print(json.dumps({
        "metric": "integrated-softmax evaluations/s (src/attribution.rs:79-123)",
        "value": evals / dt, "unit": "exp/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": dt * 1e3, "higher_is_better": True, "dtype": "f64",
        "data": "synthetic: seeded before/after logits over the Qwen3-0.6B vocabulary",
        "config": {"workload": f"{P} points x {panels} panels x {V} vocabulary rows",
                   "timing": "wall clock around lsx_integrated_credits with host arrays (2 x 39 MB uploaded)"},
        "cpu_baseline": {"value": (panels + 1) * V / cpu, "unit": "exp/s", "cores": 1, "kind": "port",
                         "sample": "one point (oracle, sequential f64 as the reference)"},
        "clocks": clocks.summary(),
    }))


def profile_run(args, local):
    """Device legs only, for ncu: prints the per-step device times."""
    import laplacesscissors_b200 as lsx
    dist = Dist(1, local)
    gpu = lsx.Gpu(local)
    out = {"profile": True}
    if args.workload in ("all", "decode"):
        dec = run_decode(gpu, build_checkpoint(local, args.layers or 28), args.steps, args.warmup, dist, e2e=False)
        out["decode_ms_per_generation"] = dec["dev_ms"] / args.steps
        out["decode_graph"] = dec["graph"]
        out["kernels_per_step"] = dec["kernels_per_step"]
    if args.workload in ("all", "readout"):
        ro = run_readout(gpu, readout_inputs(), args.steps, args.warmup, dist, e2e=False)
        out["readout_ms_per_step"] = ro["dev_ms"] / args.steps
    if args.workload in ("all", "gemv"):
        out["gemv"] = run_gemv(gpu)
    print(json.dumps(out))


def model_checkpoint(shape: str, **overrides) -> Path:
    from laplacesscissors_b200 import synth
    cfg = dict(getattr(synth, shape), **overrides)
    tag = "-".join(f"{k}{v}" for k, v in sorted(overrides.items()))
    d = Path(tempfile.gettempdir()) / f"lsx-bench-{shape.lower()}-seed7{'-' + tag if tag else ''}"
    if not (d / "model.safetensors").exists():
        synth.make_qwen3_checkpoint(d, synth.qwen3_config(**cfg), seed=7)
    return d


def weight_bytes_per_step(cfg: dict) -> int:
    """bf16 weight bytes one decode step reads: every block matrix and norm, the
    final norm and the lm_head (one embedding row is not counted)."""
    H, I, D = cfg["hidden"], cfg["intermediate"], cfg["head_dim"]
    q, kv = cfg["heads"] * D, cfg["kv_heads"] * D
    block = H * (q + 2 * kv) + q * H + 3 * H * I + 2 * H + 2 * D
    return 2 * (cfg["layers"] * block + H + cfg["vocab"] * H)


def long_decode_batch(args, local, batch: int = 16):
    """Qwen3-4B, `batch` sequences decoded together after a --prompt-token prompt
    each (lsx_model_generate_batch: one batched forward prefills all sequences into
    per-sequence f32 KV caches, then every step feeds one row per sequence).  Decode
    throughput = batch x K extra steps / (time(1 + K steps) - time(1 step)), wall
    clock around the whole call (prompts in, tokens out).  Bytes per step: the bf16
    weights once plus every sequence's f32 K and V of all cached positions."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    gpu = lsx.Gpu(local)
    cfg = synth.QWEN3_4B
    P, K = args.prompt, max(32, args.steps)
    model = lsx.Model.load(model_checkpoint("QWEN3_4B"), gpu, 64)
    prompts = np.stack([synth.prompt_tokens(7 + b, P, cfg["vocab"]) for b in range(batch)])
    model.generate_batch(prompts, 1 + K)  # warm-up: buffers, caches (largest), kernel modules
    t0 = time.perf_counter()
    model.generate_batch(prompts, 1)
    t_one = time.perf_counter() - t0
    with ClockSampler(gpu.device) as clocks:
        t0 = time.perf_counter()
        model.generate_batch(prompts, 1 + K)
        t_all = time.perf_counter() - t0
    step_s = (t_all - t_one) / K
    kv_layers = cfg["layers"] * 2 * cfg["kv_heads"] * cfg["head_dim"] * 4
    mean_ctx = P + 1 + K / 2
    step_bytes = weight_bytes_per_step(cfg) + batch * kv_layers * mean_ctx
    peaks = measured_peaks()
    achieved = step_bytes / step_s / 1e9
    print(json.dumps({
        "metric": f"decode tok/s (Qwen3-4B bs{batch} after a long prompt)",
        "value": batch / step_s, "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": 1,
        "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "dtype": "bf16 weights, f32 activations (two bf16 terms into the tensor cores) and KV",
        "data": "synthetic: random-init Qwen3-4B architecture (seed 7), seeded random prompts",
        "config": {"workload": f"Qwen3-4B bs{batch} greedy decode at context {P + 1}..{P + K}", "prompt": P,
                   "batch": batch, "kv_cache": "f32",
                   "timing": "wall clock: generate_batch(1 + K) minus generate_batch(1), host buffers"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "scope": f"{step_bytes / 1e9:.2f} GB per step: weights once + {batch} sequences' f32 KV"},
        "prefill_and_first_step_seconds": t_one,
        "clocks": clocks.summary(),
    }))


def long_decode(args, local):
    """Qwen3-4B (36 layers, hidden 2560, 32/8 heads, I 9728, tied), batch 1: a
    seeded random prompt of --prompt ids fed token by token (one persistent
    launch), then --steps greedy decode steps timed one lsx_model_advance call
    each (CUDA events on the library stream).  Bytes per decode step: the bf16
    weights plus the f32 K and V of every cached position."""
    import torch

    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    gpu = lsx.Gpu(local)
    cfg = synth.QWEN3_4B
    P = args.prompt
    model = lsx.Model.load(model_checkpoint("QWEN3_4B"), gpu, P + args.warmup + args.steps + 8)
    prompt = synth.prompt_tokens(7, P, cfg["vocab"])
    stream, event = cuda_timer(gpu)
    model.generate(prompt, 1)  # warm-up: buffers, tensor maps and kernel modules
    model.reset()
    t0 = time.perf_counter()
    tokens, _, _ = model.generate(prompt, 1)
    prefill_s = time.perf_counter() - t0
    token = int(tokens[0])
    for _ in range(args.warmup):
        token = model.advance_token(token)
    start, stop = event(), event()
    pos0 = model.position()
    with ClockSampler(gpu.device) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            token = model.advance_token(token)
        stop.record(stream)
        stop.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    kv = 2 * cfg["layers"] * cfg["kv_heads"] * cfg["head_dim"] * 4
    mean_ctx = pos0 + (args.steps + 1) / 2
    step_bytes = weight_bytes_per_step(cfg) + kv * mean_ctx
    peaks = measured_peaks()
    achieved = step_bytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "decode tok/s (Qwen3-4B bs1 after a long prompt)", "value": 1e3 / ms, "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "bf16 weights, f32 activations and KV (f32 accumulate)",
        "data": f"synthetic: random-init Qwen3-4B architecture (seed 7), {P} random prompt ids",
        "config": {"workload": f"Qwen3-4B bs1 greedy decode at context {pos0}..{pos0 + args.steps}",
                   "prompt": P, "kv_cache": "f32", "timing": "one lsx_model_advance per step, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "scope": f"{step_bytes / 1e9:.3f} GB per step (weights + f32 KV at the mean context)"},
        "prefill": {"tokens": P, "seconds": prefill_s, "tok_s": P / prefill_s,
                    "tflops": decoder_flops_per_token(cfg) * (P - 1) / prefill_s / 1e12,
                    "note": "lsx_model_generate wall clock after one warm-up call: the first P - 1 tokens in one "
                            "batched forward "
                            "(tcgen05 GEMMs, causal attention, KV cache filled), the last through the decode "
                            "engine; LSX_PREFILL_MIN=0 feeds the prompt token by token as the reference"},
        "clocks": clocks.summary(),
    }))


def decoder_flops_per_token(cfg: dict) -> int:
    """2 x the decoder's matrix parameters (the decoder flops of one token)."""
    H, I, D = cfg["hidden"], cfg["intermediate"], cfg["head_dim"]
    q, kv = cfg["heads"] * D, cfg["kv_heads"] * D
    return 2 * cfg["layers"] * (H * (q + 2 * kv) + q * H + 3 * H * I)


def scoring(args, rank, local, world):
    """Qwen3-8B (36 layers, hidden 4096, 32/8 heads, I 12288, untied lm_head)
    teacher-forced case scoring: cases of 64 random prompt ids and 8 random
    answer ids + EOS.  --batch > 0: lsx_model_score_batch over --batch cases at a
    time (the 72 fed tokens of every case through each layer together, tcgen05
    GEMMs); --batch 0: lsx_model_score per case (prefill, then per target the
    frame's loss and argmax, advancing with the target, token by token as the
    reference).  --cases of the 1024-case job are timed end to end (host arrays in,
    losses and argmaxes out)."""
    if args.batch > 0:
        return scoring_batched(args, rank, local, world)
    if rank != 0:  # the token-by-token form is a single-GPU measurement
        return
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    gpu = lsx.Gpu(local)
    cfg = synth.QWEN3_8B
    eos = 151645
    model = lsx.Model.load(model_checkpoint("QWEN3_8B"), gpu, 80)
    V = cfg["vocab"]

    def case(i):
        prompt = synth.uniform_u32(7, 1000 + i, 64, V)
        answer = synth.uniform_u32(7, 5000 + i, 8, V)
        return prompt, np.append(answer, np.uint32(eos))

    for i in range(max(1, args.warmup)):
        model.reset()
        model.score(*case(i))
    gpu.synchronize()
    n = args.cases
    with ClockSampler(gpu.device) as clocks:
        t0 = time.perf_counter()
        for i in range(n):
            model.reset()
            model.score(*case(100 + i))
        dt = time.perf_counter() - t0
    steps_per_case = 64 + 9 - 1
    step_bytes = weight_bytes_per_step(cfg)
    peaks = measured_peaks()
    achieved = n * steps_per_case * step_bytes / dt / 1e9
    print(json.dumps({
        "metric": "teacher-forced scoring cases/s (Qwen3-8B, 64-token prompt + 9 scored targets)",
        "value": n / dt, "unit": "cases/s", "n_gpus": 1, "steps": n, "warmup": args.warmup,
        "ms_per_step": dt / n * 1e3, "higher_is_better": True,
        "dtype": "bf16 weights, f32 activations and KV, f64 loss",
        "data": "synthetic: random-init Qwen3-8B architecture (seed 7), random prompt and answer ids",
        "config": {"workload": "Qwen3-8B teacher-forced scoring, 64 prompt + 8 answer + EOS per case",
                   "cases_timed": n, "job_cases": 1024, "decode_steps_per_case": steps_per_case,
                   "timing": "wall clock around lsx_model_score per case (host buffers)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "scope": f"token-by-token decode steps, {step_bytes / 1e9:.3f} GB of weights each "
                              "(a batched-prefill GEMM path would make this tensor-bound)"},
        "job_seconds_estimate": 1024 / (n / dt),
        "clocks": clocks.summary(),
    }))


def scoring_batched(args, rank, local, world):
    """Batched scoring; with several ranks (torchrun) each rank scores its own
    --cases cases of the job (cases are independent: case sharding, weak scaling)
    and the time is the maximum over ranks."""
    import laplacesscissors_b200 as lsx
    from laplacesscissors_b200 import synth
    # One writer for the 16 GB checkpoint, before the process group exists (writing it
    # takes longer than a collective may wait); the other ranks wait for its marker.
    # --layers: the same widths with fewer layers (profiling captures, one rank).
    over = {} if args.layers is None else {"layers": args.layers}
    if over and world != 1:
        raise SystemExit("score8b --layers is a one-rank profiling aid")
    marker = Path(tempfile.gettempdir()) / "lsx-bench-qwen3_8b-seed7.complete"
    if over:
        model_checkpoint("QWEN3_8B", **over)
    elif rank == 0:
        model_checkpoint("QWEN3_8B")
        marker.touch()
    else:
        t_wait = time.monotonic()
        while not marker.exists():
            if time.monotonic() - t_wait > 1800:
                raise RuntimeError("the checkpoint writer did not finish")
            time.sleep(1.0)
    dist = Dist(world, local)
    gpu = lsx.Gpu(local)
    cfg = dict(synth.QWEN3_8B, **over)  # the flop count follows the checkpoint's layers
    eos, V, P, n = 151645, cfg["vocab"], 64, 9
    model = lsx.Model.load(model_checkpoint("QWEN3_8B", **over), gpu, 80)
    first_case = 100 + rank * args.cases

    def batch(first, count):
        prompts = np.stack([synth.uniform_u32(7, 1000 + i, P, V) for i in range(first, first + count)])
        answers = np.stack([synth.uniform_u32(7, 5000 + i, n - 1, V) for i in range(first, first + count)])
        return prompts, np.concatenate([answers, np.full((count, 1), eos, np.uint32)], axis=1)

    B = args.batch
    for i in range(max(1, args.warmup)):
        model.score_batch(*batch(10_000 + i * B, B))
    gpu.synchronize()
    inputs = [batch(first_case + i, min(B, args.cases - i)) for i in range(0, args.cases, B)]
    dist.barrier()
    with ClockSampler(gpu.device) as clocks:
        t0 = time.perf_counter()
        for pr, tg in inputs:
            model.score_batch(pr, tg)
        dt = dist.max(time.perf_counter() - t0)
    dist.close()
    if rank != 0:
        return
    tokens = P + n - 1
    flops_case = decoder_flops_per_token(cfg) * tokens + 2 * n * V * cfg["hidden"]
    tflops = world * args.cases * flops_case / dt / 1e12
    peaks = measured_peaks()
    print(json.dumps({
        "metric": "teacher-forced scoring cases/s (Qwen3-8B, 64-token prompt + 9 scored targets)",
        "value": world * args.cases / dt, "unit": "cases/s", "n_gpus": world, "steps": args.cases,
        "warmup": args.warmup, "scaling": "weak (case shards)",
        "ms_per_step": dt / args.cases * 1e3, "higher_is_better": True,
        "dtype": "bf16 weights; f32 activations entering the tensor cores as two bf16 terms (f32 accumulate); "
                 "f64 loss",
        "data": "synthetic: random-init Qwen3-8B architecture (seed 7), random prompt and answer ids",
        "config": {"workload": "Qwen3-8B teacher-forced scoring, 64 prompt + 8 answer + EOS per case",
                   "cases_timed": args.cases, "cases_per_call": B, "job_cases": 1024, "fed_tokens_per_case": tokens,
                   "timing": "wall clock around lsx_model_score_batch calls (host buffers in and out)"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": world * peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / (world * peaks["bf16_tflops"]),
                     "scope": f"algorithmic {flops_case / 1e12:.3f} TFLOP per case (2 x decoder parameters x 72 "
                              "fed tokens + the lm_head on 9 rows); the two-term activations double the "
                              "tensor-core work, so 0.5 of peak is this path's ceiling"},
        "job_seconds_estimate": 1024 / (world * args.cases / dt),
        "clocks": clocks.summary(),
    }))


def reference_arm(args, rank, world):
    """The reference's CPU path on the host cores, rank 0 only: the oracle's
    restatement of the reference's CPU forward (tests/qwen_reference.rs:39-202 with
    the KV cache of Model::decode), running the headline workload itself -- one
    bench step is the whole 55-step generation of the 24-token prompt -- on the
    same checkpoint bytes, built by the oracle's own generator.  Nothing of this
    repository's library is loaded."""
    if rank != 0:
        return
    from oracle import binding as oracle
    from oracle import synth as osynth
    ckpt = osynth.cached_checkpoint(osynth.QWEN3_0_6B, "qwen3_0_6b")
    threads = cpu_threads()
    m = oracle.OracleModel(ckpt, 64, threads=threads)
    prompt = osynth.prompt_tokens(7, PROMPT, VOCAB)

    def one():
        m.cursor = 0
        return m.generate(prompt, GENERATE)[0]

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tokens = one()
    dt = time.perf_counter() - t0
    v = args.steps * STEPS_PER_GENERATION / dt
    sample = (f"the whole generation ({STEPS_PER_GENERATION} oracle decode steps) per bench step on {threads} "
              "host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 weights, f32 activations and KV (f32 accumulate)",
        "data": "synthetic: random-init Qwen3-0.6B architecture (seed 7), 24 random prompt ids",
        "config": decode_config(world),
        "cpu_baseline": {"kind": "port", "cores": threads, "value": v, "unit": "tok/s", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "first_tokens": [int(t) for t in tokens[:8]],
        "note": "the reference's Rust crate cannot be built here (no cargo); its GPU kernels are timed on the "
                "GPU by the repo arm's triton_baseline object.  One CPU process on the host cores whatever the "
                "GPU count (rank 0 alone runs)",
    }))


if __name__ == "__main__":
    main()
