"""The reference's own GPU path, timed on this machine's GPU.

The reference runs its decode and readout validation as one Triton kernel per op
(kernels/ops.py), each launched by its Rust runtime with the constexprs, grids and
num_warps = 4 of src/gpu.rs:360-559, compiled with enable_fp_fusion = False
(kernels/compile.py:34-35), in the op order of Model::decode
(src/model.rs:729-853).  Its Rust runtime cannot be built here (no cargo), so this
script launches the same unmodified kernels through Triton's own launcher, in the
same order and with the same arguments.  The module is loaded from
baseline/_ref/kernels/ops.py (python baseline/install_reference.py <reference>
puts it there); nothing of this repository's library is used.

Two timings per workload:
  runtime  the reference's runtime pattern: every op allocates its output with
           cudaMalloc and frees it with cudaFree (cuMemAlloc_v2 / cuMemFree,
           src/device.rs:256-290; PYTORCH_NO_CUDA_MEMORY_CACHING=1 makes torch do
           exactly that), kernels launched one by one from the host, and every
           decode step's Frame (hidden state and logits) read back to the host,
           where the greedy argmax runs (src/diagnosis.rs:58-70, 106-149).  Python's
           launcher costs more per launch than the reference's Rust dispatch, so
           this figure is a lower bound on the reference's speed only up to that.
  graph    the same kernel sequence with fixed token ids and positions, captured
           once in a CUDA graph and replayed: the device time of the reference's
           kernels alone, with no allocation, launch or host cost -- an upper
           bound on the reference's speed on this GPU.

Usage: python baseline/triton_reference.py --mode runtime|graph --checkpoint DIR
       [--workload decode,readout,gemv] [--steps K] [--warmup W]
Prints one JSON object.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import struct
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
KERNELS = HERE / "_ref" / "kernels"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["runtime", "graph"], required=True)
    ap.add_argument("--checkpoint", required=True)
    ap.add_argument("--workload", default="decode,readout,gemv")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=24)
    ap.add_argument("--generate", type=int, default=32)
    ap.add_argument("--readout-rows", type=int, default=256)
    return ap.parse_args()


ARGS = parse_args()
if ARGS.mode == "runtime":
    # the reference allocates and frees every op's output on the device
    os.environ["PYTORCH_NO_CUDA_MEMORY_CACHING"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

if not (KERNELS / "ops.py").exists():
    print(json.dumps({"unavailable": "baseline/_ref/kernels/ops.py is not installed "
                                     "(python baseline/install_reference.py <reference tree>)"}))
    sys.exit(0)
sys.path.insert(0, str(KERNELS))
import ops  # noqa: E402  (the reference's kernels/ops.py, unmodified)
import triton  # noqa: E402

DEV = torch.device("cuda", 0)
OPTS = {"num_warps": 4, "enable_fp_fusion": False}


def cdiv(a, b):
    return (a + b - 1) // b


def p2(n):
    return 1 << (int(n) - 1).bit_length()


def f32(x):
    return float(np.float32(x))


# ------------------------------------------------------------- Gpu ops ------
class RefGpu:
    """The ops of src/gpu.rs:360-559: each returns a new f32 tensor."""

    def __init__(self, preallocated: bool):
        self.pre = preallocated

    def out(self, n):
        return torch.empty(n, dtype=torch.float32, device=DEV)

    def embedding(self, weight, row, width):
        out = self.out(width)
        ops.take_row[(cdiv(width, 256),)](weight, out, row, WIDTH=width, TILE=256, **OPTS)
        return out

    def linear(self, x, w, bias, rows, cols):
        out = self.out(rows)
        ops.matvec[(cdiv(rows, 8),)](w, x, bias if bias is not None else x, out, ROWS=rows, COLS=cols,
                                     BIAS=bias is not None, TILE_R=8, TILE_C=256, **OPTS)
        return out

    def norm(self, x, gain, groups, width, eps):
        out = self.out(groups * width)
        ops.normalization[(groups,)](x, gain, gain, out, WIDTH=width, EPSILON=f32(eps), CENTER=False, BIAS=False,
                                     TILE=p2(width), **OPTS)
        return out

    def rope(self, x, position, heads, dim, theta, rotary):
        n = heads * dim
        out = self.out(n)
        ops.rotary_position[(cdiv(n, 256),)](x, out, position, HEAD_DIM=dim, WIDTH=n, ROTARY=rotary,
                                             BASE=f32(theta), INTERLEAVED=False, TILE=256, **OPTS)
        return out

    def attention(self, q, k, v, keys, values, position, qheads, kvheads, dim, scale):
        width = kvheads * dim
        ops.cache_write[(cdiv(width, 256),)](k, v, keys, values, position, WIDTH=width, TILE=256, **OPTS)
        out = self.out(qheads * dim)
        ops.causal_attention[(qheads,)](q, keys, values, out, position, Q_HEADS=qheads, KV_HEADS=kvheads, DIM=dim,
                                        SCALE=f32(scale), TILE_T=32, TILE_D=p2(dim), **OPTS)
        return out

    def gated(self, gate, up, kind):
        out = self.out(gate.numel())
        ops.gated_product[(cdiv(gate.numel(), 256),)](gate, up, out, WIDTH=gate.numel(), KIND=kind, TILE=256,
                                                      **OPTS)
        return out

    def combine(self, x, y, factor):
        out = self.out(x.numel())
        ops.vector_sum[(cdiv(x.numel(), 256),)](x, y, out, f32(factor), WIDTH=x.numel(), TILE=256, **OPTS)
        return out


# ------------------------------------------------------------ checkpoint ----
def read_checkpoint(root: Path):
    path = root / "model.safetensors"
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    tensors = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        assert e["dtype"] == "BF16", (name, e["dtype"])
        b, en = e["data_offsets"]
        raw = np.asarray(mm[8 + n + b: 8 + n + en]).view(np.int16)
        tensors[name] = torch.from_numpy(raw.copy()).view(torch.bfloat16).to(DEV)  # Bank::take: raw upload
    return tensors, json.loads((root / "config.json").read_text())


class RefModel:
    """Model::load + Model::decode (src/model.rs:411-853) for a Qwen3-layout checkpoint
    on the reference's kernels."""

    def __init__(self, root: Path, gpu: RefGpu, capacity: int):
        self.t, c = read_checkpoint(root)
        self.gpu = gpu
        self.H, self.V, self.L = c["hidden_size"], c["vocab_size"], c["num_hidden_layers"]
        self.QH, self.KVH, self.D = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        self.I, self.theta, self.eps = c["intermediate_size"], c["rope_theta"], c["rms_norm_eps"]
        self.scale = 1.0 / math.sqrt(self.D)
        self.embed = self.t["model.embed_tokens.weight"]
        self.head = self.t.get("lm_head.weight", self.embed)
        kw = self.KVH * self.D
        self.keys = [torch.zeros(capacity * kw, dtype=torch.float32, device=DEV) for _ in range(self.L)]
        self.values = [torch.zeros(capacity * kw, dtype=torch.float32, device=DEV) for _ in range(self.L)]
        self.cursor = 0

    def w(self, i, name):
        return self.t[f"model.layers.{i}.{name}.weight"]

    def decode(self, token: int):
        """One token through every block, the final norm and the readout."""
        g, H, D, QH, KVH, I = self.gpu, self.H, self.D, self.QH, self.KVH, self.I
        residual = g.embedding(self.embed, token, H)
        for i in range(self.L):
            norm = g.norm(residual, self.w(i, "input_layernorm"), 1, H, self.eps)
            q = g.linear(norm, self.w(i, "self_attn.q_proj"), None, QH * D, H)
            k = g.linear(norm, self.w(i, "self_attn.k_proj"), None, KVH * D, H)
            v = g.linear(norm, self.w(i, "self_attn.v_proj"), None, KVH * D, H)
            q = g.norm(q, self.w(i, "self_attn.q_norm"), QH, D, self.eps)
            k = g.norm(k, self.w(i, "self_attn.k_norm"), KVH, D, self.eps)
            q = g.rope(q, self.cursor, QH, D, self.theta, D)
            k = g.rope(k, self.cursor, KVH, D, self.theta, D)
            mixed = g.attention(q, k, v, self.keys[i], self.values[i], self.cursor, QH, KVH, D, self.scale)
            projected = g.linear(mixed, self.w(i, "self_attn.o_proj"), None, H, QH * D)
            residual = g.combine(residual, projected, 1.0)
            norm = g.norm(residual, self.w(i, "post_attention_layernorm"), 1, H, self.eps)
            gate = g.linear(norm, self.w(i, "mlp.gate_proj"), None, I, H)
            up = g.linear(norm, self.w(i, "mlp.up_proj"), None, I, H)
            feature = g.gated(gate, up, 0)
            down = g.linear(feature, self.w(i, "mlp.down_proj"), None, H, I)
            residual = g.combine(residual, down, 1.0)
        hidden = g.norm(residual, self.t["model.norm.weight"], 1, H, self.eps)
        logits = g.linear(hidden, self.head, None, self.V, H)
        self.cursor += 1
        return hidden, logits


def first_argmax(values: np.ndarray) -> int:  # src/diagnosis.rs:58-70
    if not np.all(np.isfinite(values)):
        raise ValueError("non-finite scores")
    return int(np.argmax(values))


def synth_prompt(n: int, vocab: int, seed: int = 7) -> list[int]:
    """The prompt ids of the decode workload: the counter-based generator of the
    benchmark (SplitMix64 finaliser, stream 2^32, uniform in [0, vocab))."""
    def mix(z):
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9 & 0xFFFFFFFFFFFFFFFF
        z = (z ^ (z >> 27)) * 0x94D049BB133111EB & 0xFFFFFFFFFFFFFFFF
        return z ^ (z >> 31)
    golden = 0x9E3779B97F4A7C15
    key = mix(seed ^ mix(((1 << 32) + golden) & 0xFFFFFFFFFFFFFFFF))
    out = []
    for i in range(n):
        bits = mix((key + (i + 1) * golden) & 0xFFFFFFFFFFFFFFFF)
        out.append(((bits >> 32) * vocab) >> 32)
    return out


# ------------------------------------------------------------- workloads ----
def decode_runtime(model: RefModel, prompt, generate, steps, warmup):
    """generate_frames (src/diagnosis.rs:106-149): the prompt token by token, then
    greedy argmax on the host; every step's Frame is read back."""
    def one():
        model.cursor = 0
        tokens = []
        frame = None
        for t in prompt:
            h, z = model.decode(int(t))
            frame = (h.cpu().numpy(), z.cpu().numpy())
        for position in range(generate):
            token = first_argmax(frame[1])
            tokens.append(token)
            if position + 1 == generate:
                break
            h, z = model.decode(token)
            frame = (h.cpu().numpy(), z.cpu().numpy())
        return tokens

    for _ in range(warmup):
        tokens = one()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        tokens = one()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) / steps, tokens


def decode_graph(model: RefModel, prompt, generate, steps, warmup):
    """The generation's kernels with its token ids fixed in advance, as one CUDA graph."""
    # the greedy path, computed once eagerly: the ids every step feeds
    model.cursor = 0
    feed = []
    frame = None
    for t in prompt:
        feed.append(int(t))
        _, frame = model.decode(int(t))
    for position in range(generate - 1):
        token = first_argmax(frame.cpu().numpy())
        feed.append(token)
        _, frame = model.decode(token)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        model.cursor = 0
        for t in feed:  # warm the allocator's graph pool shapes outside capture
            model.decode(t)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        model.cursor = 0
        for t in feed:
            model.decode(t)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    stop.record()
    stop.synchronize()
    return start.elapsed_time(stop) / 1e3 / steps, len(feed)


def readout_inputs(model: RefModel, rows: int, seed: int = 7):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, model.H))
    x = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + 1e-6)
    targets = rng.integers(0, model.V, rows)
    # the rank-16 joint edit (DeviceRotation::upload_edit, src/model.rs:311-341)
    basis, _ = np.linalg.qr(rng.standard_normal((model.H, 16)))
    basis = basis.T
    transform = np.eye(16)
    for p in range(8):
        a = math.radians(rng.uniform(-3, 3))
        c, s = math.cos(a), math.sin(a)
        i, j = 2 * p, 2 * p + 1
        transform[[i, i, j, j], [i, j, i, j]] = [c, -s, s, c]
    return x.astype(np.float32), targets, basis, transform


def readout_runtime(model: RefModel, rows, steps, warmup):
    """verify_cached's per-row work (src/diagnosis.rs:512-537): Model::readout with
    the joint edit (upload, DeviceRotation::apply = three matvecs and a combine,
    the lm_head matvec, logits read back), then minimum_margin and argmax on the
    host.  Seconds per row."""
    g = model.gpu
    x, targets, basis, transform = readout_inputs(model, rows)
    r = basis.shape[0]
    d_basis = torch.from_numpy(basis.astype(np.float32).reshape(-1)).to(DEV)
    d_transpose = torch.from_numpy(basis.T.astype(np.float32).reshape(-1).copy()).to(DEV)
    d_delta = torch.from_numpy((transform - np.eye(r)).astype(np.float32).reshape(-1)).to(DEV)

    def one():
        out = []
        for i in range(rows):
            h = torch.from_numpy(x[i]).to(DEV)
            coords = g.linear(h, d_basis, None, r, model.H)
            shift = g.linear(coords, d_delta, None, r, r)
            lifted = g.linear(shift, d_transpose, None, model.H, r)
            edited = g.combine(h, lifted, 1.0)
            z = g.linear(edited, model.head, None, model.V, model.H).cpu().numpy()
            t = int(targets[i])
            if not np.all(np.isfinite(z)):
                raise ValueError("non-finite scores")
            masked = z.astype(np.float64)
            zt = masked[t]
            masked[t] = -np.inf
            out.append((zt - masked.max(), first_argmax(z)))
        return out

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    return (time.perf_counter() - t0) / steps / rows


def readout_graph(model: RefModel, rows, steps, warmup):
    """The per-row kernels (edit + lm_head matvec) of `rows` rows as one CUDA graph."""
    g = model.gpu
    x, _, basis, transform = readout_inputs(model, rows)
    r = basis.shape[0]
    d_x = torch.from_numpy(x).to(DEV)
    d_basis = torch.from_numpy(basis.astype(np.float32).reshape(-1)).to(DEV)
    d_transpose = torch.from_numpy(basis.T.astype(np.float32).reshape(-1).copy()).to(DEV)
    d_delta = torch.from_numpy((transform - np.eye(r)).astype(np.float32).reshape(-1)).to(DEV)

    def rows_once():
        for i in range(rows):
            h = d_x[i]
            coords = g.linear(h, d_basis, None, r, model.H)
            shift = g.linear(coords, d_delta, None, r, r)
            lifted = g.linear(shift, d_transpose, None, model.H, r)
            edited = g.combine(h, lifted, 1.0)
            g.linear(edited, model.head, None, model.V, model.H)

    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        rows_once()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        rows_once()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    stop.record()
    stop.synchronize()
    return start.elapsed_time(stop) / 1e3 / steps / rows


GEMV_SHAPES = [(2048, 1024), (6144, 1024), (1024, 3072), (151936, 1024), (12288, 4096)]


def gemv_graph(gpu: RefGpu, iters: int = 20):
    """The reference's matvec (TILE_R 8, TILE_C 256, 4 warps) on the GEMV shapes:
    launches over enough weight copies to exceed L2 captured in a CUDA graph,
    bytes = 2NK + 4K + 4N per launch."""
    out = {}
    for n, k in GEMV_SHAPES:
        copies = max(2, min(64, -(-256_000_000 // (2 * n * k))))
        ws = [(torch.randn(n * k, device=DEV) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn(k, device=DEV).to(torch.bfloat16).float()
        y = torch.empty(n, dtype=torch.float32, device=DEV)

        def launch_all():
            for w in ws:
                ops.matvec[(cdiv(n, 8),)](w, x, x, y, ROWS=n, COLS=k, BIAS=False, TILE_R=8, TILE_C=256, **OPTS)

        launch_all()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        with torch.cuda.graph(graph, stream=stream):
            launch_all()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            graph.replay()
        stop.record()
        stop.synchronize()
        s = start.elapsed_time(stop) / 1e3 / (iters * copies)
        out[f"{n}x{k}"] = {"us": s * 1e6, "GB/s": (2 * n * k + 4 * k + 4 * n) / s / 1e9}
        del ws, graph
    return out


def main():
    a = ARGS
    work = set(a.workload.split(","))
    gpu = RefGpu(preallocated=a.mode == "graph")
    result = {"mode": a.mode, "triton": triton.__version__, "kernels": "kernels/ops.py (unmodified)",
              "launch": "num_warps 4, enable_fp_fusion False, src/gpu.rs constexprs and grids"}
    inst = HERE / "_ref" / "INSTALLED.json"
    if inst.exists():
        result["ops_sha256"] = json.loads(inst.read_text())["sha256"]
    model = None
    if work & {"decode", "readout"}:
        model = RefModel(Path(a.checkpoint), gpu, a.prompt + a.generate + 8)
    prompt = synth_prompt(a.prompt, model.V) if model else None
    steps_per_generation = a.prompt + a.generate - 1
    if "decode" in work:
        if a.mode == "runtime":
            s, tokens = decode_runtime(model, prompt, a.generate, a.steps, a.warmup)
            result["decode"] = {"tok_s": steps_per_generation / s, "ms_per_generation": s * 1e3,
                                "first_tokens": tokens[:8]}
        else:
            s, n = decode_graph(model, prompt, a.generate, a.steps, a.warmup)
            result["decode"] = {"tok_s": n / s, "ms_per_generation": s * 1e3}
    if "readout" in work:
        fn = readout_runtime if a.mode == "runtime" else readout_graph
        s = fn(model, a.readout_rows, a.steps, a.warmup)
        result["readout"] = {"rows_s": 1.0 / s, "rows_timed": a.readout_rows}
    if "gemv" in work and a.mode == "graph":
        result["gemv"] = gemv_graph(gpu)
    print(json.dumps(result))


if __name__ == "__main__":
    main()
