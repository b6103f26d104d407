"""Seeded synthetic checkpoints and inputs in the reference's formats.

Checkpoints are HF-layout folders (config.json + model.safetensors) that the
reference's GraphSpec::from_config (src/graph.rs:231-411) and this library's
loader both accept.  Values come from the counter-based generator of
csrc/synth.cu (lsx_synth_normal / lsx_synth_uniform_u32): tensor number i in
sorted-name order draws stream i; inputs use the fixed streams below.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct
from pathlib import Path

import numpy as np

from ._lib import BF16, F32, check, lib

# Streams reserved for inputs (tensor streams count up from 0).
STREAM_PROMPT = 1 << 32
STREAM_HIDDEN = (1 << 32) + 1
STREAM_TARGETS = (1 << 32) + 2
STREAM_EDIT_BASIS = (1 << 32) + 3
STREAM_EDIT_ANGLES = (1 << 32) + 4


def normal_bf16(seed: int, stream: int, count: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    """bf16 bit patterns (uint16) of seeded N(0, std^2) draws."""
    out = np.empty(count, dtype=np.uint16)
    check(lib.lsx_synth_normal(seed, stream, offset, count, float(std), BF16, out.ctypes.data_as(C.c_void_p)))
    return out


def normal_f32(seed: int, stream: int, count: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    check(lib.lsx_synth_normal(seed, stream, offset, count, float(std), F32, out.ctypes.data_as(C.c_void_p)))
    return out


def uniform_u32(seed: int, stream: int, count: int, bound: int, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    check(lib.lsx_synth_uniform_u32(seed, stream, offset, count, int(bound),
                                    out.ctypes.data_as(C.POINTER(C.c_uint32))))
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


_DTYPE_NAME = {np.dtype(np.float32): "F32", np.dtype(np.uint16): "BF16", np.dtype(np.float16): "F16"}


def write_safetensors(path: str | os.PathLike, tensors: dict[str, np.ndarray],
                      dtypes: dict[str, str] | None = None) -> None:
    """Writes tensors in safetensors layout; uint16 arrays are stored as BF16
    unless `dtypes` names another 2-byte kind."""
    names = sorted(tensors)
    header: dict = {}
    offset = 0
    for n in names:
        a = tensors[n]
        kind = (dtypes or {}).get(n) or _DTYPE_NAME[a.dtype]
        header[n] = {"dtype": kind, "shape": list(a.shape), "data_offsets": [offset, offset + a.nbytes]}
        offset += a.nbytes
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for n in names:
            f.write(np.ascontiguousarray(tensors[n]).tobytes())


def read_safetensors(path: str | os.PathLike) -> dict[str, tuple[str, tuple, np.memmap]]:
    """Maps a safetensors file: name -> (dtype, shape, raw array view)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        b, en = e["data_offsets"]
        raw = mm[8 + n + b: 8 + n + en]
        np_dtype = {"F32": np.float32, "BF16": np.uint16, "F16": np.float16}[e["dtype"]]
        out[name] = (e["dtype"], tuple(e["shape"]), raw.view(np_dtype).reshape(e["shape"]))
    return out


def qwen3_config(hidden: int, layers: int, heads: int, kv_heads: int, head_dim: int, intermediate: int,
                 vocab: int, tie: bool = True, theta: float = 1e6, eps: float = 1e-6,
                 max_positions: int = 40960, eos: int | None = None) -> dict:
    c = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": hidden,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv_heads,
        "head_dim": head_dim, "intermediate_size": intermediate, "vocab_size": vocab,
        "tie_word_embeddings": tie, "rope_theta": theta, "rms_norm_eps": eps,
        "max_position_embeddings": max_positions, "hidden_act": "silu", "torch_dtype": "bfloat16",
    }
    if eos is not None:
        c["eos_token_id"] = eos
    return c


QWEN3_0_6B = dict(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=151936,
                  tie=True)
QWEN3_4B = dict(hidden=2560, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=9728, vocab=151936,
                tie=True)
QWEN3_8B = dict(hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=12288, vocab=151936,
                tie=False)


def qwen3_tensor_shapes(config: dict) -> dict[str, tuple]:
    H, I, V = config["hidden_size"], config["intermediate_size"], config["vocab_size"]
    hd, q, kv = config["head_dim"], config["num_attention_heads"], config["num_key_value_heads"]
    shapes = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    for i in range(config["num_hidden_layers"]):
        p = f"model.layers.{i}"
        shapes.update({
            f"{p}.input_layernorm.weight": (H,), f"{p}.post_attention_layernorm.weight": (H,),
            f"{p}.self_attn.q_proj.weight": (q * hd, H), f"{p}.self_attn.k_proj.weight": (kv * hd, H),
            f"{p}.self_attn.v_proj.weight": (kv * hd, H), f"{p}.self_attn.o_proj.weight": (H, q * hd),
            f"{p}.self_attn.q_norm.weight": (hd,), f"{p}.self_attn.k_norm.weight": (hd,),
            f"{p}.mlp.gate_proj.weight": (I, H), f"{p}.mlp.up_proj.weight": (I, H),
            f"{p}.mlp.down_proj.weight": (H, I),
        })
    if not config.get("tie_word_embeddings", False):
        shapes["lm_head.weight"] = (V, H)
    return shapes


def make_qwen3_checkpoint(root: str | os.PathLike, config: dict, seed: int = 7, std: float = 0.02,
                          gain_std: float = 0.0) -> Path:
    """Writes a random-init Qwen3-architecture checkpoint: matrices N(0, std^2) in
    bf16, norm gains 1.0 (plus N(0, gain_std^2) when gain_std > 0), tensor i in
    sorted-name order drawing stream i of `seed`.  Tensors are generated and
    written one at a time, so memory stays at one tensor (the 8B model's 16 GB
    never sits in host memory at once); the file equals write_safetensors' of the
    same tensors."""
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    shapes = qwen3_tensor_shapes(config)
    names = sorted(shapes)
    header: dict = {}
    offset = 0
    for n in names:
        nbytes = 2 * int(np.prod(shapes[n]))
        header[n] = {"dtype": "BF16", "shape": list(shapes[n]), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    with open(root / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for stream, name in enumerate(names):
            count = int(np.prod(shapes[name]))
            if len(shapes[name]) == 1:
                g = np.ones(count, dtype=np.float32)
                if gain_std > 0:
                    g = g + normal_f32(seed, stream, count, gain_std)
                f.write(f32_to_bf16(g).tobytes())
            else:
                f.write(normal_bf16(seed, stream, count, std).tobytes())
    (root / "config.json").write_text(json.dumps(config, indent=1))
    return root


def cached_checkpoint(shape: str, seed: int = 7, **overrides) -> Path:
    """The checkpoint make_qwen3_checkpoint writes for the named shape (QWEN3_0_6B,
    QWEN3_4B, QWEN3_8B) with `overrides`, kept under the system temporary folder so
    later runs on the same machine reuse it.  It is written to a private folder and
    renamed into place when complete, so an interrupted write is never reused."""
    import shutil
    import tempfile
    cfg = dict(globals()[shape], **overrides)
    tag = "".join(f"-{k}{v}" for k, v in sorted(overrides.items()))
    root = Path(tempfile.gettempdir()) / f"lsx-bench-{shape.lower()}-seed{seed}{tag}"
    if (root / "model.safetensors").exists() and (root / "config.json").exists():
        return root
    work = Path(tempfile.mkdtemp(prefix=root.name + ".partial-", dir=root.parent))
    try:
        make_qwen3_checkpoint(work, qwen3_config(**cfg), seed=seed)
        try:
            os.replace(work, root)
        except OSError:  # another process completed it first
            if not (root / "config.json").exists():
                raise
    finally:
        if work.exists():
            shutil.rmtree(work, ignore_errors=True)
    return root


def prompt_tokens(seed: int, length: int, vocab: int) -> np.ndarray:
    return uniform_u32(seed, STREAM_PROMPT, length, vocab)


def readout_hidden(seed: int, rows: int, width: int, eps: float = 1e-6, first: int = 0) -> np.ndarray:
    """Hidden states of the readout-validation workload: N(0, 1) rows, RMSNorm'd
    (gain 1) in f64, rounded to bf16.  Returns bf16 bit patterns [rows, width] of
    rows first .. first + rows - 1 of the seed's row sequence (any shard of the
    global set is generated independently)."""
    x = normal_f32(seed, STREAM_HIDDEN, rows * width, offset=first * width).astype(np.float64).reshape(rows, width)
    x = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + eps)
    return f32_to_bf16(x.astype(np.float32))


def readout_targets(seed: int, rows: int, vocab: int, first: int = 0) -> np.ndarray:
    return uniform_u32(seed, STREAM_TARGETS, rows, vocab, offset=first)


__all__ = [
    "normal_bf16", "normal_f32", "uniform_u32", "bf16_to_f32", "f32_to_bf16", "write_safetensors",
    "read_safetensors", "qwen3_config", "qwen3_tensor_shapes", "make_qwen3_checkpoint", "cached_checkpoint",
    "prompt_tokens",
    "readout_hidden", "readout_targets", "QWEN3_0_6B", "QWEN3_4B", "QWEN3_8B",
]
