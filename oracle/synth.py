"""TEST INFRASTRUCTURE ONLY: the benchmark's synthetic inputs built with the
oracle's own generator (lsxo_synth_normal / lsxo_synth_uniform_u32), so that the
CPU baseline and the reference arms of bench.py never load the library they are
measured against.  The files are byte-identical to the library's
(laplacesscissors_b200.synth), which tests/test_oracle_synth.py checks.

Checkpoints are HF-layout folders (config.json + model.safetensors, the tensor
names of the reference's src/graph.rs:326-384): matrices N(0, std^2) in bf16,
norm gains 1.0, tensor i in sorted-name order drawing stream i of the seed.
"""
from __future__ import annotations

import json
import os
import shutil
import struct
import tempfile
from pathlib import Path

import numpy as np

from .binding import BF16, F32, lib, ptr

STREAM_PROMPT = 1 << 32

QWEN3_0_6B = dict(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=151936,
                  tie=True)
QWEN3_4B = dict(hidden=2560, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=9728, vocab=151936,
                tie=True)
QWEN3_8B = dict(hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=12288, vocab=151936,
                tie=False)


def normal_bf16(seed: int, stream: int, count: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib.lsxo_synth_normal(seed, stream, offset, count, float(std), BF16, ptr(out))
    return out


def normal_f32(seed: int, stream: int, count: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib.lsxo_synth_normal(seed, stream, offset, count, float(std), F32, ptr(out))
    return out


def uniform_u32(seed: int, stream: int, count: int, bound: int, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    lib.lsxo_synth_uniform_u32(seed, stream, offset, count, int(bound), ptr(out))
    return out


def prompt_tokens(seed: int, length: int, vocab: int) -> np.ndarray:
    return uniform_u32(seed, STREAM_PROMPT, length, vocab)


def config(hidden, layers, heads, kv_heads, head_dim, intermediate, vocab, tie=True) -> dict:
    return {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": hidden,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv_heads,
        "head_dim": head_dim, "intermediate_size": intermediate, "vocab_size": vocab,
        "tie_word_embeddings": tie, "rope_theta": 1e6, "rms_norm_eps": 1e-6,
        "max_position_embeddings": 40960, "hidden_act": "silu", "torch_dtype": "bfloat16",
    }


def shapes(c: dict) -> dict[str, tuple]:
    H, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    hd, q, kv = c["head_dim"], c["num_attention_heads"], c["num_key_value_heads"]
    out = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}"
        out.update({
            f"{p}.input_layernorm.weight": (H,), f"{p}.post_attention_layernorm.weight": (H,),
            f"{p}.self_attn.q_proj.weight": (q * hd, H), f"{p}.self_attn.k_proj.weight": (kv * hd, H),
            f"{p}.self_attn.v_proj.weight": (kv * hd, H), f"{p}.self_attn.o_proj.weight": (H, q * hd),
            f"{p}.self_attn.q_norm.weight": (hd,), f"{p}.self_attn.k_norm.weight": (hd,),
            f"{p}.mlp.gate_proj.weight": (I, H), f"{p}.mlp.up_proj.weight": (I, H),
            f"{p}.mlp.down_proj.weight": (H, I),
        })
    if not c.get("tie_word_embeddings", False):
        out["lm_head.weight"] = (V, H)
    return out


def write_checkpoint(root: Path, c: dict, seed: int = 7, std: float = 0.02) -> Path:
    root.mkdir(parents=True, exist_ok=True)
    sh = shapes(c)
    names = sorted(sh)
    header, offset = {}, 0
    for n in names:
        nbytes = 2 * int(np.prod(sh[n]))
        header[n] = {"dtype": "BF16", "shape": list(sh[n]), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    one = np.uint16(0x3F80)  # bf16 1.0
    with open(root / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for stream, n in enumerate(names):
            count = int(np.prod(sh[n]))
            if len(sh[n]) == 1:
                f.write(np.full(count, one, dtype=np.uint16).tobytes())
            else:
                f.write(normal_bf16(seed, stream, count, std).tobytes())
    (root / "config.json").write_text(json.dumps(c, indent=1))
    return root


def cached_checkpoint(shape: dict, name: str, seed: int = 7) -> Path:
    """write_checkpoint under the system temporary folder, reused when complete."""
    root = Path(tempfile.gettempdir()) / f"lsx-oracle-{name}-seed{seed}"
    if (root / "model.safetensors").exists() and (root / "config.json").exists():
        return root
    work = Path(tempfile.mkdtemp(prefix=root.name + ".partial-", dir=root.parent))
    try:
        write_checkpoint(work, config(**shape), seed)
        try:
            os.replace(work, root)
        except OSError:
            if not (root / "config.json").exists():
                raise
    finally:
        if work.exists():
            shutil.rmtree(work, ignore_errors=True)
    return root
