"""TEST INFRASTRUCTURE ONLY: ctypes binding of the oracle (liblsx_oracle.so).

Loaded by tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py
as the checker of the CUDA path; the product never imports it.  Besides the raw
functions it offers OracleModel, which reads a checkpoint folder on its own
(safetensors + config.json or laplace.graph.json, following src/graph.rs) and
runs Model::decode (src/model.rs:729-853) with the oracle's f64 reductions.
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liblsx_oracle.so"

F32, F16, BF16 = 0, 1, 2


def build() -> Path:
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < max((HERE / "lsx_oracle.c").stat().st_mtime,
                                                               (HERE / "lsx_oracle.h").stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


class Block(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, C.c_void_p) for n in ("q_bias", "k_bias", "v_bias", "o_bias", "gate_bias", "up_bias",
                                          "down_bias")] + \
               [("kind", C.c_int)] + \
               [(n, C.c_void_p) for n in ("input_gain", "post_gain", "input_bias", "post_bias", "q_gain", "k_gain",
                                          "keys", "values")]


class ModelStruct(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("hidden", "vocab", "layers", "qheads", "kvheads", "head_dim",
                                          "intermediate", "rotary", "capacity")] + \
               [("theta", C.c_double), ("score_scale", C.c_double), ("epsilon", C.c_float),
                ("qk_epsilon", C.c_float), ("center", C.c_int), ("interleaved", C.c_int), ("activation", C.c_int),
                ("embedding_scale", C.c_float), ("embedding", C.c_void_p), ("embedding_kind", C.c_int),
                ("head", C.c_void_p), ("head_kind", C.c_int), ("head_bias", C.c_void_p),
                ("final_gain", C.c_void_p), ("final_bias", C.c_void_p), ("blocks", C.POINTER(Block))]


class FeasibleStruct(C.Structure):
    _fields_ = [("bound", C.c_double), ("lower", C.c_void_p), ("upper", C.c_void_p), ("count", C.c_size_t),
                ("capacity", C.c_size_t), ("work", C.c_uint64 * 4)]


def _load() -> C.CDLL:
    lib = C.CDLL(str(build()))
    V, SZ, I, D, F = C.c_void_p, C.c_size_t, C.c_int, C.c_double, C.c_float
    sig = {
        "lsxo_take_row": (None, [V, I, SZ, SZ, V]),
        "lsxo_matvec": (None, [V, I, V, V, SZ, SZ, V, I]),
        "lsxo_norm": (None, [V, V, V, SZ, SZ, F, I, V]),
        "lsxo_rope": (None, [V, SZ, SZ, D, SZ, I, SZ, V]),
        "lsxo_cache_write": (None, [V, V, V, V, SZ, SZ]),
        "lsxo_attention": (None, [V, V, V, SZ, SZ, SZ, SZ, D, V]),
        "lsxo_gated": (None, [V, V, SZ, I, V]),
        "lsxo_combine": (None, [V, V, F, SZ, V]),
        "lsxo_plane_rotation": (None, [V, V, V, F, F, SZ, V]),
        "lsxo_plane_coefficients": (None, [D, C.POINTER(D), C.POINTER(D)]),
        "lsxo_plane_apply": (None, [V, V, D, SZ, V, V]),
        "lsxo_subspace_apply": (None, [V, V, SZ, SZ, V, V]),
        "lsxo_argmax": (C.c_uint32, [V, SZ]),
        "lsxo_other": (SZ, [V, SZ, C.c_uint32]),
        "lsxo_minimum_margin": (D, [V, SZ, C.c_uint32]),
        "lsxo_loss": (D, [V, SZ, C.c_uint32]),
        "lsxo_decode": (None, [C.POINTER(ModelStruct), SZ, V, V, V, I]),
        "lsxo_embedding": (None, [C.POINTER(ModelStruct), C.c_uint32, V]),
        "lsxo_readout_rows": (None, [V, I, V, SZ, SZ, V, SZ, V, V, V, V, I]),
        "lsxo_version": (C.c_char_p, []),
        "lsxo_feasible_init": (I, [C.POINTER(FeasibleStruct), D]),
        "lsxo_feasible_free": (None, [C.POINTER(FeasibleStruct)]),
        "lsxo_feasible_constrain": (I, [C.POINTER(FeasibleStruct), D, D, D]),
        "lsxo_feasible_is_empty": (I, [C.POINTER(FeasibleStruct)]),
        "lsxo_feasible_nearest": (I, [C.POINTER(FeasibleStruct), C.POINTER(D)]),
        "lsxo_feasible_intervals": (SZ, [C.POINTER(FeasibleStruct), V, SZ]),
        "lsxo_plane_feasible": (I, [C.POINTER(FeasibleStruct), V, V, SZ, V, V, V, V, SZ, D, D]),
        "lsxo_restored_loss": (D, [V, SZ, SZ, F, C.c_uint32]),
        "lsxo_integrated_credits": (None, [V, V, V, V, SZ, SZ, SZ, V, V]),
        "lsxo_synth_normal": (None, [C.c_uint64, C.c_uint64, C.c_uint64, SZ, D, I, V]),
        "lsxo_synth_uniform_u32": (None, [C.c_uint64, C.c_uint64, C.c_uint64, SZ, C.c_uint32, V]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------ op wrappers ---
def matvec(w: np.ndarray, kind: int, x, bias, rows: int, cols: int, threads: int = 0) -> np.ndarray:
    out = np.empty(rows, dtype=np.float32)
    x = f32(x)
    b = None if bias is None else f32(bias)
    lib.lsxo_matvec(ptr(np.ascontiguousarray(w)), kind, ptr(x), ptr(b), rows, cols, ptr(out), threads)
    return out


def take_row(w: np.ndarray, kind: int, row: int, width: int) -> np.ndarray:
    out = np.empty(width, dtype=np.float32)
    lib.lsxo_take_row(ptr(np.ascontiguousarray(w)), kind, row, width, ptr(out))
    return out


def norm(x, gain, bias, groups, width, eps, center) -> np.ndarray:
    x, g = f32(x), f32(gain)
    b = None if bias is None else f32(bias)
    out = np.empty(groups * width, dtype=np.float32)
    lib.lsxo_norm(ptr(x), ptr(g), ptr(b), groups, width, float(eps), int(center), ptr(out))
    return out


def rope(x, heads, dim, theta, rotary, interleaved, position) -> np.ndarray:
    x = f32(x)
    out = np.empty_like(x)
    lib.lsxo_rope(ptr(x), heads, dim, float(theta), rotary, int(interleaved), position, ptr(out))
    return out


def attention(q, keys, values, position, qheads, kvheads, dim, scale) -> np.ndarray:
    q, k, v = f32(q), f32(keys), f32(values)
    out = np.empty(qheads * dim, dtype=np.float32)
    lib.lsxo_attention(ptr(q), ptr(k), ptr(v), position, qheads, kvheads, dim, float(scale), ptr(out))
    return out


def gated(gate, up, kind) -> np.ndarray:
    g, u = f32(gate), f32(up)
    out = np.empty_like(g)
    lib.lsxo_gated(ptr(g), ptr(u), g.size, int(kind), ptr(out))
    return out


def combine(x, y, factor) -> np.ndarray:
    x, y = f32(x), f32(y)
    out = np.empty_like(x)
    lib.lsxo_combine(ptr(x), ptr(y), float(factor), x.size, ptr(out))
    return out


def plane_rotation(h, u, v, a, b) -> np.ndarray:
    h, u, v = f32(h), f32(u), f32(v)
    out = np.empty_like(h)
    lib.lsxo_plane_rotation(ptr(h), ptr(u), ptr(v), float(a), float(b), h.size, ptr(out))
    return out


def plane_apply(u, v, tangent, h) -> np.ndarray:
    u, v, h = (np.ascontiguousarray(a, dtype=np.float64) for a in (u, v, h))
    out = np.empty_like(h)
    lib.lsxo_plane_apply(ptr(u), ptr(v), float(tangent), h.size, ptr(h), ptr(out))
    return out


def subspace_apply(basis, transform, h) -> np.ndarray:
    b, t, h = (np.ascontiguousarray(a, dtype=np.float64) for a in (basis, transform, h))
    out = np.empty_like(h)
    lib.lsxo_subspace_apply(ptr(b), ptr(t), b.shape[0], b.shape[1], ptr(h), ptr(out))
    return out


def argmax(z) -> int:
    z = f32(z)
    return int(lib.lsxo_argmax(ptr(z), z.size))


def other(z, target) -> int:
    z = f32(z)
    return int(lib.lsxo_other(ptr(z), z.size, int(target)))


def minimum_margin(z, target) -> float:
    z = f32(z)
    return float(lib.lsxo_minimum_margin(ptr(z), z.size, int(target)))


def loss(z, target) -> float:
    z = f32(z)
    return float(lib.lsxo_loss(ptr(z), z.size, int(target)))


def readout_rows(w: np.ndarray, kind: int, bias, vocab: int, width: int, inputs: np.ndarray, targets,
                 threads: int = 0):
    """Margin (f64), first argmax and target logit of every f32 input row."""
    x = f32(inputs)
    t = np.ascontiguousarray(targets, dtype=np.uint32)
    n = t.size
    margin = np.empty(n, dtype=np.float64)
    amax = np.empty(n, dtype=np.uint32)
    tl = np.empty(n, dtype=np.float32)
    b = None if bias is None else f32(bias)
    lib.lsxo_readout_rows(ptr(np.ascontiguousarray(w)), kind, ptr(b), vocab, width, ptr(x), n, ptr(t), ptr(margin),
                          ptr(amax), ptr(tl), threads)
    return margin, amax, tl


# ------------------------------------------------------- checkpoint reader --
_KIND = {"F32": F32, "F16": F16, "BF16": BF16}
_NP = {"F32": np.float32, "F16": np.uint16, "BF16": np.uint16}


def read_checkpoint(root: Path) -> dict[str, tuple[int, tuple, np.ndarray]]:
    path = Path(root) / "model.safetensors"
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        b, en = e["data_offsets"]
        out[name] = (_KIND[e["dtype"]], tuple(e["shape"]), mm[8 + n + b: 8 + n + en].view(_NP[e["dtype"]]))
    return out


def widen(kind: int, raw: np.ndarray) -> np.ndarray:
    if kind == F32:
        return np.asarray(raw, dtype=np.float32)
    if kind == BF16:
        return (np.asarray(raw, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    return np.asarray(raw, dtype=np.uint16).view(np.float16).astype(np.float32)


def graph_of(root: Path, tensors: dict) -> dict:
    """GraphSpec::load (src/graph.rs:151-163) for laplace.graph.json or a
    Qwen/Llama-style config.json."""
    g = Path(root) / "laplace.graph.json"
    if g.is_file():
        return json.loads(g.read_text())
    c = json.loads((Path(root) / "config.json").read_text())
    eps = c["rms_norm_eps"]
    heads = c["num_attention_heads"]
    kv = c.get("num_key_value_heads", heads)
    hd = c.get("head_dim", c["hidden_size"] // heads)
    rotary = int(hd * c.get("partial_rotary_factor", 1.0))
    theta = c.get("rope_theta", (c.get("rope_parameters") or {}).get("rope_theta"))
    rms = lambda n: {"weight": n + ".weight", "kind": "rms", "epsilon": eps}  # noqa: E731
    lin = lambda n: {"weight": n + ".weight", **({"bias": n + ".bias"} if n + ".bias" in tensors else {})}  # noqa
    blocks = []
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}"
        att = {"query": lin(f"{p}.self_attn.q_proj"), "key": lin(f"{p}.self_attn.k_proj"),
               "value": lin(f"{p}.self_attn.v_proj"), "output": lin(f"{p}.self_attn.o_proj"),
               "query_heads": heads, "kv_heads": kv, "head_dim": hd, "rotary_dim": rotary, "rope_theta": theta,
               "score_scale": float(np.float32(1.0) / np.sqrt(np.float32(hd)))}
        if f"{p}.self_attn.q_norm.weight" in tensors:
            att["query_norm"] = rms(f"{p}.self_attn.q_norm")
        if f"{p}.self_attn.k_norm.weight" in tensors:
            att["key_norm"] = rms(f"{p}.self_attn.k_norm")
        blocks.append({"input_norm": rms(f"{p}.input_layernorm"),
                       "post_attention_norm": rms(f"{p}.post_attention_layernorm"), "attention": att,
                       "mlp": {"gate": lin(f"{p}.mlp.gate_proj"), "up": lin(f"{p}.mlp.up_proj"),
                               "down": lin(f"{p}.mlp.down_proj"), "intermediate_size": c["intermediate_size"],
                               "activation": c.get("hidden_act", "silu")}})
    tied = c.get("tie_word_embeddings", False) is True
    return {"hidden_size": c["hidden_size"], "vocab_size": c["vocab_size"], "embedding": "model.embed_tokens.weight",
            "final_norm": rms("model.norm"),
            "readout": {"weight": "model.embed_tokens.weight"} if tied else lin("lm_head"), "blocks": blocks,
            "eos_token_ids": [c["eos_token_id"]] if isinstance(c.get("eos_token_id"), int) else
            c.get("eos_token_id") or []}


ACTIVATION = {"silu": 0, "swish": 0, "gelu": 1, "relu": 2, "gelu_tanh": 3, "gelu_new": 3, "gelu_pytorch_tanh": 3}


class OracleModel:
    """Model::load + Model::decode (src/model.rs:411-853) on the oracle."""

    def __init__(self, root, capacity: int, threads: int = 0):
        root = Path(root)
        self.tensors = read_checkpoint(root)
        self.graph = graph_of(root, self.tensors)
        self.capacity = capacity
        self.threads = threads
        self.cursor = 0
        self._keep = []
        g = self.graph
        b0 = g["blocks"][0]
        a0 = b0["attention"]
        m = ModelStruct()
        m.hidden, m.vocab, m.layers = g["hidden_size"], g["vocab_size"], len(g["blocks"])
        m.qheads, m.kvheads, m.head_dim = a0["query_heads"], a0["kv_heads"], a0["head_dim"]
        m.intermediate, m.rotary, m.capacity = b0["mlp"]["intermediate_size"], a0["rotary_dim"], capacity
        m.theta, m.score_scale = float(np.float32(a0["rope_theta"])), float(np.float32(a0["score_scale"]))
        m.epsilon = b0["input_norm"]["epsilon"]
        qn = a0.get("query_norm") or a0.get("key_norm")
        m.qk_epsilon = qn["epsilon"] if qn else m.epsilon
        m.center = 1 if b0["input_norm"]["kind"] == "layer" else 0
        m.interleaved = 1 if a0.get("rotary_interleaved") else 0
        m.activation = ACTIVATION[b0["mlp"]["activation"]]
        m.embedding_scale = g.get("embedding_scale", 1.0)
        k, _, raw = self.tensors[g["embedding"]]
        m.embedding, m.embedding_kind = self._hold(raw), k
        k, _, raw = self.tensors[g["readout"]["weight"]]
        m.head, m.head_kind = self._hold(raw), k
        m.head_bias = self._vec(g["readout"].get("bias"))
        m.final_gain = self._gain(g["final_norm"])
        m.final_bias = self._vec(g["final_norm"].get("bias"))
        blocks = (Block * m.layers)()
        self.caches = []
        for i, b in enumerate(g["blocks"]):
            a, mlp = b["attention"], b["mlp"]
            kinds = set()
            for fld, spec in (("q", a["query"]), ("k", a["key"]), ("v", a["value"]), ("o", a["output"]),
                              ("gate", mlp["gate"]), ("up", mlp["up"]), ("down", mlp["down"])):
                kk, _, raw = self.tensors[spec["weight"]]
                kinds.add(kk)
                setattr(blocks[i], fld, self._hold(raw))
                setattr(blocks[i], fld + "_bias", self._vec(spec.get("bias")))
            assert len(kinds) == 1, "the oracle expects one storage kind per block"
            blocks[i].kind = kinds.pop()
            blocks[i].input_gain = self._gain(b["input_norm"])
            blocks[i].post_gain = self._gain(b["post_attention_norm"])
            blocks[i].input_bias = self._vec(b["input_norm"].get("bias"))
            blocks[i].post_bias = self._vec(b["post_attention_norm"].get("bias"))
            blocks[i].q_gain = self._gain(a["query_norm"]) if a.get("query_norm") else None
            blocks[i].k_gain = self._gain(a["key_norm"]) if a.get("key_norm") else None
            n = capacity * a["kv_heads"] * a["head_dim"]
            keys, values = np.zeros(n, np.float32), np.zeros(n, np.float32)
            self.caches.append((keys, values))
            blocks[i].keys, blocks[i].values = ptr(keys), ptr(values)
        m.blocks = blocks
        self._blocks = blocks
        self.m = m

    def _hold(self, raw):
        a = np.ascontiguousarray(raw)
        self._keep.append(a)
        return ptr(a)

    def _vec(self, name):
        if not name:
            return None
        k, _, raw = self.tensors[name]
        return self._hold(widen(k, raw))

    def _gain(self, spec):
        k, _, raw = self.tensors[spec["weight"]]
        return self._hold(widen(k, raw) + np.float32(spec.get("gain_offset", 0.0)))

    def embedding(self, token: int) -> np.ndarray:
        out = np.empty(self.m.hidden, dtype=np.float32)
        lib.lsxo_embedding(C.byref(self.m), int(token), ptr(out))
        return out

    def decode(self, residual: np.ndarray, logits: bool = True):
        hidden = np.empty(self.m.hidden, dtype=np.float32)
        z = np.empty(self.m.vocab, dtype=np.float32) if logits else None
        r = f32(residual)
        lib.lsxo_decode(C.byref(self.m), self.cursor, ptr(r), ptr(hidden), ptr(z), self.threads)
        self.cursor += 1
        return hidden, z

    def advance(self, token: int):
        return self.decode(self.embedding(token))

    def head(self):
        k, shape, raw = self.tensors[self.graph["readout"]["weight"]]
        return k, raw

    def readout(self, hidden, edit=None) -> np.ndarray:
        """Model::readout with an optional f64 edit (SubspaceRotation/ReadoutRotation .apply)."""
        x = np.asarray(hidden, dtype=np.float64)
        if edit is not None:
            x = edit(x)
        k, raw = self.head()
        bias = self.graph["readout"].get("bias")
        b = widen(*self.tensors[bias][::2]) if bias else None
        return matvec(raw, k, x.astype(np.float32), b, self.m.vocab, self.m.hidden, self.threads)

    def generate(self, prompt, maximum: int, stop=()):
        """generate_frames (src/diagnosis.rs:106-149): tokens and frames."""
        self.cursor = 0
        frame = None
        for t in prompt:
            frame = self.advance(int(t))
        tokens, frames = [], []
        for position in range(maximum):
            tok = argmax(frame[1])
            tokens.append(tok)
            frames.append(frame)
            if tok in stop or position + 1 == maximum:
                break
            frame = self.advance(tok)
        return tokens, frames


__all__ = ["lib", "OracleModel", "readout_rows", "matvec", "norm", "rope", "attention", "gated", "combine",
           "plane_rotation", "plane_apply", "subspace_apply", "argmax", "other", "minimum_margin", "loss",
           "take_row", "read_checkpoint", "widen", "build"]


# ------------------------------------------------------------ FeasibleSet ---
class Feasible:
    """src/interval.rs:47-212 (the oracle's C restatement)."""

    def __init__(self, bound: float):
        self._s = FeasibleStruct()
        if lib.lsxo_feasible_init(C.byref(self._s), float(bound)) != 0:
            raise ValueError("the half-angle bound must lie in (0, 1e6]")

    def __del__(self):
        try:
            lib.lsxo_feasible_free(C.byref(self._s))
        except Exception:
            pass

    def constrain(self, a: float, b: float, c: float) -> None:
        if lib.lsxo_feasible_constrain(C.byref(self._s), float(a), float(b), float(c)) != 0:
            raise ValueError("finite quadratic coefficients are required")

    def is_empty(self) -> bool:
        return bool(lib.lsxo_feasible_is_empty(C.byref(self._s)))

    def nearest(self):
        t = C.c_double()
        return t.value if lib.lsxo_feasible_nearest(C.byref(self._s), C.byref(t)) else None

    def intervals(self) -> list[tuple[float, float]]:
        n = lib.lsxo_feasible_intervals(C.byref(self._s), None, 0)
        out = np.empty(2 * max(n, 1), dtype=np.float64)
        lib.lsxo_feasible_intervals(C.byref(self._s), ptr(out), n)
        return [(float(out[2 * i]), float(out[2 * i + 1])) for i in range(n)]

    def work(self) -> tuple[int, int, int, int]:
        return tuple(int(x) for x in self._s.work)

    def plane(self, wu, wv, logits, targets, hu, hv, margin: float, guard: float) -> None:
        """The constraint loop of src/diagnosis.rs:1118-1143 (sequential, on the host)."""
        wu, wv = f32(wu), f32(wv)
        z = f32(logits)
        t = np.ascontiguousarray(targets, dtype=np.uint32)
        hu = np.ascontiguousarray(hu, dtype=np.float64)
        hv = np.ascontiguousarray(hv, dtype=np.float64)
        if lib.lsxo_plane_feasible(C.byref(self._s), ptr(wu), ptr(wv), wu.size, ptr(z), ptr(t), ptr(hu), ptr(hv),
                                   t.size, float(margin), float(guard)) != 0:
            raise ValueError("finite quadratic coefficients are required")


# ------------------------------------------------------------ attribution ---
def restored_loss(z, row: int, original: float, target: int) -> float:
    z = f32(z)
    return float(lib.lsxo_restored_loss(ptr(z), z.size, int(row), float(original), int(target)))


def integrated_credits(before, after, targets, weights, panels: int, gradients: bool = False):
    """src/attribution.rs:79-123: (credits [vocab], integrals [points, vocab] or None)."""
    b, a = f32(before), f32(after)
    points, vocab = b.shape
    t = np.ascontiguousarray(targets, dtype=np.uint32)
    w = np.ascontiguousarray(weights, dtype=np.float64)
    credits = np.empty(vocab, dtype=np.float64)
    grads = np.empty((points, vocab), dtype=np.float64) if gradients else None
    lib.lsxo_integrated_credits(ptr(b), ptr(a), ptr(t), ptr(w), points, vocab, int(panels), ptr(credits),
                                ptr(grads))
    return credits, grads
