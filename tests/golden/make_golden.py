"""Generates the golden vectors in tests/golden/ from the reference itself.

Runs ONLY in a container that has the reference tree, named by the required
environment variable LSX_REFERENCE (the folder holding the reference's
kernels/ops.py, src/ and tests/): it imports the reference's unmodified
kernels/ops.py and executes its Triton kernels with Triton's CPU interpreter
(TRITON_INTERPRET=1), launched with the constexprs and grids of src/gpu.rs:360-559
and, for whole-model cases, in the op order of Model::decode (src/model.rs:729-853).

Outputs (committed):
  ops_kat.json        the known-answer inputs of tests/gpu.rs:19-264 and the
                      reference kernels' outputs for them
  ops_random.npz      seeded random cases for every op at odd shapes
  tiny_qwen3/         a small random-init Qwen3-layout checkpoint (bf16)
  tiny_decode.npz     greedy decode of tiny_qwen3 through the reference's ops:
                      per-step tokens, hidden states and logits, plus plane and
                      joint-edit readouts of the last hidden state
  rotation_fixture/   the 4-wide f32 fixture of tests/model_rotation.rs:19-82
  rotation_decode.npz its decode through the reference's ops

libdevice erf/tanh (GELU kinds 1 and 3) cannot run in the interpreter; those two
activations are pinned by the reference's own KAT formulas instead.
"""
from __future__ import annotations

import json
import math
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("LSX_REFERENCE"):
    sys.exit("make_golden.py: set LSX_REFERENCE to the reference tree (the folder holding kernels/ops.py)")
REFERENCE = Path(os.environ["LSX_REFERENCE"])
sys.path.insert(0, str(REFERENCE / "kernels"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import ops  # noqa: E402  (the reference's kernels/ops.py)

from laplacesscissors_b200 import synth  # noqa: E402  (only to write the fixture checkpoint)


def cdiv(a, b):
    return (a + b - 1) // b


def p2(n):
    return 1 << (int(n) - 1).bit_length()


def f32(x):
    return float(np.float32(x))


def t32(a):
    return torch.tensor(np.asarray(a, dtype=np.float32))


# ---- Gpu methods of src/gpu.rs, each launching the reference kernel as gpu.rs does.
def take_row(weight: torch.Tensor, row: int, width: int) -> torch.Tensor:
    out = torch.zeros(width, dtype=torch.float32)
    ops.take_row[(cdiv(width, 256),)](weight, out, row, WIDTH=width, TILE=256)
    return out


def linear(x, w, bias, rows, cols):
    out = torch.zeros(rows, dtype=torch.float32)
    ops.matvec[(cdiv(rows, 8),)](w, x, bias if bias is not None else x, out, ROWS=rows, COLS=cols,
                                 BIAS=bias is not None, TILE_R=8, TILE_C=256)
    return out


def norm(x, gain, bias, groups, width, eps, center):
    out = torch.zeros(groups * width, dtype=torch.float32)
    ops.normalization[(groups,)](x, gain, bias if bias is not None else gain, out, WIDTH=width, EPSILON=f32(eps),
                                 CENTER=bool(center), BIAS=bias is not None, TILE=p2(width))
    return out


def rope(x, position, heads, dim, theta, rotary, interleaved):
    n = heads * dim
    out = torch.zeros(n, dtype=torch.float32)
    ops.rotary_position[(cdiv(n, 256),)](x, out, position, HEAD_DIM=dim, WIDTH=n, ROTARY=rotary, BASE=f32(theta),
                                         INTERLEAVED=bool(interleaved), TILE=256)
    return out


def attention(q, k, v, keys, values, position, qheads, kvheads, dim, scale):
    width = kvheads * dim
    ops.cache_write[(cdiv(width, 256),)](k, v, keys, values, position, WIDTH=width, TILE=256)
    out = torch.zeros(qheads * dim, dtype=torch.float32)
    ops.causal_attention[(qheads,)](q, keys, values, out, position, Q_HEADS=qheads, KV_HEADS=kvheads, DIM=dim,
                                    SCALE=f32(scale), TILE_T=32, TILE_D=p2(dim))
    return out


def gated(gate, up, kind):
    out = torch.zeros(len(gate), dtype=torch.float32)
    ops.gated_product[(cdiv(len(gate), 256),)](gate, up, out, WIDTH=len(gate), KIND=kind, TILE=256)
    return out


def combine(x, y, factor):
    out = torch.zeros(len(x), dtype=torch.float32)
    ops.vector_sum[(cdiv(len(x), 256),)](x, y, out, f32(factor), WIDTH=len(x), TILE=256)
    return out


def rotate(h, u, v, a, b):
    out = torch.zeros(len(h), dtype=torch.float32)
    ops.plane_rotation[(1,)](h, u, v, out, f32(a), f32(b), WIDTH=len(h), TILE=p2(len(h)))
    return out


def arr(t):
    return t.detach().cpu().numpy().astype(np.float32)


# ---------------------------------------------------------------- KATs ------
def kat_cases() -> dict:
    """tests/gpu.rs:19-264 inputs and the reference kernels' outputs."""
    x = [0.25, -2.0, 1.5, 0.75, -0.3]
    w = [(i - 7.0) / 9.0 for i in range(15)]
    bias = [0.3, -0.4, 0.5]
    out = {"x": x, "w": w, "bias": bias}
    xt = t32(x)
    for kind, name in ((0, "F32"), (1, "F16"), (2, "BF16")):
        if kind == 0:
            wt = t32(w)
        elif kind == 1:
            wt = torch.tensor(w, dtype=torch.float32).to(torch.float16)
        else:
            wt = torch.tensor(w, dtype=torch.float32).to(torch.bfloat16)
        out[f"linear_{name}"] = arr(linear(xt, wt, t32(bias), 3, 5)).tolist()
        out[f"embedding_{name}"] = arr(take_row(wt, 2, 5)).tolist()
    gain = [1.0, 0.5, 1.2, 0.8, 1.5]
    out["gain"] = gain
    for center in (False, True):
        out[f"norm_center{int(center)}"] = arr(norm(xt, t32(gain), xt, 1, 5, 1e-5, center)).tolist()
    rin = [i / 7.0 - 1.0 for i in range(12)]
    out["rope_input"] = rin
    for inter in (False, True):
        out[f"rope_interleaved{int(inter)}"] = arr(rope(t32(rin), 7, 2, 6, 10000.0, 4, inter)).tolist()
    out["gated_silu"] = arr(gated(xt, xt, 0)).tolist()
    out["gated_relu"] = arr(gated(xt, xt, 2)).tolist()
    out["combine"] = arr(combine(xt, xt, -0.25)).tolist()
    keys = torch.zeros(35 * 6)
    values = torch.zeros(35 * 6)
    queries = [i / 11.0 - 0.4 for i in range(12)]
    out["queries"] = queries
    att = {}
    for time in range(35):
        k = [float(np.float32(np.sin(np.float32((time * 6 + d) / np.float32(13.0))))) for d in range(6)]
        v = [float(np.float32(np.cos(np.float32((time * 6 + d) / np.float32(17.0))))) for d in range(6)]
        res = attention(t32(queries), t32(k), t32(v), keys, values, time, 4, 2, 3, 0.7)
        if time in (0, 31, 34):
            att[str(time)] = arr(res).tolist()
    out["attention_keys"] = arr(keys).tolist()
    out["attention_values"] = arr(values).tolist()
    out["attention"] = att
    u = [0.6, 0.8, 0.0, 0.0, 0.0]
    vv = [0.0, 0.0, 1.0, 0.0, 0.0]
    t = -0.37
    a, b = -2 * t * t / (1 + t * t), 2 * t / (1 + t * t)
    out["rotate_u"], out["rotate_v"], out["rotate_tangent"] = u, vv, t
    out["rotate"] = arr(rotate(xt, t32(u), t32(vv), a, b)).tolist()
    return out


# --------------------------------------------------------- random cases -----
def random_cases() -> dict:
    rng = np.random.default_rng(20261201)
    out = {}
    for kind, name, rows, cols in ((2, "bf16", 37, 300), (0, "f32", 19, 77), (1, "f16", 13, 264), (2, "bf16b", 64, 1024)):
        w = rng.standard_normal(rows * cols).astype(np.float32) * 0.05
        x = rng.standard_normal(cols).astype(np.float32)
        bias = rng.standard_normal(rows).astype(np.float32)
        wt = torch.tensor(w)
        if kind == 1:
            wt = wt.to(torch.float16)
            stored = wt.numpy().view(np.uint16)
        elif kind == 2:
            wt = wt.to(torch.bfloat16)
            stored = wt.view(torch.int16).numpy().view(np.uint16)
        else:
            stored = w
        out[f"mv_{name}_w"] = stored
        out[f"mv_{name}_x"] = x
        out[f"mv_{name}_b"] = bias
        out[f"mv_{name}_y"] = arr(linear(t32(x), wt, t32(bias), rows, cols))
        out[f"mv_{name}_shape"] = np.array([kind, rows, cols])
    x = rng.standard_normal(3 * 50).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(50)).astype(np.float32)
    bb = rng.standard_normal(50).astype(np.float32)
    out["norm_x"], out["norm_g"], out["norm_b"] = x, g, bb
    out["norm_rms"] = arr(norm(t32(x), t32(g), None, 3, 50, 1e-6, False))
    out["norm_layer"] = arr(norm(t32(x), t32(g), t32(bb), 3, 50, 1e-5, True))
    x = rng.standard_normal(3 * 10).astype(np.float32)
    out["rope_x"] = x
    for inter in (0, 1):
        for pos in (0, 41, 1000):
            out[f"rope_{inter}_{pos}"] = arr(rope(t32(x), pos, 3, 10, 1e6, 6, inter))
    qh, kvh, dim, n = 6, 2, 16, 40
    q = rng.standard_normal(qh * dim).astype(np.float32)
    ks = rng.standard_normal(n * kvh * dim).astype(np.float32)
    vs = rng.standard_normal(n * kvh * dim).astype(np.float32)
    out["att_q"], out["att_k"], out["att_v"] = q, ks, vs
    keys = torch.zeros(n * kvh * dim)
    values = torch.zeros(n * kvh * dim)
    for t in range(n):
        res = attention(t32(q), t32(ks[t * kvh * dim:(t + 1) * kvh * dim]), t32(vs[t * kvh * dim:(t + 1) * kvh * dim]),
                        keys, values, t, qh, kvh, dim, 1 / math.sqrt(dim))
        if t in (0, 17, 39):
            out[f"att_out_{t}"] = arr(res)
    gx = (3 * rng.standard_normal(300)).astype(np.float32)
    gu = rng.standard_normal(300).astype(np.float32)
    out["gated_gate"], out["gated_up"] = gx, gu
    out["gated_0"] = arr(gated(t32(gx), t32(gu), 0))
    out["gated_2"] = arr(gated(t32(gx), t32(gu), 2))
    y = rng.standard_normal(300).astype(np.float32)
    out["combine_y"] = y
    out["combine"] = arr(combine(t32(gx), t32(y), 0.37))
    h = rng.standard_normal(130).astype(np.float32)
    u = rng.standard_normal(130)
    u /= np.linalg.norm(u)
    v = rng.standard_normal(130)
    v -= (v @ u) * u
    v /= np.linalg.norm(v)
    out["rot_h"], out["rot_u"], out["rot_v"] = h, u, v
    tan = 0.21
    a, b = -2 * tan * tan / (1 + tan * tan), 2 * tan / (1 + tan * tan)
    out["rot_ab"] = np.array([a, b])
    out["rot_out"] = arr(rotate(t32(h), t32(u), t32(v), a, b))
    return out


# -------------------------------------------------------------- decoders ----
class RefModel:
    """Model::load + Model::decode (src/model.rs:411-853) over the reference ops."""

    def __init__(self, tensors: dict, graph: dict, capacity: int):
        self.t = tensors
        self.g = graph
        self.capacity = capacity
        self.cursor = 0
        self.blocks = graph["blocks"]
        self.cache = []
        for b in self.blocks:
            a = b["attention"]
            n = capacity * a["kv_heads"] * a["head_dim"]
            self.cache.append((torch.zeros(n), torch.zeros(n)))

    def tensor(self, name):
        return self.t[name]

    def gain(self, spec):
        return t32(self.t[spec["weight"]].float().numpy() + spec.get("gain_offset", 0.0))

    def run_norm(self, spec, x, groups, width):
        bias = self.t[spec["bias"]].float() if spec.get("bias") else None
        return norm(x, self.gain(spec), bias, groups, width, spec["epsilon"], spec["kind"] == "layer")

    def run_linear(self, spec, x, rows, cols, with_bias=True):
        bias = self.t[spec["bias"]].float() if (with_bias and spec.get("bias")) else None
        return linear(x, self.t[spec["weight"]], bias, rows, cols)

    def embedding(self, token):
        row = take_row(self.t[self.g["embedding"]], token, self.g["hidden_size"])
        s = self.g.get("embedding_scale", 1.0)
        return row if s == 1.0 else combine(row, row, s - 1.0)

    def decode(self, residual, rotation=None):
        H = self.g["hidden_size"]
        for b, (keys, values) in zip(self.blocks, self.cache):
            a = b["attention"]
            qh, kvh, hd = a["query_heads"], a["kv_heads"], a["head_dim"]
            nrm = self.run_norm(b["input_norm"], residual, 1, H)
            q = self.run_linear(a["query"], nrm, qh * hd, H)
            k = self.run_linear(a["key"], nrm, kvh * hd, H)
            v = self.run_linear(a["value"], nrm, kvh * hd, H)
            if a.get("query_norm"):
                q = self.run_norm(a["query_norm"], q, qh, hd)
            if a.get("key_norm"):
                k = self.run_norm(a["key_norm"], k, kvh, hd)
            if a["rotary_dim"] > 0:
                q = rope(q, self.cursor, qh, hd, a["rope_theta"], a["rotary_dim"], a.get("rotary_interleaved", False))
                k = rope(k, self.cursor, kvh, hd, a["rope_theta"], a["rotary_dim"], a.get("rotary_interleaved", False))
            mixed = attention(q, k, v, keys, values, self.cursor, qh, kvh, hd, a["score_scale"])
            proj = self.run_linear(a["output"], mixed, H, qh * hd)
            residual = combine(residual, proj, 1.0)
            nrm = self.run_norm(b["post_attention_norm"], residual, 1, H)
            m = b["mlp"]
            I = m["intermediate_size"]
            gate = self.run_linear(m["gate"], nrm, I, H)
            up = self.run_linear(m["up"], nrm, I, H)
            feat = gated(gate, up, {"silu": 0, "gelu": 1, "relu": 2, "gelu_tanh": 3}[m["activation"]])
            down = self.run_linear(m["down"], feat, H, I)
            residual = combine(residual, down, 1.0)
        hidden = self.run_norm(self.g["final_norm"], residual, 1, H)
        x = rotation(hidden) if rotation else hidden
        logits = self.run_linear(self.g["readout"], x, self.g["vocab_size"], H)
        self.cursor += 1
        return arr(hidden), arr(logits)

    def readout(self, hidden, rotation=None):
        x = t32(hidden)
        if rotation:
            x = rotation(x)
        return arr(self.run_linear(self.g["readout"], x, self.g["vocab_size"], self.g["hidden_size"]))


def load_tensors(path: Path) -> dict:
    out = {}
    for name, (dtype, shape, raw) in synth.read_safetensors(path).items():
        a = np.array(raw)
        if dtype == "BF16":
            out[name] = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).reshape(-1)
        elif dtype == "F16":
            out[name] = torch.from_numpy(a.copy()).reshape(-1)
        else:
            out[name] = torch.from_numpy(a.astype(np.float32).copy()).reshape(-1)
    return out


def qwen_graph(c: dict) -> dict:
    """GraphSpec::from_config (src/graph.rs:231-411) for a Qwen3-layout config."""
    eps = c["rms_norm_eps"]
    hd = c["head_dim"]
    rms = lambda n: {"weight": n + ".weight", "kind": "rms", "epsilon": eps}  # noqa: E731
    lin = lambda n: {"weight": n + ".weight"}  # noqa: E731
    blocks = []
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}"
        blocks.append({
            "input_norm": rms(f"{p}.input_layernorm"), "post_attention_norm": rms(f"{p}.post_attention_layernorm"),
            "attention": {"query": lin(f"{p}.self_attn.q_proj"), "key": lin(f"{p}.self_attn.k_proj"),
                          "value": lin(f"{p}.self_attn.v_proj"), "output": lin(f"{p}.self_attn.o_proj"),
                          "query_norm": rms(f"{p}.self_attn.q_norm"), "key_norm": rms(f"{p}.self_attn.k_norm"),
                          "query_heads": c["num_attention_heads"], "kv_heads": c["num_key_value_heads"],
                          "head_dim": hd, "rotary_dim": hd, "rope_theta": c["rope_theta"],
                          "score_scale": f32(1.0 / math.sqrt(np.float32(hd)))},
            "mlp": {"gate": lin(f"{p}.mlp.gate_proj"), "up": lin(f"{p}.mlp.up_proj"),
                    "down": lin(f"{p}.mlp.down_proj"), "intermediate_size": c["intermediate_size"],
                    "activation": "silu"}})
    return {"hidden_size": c["hidden_size"], "vocab_size": c["vocab_size"], "embedding": "model.embed_tokens.weight",
            "final_norm": rms("model.norm"),
            "readout": {"weight": "model.embed_tokens.weight" if c["tie_word_embeddings"] else "lm_head.weight"},
            "blocks": blocks}


def plane_fn(u, v, tangent):
    a, b = -2 * tangent * tangent / (1 + tangent * tangent), 2 * tangent / (1 + tangent * tangent)
    return lambda h: rotate(h, t32(u), t32(v), a, b)


def joint_fn(basis, transform):
    """DeviceRotation::apply Joint (src/model.rs:350-361): three matvecs and a combine."""
    r, w = basis.shape
    bt = t32(basis.reshape(-1))
    tr = t32(basis.T.reshape(-1))
    de = t32((transform - np.eye(r)).reshape(-1))

    def apply(h):
        coords = linear(h, bt, None, r, w)
        shift = linear(coords, de, None, r, r)
        lifted = linear(shift, tr, None, w, r)
        return combine(h, lifted, 1.0)
    return apply


def tiny_decode(out_dir: Path) -> dict:
    config = synth.qwen3_config(hidden=128, layers=2, heads=2, kv_heads=1, head_dim=64, intermediate=192, vocab=512,
                                tie=True, theta=1e6, eps=1e-6, max_positions=64)
    root = synth.make_qwen3_checkpoint(out_dir / "tiny_qwen3", config, seed=11, std=0.15, gain_std=0.1)
    model = RefModel(load_tensors(root / "model.safetensors"), qwen_graph(config), 32)
    prompt = [int(t) for t in synth.prompt_tokens(11, 5, config["vocab_size"])]
    hiddens, logits, tokens = [], [], []
    frame = None
    for tok in prompt:  # prefill (src/diagnosis.rs:81-99)
        frame = model.decode(model.embedding(tok))
    for i in range(6):  # greedy (src/diagnosis.rs:122-145)
        tok = int(np.argmax(frame[1]))
        tokens.append(tok)
        hiddens.append(frame[0])
        logits.append(frame[1])
        if i == 5:
            break
        frame = model.decode(model.embedding(tok))
    rng = np.random.default_rng(5)
    width = config["hidden_size"]
    u = rng.standard_normal(width)
    u /= np.linalg.norm(u)
    v = rng.standard_normal(width)
    v -= (v @ u) * u
    v /= np.linalg.norm(v)
    q, _ = np.linalg.qr(rng.standard_normal((width, 4)))
    basis = q.T.copy()
    th = 0.3
    R = np.eye(4)
    R[0, 0] = R[1, 1] = math.cos(th)
    R[0, 1], R[1, 0] = -math.sin(th), math.sin(th)
    R2 = np.eye(4)
    R2[2, 2] = R2[3, 3] = math.cos(0.2)
    R2[2, 3], R2[3, 2] = -math.sin(0.2), math.sin(0.2)
    R = R2 @ R
    last = hiddens[-1]
    return {
        "prompt": np.array(prompt, dtype=np.uint32), "tokens": np.array(tokens, dtype=np.uint32),
        "hidden": np.stack(hiddens), "logits": np.stack(logits),
        "plane_u": u, "plane_v": v, "plane_tangent": np.array(0.4),
        "plane_logits": model.readout(last, plane_fn(u, v, 0.4)),
        "joint_basis": basis, "joint_transform": R,
        "joint_logits": model.readout(last, joint_fn(basis, R)),
    }


def rotation_fixture(out_dir: Path) -> dict:
    """tests/model_rotation.rs:19-82 fixture with head bias -0.2, tied=False."""
    root = out_dir / "rotation_fixture"
    root.mkdir(parents=True, exist_ok=True)
    t = {
        "embed": np.array([0, 0, -1, 0, 0, 0, 0, 1, 1, 0, 0, 0, 0, 0, 1, 0, 0, 1, 0, 0, 0, 0, 0, 1],
                          dtype=np.float32).reshape(6, 4),
        "head": np.array([0, -1, 1, 0] + [0] * 20, dtype=np.float32).reshape(6, 4),
        "bias": np.array([-0.2, 0, -10, -10, -10, -10], dtype=np.float32),
        "norm": np.full(4, np.sqrt(np.float32(0.25) + np.float32(1e-5)), dtype=np.float32),
    }
    for name, rows, cols in (("q", 4, 4), ("k", 2, 4), ("v", 2, 4), ("o", 4, 4), ("gate", 3, 4), ("up", 3, 4),
                             ("down", 4, 3)):
        t[name] = np.zeros((rows, cols), dtype=np.float32)
    synth.write_safetensors(root / "model.safetensors", t)
    norm_spec = {"weight": "norm", "kind": "rms", "epsilon": 1e-5}
    lin = lambda n: {"weight": n}  # noqa: E731
    graph = {"version": 1, "source": "regression_fixture", "hidden_size": 4, "vocab_size": 6, "max_context": 16,
             "embedding": "embed", "final_norm": norm_spec, "readout": {"weight": "head", "bias": "bias"},
             "blocks": [{"input_norm": norm_spec, "post_attention_norm": norm_spec,
                         "attention": {"query": lin("q"), "key": lin("k"), "value": lin("v"), "output": lin("o"),
                                       "query_heads": 2, "kv_heads": 1, "head_dim": 2, "rotary_dim": 2,
                                       "rope_theta": 10000.0, "score_scale": 0.70710677},
                         "mlp": {"gate": lin("gate"), "up": lin("up"), "down": lin("down"), "intermediate_size": 3,
                                 "activation": "silu"}}],
             "eos_token_ids": [1]}
    (root / "laplace.graph.json").write_text(json.dumps(graph))
    (root / "config.json").write_text('{"eos_token_id":1}')
    model = RefModel(load_tensors(root / "model.safetensors"), graph, 16)
    h0, z0 = model.decode(model.embedding(2))
    model.cursor = 0
    plane = plane_fn([1, 0, 0, 0], [0, 1, 0, 0], 1.0 / 3.0)
    h1, z1 = model.decode(model.embedding(2), plane)
    h2, z2 = model.decode(model.embedding(0), plane)
    return {"token2_hidden": h0, "token2_logits": z0, "rotated_hidden": h1, "rotated_logits": z1,
            "next_hidden": h2, "next_logits": z2}


def main() -> None:
    HERE.mkdir(parents=True, exist_ok=True)
    (HERE / "ops_kat.json").write_text(json.dumps(kat_cases(), indent=0))
    np.savez_compressed(HERE / "ops_random.npz", **random_cases())
    np.savez_compressed(HERE / "tiny_decode.npz", **tiny_decode(HERE))
    np.savez_compressed(HERE / "rotation_decode.npz", **rotation_fixture(HERE))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
