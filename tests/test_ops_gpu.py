"""Per-op parity of the CUDA kernels (the Gpu surface, src/gpu.rs:360-559)
against the reference's known answers (tests/gpu.rs:19-264), the reference
kernels' outputs and the oracle."""
import math

import numpy as np
import pytest

from conftest import close
from laplacesscissors_b200 import AttentionConfig, NormConfig, RopeConfig, synth
from laplacesscissors_b200._lib import BF16, F16, F32

pytestmark = pytest.mark.gpu


def test_linear_and_embedding_kat(gpu, golden_kat):
    """tests/gpu.rs:26-71 with the reference's tolerances."""
    x = np.array(golden_kat["x"], np.float32)
    w = np.array(golden_kat["w"], np.float32)
    bias = np.array(golden_kat["bias"], np.float32)
    xin, b = gpu.upload_f32(x), gpu.upload_f32(bias)
    for kind, name in ((F32, "F32"), (F16, "F16"), (BF16, "BF16")):
        if kind == F32:
            stored, rounded = w, w
        elif kind == F16:
            stored, rounded = w.astype(np.float16), w.astype(np.float16).astype(np.float32)
        else:
            stored = synth.f32_to_bf16(w)
            rounded = synth.bf16_to_f32(stored)
        weight = gpu.upload_raw(stored, kind)
        out = gpu.read(gpu.linear(xin, weight, b, 3, 5))
        close(out, rounded.astype(np.float64).reshape(3, 5) @ x.astype(np.float64) + bias, 2e-6)
        close(out, golden_kat[f"linear_{name}"], 2e-6)
        row = gpu.read(gpu.embedding(weight, 2, 5))
        close(row, rounded[10:], 0.0)


def test_norm_rope_gated_combine_kat(gpu, golden_kat, oracle):
    x = np.array(golden_kat["x"], np.float32)
    xin = gpu.upload_f32(x)
    gain = gpu.upload_f32(golden_kat["gain"])
    for center in (False, True):
        out = gpu.read(gpu.norm(xin, gain, xin, NormConfig(1, 5, 1e-5, center)))
        close(out, golden_kat[f"norm_center{int(center)}"], 2e-6)
        close(out, oracle.norm(x, golden_kat["gain"], x, 1, 5, 1e-5, center), 2e-6)
    rin = np.array(golden_kat["rope_input"], np.float32)
    r = gpu.upload_f32(rin)
    for inter in (False, True):
        out = gpu.read(gpu.rope(r, 7, RopeConfig(2, 6, 10000.0, 4, inter)))
        close(out, golden_kat[f"rope_interleaved{int(inter)}"], 4e-6)
        close(out, oracle.rope(rin, 2, 6, 10000.0, 4, inter, 7), 4e-6)
    for kind in range(4):
        out = gpu.read(gpu.gated(xin, xin, kind))
        close(out, oracle.gated(x, x, kind), 3e-6)
    close(gpu.read(gpu.gated(xin, xin, 0)), golden_kat["gated_silu"], 3e-6)
    out = gpu.read(gpu.combine(xin, xin, -0.25))
    assert np.array_equal(out, np.array(golden_kat["combine"], np.float32))  # same roundings as the reference


def test_attention_kat(gpu, golden_kat, oracle):
    """tests/gpu.rs:180-241: 35 appended positions, checked at 0, 31, 34."""
    keys, values = gpu.zeros(35 * 6), gpu.zeros(35 * 6)
    queries = np.array(golden_kat["queries"], np.float32)
    q = gpu.upload_f32(queries)
    all_k = np.array(golden_kat["attention_keys"], np.float32).reshape(35, 6)
    all_v = np.array(golden_kat["attention_values"], np.float32).reshape(35, 6)
    for time in range(35):
        out = gpu.read(gpu.attention(q, gpu.upload_f32(all_k[time]), gpu.upload_f32(all_v[time]), (keys, values),
                                     time, AttentionConfig(4, 2, 3, 0.7)))
        if time in (0, 31, 34):
            close(out, golden_kat["attention"][str(time)], 5e-6)
            close(out, oracle.attention(queries, all_k.reshape(-1), all_v.reshape(-1), time, 4, 2, 3,
                                        np.float32(0.7)), 5e-6)
    assert np.array_equal(gpu.read(keys), all_k.reshape(-1))  # cache_write (kernels/ops.py:69-73)


def test_rotate_kat(gpu, golden_kat, oracle):
    x = np.array(golden_kat["x"], np.float32)
    t = golden_kat["rotate_tangent"]
    a, b = -2 * t * t / (1 + t * t), 2 * t / (1 + t * t)
    out = gpu.read(gpu.rotate(gpu.upload_f32(x), gpu.upload_f32(golden_kat["rotate_u"]),
                              gpu.upload_f32(golden_kat["rotate_v"]), a, b))
    close(out, oracle.plane_apply(golden_kat["rotate_u"], golden_kat["rotate_v"], t, x), 2e-6)
    close(out, golden_kat["rotate"], 2e-6)


def test_random_ops_against_reference_kernels(gpu, golden_random):
    g = golden_random
    for name in ("bf16", "f32", "f16", "bf16b"):
        kind, rows, cols = (int(v) for v in g[f"mv_{name}_shape"])
        w = gpu.upload_raw(g[f"mv_{name}_w"], kind)
        out = gpu.read(gpu.linear(gpu.upload_f32(g[f"mv_{name}_x"]), w, gpu.upload_f32(g[f"mv_{name}_b"]), rows,
                                  cols))
        close(out, g[f"mv_{name}_y"], 2e-6)
    x = gpu.upload_f32(g["norm_x"])
    close(gpu.read(gpu.norm(x, gpu.upload_f32(g["norm_g"]), None, NormConfig(3, 50, 1e-6, False))), g["norm_rms"],
          2e-6)
    close(gpu.read(gpu.norm(x, gpu.upload_f32(g["norm_g"]), gpu.upload_f32(g["norm_b"]),
                            NormConfig(3, 50, 1e-5, True))), g["norm_layer"], 2e-6)
    r = gpu.upload_f32(g["rope_x"])
    for inter in (0, 1):
        for pos in (0, 41, 1000):
            tol = 4e-6 if pos < 100 else 3e-4  # the reference's own f32 phase error at 1000
            close(gpu.read(gpu.rope(r, pos, RopeConfig(3, 10, 1e6, 6, bool(inter)))), g[f"rope_{inter}_{pos}"], tol)
    qh, kvh, dim, n = 6, 2, 16, 40
    keys, values = gpu.zeros(n * kvh * dim), gpu.zeros(n * kvh * dim)
    q = gpu.upload_f32(g["att_q"])
    for t in range(n):
        sl = slice(t * kvh * dim, (t + 1) * kvh * dim)
        out = gpu.read(gpu.attention(q, gpu.upload_f32(g["att_k"][sl]), gpu.upload_f32(g["att_v"][sl]),
                                     (keys, values), t, AttentionConfig(qh, kvh, dim, 1 / math.sqrt(dim))))
        if t in (0, 17, 39):
            close(out, g[f"att_out_{t}"], 5e-6)
    gg, gu = gpu.upload_f32(g["gated_gate"]), gpu.upload_f32(g["gated_up"])
    close(gpu.read(gpu.gated(gg, gu, 0)), g["gated_0"], 3e-6)
    close(gpu.read(gpu.gated(gg, gu, 2)), g["gated_2"], 3e-6)
    assert np.array_equal(gpu.read(gpu.combine(gg, gpu.upload_f32(g["combine_y"]), 0.37)), g["combine"])
    a, b = g["rot_ab"]
    close(gpu.read(gpu.rotate(gpu.upload_f32(g["rot_h"]), gpu.upload_f32(g["rot_u"]), gpu.upload_f32(g["rot_v"]),
                              a, b)), g["rot_out"], 2e-6)


@pytest.mark.parametrize("rows,cols", [(2048, 1024), (6144, 1024), (1024, 3072), (151936, 1024), (12288, 4096)])
def test_gemv_shapes_against_oracle(gpu, oracle, rows, cols):
    """The GEMV microbench shapes: bf16 W N(0, 0.02), f32 x from bf16 N(0, 1)."""
    w = synth.normal_bf16(7, 0, rows * cols, 0.02)
    x = synth.bf16_to_f32(synth.normal_bf16(7, 1, cols, 1.0))
    out = gpu.read(gpu.linear(gpu.upload_f32(x), gpu.upload_raw(w, BF16), None, rows, cols))
    close(out, oracle.matvec(w, oracle.BF16, x, None, rows, cols), 2e-6 * math.sqrt(cols / 5))


def test_argument_checks(gpu):
    """The reference's ensure! rejections (src/gpu.rs:378-559) surface as errors."""
    from laplacesscissors_b200 import LsxError
    x = gpu.upload_f32(np.ones(5, np.float32))
    w = gpu.upload_f32(np.ones(15, np.float32))
    with pytest.raises(LsxError):
        gpu.linear(x, w, None, 4, 5)
    with pytest.raises(LsxError):
        gpu.embedding(w, 3, 5)
    with pytest.raises(LsxError):
        gpu.rope(x, 0, RopeConfig(1, 5, 1e4, 3, False))
    with pytest.raises(LsxError):
        gpu.norm(x, gpu.upload_f32(np.ones(4, np.float32)), None, NormConfig(1, 5, 1e-5, False))
    with pytest.raises(LsxError):
        gpu.gated(x, x, 4)
    with pytest.raises(LsxError):
        gpu.combine(x, x, float("inf"))
