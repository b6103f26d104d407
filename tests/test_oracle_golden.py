"""Pins the oracle (the checker of the CUDA path) to the reference.

Two kinds of evidence, both committed under tests/golden/:
  * the known-answer tests of the reference (tests/gpu.rs:19-264,
    src/rotation.rs:226-396) restated with their inputs, formulas and tolerances;
  * outputs of the reference's own kernels/ops.py executed by Triton's CPU
    interpreter (tests/golden/make_golden.py), including whole-model decodes.
"""
import math

import numpy as np
import pytest

from conftest import close


# ----------------------------------------------------- tests/gpu.rs KATs ----
def test_linear_and_embedding_kat(oracle, golden_kat):
    x = np.array(golden_kat["x"], np.float32)
    w = np.array(golden_kat["w"], np.float32)
    bias = np.array(golden_kat["bias"], np.float32)
    for kind, name in ((oracle.F32, "F32"), (oracle.F16, "F16"), (oracle.BF16, "BF16")):
        if kind == oracle.F32:
            stored, rounded = w, w
        elif kind == oracle.F16:
            stored = w.astype(np.float16).view(np.uint16)
            rounded = w.astype(np.float16).astype(np.float32)
        else:
            from laplacesscissors_b200.synth import bf16_to_f32, f32_to_bf16
            stored = f32_to_bf16(w)
            rounded = bf16_to_f32(stored)
        expected = rounded.astype(np.float64).reshape(3, 5) @ x.astype(np.float64) + bias  # tests/gpu.rs:47-58
        got = oracle.matvec(stored, kind, x, bias, 3, 5)
        close(got, expected, 2e-6)
        close(got, golden_kat[f"linear_{name}"], 2e-6)  # the reference kernel
        row = oracle.take_row(stored, kind, 2, 5)
        close(row, rounded[10:], 0.0)
        close(row, golden_kat[f"embedding_{name}"], 0.0)


def test_norm_kat(oracle, golden_kat):
    x = np.array(golden_kat["x"], np.float64)
    gain = np.array(golden_kat["gain"], np.float64)
    for center in (False, True):
        got = oracle.norm(x, gain, x, 1, 5, 1e-5, center)
        mean = x.mean() if center else 0.0
        var = ((x - mean) ** 2).mean()
        expected = (x - mean) / math.sqrt(var + 1e-5) * gain + x  # tests/gpu.rs:83-102
        close(got, expected, 2e-6)
        close(got, golden_kat[f"norm_center{int(center)}"], 2e-6)


def test_rope_kat(oracle, golden_kat):
    rin = np.array(golden_kat["rope_input"], np.float32)
    for inter in (False, True):
        got = oracle.rope(rin, 2, 6, 10000.0, 4, inter, 7)
        expected = rin.astype(np.float64).copy()
        for head in range(2):
            for pair in range(2):
                a, b = (head * 6 + 2 * pair, head * 6 + 2 * pair + 1) if inter else (head * 6 + pair,
                                                                                     head * 6 + pair + 2)
                phase = 7.0 / 10000.0 ** (pair / 2.0)
                s, c = math.sin(phase), math.cos(phase)
                expected[a] = rin[a] * c - rin[b] * s
                expected[b] = rin[b] * c + rin[a] * s
        close(got, expected, 4e-6)
        close(got, golden_kat[f"rope_interleaved{int(inter)}"], 4e-6)


def _erf_as(z):
    """The Abramowitz-Stegun form tests/gpu.rs:146-158 uses for its expectation."""
    sign = math.copysign(1.0, z)
    t = 1.0 / (1.0 + 0.3275911 * abs(z))
    return sign * (1 - (((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t
                        + 0.254829592) * t * math.exp(-z * z))


def test_gated_kat(oracle, golden_kat):
    x = np.array(golden_kat["x"], np.float32)
    for kind in range(4):
        got = oracle.gated(x, x, kind)
        exp = []
        for v in x.astype(np.float64):
            if kind == 0:
                a = v / (1 + math.exp(-v))
            elif kind == 1:
                a = 0.5 * v * (1 + _erf_as(v / math.sqrt(2)))
            elif kind == 2:
                a = max(v, 0.0)
            else:
                a = 0.5 * v * (1 + math.tanh(2 / math.sqrt(math.pi) / math.sqrt(2) * (v + 0.044715 * v ** 3)))
            exp.append(a * v)
        close(got, exp, 3e-6)
    close(oracle.gated(x, x, 0), golden_kat["gated_silu"], 3e-6)
    close(oracle.gated(x, x, 2), golden_kat["gated_relu"], 3e-6)


def test_combine_kat(oracle, golden_kat):
    x = np.array(golden_kat["x"], np.float32)
    got = oracle.combine(x, x, -0.25)
    close(got, x.astype(np.float64) * 0.75, 2e-7)
    assert np.array_equal(got, np.array(golden_kat["combine"], np.float32))  # same two roundings


def test_attention_kat(oracle, golden_kat):
    keys = np.array(golden_kat["attention_keys"], np.float32)
    values = np.array(golden_kat["attention_values"], np.float32)
    q = np.array(golden_kat["queries"], np.float32)
    for time in (0, 31, 34):
        got = oracle.attention(q, keys, values, time, 4, 2, 3, np.float32(0.7))
        exp = []
        for head in range(4):
            kv = head // 2
            sc = np.array([sum(float(q[head * 3 + d]) * float(keys[t * 6 + kv * 3 + d]) for d in range(3)) * 0.7
                           for t in range(time + 1)])
            wgt = np.exp(sc - sc.max())
            for d in range(3):
                exp.append(float((wgt * values[[t * 6 + kv * 3 + d for t in range(time + 1)]]).sum() / wgt.sum()))
        close(got, exp, 5e-6)
        close(got, golden_kat["attention"][str(time)], 5e-6)


def test_plane_rotation_kat(oracle, golden_kat):
    x = np.array(golden_kat["x"], np.float32)
    u, v, t = golden_kat["rotate_u"], golden_kat["rotate_v"], golden_kat["rotate_tangent"]
    a = -2 * t * t / (1 + t * t)
    b = 2 * t / (1 + t * t)
    got = oracle.plane_rotation(x, u, v, a, b)
    close(got, oracle.plane_apply(u, v, t, x), 2e-6)
    close(got, golden_kat["rotate"], 2e-6)


# --------------------------------------------- src/rotation.rs unit tests ----
def test_rotation_known_answer(oracle):
    """src/rotation.rs:312-329: t = 1/3 maps the repair and protected axes."""
    u, v = [1.0, 0, 0], [0, 1.0, 0]
    w = np.array([0.0, -1.0, 1.0])
    first = w @ oracle.plane_apply(u, v, 1 / 3, [1.0, 0, 0])
    second = w @ oracle.plane_apply(u, v, 1 / 3, [0, 1.0, 0])
    assert abs(first - 0.6) < 1e-12 and abs(second + 0.8) < 1e-12
    assert np.array_equal(oracle.plane_apply(u, v, 1 / 3, [0, 0, 1.0]), [0, 0, 1.0])


def test_rotation_preserves_row_gram(oracle):
    """src/rotation.rs:230-268: a finite plane rotation keeps every row Gram entry."""
    u, v, t = [0.6, 0.8, 0, 0], [0, 0, 1.0, 0], 0.73
    rows = np.array([[math.sin((r * 4 + c) / 3) for c in range(4)] for r in range(7)])
    cols = np.stack([oracle.plane_apply(u, v, t, np.eye(4)[j]) for j in range(4)])
    changed = rows @ cols.T
    assert np.max(np.abs(rows @ rows.T - changed @ changed.T)) < 2e-14
    p = np.array([-0.8, 0.6, 0, 2.0])
    assert np.max(np.abs(rows @ p - changed @ p)) < 2e-14


def test_subspace_apply_matches_plane(oracle):
    rng = np.random.default_rng(3)
    u = rng.standard_normal(9)
    u /= np.linalg.norm(u)
    v = rng.standard_normal(9)
    v -= (v @ u) * u
    v /= np.linalg.norm(v)
    t = 0.41
    a, b = -2 * t * t / (1 + t * t), 2 * t / (1 + t * t)
    h = rng.standard_normal(9)
    # ReadoutEdit::subspace (src/response.rs:240-251)
    got = oracle.subspace_apply(np.stack([u, v]), np.array([[1 + a, b], [-b, 1 + a]]), h)
    assert np.max(np.abs(got - oracle.plane_apply(u, v, t, h))) < 1e-13


def test_argmax_other_margin_rules(oracle):
    """src/diagnosis.rs:58-80: first maximum; competitor with lowest index on ties."""
    z = np.array([1.0, 3.0, 3.0, 2.0, 3.0], np.float32)
    assert oracle.argmax(z) == 1
    assert oracle.other(z, 1) == 2
    assert oracle.other(z, 0) == 1
    assert oracle.minimum_margin(z, 3) == -1.0
    assert oracle.minimum_margin(z, 1) == 0.0
    z = np.array([-1.0, -1.0], np.float32)
    assert oracle.other(z, 0) == 1 and oracle.other(z, 1) == 0


# ---------------------------------- reference kernels (Triton interpreter) ---
def test_matvec_random_against_reference_kernel(oracle, golden_random):
    for name in ("bf16", "f32", "f16", "bf16b"):
        kind, rows, cols = (int(v) for v in golden_random[f"mv_{name}_shape"])
        got = oracle.matvec(golden_random[f"mv_{name}_w"], kind, golden_random[f"mv_{name}_x"],
                            golden_random[f"mv_{name}_b"], rows, cols)
        close(got, golden_random[f"mv_{name}_y"], 2e-6)


def test_norm_rope_attention_random_against_reference_kernel(oracle, golden_random):
    g = golden_random
    close(oracle.norm(g["norm_x"], g["norm_g"], None, 3, 50, 1e-6, False), g["norm_rms"], 2e-6)
    close(oracle.norm(g["norm_x"], g["norm_g"], g["norm_b"], 3, 50, 1e-5, True), g["norm_layer"], 2e-6)
    for inter in (0, 1):
        for pos in (0, 41, 1000):
            # The reference forms the phase in f32 (kernels/ops.py:62): at position
            # 1000 its own rounding reaches ~1e-4 rad, so the tolerance widens with it.
            tol = 4e-6 if pos < 100 else 3e-4
            close(oracle.rope(g["rope_x"], 3, 10, 1e6, 6, inter, pos), g[f"rope_{inter}_{pos}"], tol)
    qh, kvh, dim = 6, 2, 16
    for t in (0, 17, 39):
        got = oracle.attention(g["att_q"], g["att_k"], g["att_v"], t, qh, kvh, dim, np.float32(1 / math.sqrt(dim)))
        close(got, g[f"att_out_{t}"], 5e-6)
    close(oracle.gated(g["gated_gate"], g["gated_up"], 0), g["gated_0"], 3e-6)
    close(oracle.gated(g["gated_gate"], g["gated_up"], 2), g["gated_2"], 3e-6)
    assert np.array_equal(oracle.combine(g["gated_gate"], g["combine_y"], 0.37), g["combine"])
    a, b = g["rot_ab"]
    close(oracle.plane_rotation(g["rot_h"], g["rot_u"], g["rot_v"], a, b), g["rot_out"], 2e-6)


def test_tiny_model_decode_against_reference(oracle, golden_tiny):
    """Greedy decode of tests/golden/tiny_qwen3 through the reference's ops vs the
    oracle: identical tokens, and logits within the whole-model rule of
    tests/qwen_reference.rs:266-273 (relative L2 < sqrt(eps_f32))."""
    from conftest import GOLDEN
    m = oracle.OracleModel(GOLDEN / "tiny_qwen3", capacity=32)
    tokens, frames = m.generate(golden_tiny["prompt"], 6)
    assert tokens == [int(t) for t in golden_tiny["tokens"]]
    for i, (h, z) in enumerate(frames):
        ref_z = golden_tiny["logits"][i]
        rel = np.linalg.norm(z.astype(np.float64) - ref_z) / np.linalg.norm(ref_z)
        assert rel < math.sqrt(np.finfo(np.float32).eps), (i, rel)
        close(h, golden_tiny["hidden"][i], 1e-4)


def test_tiny_model_edited_readouts_against_reference(oracle, golden_tiny):
    from conftest import GOLDEN
    m = oracle.OracleModel(GOLDEN / "tiny_qwen3", capacity=32)
    last = golden_tiny["hidden"][-1]
    u, v, t = golden_tiny["plane_u"], golden_tiny["plane_v"], float(golden_tiny["plane_tangent"])
    plane = m.readout(last, lambda h: oracle.plane_apply(u, v, t, h))
    close(plane, golden_tiny["plane_logits"], 2e-5)
    basis, R = golden_tiny["joint_basis"], golden_tiny["joint_transform"]
    joint = m.readout(last, lambda h: oracle.subspace_apply(basis, R, h))
    close(joint, golden_tiny["joint_logits"], 2e-5)


def test_rotation_fixture_against_reference(oracle, golden_rotation):
    """tests/model_rotation.rs fixture: the plane edit t = 1/3 repairs the path to
    [0, 1] and leaves the hidden state unchanged (tests/model_rotation.rs:267-272)."""
    from conftest import GOLDEN
    m = oracle.OracleModel(GOLDEN / "rotation_fixture", capacity=16)
    h, z = m.advance(2)
    close(h, golden_rotation["token2_hidden"], 1e-6)
    close(z, golden_rotation["token2_logits"], 1e-6)
    assert oracle.argmax(z) == 1  # the unedited path ends at once (EOS = 1)
    edit = lambda x: oracle.plane_apply([1.0, 0, 0, 0], [0, 1.0, 0, 0], 1 / 3, x)  # noqa: E731
    zr = m.readout(h, edit)
    close(zr, golden_rotation["rotated_logits"], 1e-6)
    assert oracle.argmax(zr) == 0
    h2, _ = m.advance(0)
    z2 = m.readout(h2, edit)
    close(z2, golden_rotation["next_logits"], 1e-6)
    assert oracle.argmax(z2) == 1  # tokens [0, 1]


def test_readout_rows_matches_rules(oracle):
    rng = np.random.default_rng(9)
    V, H, n = 301, 40, 13
    w = rng.standard_normal((V, H)).astype(np.float32)
    x = rng.standard_normal((n, H)).astype(np.float32)
    t = rng.integers(0, V, n).astype(np.uint32)
    margin, amax, tl = oracle.readout_rows(w, oracle.F32, None, V, H, x, t)
    for i in range(n):
        z = oracle.matvec(w, oracle.F32, x[i], None, V, H)
        assert amax[i] == oracle.argmax(z)
        assert margin[i] == oracle.minimum_margin(z, int(t[i]))
        assert tl[i] == z[t[i]]
