"""The C-ABI library loads and exports every entry point include/lsx.h declares,
and its host-only entry points (synthetic inputs) behave as documented.  No GPU."""
import ctypes as C
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "lsx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lsx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import laplacesscissors_b200 as lsx
    lib = C.CDLL(lsx.library_path())
    names = declared_functions()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    from laplacesscissors_b200 import _lib
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_version_and_error_channel():
    from laplacesscissors_b200._lib import lib
    assert lib.lsx_version().startswith(b"liblsx")
    ctx = C.c_void_p()
    status = lib.lsx_ctx_create(0, None)  # NULL output pointer is rejected before touching CUDA
    assert status == 1
    assert b"NULL" in lib.lsx_last_error()


def test_synth_normal_matches_restatement():
    """lsx_synth_normal against an independent numpy restatement of its generator."""
    from laplacesscissors_b200 import synth
    M = (1 << 64) - 1

    def mix(z):
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    seed, stream, golden = 7, 5, 0x9E3779B97F4A7C15
    key = mix(seed ^ mix((stream + golden) & M))
    bits = lambda i: mix((key + (i + 1) * golden) & M)  # noqa: E731
    vals = []
    for i in range(64):
        p = i >> 1
        u1 = ((bits(2 * p) >> 11) + 1) * 2.0 ** -53
        u2 = (bits(2 * p + 1) >> 11) * 2.0 ** -53
        r = np.sqrt(-2 * np.log(u1))
        vals.append(0.02 * (r * np.sin(2 * np.pi * u2) if i & 1 else r * np.cos(2 * np.pi * u2)))
    expect = synth.f32_to_bf16(np.array(vals, dtype=np.float64).astype(np.float32))
    got = synth.normal_bf16(seed, stream, 64, 0.02)
    # libm vs numpy transcendental results may differ in the last f64 bit; that moves
    # a bf16 rounding only at an exact tie, so allow at most one ulp on rare elements.
    diff = np.abs(got.astype(np.int32) - expect.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).sum() <= 1
    # Slices are position-addressable.
    assert np.array_equal(synth.normal_bf16(seed, stream, 16, 0.02, offset=32), got[32:48])
    u = synth.uniform_u32(seed, stream, 1000, 151936)
    assert u.max() < 151936 and len(set(u.tolist())) > 990


def test_safetensors_roundtrip(tmp_path):
    from laplacesscissors_b200 import synth
    cfg = synth.qwen3_config(hidden=32, layers=1, heads=2, kv_heads=1, head_dim=16, intermediate=48, vocab=50)
    synth.make_qwen3_checkpoint(tmp_path, cfg, seed=3)
    t = synth.read_safetensors(tmp_path / "model.safetensors")
    shapes = synth.qwen3_tensor_shapes(cfg)
    assert set(t) == set(shapes)
    for n, (dtype, shape, raw) in t.items():
        assert dtype == "BF16" and shape == shapes[n]
    gain = synth.bf16_to_f32(t["model.norm.weight"][2])
    assert np.all(gain == 1.0)
    w = synth.bf16_to_f32(t["model.embed_tokens.weight"][2])
    assert 0.015 < w.std() < 0.025
