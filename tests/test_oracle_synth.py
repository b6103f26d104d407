"""The oracle's input generator (oracle/synth.py, used by the CPU baseline and the
reference arms of bench.py) against the library's (laplacesscissors_b200.synth):
the same values and byte-identical checkpoint files, so both arms of the
benchmark measure the same inputs."""
import filecmp
import json
import tempfile
from pathlib import Path

import numpy as np

from laplacesscissors_b200 import synth
from oracle import synth as osynth


def test_generators_agree():
    for seed, stream, offset in ((7, 0, 0), (7, 5, 12345), (3, 1 << 32, 7)):
        assert np.array_equal(synth.normal_bf16(seed, stream, 4097, 0.02, offset),
                              osynth.normal_bf16(seed, stream, 4097, 0.02, offset))
        assert np.array_equal(synth.normal_f32(seed, stream, 1001, 1.0, offset),
                              osynth.normal_f32(seed, stream, 1001, 1.0, offset))
        assert np.array_equal(synth.uniform_u32(seed, stream, 999, 151936, offset),
                              osynth.uniform_u32(seed, stream, 999, 151936, offset))
    assert np.array_equal(synth.prompt_tokens(7, 24, 151936), osynth.prompt_tokens(7, 24, 151936))


def test_checkpoints_byte_identical():
    shape = dict(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, intermediate=96, vocab=300, tie=False)
    with tempfile.TemporaryDirectory() as t:
        a, b = Path(t) / "a", Path(t) / "b"
        synth.make_qwen3_checkpoint(a, synth.qwen3_config(**shape), seed=7)
        osynth.write_checkpoint(b, osynth.config(**shape), seed=7)
        assert filecmp.cmp(a / "model.safetensors", b / "model.safetensors", shallow=False)
        assert json.loads((a / "config.json").read_text()) == json.loads((b / "config.json").read_text())
