"""Decode parity at the other measured model widths: Qwen3-4B
(hidden 2560, 32/8 heads, I 9728, tied) and Qwen3-8B (hidden 4096, I 12288,
untied head) shapes with 2 layers, through the persistent engine, against the
oracle: greedy tokens identical except at oracle near-ties (|margin| < 1e-3),
logits within 2e-2 abs / 1e-2 relative-L2."""
import math
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import close
from laplacesscissors_b200 import synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("shape,vocab", [("QWEN3_4B", 151936), ("QWEN3_8B", 8192)])
def test_wide_shapes_match_oracle(gpu, oracle, shape, vocab):
    d = Path(tempfile.mkdtemp(prefix=f"lsx-{shape.lower()}-"))
    cfg = dict(getattr(synth, shape), layers=2, vocab=vocab)
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**cfg), seed=9)
    model = lsx.Model.load(d, gpu, 32)
    assert model.fused and model.info().persistent
    prompt = synth.prompt_tokens(9, 8, vocab)
    tokens, _, frames = model.generate(prompt, 6, frames=True)
    ref = oracle.OracleModel(d, 32)
    ref_tokens, ref_frames = ref.generate(prompt, 6)
    for i, (t, rt) in enumerate(zip(tokens, ref_tokens)):
        if int(t) != rt:
            assert abs(oracle.minimum_margin(ref_frames[i][1], rt)) < 1e-3, (i, t, rt)
            break
        assert rel_l2(frames[i].logits, ref_frames[i][1]) < 1e-2
        close(frames[i].logits, ref_frames[i][1], 2e-2)
        close(frames[i].hidden, ref_frames[i][0], 2e-2)
    else:
        assert list(map(int, tokens)) == ref_tokens


def test_full_depth_qwen3_4b_matches_oracle(gpu, oracle):
    """All 36 layers of the Qwen3-4B architecture (hidden 2560, 32/8 heads, I 9728,
    vocab 151936, tied; random init, seed 7 — the long-context decode workload's
    checkpoint) through the persistent engine: a 4-token prompt and 4 greedy
    tokens, the first two steps' tokens, logits and hidden states against the
    oracle."""
    d = synth.cached_checkpoint("QWEN3_4B")
    model = lsx.Model.load(d, gpu, 16)
    assert model.fused and model.info().persistent
    prompt = synth.prompt_tokens(7, 4, 151936)
    tokens, _, frames = model.generate(prompt, 4, frames=True)
    ref_tokens, ref_frames = oracle.OracleModel(d, 16).generate(prompt, 2)
    for i, rt in enumerate(ref_tokens):
        if int(tokens[i]) != rt:
            assert abs(oracle.minimum_margin(ref_frames[i][1], rt)) < 1e-3, (i, tokens[i], rt)
            break
        assert rel_l2(frames[i].logits, ref_frames[i][1]) < 1e-2
        close(frames[i].logits, ref_frames[i][1], 2e-2)
        close(frames[i].hidden, ref_frames[i][0], 2e-2)
