"""Split attention of the persistent decode kernel (long contexts: each KV group's
positions spread over the CTAs in fixed blocks, per-head partial softmax states
merged by the head's CTA) against the oracle's attention (kernels/ops.py:69-101,
restated from tests/qwen_reference.rs:78-117): greedy tokens identical except at
oracle near-ties (|margin| < 1e-3), logits within 2e-2 abs / 1e-2 rel-L2.

LSX_DECODE_SPLIT_MIN sets the first position (+1) at which the kernel splits;
1 splits every step, so short cases cover the split path at every group ratio."""
import math
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN, close
from laplacesscissors_b200 import synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def load(gpu, root, capacity, split_min):
    saved = os.environ.get("LSX_DECODE_SPLIT_MIN")
    os.environ["LSX_DECODE_SPLIT_MIN"] = str(split_min)
    try:
        model = lsx.Model.load(root, gpu, capacity)
    finally:
        if saved is None:
            os.environ.pop("LSX_DECODE_SPLIT_MIN", None)
        else:
            os.environ["LSX_DECODE_SPLIT_MIN"] = saved
    assert model.fused and model.info().persistent
    return model


def check_against_oracle(oracle, root, capacity, prompt, tokens, frames, n):
    ref = oracle.OracleModel(root, capacity)
    ref_tokens, ref_frames = ref.generate(prompt, n)
    for i, (t, rt) in enumerate(zip(tokens, ref_tokens)):
        if int(t) != rt:
            assert abs(oracle.minimum_margin(ref_frames[i][1], rt)) < 1e-3, (i, t, rt)
            return
        assert rel_l2(frames[i].logits, ref_frames[i][1]) < 1e-2
        close(frames[i].logits, ref_frames[i][1], 2e-2)
        close(frames[i].hidden, ref_frames[i][0], 2e-2)
    assert list(map(int, tokens)) == ref_tokens


@pytest.mark.parametrize("split_min", [1, 7])
def test_tiny_split_matches_oracle(gpu, oracle, split_min):
    """Group ratio 2, head_dim 64, one KV group over 32 slots; split from the first
    step, and switching from per-head attention to the split mid-generation."""
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 64, split_min)
    prompt = synth.prompt_tokens(3, 12, 512)
    tokens, _, frames = model.generate(prompt, 24, frames=True)
    check_against_oracle(oracle, root, 64, prompt, tokens, frames, 24)


def small_long_checkpoint():
    """The tiny model's shape (hidden 128, 2/1 heads, head_dim 64) with room for
    long contexts."""
    d = Path(tempfile.mkdtemp(prefix="lsx-split-small-"))
    cfg = synth.qwen3_config(hidden=128, layers=2, heads=2, kv_heads=1, head_dim=64, intermediate=192, vocab=512,
                             max_positions=4096)
    return synth.make_qwen3_checkpoint(d, cfg, seed=4)


def test_long_context_split_matches_oracle(gpu, oracle):
    """A 600-token prompt at the default split threshold: positions past it are
    spread over the slots in blocks, several blocks per slot."""
    root = small_long_checkpoint()
    model = load(gpu, root, 640, 128)
    prompt = synth.prompt_tokens(4, 600, 512)
    tokens, _, frames = model.generate(prompt, 12, frames=True)
    check_against_oracle(oracle, root, 640, prompt, tokens, frames, 12)


def test_split_and_per_head_attention_agree(gpu):
    """The two attention paths of one model give the same greedy path and logits
    within float reassociation."""
    root = small_long_checkpoint()
    a = load(gpu, root, 160, 0)
    b = load(gpu, root, 160, 1)
    prompt = synth.prompt_tokens(5, 100, 512)
    ta, _, fa = a.generate(prompt, 16, frames=True)
    tb, _, fb = b.generate(prompt, 16, frames=True)
    assert list(ta) == list(tb)
    for x, y in zip(fa, fb):
        assert rel_l2(x.logits, y.logits) < 1e-5


@pytest.mark.parametrize("shape,ratio", [("QWEN3_0_6B", 2), ("QWEN3_4B", 4)])
def test_wide_split_matches_oracle(gpu, oracle, shape, ratio):
    """Qwen3-0.6B (ratio 2, register-resident x) and Qwen3-4B (ratio 4) widths with
    2 layers and an 8192-entry vocabulary; a 160-token prompt crosses the default
    threshold, then every step splits."""
    cfg = dict(getattr(synth, shape), layers=2, vocab=8192)
    assert cfg["heads"] // cfg["kv_heads"] == ratio
    d = Path(tempfile.mkdtemp(prefix=f"lsx-split-{shape.lower()}-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**cfg), seed=11)
    model = load(gpu, d, 192, 128)
    prompt = synth.prompt_tokens(11, 160, 8192)
    tokens, _, frames = model.generate(prompt, 8, frames=True)
    check_against_oracle(oracle, d, 192, prompt, tokens, frames, 8)


def test_batched_prefill_matches_token_by_token(gpu, oracle):
    """A prompt of 200 tokens is prefilled in one batched forward (tensor-core
    GEMMs filling the KV cache) before the decode engine continues; the generation
    matches the token-by-token prefill (LSX_PREFILL_MIN=0) and the oracle."""
    root = small_long_checkpoint()
    prompt = synth.prompt_tokens(8, 200, 512)
    saved = os.environ.get("LSX_PREFILL_MIN")
    try:
        os.environ["LSX_PREFILL_MIN"] = "0"
        slow = load(gpu, root, 256, 128)
        ts, _, fs = slow.generate(prompt, 10, frames=True)
        os.environ["LSX_PREFILL_MIN"] = "64"
        fast = load(gpu, root, 256, 128)
        tf, _, ff = fast.generate(prompt, 10, frames=True)
    finally:
        if saved is None:
            os.environ.pop("LSX_PREFILL_MIN", None)
        else:
            os.environ["LSX_PREFILL_MIN"] = saved
    assert fast.position() == slow.position() == 200 + 9
    check_against_oracle(oracle, root, 256, prompt, tf, ff, 10)
    n = next((i for i, (a, b) in enumerate(zip(ts, tf)) if a != b), len(ts))
    for i in range(n):
        assert rel_l2(ff[i].logits, fs[i].logits) < 1e-3
