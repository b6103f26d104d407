"""Batched greedy generation (lsx_model_generate_batch): several sequences decoded
together, each row's tokens equal to that prompt's own greedy generation by the
oracle (the reference decodes one sequence at a time, so a batch is that many
independent generations), except that a path may part at an oracle near-tie
(|margin| < 1e-3), the rule of the single-sequence decode tests."""
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN
from laplacesscissors_b200 import synth

pytestmark = pytest.mark.gpu


def check_rows(tokens, prompts, ref_model, oracle, maximum):
    for b, prompt in enumerate(prompts):
        ref_model.cursor = 0
        ref_tokens, ref_frames = ref_model.generate(prompt, maximum)
        for i, (t, rt) in enumerate(zip(tokens[b], ref_tokens)):
            if int(t) != rt:
                assert abs(oracle.minimum_margin(ref_frames[i][1], rt)) < 1e-3, (b, i, t, rt)
                break
        else:
            assert list(map(int, tokens[b])) == ref_tokens, b


def test_tiny_batch_matches_oracle(gpu, oracle):
    root = GOLDEN / "tiny_qwen3"
    model = lsx.Model.load(root, gpu, 32)
    prompts = np.stack([synth.prompt_tokens(20 + b, 9, 512) for b in range(5)])
    tokens = model.generate_batch(prompts, 7)
    assert tokens.shape == (5, 7)
    check_rows(tokens, prompts, oracle.OracleModel(root, 32), oracle, 7)


@pytest.mark.parametrize("shape,vocab", [("QWEN3_0_6B", 151936), ("QWEN3_4B", 8192)])
def test_wide_batch_matches_oracle(gpu, oracle, shape, vocab):
    d = Path(tempfile.mkdtemp(prefix=f"lsx-batch-{shape.lower()}-"))
    cfg = dict(getattr(synth, shape), layers=2, vocab=vocab)
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**cfg), seed=11)
    model = lsx.Model.load(d, gpu, 48)
    prompts = np.stack([synth.prompt_tokens(30 + b, 12, vocab) for b in range(4)])
    tokens = model.generate_batch(prompts, 6)
    check_rows(tokens, prompts, oracle.OracleModel(d, 48), oracle, 6)


# ---- long contexts: the attention walk's ring wraps and its splits end ragged ----

LONG_P, LONG_MAX = 653, 4  # an odd prompt length: no split ends on a 16-position walker boundary


@pytest.fixture(scope="module")
def long_case(oracle):
    """Qwen3-4B width (2 layers, vocab 8192), three 653-token prompts, and each
    prompt's greedy generation by the oracle."""
    d = synth.cached_checkpoint("QWEN3_4B", seed=13, layers=2, vocab=8192)
    prompts = np.stack([synth.prompt_tokens(40 + b, LONG_P, 8192) for b in range(3)])
    ref = oracle.OracleModel(d, LONG_P + LONG_MAX + 4)
    expected = []
    for prompt in prompts:
        ref.cursor = 0
        expected.append(ref.generate(prompt, LONG_MAX))
    return d, prompts, expected


@pytest.mark.parametrize("splits", [None, "2", "64"])
def test_long_context_batch_matches_oracle(gpu, oracle, long_case, monkeypatch, splits):
    """Batched generation after 653-token prompts against each prompt's own greedy
    generation by the oracle.  With 2 position splits every half-warp walker of
    cached_attention_part_kernel makes about 21 trips, so its 6-slot cp.async ring
    wraps three times and the splits end mid-walker; with 64 splits the last splits
    hold no position at all; the default split count sits between."""
    d, prompts, expected = long_case
    if splits is None:
        monkeypatch.delenv("LSX_BATCH_ATTENTION_SPLITS", raising=False)
    else:
        monkeypatch.setenv("LSX_BATCH_ATTENTION_SPLITS", splits)
    model = lsx.Model.load(d, gpu, LONG_P + LONG_MAX + 4)
    tokens = model.generate_batch(prompts, LONG_MAX)
    for b, (ref_tokens, ref_frames) in enumerate(expected):
        for i, (t, rt) in enumerate(zip(tokens[b], ref_tokens)):
            if int(t) != rt:
                assert abs(oracle.minimum_margin(ref_frames[i][1], rt)) < 1e-3, (splits, b, i, t, rt)
                break
        else:
            assert list(map(int, tokens[b])) == ref_tokens, (splits, b)
