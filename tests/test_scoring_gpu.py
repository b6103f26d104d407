"""Teacher-forced case scoring (src/scaling.rs:181-216 with attribution::loss,
src/attribution.rs:49-60) through lsx_model_score on every decode plan, against
the oracle: per-position losses within tolerance, argmax identical except at
oracle near-ties, edited ("after") scores from the edited readout of the unedited
hidden state, and the case aggregation of scaling::evaluate."""
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN
from laplacesscissors_b200 import DeviceRotation, ReadoutRotation, diagnosis, synth

pytestmark = pytest.mark.gpu


def load(gpu, root, capacity, plan=None):
    keys = {"ops": ("LSX_DECODE_PLAN", "ops"), "graph": ("LSX_DECODE_ENGINE", "graph")}
    saved = {k: os.environ.get(k) for k in ("LSX_DECODE_PLAN", "LSX_DECODE_ENGINE")}
    if plan:
        os.environ[keys[plan][0]] = keys[plan][1]
    try:
        return lsx.Model.load(root, gpu, capacity)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def oracle_scores(oracle, root, prompt, targets, edit=None, capacity=64):
    ref = oracle.OracleModel(root, capacity)
    frame = None
    for t in prompt:
        frame = ref.advance(int(t))
    nll, amax = [], []
    for k, t in enumerate(targets):
        z = frame[1] if edit is None else ref.readout(frame[0], edit)
        nll.append(oracle.loss(z, int(t)))
        amax.append(oracle.argmax(z))
        if k + 1 < len(targets):
            frame = ref.advance(int(t))
    return np.array(nll), np.array(amax, dtype=np.uint32)


def check_argmax(got, want, oracle, root, prompt, targets):
    """Equal, except where the oracle's own top two are within 1e-3."""
    if np.array_equal(got, want):
        return
    ref = oracle.OracleModel(root, 64)
    frame = None
    for t in prompt:
        frame = ref.advance(int(t))
    for k, t in enumerate(targets):
        if got[k] != want[k]:
            z = frame[1]
            assert abs(oracle.minimum_margin(z, int(got[k]))) < 1e-3, (k, got[k], want[k])
        if k + 1 < len(targets):
            frame = ref.advance(int(t))


@pytest.mark.parametrize("plan", [None, "graph", "ops"])
def test_scores_match_oracle(gpu, oracle, plan):
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 32, plan)
    prompt, targets = [1, 2, 3], [5, 9, 200, 7, 7]
    nll, amax, frames = model.score(prompt, targets, frames=True)
    ref_nll, ref_amax = oracle_scores(oracle, root, prompt, targets)
    assert np.all(np.abs(nll - ref_nll) <= 1e-4 * (1 + np.abs(ref_nll))), (nll, ref_nll)
    check_argmax(amax, ref_amax, oracle, root, prompt, targets)
    assert model.position() == len(prompt) + len(targets) - 1
    # the frames are the teacher-forced path's: same as advancing by hand
    model.reset()
    hand = None
    for t in prompt:
        hand = model.advance(gpu, t)
    for k, t in enumerate(targets):
        np.testing.assert_allclose(frames[k].logits, hand.logits, rtol=1e-5, atol=1e-5)
        if k + 1 < len(targets):
            hand = model.advance(gpu, t)


def test_single_target_and_bad_arguments(gpu, oracle):
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 8)
    nll, amax, _ = model.score([4], [9])
    ref_nll, ref_amax = oracle_scores(oracle, root, [4], [9])
    assert abs(nll[0] - ref_nll[0]) <= 1e-4 * (1 + abs(ref_nll[0]))
    with pytest.raises(lsx.LsxError):
        model.score([1] * 6, [2] * 4)  # 6 + 4 - 1 > capacity 8
    with pytest.raises(lsx.LsxError):
        model.score([1], [model.vocab_size()])


def test_edited_scores_use_edited_readout(gpu, oracle, golden_tiny):
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 32)
    spec = ReadoutRotation(golden_tiny["plane_u"], golden_tiny["plane_v"], float(golden_tiny["plane_tangent"]))
    edit = DeviceRotation.upload(gpu, spec, model.hidden_size)
    prompt, targets = [7, 3], [11, 400, 2]
    nll, amax, frames = model.score(prompt, targets, edit, frames=True)
    ref_nll, ref_amax = oracle_scores(oracle, root, prompt, targets, edit=spec.apply)
    assert np.all(np.abs(nll - ref_nll) <= 1e-4 * (1 + np.abs(ref_nll))), (nll, ref_nll)
    plain_nll, _, plain = model.score(prompt, targets, frames=True)
    for a, b in zip(frames, plain):  # an edit changes logits, never the hidden state
        assert np.array_equal(a.hidden, b.hidden)


def test_evaluate_cases_aggregates_like_reference(gpu):
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 32)
    cases = [([1, 2, 3], [5, 9], 4), ([8], [1, 1, 2], 0)]
    ev = diagnosis.evaluate_cases(model, cases)
    nll0, amax0, _ = model.score(*cases[0][:2])
    nll1, amax1, _ = model.score(*cases[1][:2])
    want = nll0.sum() / (2 * 4) + nll1.sum() / (2 * 1)
    assert abs(ev.loss_before - want) <= 1e-12 * abs(want)
    assert ev.loss_after == ev.loss_before
    assert ev.correct_before == int(np.array_equal(amax0, [5, 9])) + int(np.array_equal(amax1, [1, 1, 2]))
    assert [c.target_tokens for c in ev.cases] == [[5, 9], [1, 1, 2]]


def test_qwen3_0_6b_case_scores(gpu, oracle):
    d = Path(tempfile.mkdtemp(prefix="lsx-score-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**dict(synth.QWEN3_0_6B, layers=2)), seed=5)
    model = lsx.Model.load(d, gpu, 64)
    assert model.info().persistent
    prompt = synth.prompt_tokens(5, 16, 151936)
    targets = synth.prompt_tokens(6, 6, 151936)
    nll, amax, _ = model.score(prompt, targets)
    ref_nll, ref_amax = oracle_scores(oracle, d, prompt, targets)
    assert np.all(np.abs(nll - ref_nll) <= 2e-2), (nll, ref_nll)
    check_argmax(amax, ref_amax, oracle, d, prompt, targets)
