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


def check_argmax(got, want, oracle, root, prompt, targets, capacity=64):
    """Equal, except where the oracle's own top two are within 1e-3."""
    if np.array_equal(got, want):
        return
    ref = oracle.OracleModel(root, capacity)
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


# ---- batched teacher forcing (lsx_model_score_batch) ----------------------------

def batch_cases(seed, cases, P, n, vocab):
    prompts = np.stack([synth.uniform_u32(seed, 100 + c, P, vocab) for c in range(cases)])
    targets = np.stack([synth.uniform_u32(seed, 900 + c, n, vocab) for c in range(cases)])
    return prompts, targets


def test_batched_scores_match_oracle_tiny(gpu, oracle):
    """Every case of the batch against the oracle's token-by-token scoring: losses
    within 1e-3 (the f32 activations enter the GEMMs as two bf16 terms), argmax
    equal except at oracle near-ties."""
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 32)
    prompts, targets = batch_cases(3, 5, 7, 4, 512)
    nll, amax, margin, lg = model.score_batch(prompts, targets, logits=True)
    for c in range(len(prompts)):
        ref_nll, ref_amax = oracle_scores(oracle, root, prompts[c], targets[c])
        assert np.all(np.abs(nll[c] - ref_nll) <= 1e-3 * (1 + np.abs(ref_nll))), (c, nll[c], ref_nll)
        check_argmax(amax[c], ref_amax, oracle, root, prompts[c], targets[c])
        # the logits are the frames of the sequential path; margins follow
        # minimum_margin (src/diagnosis.rs:490-492) of those logits
        _, _, frames = model.score(prompts[c], targets[c], frames=True)
        for k in range(targets.shape[1]):
            np.testing.assert_allclose(lg[c, k], frames[k].logits, rtol=2e-3, atol=2e-3)
            want = oracle.minimum_margin(lg[c, k], int(targets[c, k]))
            assert abs(margin[c, k] - want) <= 1e-9 * (1 + abs(want))


def test_batched_single_case_single_target_and_checks(gpu, oracle):
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 8)
    nll, amax, _, _ = model.score_batch([[4]], [[9]])
    ref_nll, ref_amax = oracle_scores(oracle, root, [4], [9])
    assert abs(nll[0, 0] - ref_nll[0]) <= 1e-3 * (1 + abs(ref_nll[0]))
    model.reset()
    before = model.position()
    model.score_batch([[1, 2, 3]], [[4, 5]])
    assert model.position() == before  # the decode state is untouched
    with pytest.raises(lsx.LsxError):
        model.score_batch([[1] * 6], [[2] * 4])  # 6 + 4 - 1 > capacity 8
    with pytest.raises(lsx.LsxError):
        model.score_batch([[1]], [[model.vocab_size()]])


@pytest.mark.parametrize("shape,vocab", [("QWEN3_0_6B", 151936), ("QWEN3_8B", 8192)])
def test_batched_scores_wide_shapes(gpu, oracle, shape, vocab):
    """Qwen3-0.6B and Qwen3-8B widths (2 layers): several cases of a 64-token prompt
    and 9 targets, against the sequential path and the oracle on every case (losses
    within 2e-2, the decode tolerance)."""
    d = Path(tempfile.mkdtemp(prefix=f"lsx-batch-{shape.lower()}-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**dict(getattr(synth, shape), layers=2, vocab=vocab)), seed=6)
    model = lsx.Model.load(d, gpu, 80)
    prompts, targets = batch_cases(6, 3, 64, 9, vocab)
    nll, amax, _, _ = model.score_batch(prompts, targets)
    for c in range(len(prompts)):
        seq_nll, seq_amax, _ = model.score(prompts[c], targets[c])
        assert np.all(np.abs(nll[c] - seq_nll) <= 2e-2), (c, nll[c], seq_nll)
    for c in range(len(prompts)):
        ref_nll, ref_amax = oracle_scores(oracle, d, prompts[c], targets[c], capacity=80)
        assert np.all(np.abs(nll[c] - ref_nll) <= 2e-2), (c, nll[c], ref_nll)
        check_argmax(amax[c], ref_amax, oracle, d, prompts[c], targets[c], capacity=80)


def test_gated_epilogue_equals_two_kernel_form(gpu):
    """The gate/up GEMM writing act(gate) * up as the down GEMM's bf16 planes from
    its epilogue, against the two-kernel form (the f32 gate/up product, then
    gated_planes_kernel; LSX_GEMM_GATED=0): the batched losses, argmaxes, margins and
    logits are the same bits.  216 rows, so the CTA-pair GEMMs carry the epilogue."""
    vocab = 8192
    d = Path(tempfile.mkdtemp(prefix="lsx-gated-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**dict(synth.QWEN3_0_6B, layers=2, vocab=vocab)), seed=8)
    model = lsx.Model.load(d, gpu, 80)
    prompts, targets = batch_cases(8, 3, 64, 9, vocab)
    fused = model.score_batch(prompts, targets, logits=True)
    saved = os.environ.get("LSX_GEMM_GATED")
    os.environ["LSX_GEMM_GATED"] = "0"
    try:
        plain = model.score_batch(prompts, targets, logits=True)
    finally:
        if saved is None:
            os.environ.pop("LSX_GEMM_GATED", None)
        else:
            os.environ["LSX_GEMM_GATED"] = saved
    for a, b in zip(fused, plain):
        assert np.array_equal(a, b)


def test_per_case_attention_equals_query_tile_blocks(gpu):
    """Short cases' attention with one block per (case, KV group) staging all keys
    once, against one block per 16-query tile (LSX_ATTENTION_PER_CASE=0): the same
    per-tile arithmetic, so the batched results are the same bits."""
    vocab = 8192
    d = Path(tempfile.mkdtemp(prefix="lsx-attcase-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**dict(synth.QWEN3_8B, layers=2, vocab=vocab)), seed=9)
    model = lsx.Model.load(d, gpu, 80)
    prompts, targets = batch_cases(9, 3, 64, 9, vocab)
    per_case = model.score_batch(prompts, targets, logits=True)
    saved = os.environ.get("LSX_ATTENTION_PER_CASE")
    os.environ["LSX_ATTENTION_PER_CASE"] = "0"
    try:
        tiles = model.score_batch(prompts, targets, logits=True)
    finally:
        if saved is None:
            os.environ.pop("LSX_ATTENTION_PER_CASE", None)
        else:
            os.environ["LSX_ATTENTION_PER_CASE"] = saved
    for a, b in zip(per_case, tiles):
        assert np.array_equal(a, b)


def test_batched_edited_scores_match_sequential(gpu, golden_tiny):
    """The "after" pass (src/scaling.rs:199-203): the edited readout of the
    unedited hidden states, batched, against lsx_model_score with the same plane
    and joint edits."""
    root = GOLDEN / "tiny_qwen3"
    model = load(gpu, root, 32)
    prompts, targets = batch_cases(4, 3, 6, 3, 512)
    plane = DeviceRotation.upload(gpu, ReadoutRotation(golden_tiny["plane_u"], golden_tiny["plane_v"],
                                                       float(golden_tiny["plane_tangent"])), model.hidden_size)
    rng = np.random.default_rng(2)
    basis, _ = np.linalg.qr(rng.standard_normal((model.hidden_size, 4)))
    q, _ = np.linalg.qr(rng.standard_normal((4, 4)))
    if np.linalg.det(q) < 0:
        q[:, 0] *= -1
    joint = DeviceRotation.upload_edit(gpu, lsx.SubspaceRotation(basis.T.copy(), q), model.hidden_size)
    for edit in (plane, joint):
        nll, amax, margin, _ = model.score_batch(prompts, targets, rotation=edit)
        plain, _, _, _ = model.score_batch(prompts, targets)
        assert not np.allclose(nll, plain)
        for c in range(len(prompts)):
            seq_nll, seq_amax, _ = model.score(prompts[c], targets[c], edit)
            assert np.all(np.abs(nll[c] - seq_nll) <= 1e-3 * (1 + np.abs(seq_nll))), (c, nll[c], seq_nll)
