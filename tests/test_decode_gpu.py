"""Decode parity: Model::advance / generate_frames through the C ABI against the
reference's own kernels (golden) and the oracle, for the fused engine and the
per-op plan, plus the state contracts of tests/model_rotation.rs and
tests/injection.rs (hidden unchanged by an edit, KV rewind replays bit-identically,
token path == injected path)."""
import math
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN, close
from laplacesscissors_b200 import DeviceRotation, ReadoutRotation, SubspaceRotation, synth

pytestmark = pytest.mark.gpu

REL_L2 = math.sqrt(np.finfo(np.float32).eps)  # tests/qwen_reference.rs:266-273


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def load(gpu, root, capacity, plan=None):
    """plan: None (persistent engine), "graph" (PDL kernel chain) or "ops" (per-op kernels)."""
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


@pytest.mark.parametrize("plan", [None, "graph", "ops"])
def test_tiny_generate_matches_reference_kernels(gpu, golden_tiny, plan):
    model = load(gpu, GOLDEN / "tiny_qwen3", 32, plan)
    assert model.fused == (plan != "ops")
    assert bool(model.info().persistent) == (plan is None)
    tokens, stopped, frames = model.generate(golden_tiny["prompt"], 6, frames=True)
    assert list(map(int, tokens)) == list(map(int, golden_tiny["tokens"]))
    assert not stopped
    for i, f in enumerate(frames):
        assert rel_l2(f.logits, golden_tiny["logits"][i]) < REL_L2
        close(f.hidden, golden_tiny["hidden"][i], 1e-4)
    assert model.position() == len(golden_tiny["prompt"]) + 5


def test_tiny_advance_matches_generate_and_oracle(gpu, oracle, golden_tiny):
    model = load(gpu, GOLDEN / "tiny_qwen3", 32)
    ref = oracle.OracleModel(GOLDEN / "tiny_qwen3", 32)
    for t in golden_tiny["prompt"]:
        f = model.advance(gpu, int(t))
        h, z = ref.advance(int(t))
        assert rel_l2(f.logits, z) < REL_L2
        close(f.hidden, h, 1e-4)
    assert int(np.argmax(f.logits)) == int(golden_tiny["tokens"][0])


@pytest.mark.parametrize("engine", [None, "graph"])
def test_fused_and_per_op_plans_agree(gpu, engine):
    fused = load(gpu, GOLDEN / "tiny_qwen3", 32, engine)
    ops = load(gpu, GOLDEN / "tiny_qwen3", 32, "ops")
    for t in [3, 77, 500, 12, 9, 9, 1]:
        a = fused.advance(gpu, t)
        b = ops.advance(gpu, t)
        assert rel_l2(a.logits, b.logits) < 1e-5
        close(a.hidden, b.hidden, 1e-5)


def test_edits_leave_hidden_and_match_reference(gpu, golden_tiny):
    model = load(gpu, GOLDEN / "tiny_qwen3", 32)
    plane = ReadoutRotation(golden_tiny["plane_u"], golden_tiny["plane_v"], float(golden_tiny["plane_tangent"]))
    joint = SubspaceRotation(golden_tiny["joint_basis"], golden_tiny["joint_transform"])
    dp = DeviceRotation.upload(gpu, plane, model.hidden_size)
    dj = DeviceRotation.upload_edit(gpu, joint, model.hidden_size)
    last = golden_tiny["hidden"][-1]
    close(model.readout(gpu, last, dp), golden_tiny["plane_logits"], 2e-5)
    close(model.readout(gpu, last, dj), golden_tiny["joint_logits"], 2e-5)
    # tests/model_rotation.rs:267-272: an edit changes logits, never the hidden state.
    token = int(golden_tiny["prompt"][0])
    model.reset()
    original = model.advance(gpu, token)
    model.reset()
    edited = model.advance(gpu, token, dp)
    assert np.array_equal(original.hidden, edited.hidden)
    assert not np.array_equal(original.logits, edited.logits)
    close(edited.logits, model.readout(gpu, original.hidden, dp), 1e-5)
    model.reset()
    joint_step = model.advance(gpu, token, dj)
    assert np.array_equal(original.hidden, joint_step.hidden)
    close(joint_step.logits, model.readout(gpu, original.hidden, dj), 1e-5)


@pytest.mark.parametrize("engine", [None, "graph"])
def test_kv_rewind_replays_bit_identically(gpu, engine):
    """tests/model_rotation.rs:273-279."""
    model = load(gpu, GOLDEN / "tiny_qwen3", 16, engine)
    model.advance(gpu, 5)
    branch = model.advance(gpu, 7)
    model.rewind(1)
    replay = model.advance(gpu, 7)
    assert np.array_equal(branch.hidden, replay.hidden)
    assert np.array_equal(branch.logits, replay.logits)
    with pytest.raises(lsx.LsxError):
        model.rewind(9)
    with pytest.raises(lsx.LsxError):
        model.step(gpu, model.vocab_size(), None)


def test_context_capacity_is_enforced(gpu):
    model = load(gpu, GOLDEN / "tiny_qwen3", 4)
    for t in range(4):
        model.advance(gpu, t)
    with pytest.raises(lsx.LsxError):
        model.advance(gpu, 0)
    with pytest.raises(lsx.LsxError):
        lsx.Model.load(GOLDEN / "tiny_qwen3", gpu, 65)  # above max_position_embeddings


def test_token_path_equals_injected_path(gpu):
    """tests/injection.rs:115-124: feeding the embedding vector reproduces the token path bit-exactly."""
    for plan in (None, "graph", "ops"):
        model = load(gpu, GOLDEN / "tiny_qwen3", 16, plan)
        vec = model.embedding_vector(gpu, 42)
        a = model.advance(gpu, 42)
        model.reset()
        b = model.inject(gpu, vec)
        assert np.array_equal(a.hidden, b.hidden) and np.array_equal(a.logits, b.logits)


def test_rotation_fixture(gpu, golden_rotation):
    """tests/model_rotation.rs: f32 fixture (per-op plan) repaired by the plane t = 1/3."""
    model = load(gpu, GOLDEN / "rotation_fixture", 16)
    assert not model.fused
    f = model.advance(gpu, 2)
    close(f.logits, golden_rotation["token2_logits"], 1e-6)
    plane = DeviceRotation.upload(gpu, ReadoutRotation([1.0, 0, 0, 0], [0, 1.0, 0, 0], 1 / 3), 4)
    model.reset()
    r = model.advance(gpu, 2, plane)
    assert np.array_equal(f.hidden, r.hidden)
    close(r.logits, golden_rotation["rotated_logits"], 1e-6)
    tokens, stopped, _ = model.generate([2], 3, stop_tokens=[1], rotation=plane)
    assert list(tokens) == [0, 1] and stopped  # tests/model_rotation.rs:231-237
    tokens, stopped, _ = model.generate([2], 3, stop_tokens=[1])
    assert list(tokens) == [1] and stopped
    assert np.all(model.head_image(gpu, np.zeros(4)) == 0)  # tests/model_rotation.rs:298-299


def test_generate_stops_and_positions_like_reference(gpu, oracle):
    model = load(gpu, GOLDEN / "tiny_qwen3", 32)
    ref = oracle.OracleModel(GOLDEN / "tiny_qwen3", 32)
    prompt = [1, 2, 3]
    full, _ = ref.generate(prompt, 8)
    stop = [full[3]]
    ref_tokens, _ = ref.generate(prompt, 8, stop=stop)
    tokens, stopped, frames = model.generate(prompt, 8, stop_tokens=stop, frames=True)
    assert list(map(int, tokens)) == ref_tokens and stopped
    assert len(frames) == len(ref_tokens)
    assert model.position() == len(prompt) + len(ref_tokens) - 1


@pytest.fixture(scope="module")
def qwen06b_dir():
    d = Path(tempfile.mkdtemp(prefix="lsx-qwen06b-"))
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**synth.QWEN3_0_6B), seed=7)
    return d


def test_qwen3_0_6b_greedy_tokens_identical_to_oracle(gpu, oracle, qwen06b_dir):
    """The decode workload: Qwen3-0.6B architecture, random-init bf16, 24-token
    prompt, 32 greedy tokens; token-identical to the oracle's decode."""
    prompt = synth.prompt_tokens(7, 24, 151936)
    model = lsx.Model.load(qwen06b_dir, gpu, 64)
    assert model.fused and model.info().persistent
    tokens, _, frames = model.generate(prompt, 32, frames=True)
    ref = oracle.OracleModel(qwen06b_dir, 64)
    ref_tokens, ref_frames = ref.generate(prompt, 32)
    # Greedy paths may only part at a near-tie of the oracle's logits (|margin| < 1e-3).
    for i, (t, rt) in enumerate(zip(tokens, ref_tokens)):
        if int(t) != rt:
            z = ref_frames[i][1]
            assert abs(oracle.minimum_margin(z, rt)) < 1e-3, (i, t, rt)
            break
        assert rel_l2(frames[i].logits, ref_frames[i][1]) < 1e-2
        close(frames[i].logits, ref_frames[i][1], 2e-2)
    else:
        assert list(map(int, tokens)) == ref_tokens


def test_qwen3_0_6b_engines_agree(gpu, qwen06b_dir):
    """The persistent engine and the PDL kernel chain give the same greedy path."""
    prompt = synth.prompt_tokens(7, 24, 151936)
    a = load(gpu, qwen06b_dir, 64)
    b = load(gpu, qwen06b_dir, 64, "graph")
    ta, _, fa = a.generate(prompt, 8, frames=True)
    tb, _, fb = b.generate(prompt, 8, frames=True)
    assert list(ta) == list(tb)
    for x, y in zip(fa, fb):
        assert rel_l2(x.logits, y.logits) < 1e-5


def test_qwen3_0_6b_weight_stream_depth_changes_no_bits(gpu, qwen06b_dir):
    """How many weight chunks the persistent kernel keeps in flight during the layers
    (two by default at this width, LSX_DECODE_INFLIGHT_LAYERS) only changes when the
    weights arrive, never what is computed: tokens, hidden states and logits are the
    same bits with one, two and six chunks."""
    prompt = synth.prompt_tokens(7, 24, 151936)
    runs = []
    saved = os.environ.get("LSX_DECODE_INFLIGHT_LAYERS")
    try:
        for depth in ("1", "2", "6"):
            os.environ["LSX_DECODE_INFLIGHT_LAYERS"] = depth
            model = lsx.Model.load(qwen06b_dir, gpu, 64)
            assert model.info().persistent
            runs.append(model.generate(prompt, 6, frames=True))
            del model
    finally:
        if saved is None:
            os.environ.pop("LSX_DECODE_INFLIGHT_LAYERS", None)
        else:
            os.environ["LSX_DECODE_INFLIGHT_LAYERS"] = saved
    t0, _, f0 = runs[0]
    for t, _, f in runs[1:]:
        assert list(map(int, t)) == list(map(int, t0))
        for a, b in zip(f, f0):
            assert np.array_equal(a.hidden, b.hidden) and np.array_equal(a.logits, b.logits)
