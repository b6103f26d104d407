"""Batched head images and the fused compact readout.

Model.head_images (lsx_model_head_images) must give what head_image gives per
direction (src/model.rs:643-652) within the reference's linear tolerance
(tests/gpu.rs: 2e-6 (1 + |e|)), and agree with an f64 product of the bf16 head
and the f32 direction.  CompactReadout.evaluate_margins (lsx_compact_margin) must
give, per observation, minimum_margin / other / argmax (src/diagnosis.rs:58-80,
490-492) of the scores CompactReadout.evaluate computes (src/diagnosis.rs:643-665):
the competitor and argmax exactly except at near-ties (|margin| < 1e-3), the
margin within 1e-5 (1 + |m|)."""
import tempfile
from pathlib import Path

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN, close
from laplacesscissors_b200 import diagnosis, synth

pytestmark = pytest.mark.gpu


def directions(count, width, seed):
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((count, width))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


@pytest.fixture(scope="module")
def wide_model(gpu):
    d = Path(tempfile.mkdtemp(prefix="lsx-head-images-"))
    cfg = dict(synth.QWEN3_0_6B, layers=1)
    synth.make_qwen3_checkpoint(d, synth.qwen3_config(**cfg), seed=5)
    return lsx.Model.load(d, gpu, 8), d


@pytest.mark.parametrize("count", [1, 5, 40])
def test_head_images_match_head_image_tiny(gpu, count):
    model = lsx.Model.load(GOLDEN / "tiny_qwen3", gpu, 8)
    u = directions(count, model.hidden_size, 3 + count)
    batched = model.head_images(gpu, u)
    assert batched.shape == (count, model.vocab_size())
    for k in range(count):
        close(batched[k], model.head_image(gpu, u[k]), 2e-6)


def test_head_images_full_vocab(gpu, oracle, wide_model):
    model, root = wide_model
    H, V = model.hidden_size, model.vocab_size()
    u = directions(16, H, 11)
    batched = model.head_images(gpu, u)
    for k in (0, 7, 15):
        close(batched[k], model.head_image(gpu, u[k]), 2e-6)
    ref = oracle.OracleModel(root, 8)
    kind, raw = ref.head()
    w = oracle.widen(kind, raw).reshape(V, H).astype(np.float64)
    exact = w @ u.astype(np.float32).astype(np.float64).T  # [V, 16]
    close(batched.T, exact, 2e-6)


def reference_rules(scores, targets):
    m = np.array([diagnosis.minimum_margin(z, int(t)) for z, t in zip(scores, targets)])
    o = np.array([diagnosis.other(z, int(t)) for z, t in zip(scores, targets)], dtype=np.uint32)
    a = np.array([diagnosis.argmax(z) for z in scores], dtype=np.uint32)
    return m, o, a


def check_margins(got, ref):
    m, o, a = got
    m_ref, o_ref, a_ref = ref
    near = np.abs(m_ref) < 1e-3
    assert np.array_equal(o[~near], o_ref[~near]), np.nonzero(o != o_ref)[0][:8]
    assert np.array_equal(a[~near], a_ref[~near]), np.nonzero(a != a_ref)[0][:8]
    assert np.all(np.abs(m - m_ref) <= 1e-5 * (1 + np.abs(m_ref)))


@pytest.mark.parametrize("V,rank,n", [(512, 2, 3), (3001, 16, 37), (151936, 16, 20), (2053, 130, 9)])
def test_compact_margins_match_evaluate(gpu, V, rank, n):
    rng = np.random.default_rng(V + rank + n)
    images = [rng.standard_normal(V).astype(np.float32) * 0.3 for _ in range(rank)]
    baseline = [rng.standard_normal(V).astype(np.float32) * 3 for _ in range(n)]
    coordinates = [rng.standard_normal(rank) for _ in range(n)]
    targets = rng.integers(0, V, n).astype(np.uint32)
    compact = diagnosis.CompactReadout(gpu, images, baseline, coordinates)
    q, _ = np.linalg.qr(np.eye(rank) + 0.05 * rng.standard_normal((rank, rank)))
    deadline = diagnosis.Deadline(1e9)
    scores = compact.evaluate(gpu, q, deadline)
    ref = reference_rules(scores, targets)
    got = compact.evaluate_margins(gpu, q, targets, deadline)
    check_margins(got, ref)
    # a second call reuses the uploaded baselines
    check_margins(compact.evaluate_margins(gpu, q, targets, deadline), ref)


def test_compact_margin_ties(gpu):
    """Equal scores: other() takes the lowest index, argmax the first maximum."""
    V, rank, n = 700, 4, 4
    images = [np.zeros(V, np.float32) for _ in range(rank)]
    base = np.zeros(V, np.float32)
    base[[50, 20, 600]] = 5.0
    baseline = [base.copy() for _ in range(n)]
    coordinates = [np.zeros(rank) for _ in range(n)]
    targets = np.array([20, 50, 600, 3], dtype=np.uint32)
    compact = diagnosis.CompactReadout(gpu, images, baseline, coordinates)
    m, o, a = compact.evaluate_margins(gpu, np.eye(rank), targets)
    assert list(o) == [50, 20, 20, 20]
    assert list(a) == [20, 20, 20, 20]
    assert np.all(m[:3] == 0.0) and m[3] == -5.0
