"""Attribution on the GPU (lsx_integrated_credits) against the oracle's
sequential restatement of src/attribution.rs:49-123: credits and integrals
within 1e-9 (1 + |e|) (the same f64 arithmetic with reassociated vocabulary
sums), losses and restored losses within 1e-12 (1 + |e|); the reference's own
attribution test (src/attribution.rs:246-263) through the GPU path; and analyze's
panel doubling and ranking against the oracle-driven computation."""
import numpy as np
import pytest

from laplacesscissors_b200 import attribution
from laplacesscissors_b200.attribution import LossPoint

pytestmark = pytest.mark.gpu


def near(a, e, tol):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    assert a.shape == e.shape
    assert np.all(np.abs(a - e) <= tol * (1 + np.abs(e))), np.max(np.abs(a - e) / (1 + np.abs(e)))


def test_reference_attribution_example(gpu, oracle):
    """src/attribution.rs:246-263: credits sum to the finite loss change."""
    before = np.array([[3.0, -1.0, 0.0]], np.float32)
    after = np.array([[0.0, 2.0, 1.0]], np.float32)
    c, _, losses = attribution.integrated_credits(gpu, before, after, [1], [1.0], 128, rows=[1])
    expected = oracle.loss(before[0], 1) - oracle.loss(after[0], 1)
    assert abs(c.sum() - expected) < 1e-8
    assert c[2] < 0
    assert abs(losses[0, 2] - oracle.loss(np.array([0.0, -1.0, 1.0], np.float32), 1)) < 1e-14
    assert abs(losses[0, 0] - oracle.loss(before[0], 1)) < 1e-14


@pytest.mark.parametrize("V,P,panels", [(517, 3, 16), (5000, 7, 64), (151936, 2, 16)])
def test_credits_match_oracle(gpu, oracle, V, P, panels):
    rng = np.random.default_rng(V + P)
    before = (rng.standard_normal((P, V)) * 3).astype(np.float32)
    after = (before + rng.standard_normal((P, V)).astype(np.float32) * 0.5).astype(np.float32)
    targets = rng.integers(0, V, P).astype(np.uint32)
    weights = rng.random(P)
    rows = [int(targets[0]), 0, V - 1, V // 2]
    c, g, losses = attribution.integrated_credits(gpu, before, after, targets, weights, panels, rows=rows)
    c_ref, g_ref = oracle.integrated_credits(before, after, targets, weights, panels, gradients=True)
    near(c, c_ref, 1e-9)
    near(g, g_ref[:, rows], 1e-9)
    for p in range(P):
        assert abs(losses[p, 0] - oracle.loss(before[p], int(targets[p]))) <= 1e-12 * (1 + abs(losses[p, 0]))
        assert abs(losses[p, 1] - oracle.loss(after[p], int(targets[p]))) <= 1e-12 * (1 + abs(losses[p, 1]))
        for i, r in enumerate(rows):
            ref = oracle.restored_loss(after[p], r, before[p, r], int(targets[p]))
            assert abs(losses[p, 2 + i] - ref) <= 1e-12 * (1 + abs(ref))


def test_analyze_doubles_panels_and_ranks_rows(gpu, oracle):
    rng = np.random.default_rng(5)
    V, P, H = 3001, 4, 64
    pts = []
    for p in range(P):
        b = (rng.standard_normal(V) * 2).astype(np.float32)
        a = (b + rng.standard_normal(V).astype(np.float32) * 2.0).astype(np.float32)
        pts.append(LossPoint(b, rng.standard_normal(H).astype(np.float32), a, int(rng.integers(0, V)), 1.0 / P))
    result = attribution.analyze(gpu, pts, 5, 1e-12, "test")
    # the oracle, driven by the same doubling rule
    before = np.stack([p.before_logits for p in pts])
    after = np.stack([p.after for p in pts])
    t = [p.target for p in pts]
    w = [p.weight for p in pts]
    expected = sum(wi * (oracle.loss(before[i], t[i]) - oracle.loss(after[i], t[i])) for i, wi in enumerate(w))
    panels = 16
    while True:
        c_ref, _ = oracle.integrated_credits(before, after, t, w, panels)
        if abs(c_ref.sum() - expected) <= 1e-12 * (1 + abs(expected)) or panels >= 256:
            break
        panels *= 2
    assert result.panels == panels
    order = sorted(range(V), key=lambda j: (-abs(c_ref[j]), j))[:5]
    assert [r.row for r in result.leading_rows] == order
    near([r.credit for r in result.leading_rows], c_ref[order], 1e-9)
    assert abs(result.credit_sum - c_ref.sum()) <= 1e-9 * (1 + abs(c_ref.sum()))
