"""FeasibleSet (src/interval.rs:47-212) on the host: the product's C++ set
(lsx_feasible_*) and the oracle's C restatement both reproduce the reference's
own interval tests (src/interval.rs:214-264) exactly, and agree bit for bit
(intervals, nearest tangent, work counters) on seeded random constraint streams
that exercise screening, linear and degenerate constraints, double roots,
boundary holes and emptiness.  No GPU."""
import math

import numpy as np
import pytest

from laplacesscissors_b200.feasible import FeasibleSet


def both(bound):
    from oracle import binding
    return FeasibleSet(bound), binding.Feasible(bound)


def apply(sets, a, b, c):
    for s in sets:
        s.constrain(a, b, c)


def test_reference_touching_open_intervals():
    # src/interval.rs:216-242
    for f in both(3.0):
        f.constrain(1.0, 0.0, -2.0)
        f.constrain(-1.0, 0.0, 2.0)
        r2 = math.sqrt(2.0)
        assert f.intervals() == [(-r2, -r2), (r2, r2)]
        assert f.nearest() == -r2
    for d in both(1.0):
        d.constrain(-9000.0, 600.0, -10.0)
        assert d.nearest() == 1.0 / 30.0
        d.constrain(0.0, 1.0, -0.1)
        assert d.is_empty()


def test_reference_boundary_holes_and_screening():
    # src/interval.rs:243-263
    for f in both(1.0):
        f.constrain(1.0, 0.0, -1.0)
        assert f.intervals() == [(-1.0, -1.0), (1.0, 1.0)]
        f.constrain(0.0, 1.0, 0.0)
        assert f.nearest() == 1.0
        f.constrain(1.0, 0.0, 1.0)
        assert f.work()[1] == 1
        f.constrain(0.0, -1.0, 0.5)
        assert f.is_empty()


def test_rejects_non_finite_and_bad_bounds():
    from laplacesscissors_b200._lib import LsxError
    f = FeasibleSet(1.0)
    with pytest.raises(LsxError):
        f.constrain(math.nan, 0.0, 1.0)
    with pytest.raises(LsxError):
        FeasibleSet(0.0)
    with pytest.raises(LsxError):
        FeasibleSet(2e6)


def stream(rng, n):
    """Constraints of the kinds the plane search produces, plus degenerate ones."""
    out = []
    for _ in range(n):
        kind = rng.integers(0, 10)
        if kind == 0:
            out.append((0.0, 0.0, float(rng.choice([-1.0, 0.0, 1.0]))))
        elif kind == 1:
            out.append((0.0, float(rng.normal()), float(rng.normal())))
        elif kind == 2:  # exact double root: b^2 = 4ac with powers of two
            e = float(2.0 ** rng.integers(-3, 4))
            r = float(rng.integers(-8, 9)) / 16.0
            a = -e if rng.integers(0, 2) else e
            out.append((a, -2.0 * a * r, a * r * r))
        elif kind == 3:
            out.append((0.0, 0.0, 0.0))
        else:
            s = 10.0 ** rng.uniform(-6, 6)
            c = float(rng.normal()) * 0.2 + 0.05
            out.append((float(rng.normal()) * s * 0.1, float(rng.normal()) * s, c * s))
    return out


@pytest.mark.parametrize("seed", range(12))
def test_product_equals_oracle_on_random_streams(seed):
    rng = np.random.default_rng(seed)
    bound = float(rng.choice([0.05, 0.3, 1.0, 7.0]))
    prod, orc = both(bound)
    for a, b, c in stream(rng, 400):
        apply((prod, orc), a, b, c)
        assert prod.is_empty() == orc.is_empty()
        if prod.is_empty():
            break
    assert prod.intervals() == orc.intervals()
    assert prod.nearest() == orc.nearest()
    assert prod.work() == orc.work()
