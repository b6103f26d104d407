"""The plane search's constraint loop (src/diagnosis.rs:1118-1143) with every
(point, vocabulary entry) constraint formed and screened on the GPU
(lsx_plane_feasible) against the oracle's sequential host loop: the feasible
intervals, the nearest tangent and the work counters (constraints, screened,
square roots, inserted intervals) must be identical, including runs whose hull
moves many times and runs that end empty."""
import math

import numpy as np
import pytest

from laplacesscissors_b200.feasible import FeasibleSet, plane_constraints

pytestmark = pytest.mark.gpu


def inputs(V, P, seed, spread=0.5):
    rng = np.random.default_rng(seed)
    wu = rng.standard_normal(V).astype(np.float32)
    wv = rng.standard_normal(V).astype(np.float32)
    z = (rng.standard_normal((P, V)) * 3).astype(np.float32)
    t = rng.integers(0, V, P).astype(np.uint32)
    for p in range(P):  # the target near the top, so a few competitors bind
        z[p, t[p]] = np.float32(z[p].max() + rng.uniform(-spread, spread))
    hu = rng.standard_normal(P) * 3
    hv = rng.standard_normal(P) * 3
    return wu, wv, z, t, hu, hv


def run_both(gpu, args, margin, guard, angle):
    from oracle import binding
    bound = math.tan(math.radians(angle) / 2.0)
    prod = FeasibleSet(bound)
    plane_constraints(gpu, prod, *args, margin, guard)
    ref = binding.Feasible(bound)
    ref.plane(*args, margin, guard)
    return prod, ref


def same(prod, ref):
    assert prod.is_empty() == ref.is_empty()
    assert prod.intervals() == ref.intervals()
    assert prod.nearest() == ref.nearest()
    assert prod.work() == ref.work()


@pytest.mark.parametrize("V,P,seed,margin,angle", [
    (3001, 6, 1, 0.2, 30.0),
    (3001, 6, 2, 0.05, 10.0),
    (517, 40, 3, 0.5, 60.0),
    (4099, 3, 4, 1.5, 20.0),
    (151936, 3, 5, 0.3, 30.0),
])
def test_plane_constraints_match_oracle(gpu, V, P, seed, margin, angle):
    prod, ref = run_both(gpu, inputs(V, P, seed), margin, 0.01, angle)
    same(prod, ref)
    assert prod.work()[0] > 0


def test_plane_constraints_end_empty(gpu):
    """A target far below its competitors forbids every tangent: the loop stops."""
    wu, wv, z, t, hu, hv = inputs(2053, 5, 7)
    z[2, t[2]] = np.float32(z[2].max() - 50.0)
    prod, ref = run_both(gpu, (wu, wv, z, t, hu, hv), 0.1, 0.01, 30.0)
    assert ref.is_empty()
    same(prod, ref)
    assert prod.work()[0] < 5 * 2052


def test_plane_constraints_many_hull_moves(gpu):
    """Many competitors close to the target trim the hull again and again, so the
    GPU rescreens the remaining constraints many times."""
    rng = np.random.default_rng(11)
    V, P = 1500, 4
    wu, wv, z, t, hu, hv = inputs(V, P, 11, spread=0.05)
    for p in range(P):
        top = np.argsort(z[p])[-60:]
        z[p, top] = z[p, t[p]] - np.float32(0.01) * rng.random(60).astype(np.float32)
        z[p, t[p]] = z[p].max() + np.float32(0.02)
    prod, ref = run_both(gpu, (wu, wv, z, t, hu, hv), 0.05, 0.0, 45.0)
    same(prod, ref)
