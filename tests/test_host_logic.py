"""Host-side logic of the mirror (rotation types, diagnosis rules, workload
generators) against the oracle.  No GPU."""
import numpy as np
import pytest

from laplacesscissors_b200 import diagnosis, synth
from laplacesscissors_b200.rotation import EditError, ReadoutRotation, SubspaceRotation, random_subspace_rotation


def test_readout_rotation_validate_and_apply(oracle):
    r = ReadoutRotation([0.6, 0.8, 0, 0], [0, 0, 1.0, 0], 0.73)
    r.validate(4)
    h = np.array([0.3, -1.2, 0.5, 2.0])
    assert np.allclose(r.apply(h), oracle.plane_apply(r.u, r.v, r.tangent, h), atol=1e-15)
    with pytest.raises(EditError):  # src/rotation.rs:383-394
        ReadoutRotation([1.0, 0], [1.0, 0], 0.0).validate(2)
    with pytest.raises(EditError):
        ReadoutRotation([1.0, 0], [0, 1.0], float("nan")).validate(2)
    with pytest.raises(EditError):
        ReadoutRotation([1.0, 0], [0, 1.0], 2e6).validate(2)


def test_subspace_rotation_validate_and_apply(oracle):
    s = random_subspace_rotation(64, 16, 3.0, seed=7)
    s.validate(64)
    h = np.random.default_rng(1).standard_normal(64)
    assert np.allclose(s.apply(h), oracle.subspace_apply(s.basis, s.transform, h), atol=1e-13)
    angles = np.degrees(np.arccos(np.clip(np.linalg.eigvals(s.transform).real, -1, 1)))
    assert angles.max() < 30  # a product of 120 small Givens rotations
    bad = SubspaceRotation(s.basis, -s.transform)  # det < 0 for even rank? flip one axis instead
    t = s.transform.copy()
    t[0] *= -1
    with pytest.raises(EditError):
        SubspaceRotation(s.basis, t).validate(64)
    with pytest.raises(EditError):
        SubspaceRotation(s.basis * 1.01, s.transform).validate(64)
    del bad


def test_plane_subspace_equivalence():
    r = ReadoutRotation([0.6, 0.8, 0, 0], [0, 0, 1.0, 0], -0.4)
    h = np.array([1.0, 2.0, -0.5, 0.25])
    assert np.allclose(r.subspace().apply(h), r.apply(h), atol=1e-14)


def test_diagnosis_rules_match_oracle(oracle):
    rng = np.random.default_rng(0)
    for trial in range(50):
        z = rng.integers(-3, 4, 40).astype(np.float32)  # many ties
        t = int(rng.integers(0, 40))
        assert diagnosis.argmax(z) == oracle.argmax(z)
        assert diagnosis.other(z, t) == oracle.other(z, t)
        assert diagnosis.minimum_margin(z, t) == oracle.minimum_margin(z, t)
    z = np.array([0.0, -0.0, -1.0], np.float32)
    assert diagnosis.other(z, 2) == oracle.other(z, 2) == 0  # total order puts +0 above -0
    with pytest.raises(ValueError):
        diagnosis.argmax(np.array([1.0, np.nan], np.float32))


def test_readout_workload_generators():
    h = synth.readout_hidden(7, 8, 1024)
    x = synth.bf16_to_f32(h).astype(np.float64)
    rms = np.sqrt((x * x).mean(axis=1))
    assert np.all(np.abs(rms - 1) < 0.01)
    t = synth.readout_targets(7, 4096, 151936)
    assert t.max() < 151936


def test_deadline():
    d = diagnosis.Deadline.after(-1)
    with pytest.raises(diagnosis.BudgetExpired):
        d.check()
