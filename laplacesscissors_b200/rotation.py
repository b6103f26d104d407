"""Readout edit types: ReadoutRotation (src/rotation.rs:22-77), SubspaceRotation
(src/response.rs:8-97) and ReadoutEdit (src/response.rs:222-256).

These are host-side f64 data contracts, as in the reference; the device form is
DeviceRotation in model.py.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


class EditError(ValueError):
    pass


def _ensure(cond: bool, message: str) -> None:
    if not cond:
        raise EditError(message)


@dataclass
class ReadoutRotation:
    u: np.ndarray
    v: np.ndarray
    tangent: float

    def __post_init__(self):
        self.u = np.asarray(self.u, dtype=np.float64)
        self.v = np.asarray(self.v, dtype=np.float64)
        self.tangent = float(self.tangent)

    def validate(self, width: int) -> None:  # src/rotation.rs:28-49
        _ensure(width > 1 and self.u.size == width and self.v.size == width, "check the rotation vector dimensions")
        _ensure(bool(np.all(np.isfinite(self.u)) and np.all(np.isfinite(self.v)) and np.isfinite(self.tangent)),
                "finite rotation coordinates are required")
        _ensure(abs(self.u @ self.u - 1) < 1e-8 and abs(self.v @ self.v - 1) < 1e-8 and abs(self.u @ self.v) < 1e-8,
                "the rotation plane needs orthonormal unit vectors")
        _ensure(abs(self.tangent) <= 1e6, "the half-angle coordinate must be within 1e6 in magnitude")

    def coefficients(self) -> tuple[float, float]:  # src/rotation.rs:50-53
        t = self.tangent
        return -2.0 * t * t / (1.0 + t * t), 2.0 * t / (1.0 + t * t)

    def apply(self, hidden) -> np.ndarray:  # src/rotation.rs:54-68
        h = np.asarray(hidden, dtype=np.float64)
        self.validate(h.size)
        _ensure(bool(np.all(np.isfinite(h))), "a finite hidden vector is required")
        a, b = self.coefficients()
        x = float(self.u @ h)
        y = float(self.v @ h)
        return h + self.u * (a * x + b * y) + self.v * (a * y - b * x)

    def subspace(self) -> "SubspaceRotation":  # ReadoutEdit::subspace, src/response.rs:240-251
        a, b = self.coefficients()
        return SubspaceRotation(np.stack([self.u, self.v]), np.array([[1 + a, b], [-b, 1 + a]]))


@dataclass
class SubspaceRotation:
    basis: np.ndarray      # rank x width, orthonormal rows
    transform: np.ndarray  # rank x rank orthogonal, det > 0

    def __post_init__(self):
        self.basis = np.atleast_2d(np.asarray(self.basis, dtype=np.float64))
        self.transform = np.atleast_2d(np.asarray(self.transform, dtype=np.float64))

    @property
    def rank(self) -> int:
        return self.basis.shape[0]

    def validate(self, width: int) -> None:  # src/response.rs:33-60
        n = self.rank
        _ensure(0 < n <= width and n <= 256 and self.transform.shape == (n, n),
                "check the joint rotation rank and inner matrix size")
        _ensure(self.basis.shape[1] == width and bool(np.all(np.isfinite(self.basis)))
                and bool(np.all(np.isfinite(self.transform))),
                "the joint rotation needs a finite basis and square matrix")
        gram = self.basis @ self.basis.T
        _ensure(float(np.max(np.abs(gram - np.eye(n)))) < 1e-8, "check the orthogonality of the joint basis")
        q = self.transform
        _ensure(float(np.max(np.abs(q.T @ q - np.eye(n)))) < 1e-8 and np.linalg.det(q) > 0,
                "check the orthogonality and orientation of the joint rotation")

    def coordinates(self, x) -> np.ndarray:
        return self.basis @ np.asarray(x, dtype=np.float64)

    def apply(self, h) -> np.ndarray:  # src/response.rs:67-77
        h = np.asarray(h, dtype=np.float64)
        delta = (self.transform - np.eye(self.rank)) @ self.coordinates(h)
        return h + delta @ self.basis

    def delta_row(self, row) -> np.ndarray:  # src/response.rs:78-90
        x = self.coordinates(row)
        delta = (self.transform.T - np.eye(self.rank)) @ x
        return delta @ self.basis

    def subspace(self) -> "SubspaceRotation":
        return self


ReadoutEdit = ReadoutRotation | SubspaceRotation


def random_subspace_rotation(width: int, rank: int, max_degrees: float, seed: int = 7,
                             pairs: str = "all") -> SubspaceRotation:
    """The readout-validation workload's edit: U = orthonormal `rank` rows from the
    QR of a seeded Gaussian [width, rank]; R = product of Givens rotations over all
    rank*(rank-1)/2 coordinate pairs (a < b) in lexicographic order, angles uniform
    in (-max_degrees, max_degrees), each new rotation applied on the left."""
    from . import synth

    g = synth.normal_f32(seed, synth.STREAM_EDIT_BASIS, width * rank).astype(np.float64).reshape(width, rank)
    q, r = np.linalg.qr(g)
    q = q * np.sign(np.diag(r))[None, :]
    basis = q.T.copy()
    plist = [(a, b) for a in range(rank) for b in range(a + 1, rank)] if pairs == "all" else \
        [(2 * i, 2 * i + 1) for i in range(rank // 2)]
    u = synth.uniform_u32(seed, synth.STREAM_EDIT_ANGLES, len(plist), 0xFFFFFFFF).astype(np.float64)
    angles = np.deg2rad(-max_degrees + 2 * max_degrees * (u / 4294967295.0))
    R = np.eye(rank)
    for (a, b), th in zip(plist, angles):
        G = np.eye(rank)
        c, s = np.cos(th), np.sin(th)
        G[a, a] = c
        G[b, b] = c
        G[a, b] = -s
        G[b, a] = s
        R = G @ R
    return SubspaceRotation(basis, R)


__all__ = ["ReadoutRotation", "SubspaceRotation", "ReadoutEdit", "EditError", "random_subspace_rotation"]
