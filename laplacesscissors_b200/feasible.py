"""Plane-candidate feasibility: FeasibleSet (src/interval.rs:47-212) and the
constraint loop of the plane search (src/diagnosis.rs:1113-1143), over the C ABI.

FeasibleSet is host code in liblsx (lsx_feasible_*); plane_constraints forms and
screens every (point, vocabulary entry) constraint on the GPU and merges the
survivors on the host in the reference's order (lsx_plane_feasible), so the set,
its nearest tangent and its work counters are those of the sequential loop.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from ._lib import check, lib
from .gpu import Gpu, _dp, _fp, _up


@dataclass
class FeasibleSummary:  # src/interval.rs:42-47
    intervals: list[tuple[float, float]]
    constraints: int
    screened: int
    square_roots: int
    inserted_intervals: int


class FeasibleSet:
    """Open forbidden intervals of the half-angle tangent in [-bound, bound]."""

    def __init__(self, bound: float):
        h = C.c_void_p()
        check(lib.lsx_feasible_create(float(bound), C.byref(h)))
        self._h = h
        self.bound = float(bound)

    @staticmethod
    def for_angle(max_angle_degrees: float) -> "FeasibleSet":
        """FeasibleSet::new((max_angle.to_radians() / 2).tan()) as the plane search builds it."""
        return FeasibleSet(math.tan(math.radians(max_angle_degrees) / 2.0))

    def __del__(self):
        try:
            if self._h:
                lib.lsx_feasible_free(self._h)
                self._h = None
        except Exception:
            pass

    def constrain(self, a: float, b: float, c: float) -> None:
        check(lib.lsx_feasible_constrain(self._h, float(a), float(b), float(c)))

    def is_empty(self) -> bool:
        return bool(lib.lsx_feasible_is_empty(self._h))

    def nearest(self) -> float | None:
        t = C.c_double()
        found = C.c_int()
        check(lib.lsx_feasible_nearest(self._h, C.byref(t), C.byref(found)))
        return t.value if found.value else None

    def intervals(self) -> list[tuple[float, float]]:
        n = lib.lsx_feasible_intervals(self._h, None, 0)
        out = np.empty(2 * max(n, 1), dtype=np.float64)
        lib.lsx_feasible_intervals(self._h, _dp(out), n)
        return [(float(out[2 * i]), float(out[2 * i + 1])) for i in range(n)]

    def work(self) -> tuple[int, int, int, int]:
        w = (C.c_uint64 * 4)()
        check(lib.lsx_feasible_work(self._h, w))
        return tuple(int(x) for x in w)

    def summary(self) -> FeasibleSummary:
        c, s, r, i = self.work()
        return FeasibleSummary(self.intervals(), c, s, r, i)


def plane_constraints(gpu: Gpu, feasible: FeasibleSet, wu, wv, logits, targets, hu, hv, margin: float,
                      guard: float) -> None:
    """The plane search's constraint loop into `feasible`: wu = W u and wv = W v (head
    images, f32 [vocab]); per target point its frame logits (f32 [points, vocab]),
    target token and f64 projections hu = u.h, hv = v.h."""
    wu = np.ascontiguousarray(wu, dtype=np.float32)
    wv = np.ascontiguousarray(wv, dtype=np.float32)
    z = np.ascontiguousarray(logits, dtype=np.float32)
    t = np.ascontiguousarray(targets, dtype=np.uint32)
    hu = np.ascontiguousarray(hu, dtype=np.float64)
    hv = np.ascontiguousarray(hv, dtype=np.float64)
    if z.shape != (t.size, wu.size) or wv.size != wu.size or hu.size != t.size or hv.size != t.size:
        raise ValueError("check the plane constraint shapes")
    check(lib.lsx_plane_feasible(gpu.handle, feasible._h, _fp(wu), _fp(wv), wu.size, _fp(z), _up(t), _dp(hu),
                                 _dp(hv), t.size, float(margin), float(guard)))
