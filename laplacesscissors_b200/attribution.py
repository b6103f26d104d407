"""Attribution of a readout edit's loss change to vocabulary rows
(src/attribution.rs): the numerical core runs on the GPU through
lsx_integrated_credits (Simpson integration of the softmax along the straight
chord between each point's logits before and after the edit, in f64, credits per
vocabulary row, losses and restored losses); panel doubling, ranking and the
per-coordinate split of the leading rows follow analyze (src/attribution.rs:
125-235) on the host.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from ._lib import check, lib
from .gpu import Gpu, _dp, _up


@dataclass
class LossPoint:  # src/attribution.rs:12-17
    before_logits: np.ndarray
    before_hidden: np.ndarray
    after: np.ndarray
    target: int
    weight: float


@dataclass
class CoordinateCredit:  # src/attribution.rs:18-23
    column: int
    delta_weight: float
    credit: float


@dataclass
class RowCredit:  # src/attribution.rs:24-34
    row: int
    credit: float
    restored_loss: float
    restoration_increase: float
    coordinate_sum: float
    coordinate_sum_residual: float
    leading_coordinates: list[CoordinateCredit] = field(default_factory=list)


@dataclass
class Attribution:  # src/attribution.rs:35-48
    unit: str
    loss_before: float
    loss_after: float
    credit_sum: float
    integration_residual: float
    integration_converged: bool
    panels: int
    points: int
    leading_rows: list[RowCredit]
    remaining_rows_credit: float


def integrated_credits(gpu: Gpu, before, after, targets, weights, panels: int, rows=None):
    """integrated_probabilities (src/attribution.rs:79-123) on the GPU.  before /
    after: f32 [points, vocab]; returns (credits f64 [vocab], integrals at `rows`
    f64 [points, len(rows)], losses f64 [points, 2 + len(rows)]: loss(before),
    loss(after), then restored_loss(after, row, before[row], target) per row)."""
    b = np.ascontiguousarray(before, dtype=np.float32)
    a = np.ascontiguousarray(after, dtype=np.float32)
    if b.ndim != 2 or a.shape != b.shape:
        raise ValueError("check the attribution observation conditions")
    points, vocab = b.shape
    t = np.ascontiguousarray(targets, dtype=np.uint32)
    w = np.ascontiguousarray(weights, dtype=np.float64)
    r = np.ascontiguousarray([] if rows is None else rows, dtype=np.uint32)
    credits = np.empty(vocab, dtype=np.float64)
    grads = np.empty((points, max(r.size, 1)), dtype=np.float64)
    losses = np.empty((points, 2 + r.size), dtype=np.float64)
    check(lib.lsx_integrated_credits(gpu.handle, b.ctypes.data_as(C.c_void_p), a.ctypes.data_as(C.c_void_p), _up(t),
                                     _dp(w), points, vocab, int(panels), _dp(credits),
                                     _up(r) if r.size else None, r.size, _dp(grads), _dp(losses)))
    return credits, grads[:, : r.size], losses


def _ranking(credits: np.ndarray, count: int) -> list[int]:
    """Rows by |credit| descending, lower index first on ties (src/attribution.rs:167-181)."""
    order = np.lexsort((np.arange(credits.size), -np.abs(credits)))
    return [int(i) for i in order[:count]]


def analyze(gpu: Gpu, points: list[LossPoint], row_count: int, tolerance: float, unit: str,
            head_row=None, subspace=None) -> Attribution:
    """src/attribution.rs:125-235.  `head_row(row)` gives a readout row (f32 [hidden]);
    `subspace` the edit's SubspaceRotation (for delta_row).  Without them the
    leading rows carry no coordinate split."""
    if not points or not np.isfinite(tolerance) or tolerance <= 0:
        raise ValueError("specify the attribution observations and integration tolerance")
    before = np.stack([np.asarray(p.before_logits, np.float32) for p in points])
    after = np.stack([np.asarray(p.after, np.float32) for p in points])
    targets = [int(p.target) for p in points]
    weights = np.array([p.weight for p in points], dtype=np.float64)
    vocab = before.shape[1]
    panels = 16
    while True:
        credits, _, losses = integrated_credits(gpu, before, after, targets, weights, panels)
        if panels == 16:
            loss_before = float(sum(w * l for w, l in zip(weights, losses[:, 0])))
            loss_after = float(sum(w * l for w, l in zip(weights, losses[:, 1])))
            expected = loss_before - loss_after
        residual = abs(float(np.sum(credits)) - expected)
        if residual <= tolerance * (1 + abs(expected)) or panels >= 256:
            break
        panels *= 2
    leading_rows = _ranking(credits, min(row_count, vocab))
    _, grads, losses = integrated_credits(gpu, before, after, targets, weights, panels, leading_rows)
    leading = []
    for i, row in enumerate(leading_rows):
        restored = float(sum(w * l for w, l in zip(weights, losses[:, 2 + i])))
        coordinate_sum, coords = 0.0, []
        if head_row is not None and subspace is not None:
            delta = subspace.delta_row(np.asarray(head_row(row), dtype=np.float64))
            coordinate = np.zeros(delta.size)
            for p, point in enumerate(points):
                coordinate -= point.weight * delta * np.asarray(point.before_hidden, np.float64) * grads[p, i]
            coordinate_sum = float(np.sum(coordinate))
            cols = np.lexsort((np.arange(coordinate.size), -np.abs(coordinate)))[:6]
            coords = [CoordinateCredit(int(c), float(delta[c]), float(coordinate[c])) for c in cols]
        leading.append(RowCredit(row, float(credits[row]), restored, restored - loss_after, coordinate_sum,
                                 abs(coordinate_sum - float(credits[row])), coords))
    total = float(np.sum(credits))
    return Attribution(unit, loss_before, loss_after, total, residual,
                       residual <= tolerance * (1 + abs(expected)), panels, len(points), leading,
                       total - sum(r.credit for r in leading))
