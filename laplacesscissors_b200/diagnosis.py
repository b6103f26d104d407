"""The readout-validation and generation functions of src/diagnosis.rs over liblsx.

argmax / other / minimum_margin restate the reference's host rules
(src/diagnosis.rs:58-80, 490-492) for host arrays.  generate_frames runs the
greedy loop on the device (lsx_model_generate).  verify_cached evaluates every
target prefix of every observed path in ONE fused tensor-core launch
(lsx_readout_margin: margin and first argmax without storing logits) and keeps
the reference's aggregation and acceptance rule (src/diagnosis.rs:493-580).
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass, field

import numpy as np

from ._lib import BF16, F32, check, lib
from .gpu import Gpu, Tensor, _dp, _fp, _up
from .model import DeviceRotation, Frame, Model


class BudgetExpired(RuntimeError):  # src/diagnosis.rs:22-29
    pass


class Deadline:  # src/diagnosis.rs:30-48
    def __init__(self, seconds: float):
        self.end = time.monotonic() + seconds

    @staticmethod
    def after(seconds: float) -> "Deadline":
        return Deadline(seconds)

    def check(self) -> None:
        if time.monotonic() >= self.end:
            raise BudgetExpired("the diagnosis time budget is used up")


def _finite_scores(values: np.ndarray) -> np.ndarray:
    v = np.asarray(values, dtype=np.float32)
    if v.size == 0 or not np.all(np.isfinite(v)):
        raise ValueError("finite vocabulary scores are required")
    return v


def argmax(values) -> int:  # src/diagnosis.rs:58-70: first maximum
    v = _finite_scores(values)
    return int(np.argmax(v))


def _total_key(v: np.ndarray) -> np.ndarray:
    i = v.astype(np.float32).view(np.int32).astype(np.int64)
    return np.where(i < 0, i ^ 0x7FFFFFFF, i)


def other(logits, target: int) -> int:  # src/diagnosis.rs:71-80
    v = np.asarray(logits, dtype=np.float32)
    if not (v.size > 1 and 0 <= target < v.size):
        raise ValueError("check the vocabulary range of the answer token")
    key = _total_key(v)
    key[target] = np.iinfo(np.int64).min
    return int(np.argmax(key))  # lowest index among equal keys


def minimum_margin(scores, target: int) -> float:  # src/diagnosis.rs:490-492
    v = np.asarray(scores, dtype=np.float32)
    return float(np.float64(v[target]) - np.float64(v[other(v, target)]))


def prefill(model: Model, gpu: Gpu, prompt, edit: DeviceRotation | None, deadline: Deadline) -> Frame:
    """src/diagnosis.rs:81-99: reset, then feed the prompt token by token."""
    if not (0 < len(prompt) <= model.max_context()):
        raise ValueError("check the input token length")
    model.reset()
    frame = None
    for token in prompt:
        deadline.check()
        frame = model.advance(gpu, int(token), edit)
    return frame


@dataclass
class Generation:  # src/diagnosis.rs:100-105 (token ids; text decoding is the caller's)
    tokens: list[int]
    stopped: bool


def generate_frames(model: Model, gpu: Gpu, stop_tokens, prompt, maximum: int,
                    edit: DeviceRotation | None, deadline: Deadline) -> tuple[Generation, list[Frame]]:
    """src/diagnosis.rs:106-149, with the whole loop on the device."""
    deadline.check()
    tokens, stopped, frames = model.generate(prompt, maximum, stop_tokens, edit, frames=True)
    return Generation([int(t) for t in tokens], stopped), frames


def generate(model: Model, gpu: Gpu, stop_tokens, prompt, maximum: int, edit: DeviceRotation | None,
             deadline: Deadline) -> Generation:
    deadline.check()
    tokens, stopped, _ = model.generate(prompt, maximum, stop_tokens, edit, frames=False)
    return Generation([int(t) for t in tokens], stopped)


# ------------------------------------------------------------ validation ----
def readout_margin(gpu: Gpu, weight: Tensor, bias: Tensor | None, vocab: int, width: int, hidden: np.ndarray,
                   targets: np.ndarray, rotation: DeviceRotation | None = None):
    """Fused readout margin over host rows (lsx_readout_margin).  `hidden` is
    float32 [n, width] or uint16 bf16 bits [n, width].  Returns (margin f64,
    argmax u32, target logit f32)."""
    h = np.ascontiguousarray(hidden)
    kind = BF16 if h.dtype == np.uint16 else F32
    if kind == F32:
        h = np.ascontiguousarray(h, dtype=np.float32)
    n = h.shape[0]
    t = np.ascontiguousarray(targets, dtype=np.uint32)
    margin = np.empty(n, dtype=np.float64)
    amax = np.empty(n, dtype=np.uint32)
    tl = np.empty(n, dtype=np.float32)
    check(lib.lsx_readout_margin(gpu.handle, weight.handle, bias.handle if bias else None, int(vocab), int(width),
                                 h.ctypes.data_as(C.c_void_p), kind, n, _up(t),
                                 rotation.handle if rotation else None, _dp(margin), _up(amax), _fp(tl)))
    return margin, amax, tl


@dataclass
class ObservedPath:  # the observed prefixes of one case (src/diagnosis.rs ObservedPath)
    case: int
    protected: bool
    tokens: list[int]
    frames: list[Frame]
    answer_matches: bool = True  # generation.text == case.answer() when the tokens match


@dataclass
class Verification:  # src/diagnosis.rs Verification
    method: str
    target_min_margin: float
    protected_max_logit_change: float
    protected_max_scaled_change: float
    certified_paths: list[bool]
    generations: list[Generation]
    protected_sequences_preserved: bool
    requested_answers_generated: bool
    readout_calls: int
    decoder_steps: int
    accepted: bool


def verify_cached(model: Model, gpu: Gpu, stop_tokens, edit, paths: list[ObservedPath], margin: float,
                  tolerance: float, deadline: Deadline) -> Verification:
    """src/diagnosis.rs:493-580.  Target prefixes: one fused margin/argmax launch
    for all of them.  Protected prefixes: Model::readout per prefix and the
    reference's f64 change statistics against the cached logits."""
    width = model.hidden_size
    device = DeviceRotation.upload_edit(gpu, edit, width)
    weight, bias = model.head_tensors()
    V = model.vocab_size()
    stop = set(int(s) for s in stop_tokens)
    # Fused pass over every target prefix.
    rows, targets, owners = [], [], []
    for pi, path in enumerate(paths):
        if path.protected:
            continue
        for k, (expected, frame) in enumerate(zip(path.tokens, path.frames)):
            rows.append(np.asarray(frame.hidden, dtype=np.float32))
            targets.append(int(expected))
            owners.append((pi, k))
    fused = {}
    minimum = float("inf")
    if rows:
        deadline.check()
        m, a, _ = readout_margin(gpu, weight, bias, V, width, np.stack(rows), np.asarray(targets), device)
        minimum = float(np.min(m))
        for (pi, k), am in zip(owners, a):
            fused[(pi, k)] = int(am)
    maximum = 0.0
    scaled = 0.0
    preserved = True
    repaired = True
    calls = len(rows)
    generations, certificates = [], []
    for pi, path in enumerate(paths):
        matched = True
        tokens: list[int] = []
        stopped = False
        for k, (expected, frame) in enumerate(zip(path.tokens, path.frames)):
            if path.protected:
                deadline.check()
                scores = model.readout(gpu, frame.hidden, device)
                calls += 1
                change = np.abs(frame.logits.astype(np.float64) - scores.astype(np.float64))
                maximum = max(maximum, float(change.max()))
                scaled = max(scaled, float((change / (1.0 + np.abs(frame.logits.astype(np.float64)))).max()))
                actual = argmax(scores) if matched else None
            else:
                actual = fused[(pi, k)] if matched else None
            if matched:
                tokens.append(actual)
                stopped = actual in stop
                matched = actual == int(expected)
        if path.protected:
            preserved &= matched
        else:
            repaired &= matched
        correct = matched and stopped and path.answer_matches
        if not path.protected:
            repaired &= correct
        generations.append(Generation(tokens, stopped))
        certificates.append(matched)
    accepted = minimum >= margin and scaled <= tolerance and preserved and repaired
    return Verification("native_readout_on_observed_prefixes", minimum, maximum, scaled, certificates, generations,
                        preserved, repaired, calls, 0, accepted)


class CompactReadout:
    """src/diagnosis.rs:608-666: z = z0 + F ((R - I) x) per observation, on the
    device with the f32 matvec exactly as the reference evaluates it."""

    def __init__(self, gpu: Gpu, images: list[np.ndarray], baseline: list[np.ndarray],
                 coordinates: list[np.ndarray]):
        rank = len(images)
        vocab = len(images[0])
        if not (len(baseline) == len(coordinates) and all(len(z) == vocab for z in baseline)):
            raise ValueError("check the baseline scores and observation count of the compact readout")
        rows = np.stack([np.asarray(im, dtype=np.float32) for im in images], axis=1)  # [vocab, rank]
        self.image = gpu.upload_f32(rows)
        self.baseline = [gpu.upload_f32(z) for z in baseline]
        self.coordinates = np.stack([np.asarray(c, dtype=np.float64) for c in coordinates], axis=1)  # [rank, n]
        self.vocabulary = vocab
        self.rank = rank
        self._baseline_block = None  # [n, vocab] for evaluate_margins, uploaded on first use
        self._baseline_host = baseline

    def evaluate(self, gpu: Gpu, rotation: np.ndarray, deadline: Deadline) -> list[np.ndarray]:
        rank = rotation.shape[0]
        delta = (rotation - np.eye(rank)) @ self.coordinates
        out = []
        for i, base in enumerate(self.baseline):
            deadline.check()
            coefficients = gpu.upload_f32(delta[:, i].astype(np.float32))
            scores = gpu.read(gpu.linear(coefficients, self.image, base, self.vocabulary, rank))
            if not np.all(np.isfinite(scores)):
                raise ValueError("check the finite scores of the compact readout")
            out.append(scores)
        return out

    def evaluate_margins(self, gpu: Gpu, rotation: np.ndarray, targets, deadline: Deadline | None = None):
        """evaluate() reduced on the device to what the joint search reads from each
        observation's scores (src/diagnosis.rs:790-815): minimum_margin against its
        target, the competitor other() picks and the first argmax; the V-wide
        scores are never stored or downloaded (lsx_compact_margin).  Returns
        (margin f64 [n], other u32 [n], argmax u32 [n])."""
        if deadline is not None:
            deadline.check()
        rank = rotation.shape[0]
        delta = (rotation - np.eye(rank)) @ self.coordinates  # [rank, n]
        n = delta.shape[1]
        if self._baseline_block is None:
            self._baseline_block = gpu.upload_f32(np.stack([np.asarray(z, dtype=np.float32)
                                                            for z in self._baseline_host]))
        coefficients = np.ascontiguousarray(delta.T, dtype=np.float32)  # [n, rank]
        t = np.ascontiguousarray(targets, dtype=np.uint32)
        if t.size != n:
            raise ValueError("one target per observation")
        margin = np.empty(n, dtype=np.float64)
        other_ = np.empty(n, dtype=np.uint32)
        amax = np.empty(n, dtype=np.uint32)
        check(lib.lsx_compact_margin(gpu.handle, self.image.handle, self._baseline_block.handle, self.vocabulary,
                                     rank, n, _fp(coefficients), _up(t), _dp(margin), _up(other_), _up(amax)))
        return margin, other_, amax


__all__ = [
    "argmax", "other", "minimum_margin", "prefill", "generate_frames", "generate", "Generation", "ObservedPath",
    "Verification", "verify_cached", "CompactReadout", "readout_margin", "Deadline", "BudgetExpired",
]


@dataclass
class ScoredCase:  # one case record of scaling::evaluate (src/scaling.rs:198-211)
    case: int
    prompt_tokens: list[int]
    target_tokens: list[int]
    sequence_nll_before: float
    sequence_nll_after: float
    canonical_path_before: bool
    canonical_path_after: bool


@dataclass
class Evaluation:  # the aggregates of scaling::evaluate (src/scaling.rs:178-216)
    loss_before: float
    loss_after: float
    correct_before: int
    correct_after: int
    cases: list[ScoredCase]


def evaluate_cases(model: Model, cases, rotation: DeviceRotation | None = None,
                   deadline: Deadline | None = None) -> Evaluation:
    """Teacher-forced scoring of many cases (src/scaling.rs:181-216).  `cases` holds
    (prompt token ids, target token ids, answer byte length) per case; the
    tokenizer (Text::target) is the caller's.  Per case the before scores use the
    unedited readout and the after scores the edited one; a case's weight is
    1 / (cases x max(answer bytes, 1)), as the reference's."""
    n_cases = len(cases)
    before = after = 0.0
    correct_before = correct_after = 0
    records = []
    for i, (prompt, targets, answer_bytes) in enumerate(cases):
        if deadline:
            deadline.check()
        targets = [int(t) for t in targets]
        weight = 1.0 / (n_cases * max(int(answer_bytes), 1))
        nll_b, amax_b, _ = model.score(prompt, targets)
        if rotation is not None:
            nll_a, amax_a, _ = model.score(prompt, targets, rotation)
        else:
            nll_a, amax_a = nll_b, amax_b
        case_before, case_after = float(np.sum(nll_b)), float(np.sum(nll_a))
        path_before = bool(np.all(amax_b == np.asarray(targets, dtype=np.uint32)))
        path_after = bool(np.all(amax_a == np.asarray(targets, dtype=np.uint32)))
        before += case_before * weight
        after += case_after * weight
        correct_before += int(path_before)
        correct_after += int(path_after)
        records.append(ScoredCase(i, [int(x) for x in prompt], targets, case_before, case_after, path_before,
                                  path_after))
    return Evaluation(before, after, correct_before, correct_after, records)
