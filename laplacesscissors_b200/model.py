"""Model and DeviceRotation: the reference's src/model.rs API over liblsx.

Model.load reads the same checkpoint folders as Model::load (config.json or
laplace.graph.json plus safetensors); advance/step/inject/readout/head_image/
head_row/reset/rewind keep the reference's semantics, including the Frame they
return.  `generate` runs diagnosis::generate_frames entirely on the device.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import ModelInfo, check, lib
from .gpu import Gpu, Tensor, _dp, _fp, _up
from .rotation import ReadoutRotation, SubspaceRotation


@dataclass
class Frame:  # src/model.rs:365-369
    hidden: np.ndarray
    logits: np.ndarray


class DeviceRotation:
    """An edit uploaded for the readout (src/model.rs:285-364)."""

    def __init__(self, handle: C.c_void_p, gpu: Gpu, width: int, rank: int, joint: bool):
        self._h = handle
        self.gpu = gpu
        self.width = width
        self.rank = rank
        self.joint = joint

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @staticmethod
    def upload(gpu: Gpu, spec: ReadoutRotation, width: int) -> "DeviceRotation":
        u = np.ascontiguousarray(spec.u, dtype=np.float64)
        v = np.ascontiguousarray(spec.v, dtype=np.float64)
        h = C.c_void_p()
        check(lib.lsx_rotation_plane(gpu.handle, _dp(u), _dp(v), float(spec.tangent), int(width), C.byref(h)))
        return DeviceRotation(h, gpu, width, 2, False)

    @staticmethod
    def upload_edit(gpu: Gpu, spec, width: int) -> "DeviceRotation":
        if isinstance(spec, ReadoutRotation):
            return DeviceRotation.upload(gpu, spec, width)
        assert isinstance(spec, SubspaceRotation)
        basis = np.ascontiguousarray(spec.basis, dtype=np.float64)
        transform = np.ascontiguousarray(spec.transform, dtype=np.float64)
        h = C.c_void_p()
        check(lib.lsx_rotation_joint(gpu.handle, _dp(basis), _dp(transform), basis.shape[0], int(width),
                                     C.byref(h)))
        return DeviceRotation(h, gpu, width, basis.shape[0], True)

    def apply(self, gpu: Gpu, hidden: Tensor) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_rotation_apply(gpu.handle, self._h, hidden.handle, C.byref(h)))
        return Tensor(h.value, gpu)

    def free(self) -> None:
        if self._h and self._h.value:
            lib.lsx_rotation_free(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _rot(rotation: DeviceRotation | None):
    return rotation.handle if rotation is not None else None


class Model:
    def __init__(self, handle: C.c_void_p, gpu: Gpu):
        self._h = handle
        self.gpu = gpu
        self._info = self.info()

    @staticmethod
    def load(root, gpu: Gpu, capacity: int) -> "Model":  # src/model.rs:411-529
        h = C.c_void_p()
        check(lib.lsx_model_load(gpu.handle, str(root).encode(), int(capacity), C.byref(h)))
        return Model(h, gpu)

    def free(self) -> None:
        if self._h and self._h.value:
            lib.lsx_model_free(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def info(self) -> ModelInfo:
        i = ModelInfo()
        check(lib.lsx_model_info_get(self._h, C.byref(i)))
        return i

    @property
    def fused(self) -> bool:
        return bool(lib.lsx_model_fused(self._h))

    @property
    def hidden_size(self) -> int:
        return int(self._info.hidden_size)

    def vocab_size(self) -> int:
        return int(self._info.vocab_size)

    def position(self) -> int:
        return int(self.info().position)

    def max_context(self) -> int:
        return int(self._info.capacity)

    def parameter_count(self) -> int:
        return int(self._info.parameters)

    def tensor_count(self) -> int:
        return int(self._info.tensors)

    def eos_token_ids(self) -> list[int]:
        i = self._info
        return [int(i.eos_token_ids[k]) for k in range(int(i.eos_count))]

    def reset(self) -> None:
        check(lib.lsx_model_reset(self._h))

    def rewind(self, position: int) -> None:
        check(lib.lsx_model_rewind(self._h, int(position)))

    def advance(self, gpu: Gpu, token: int, rotation: DeviceRotation | None = None) -> Frame:
        hidden = np.empty(self.hidden_size, dtype=np.float32)
        logits = np.empty(self.vocab_size(), dtype=np.float32)
        check(lib.lsx_model_advance(self._h, int(token), _rot(rotation), _fp(hidden), _fp(logits), None))
        return Frame(hidden, logits)

    def step(self, gpu: Gpu, token: int, rotation: DeviceRotation | None = None) -> np.ndarray:
        return self.advance(gpu, token, rotation).logits

    def advance_token(self, token: int, rotation: DeviceRotation | None = None) -> int:
        """advance() that returns only the first argmax of the logits (no frame copies)."""
        out = C.c_uint32()
        check(lib.lsx_model_advance(self._h, int(token), _rot(rotation), None, None, C.byref(out)))
        return int(out.value)

    def inject(self, gpu: Gpu, vector, rotation: DeviceRotation | None = None) -> Frame:
        v = np.ascontiguousarray(vector, dtype=np.float32)
        if v.size != self.hidden_size:
            raise ValueError("check the injected vector width, finiteness and context")
        hidden = np.empty(self.hidden_size, dtype=np.float32)
        logits = np.empty(self.vocab_size(), dtype=np.float32)
        check(lib.lsx_model_inject(self._h, _fp(v), _rot(rotation), _fp(hidden), _fp(logits), None))
        return Frame(hidden, logits)

    def embedding_vector(self, gpu: Gpu, token: int) -> np.ndarray:
        out = np.empty(self.hidden_size, dtype=np.float32)
        check(lib.lsx_model_embedding_vector(self._h, int(token), _fp(out)))
        return out

    def readout(self, gpu: Gpu, hidden, rotation: DeviceRotation | None = None) -> np.ndarray:
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        if h.size != self.hidden_size:
            raise ValueError("check the readout input width and finiteness")
        out = np.empty(self.vocab_size(), dtype=np.float32)
        check(lib.lsx_model_readout(self._h, _fp(h), _rot(rotation), _fp(out)))
        return out

    def head_image(self, gpu: Gpu, vector) -> np.ndarray:
        v = np.ascontiguousarray(vector, dtype=np.float64)
        if v.size != self.hidden_size:
            raise ValueError("check the readout direction dimension")
        out = np.empty(self.vocab_size(), dtype=np.float32)
        check(lib.lsx_model_head_image(self._h, _dp(v), _fp(out)))
        return out

    def generate_batch(self, prompts, maximum: int) -> np.ndarray:
        """Greedy generation of several equal-length prompts at once
        (lsx_model_generate_batch): prompts [batch, P] -> tokens [batch, maximum]."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), dtype=np.uint32)
        out = np.empty((p.shape[0], int(maximum)), dtype=np.uint32)
        check(lib.lsx_model_generate_batch(self._h, _up(p), p.shape[0], p.shape[1], int(maximum), _up(out)))
        return out

    def head_images(self, gpu: Gpu, vectors) -> np.ndarray:
        """head_image for every row of `vectors` [count, hidden] in one tensor-core
        pass over the lm_head per 32 directions; returns [count, vocab] f32."""
        v = np.ascontiguousarray(np.atleast_2d(vectors), dtype=np.float64)
        if v.shape[1] != self.hidden_size:
            raise ValueError("check the readout direction dimension")
        out = np.empty((v.shape[0], self.vocab_size()), dtype=np.float32)
        check(lib.lsx_model_head_images(self._h, _dp(v), v.shape[0], _fp(out)))
        return out

    def head_row(self, gpu: Gpu, token: int) -> np.ndarray:
        out = np.empty(self.hidden_size, dtype=np.float32)
        check(lib.lsx_model_head_row(self._h, int(token), _fp(out)))
        return out

    def head_tensors(self) -> tuple[Tensor, Tensor | None]:
        """Non-owning views of the readout weight and bias."""
        w = C.c_void_p()
        b = C.c_void_p()
        check(lib.lsx_model_head(self._h, C.byref(w), C.byref(b)))
        weight = Tensor(w.value, self.gpu, borrowed=True)
        bias = Tensor(b.value, self.gpu, borrowed=True) if b.value else None
        return weight, bias

    def generate(self, prompt, maximum: int, stop_tokens=(), rotation: DeviceRotation | None = None,
                 frames: bool = False):
        """diagnosis::generate_frames (src/diagnosis.rs:106-149) on the device.
        Returns (tokens, stopped, frames or None)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        stops = np.ascontiguousarray(list(stop_tokens), dtype=np.uint32)
        tokens = np.empty(int(maximum), dtype=np.uint32)
        n = C.c_size_t()
        stopped = C.c_int()
        H, V = self.hidden_size, self.vocab_size()
        hid = np.empty((maximum, H), dtype=np.float32) if frames else None
        lg = np.empty((maximum, V), dtype=np.float32) if frames else None
        check(lib.lsx_model_generate(self._h, _up(p), p.size, int(maximum), _up(stops) if stops.size else None,
                                     stops.size, _rot(rotation), _up(tokens), C.byref(n), C.byref(stopped),
                                     _fp(hid) if frames else None, _fp(lg) if frames else None))
        k = int(n.value)
        fr = [Frame(hid[i].copy(), lg[i].copy()) for i in range(k)] if frames else None
        return tokens[:k].copy(), bool(stopped.value), fr


    def score(self, prompt, targets, rotation: DeviceRotation | None = None, frames: bool = False):
        """Teacher-forced scoring of one case (lsx_model_score; the per-case loop of
        src/scaling.rs:181-216): per continuation position the loss
        (attribution::loss, src/attribution.rs:49-60) of its target and the argmax of
        the frame's logits.  Returns (nll f64 [n], argmax u32 [n], frames or None)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        t = np.ascontiguousarray(targets, dtype=np.uint32)
        n = t.size
        nll = np.empty(n, dtype=np.float64)
        amax = np.empty(n, dtype=np.uint32)
        H, V = self.hidden_size, self.vocab_size()
        hid = np.empty((n, H), dtype=np.float32) if frames else None
        lg = np.empty((n, V), dtype=np.float32) if frames else None
        check(lib.lsx_model_score(self._h, _up(p), p.size, _up(t), n, _rot(rotation), _dp(nll), _up(amax),
                                  _fp(hid) if frames else None, _fp(lg) if frames else None))
        fr = [Frame(hid[i].copy(), lg[i].copy()) for i in range(n)] if frames else None
        return nll, amax, fr

    def score_batch(self, prompts, targets, rotation: DeviceRotation | None = None, logits: bool = False):
        """Teacher-forced scoring of many equal-shape cases at once
        (lsx_model_score_batch): prompts [cases, P], targets [cases, n], optionally
        through the edited readout.  Returns (nll f64 [cases, n], argmax u32
        [cases, n], margin f64 [cases, n], logits f32 [cases, n, vocab] or None).
        Leaves the decode cursor and KV cache as they were."""
        p = np.ascontiguousarray(prompts, dtype=np.uint32)
        t = np.ascontiguousarray(targets, dtype=np.uint32)
        if p.ndim != 2 or t.ndim != 2 or p.shape[0] != t.shape[0]:
            raise ValueError("prompts and targets are [cases, length] arrays with one row per case")
        cases, n = t.shape
        nll = np.empty((cases, n), dtype=np.float64)
        amax = np.empty((cases, n), dtype=np.uint32)
        margin = np.empty((cases, n), dtype=np.float64)
        lg = np.empty((cases, n, self.vocab_size()), dtype=np.float32) if logits else None
        check(lib.lsx_model_score_batch(self._h, _up(p), cases, p.shape[1], _up(t), n, _rot(rotation), _dp(nll),
                                        _up(amax), _dp(margin), _fp(lg) if logits else None))
        return nll, amax, margin, lg


__all__ = ["Model", "DeviceRotation", "Frame"]
