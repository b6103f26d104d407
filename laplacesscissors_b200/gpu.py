"""Gpu and Tensor: the per-op surface of the reference's src/gpu.rs over liblsx.

Method names, argument meaning and checks follow src/gpu.rs:133-559; every op
returns a new f32 Tensor on the device.  Errors raise LsxError with the library's
message (the reference returns anyhow errors).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import BF16, F16, F32, check, lib


@dataclass(frozen=True)
class NormConfig:  # src/gpu.rs:21-27
    groups: int
    width: int
    epsilon: float
    center: bool


@dataclass(frozen=True)
class RopeConfig:  # src/gpu.rs:28-35
    heads: int
    dim: int
    theta: float
    rotary: int
    interleaved: bool


@dataclass(frozen=True)
class AttentionConfig:  # src/gpu.rs:36-42
    qheads: int
    kvheads: int
    dim: int
    scale: float


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _dp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_double))


def _up(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


class Tensor:
    """Owned device buffer (src/gpu.rs:55-76); freed when dropped."""

    def __init__(self, handle: int, gpu: "Gpu", borrowed: bool = False):
        self._h = C.c_void_p(handle)
        self.gpu = gpu
        # A borrowed handle belongs to another object (e.g. a model's readout weight)
        # and is never released from here.
        self._borrowed = borrowed

    def __len__(self) -> int:
        return int(lib.lsx_tensor_len(self._h))

    @property
    def dtype(self) -> int:
        return int(lib.lsx_tensor_dtype(self._h))

    @property
    def data_ptr(self) -> int:
        return int(lib.lsx_tensor_data(self._h) or 0)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def free(self) -> None:
        if self._h and self._h.value and not self._borrowed:
            lib.lsx_tensor_free(self._h)  # for lsx_tensor_wrap views this frees the view only
        self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Gpu:
    """A device context and stream (Gpu + Device in the reference)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib.lsx_ctx_create(int(device), C.byref(h)))
        self._h = h
        self.device = int(device)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def close(self) -> None:
        if self._h and self._h.value:
            lib.lsx_ctx_destroy(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def name(self) -> str:
        buf = C.create_string_buffer(256)
        check(lib.lsx_ctx_name(self._h, buf, 256))
        return buf.value.decode()

    def backend(self) -> str:
        return "cuda"

    def architecture(self) -> str:
        a = C.c_int()
        check(lib.lsx_ctx_architecture(self._h, C.byref(a)))
        return str(a.value)

    def synchronize(self) -> None:
        check(lib.lsx_ctx_synchronize(self._h))

    def stream(self) -> int:
        s = C.c_void_p()
        check(lib.lsx_ctx_stream(self._h, C.byref(s)))
        return int(s.value or 0)

    # ---- buffers (src/gpu.rs:204-247)
    def _tensor(self, h: C.c_void_p) -> Tensor:
        return Tensor(h.value, self)

    def upload_raw(self, data: bytes | np.ndarray, kind: int) -> Tensor:
        buf = np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else \
            np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        h = C.c_void_p()
        check(lib.lsx_upload_raw(self._h, buf.ctypes.data_as(C.c_void_p), buf.nbytes, int(kind), C.byref(h)))
        return self._tensor(h)

    def upload_f32(self, data) -> Tensor:
        a = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
        h = C.c_void_p()
        check(lib.lsx_upload_f32(self._h, _fp(a), a.size, C.byref(h)))
        return self._tensor(h)

    def zeros(self, count: int) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_zeros(self._h, int(count), C.byref(h)))
        return self._tensor(h)

    def read(self, t: Tensor) -> np.ndarray:
        out = np.empty(len(t), dtype=np.float32)
        check(lib.lsx_read(self._h, t.handle, _fp(out), out.size))
        return out

    def wrap(self, device_pointer: int, count: int, kind: int) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_tensor_wrap(self._h, C.c_void_p(device_pointer), int(count), int(kind), C.byref(h)))
        return Tensor(h.value, self)

    # ---- ops (src/gpu.rs:360-559)
    def embedding(self, weight: Tensor, row: int, width: int) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_embedding(self._h, weight.handle, int(row), int(width), C.byref(h)))
        return self._tensor(h)

    def linear(self, x: Tensor, w: Tensor, bias: Tensor | None, rows: int, cols: int) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_linear(self._h, x.handle, w.handle, bias.handle if bias else None, int(rows), int(cols),
                             C.byref(h)))
        return self._tensor(h)

    def linear_into(self, x: Tensor, w: Tensor, bias: Tensor | None, rows: int, cols: int, out: Tensor) -> None:
        """linear() into an existing F32 tensor (no allocation, enqueue only)."""
        check(lib.lsx_linear_into(self._h, x.handle, w.handle, bias.handle if bias else None, int(rows), int(cols),
                                  out.handle))

    def norm(self, x: Tensor, gain: Tensor, bias: Tensor | None, config: NormConfig) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_norm(self._h, x.handle, gain.handle, bias.handle if bias else None, config.groups,
                           config.width, float(config.epsilon), int(config.center), C.byref(h)))
        return self._tensor(h)

    def rope(self, x: Tensor, position: int, config: RopeConfig) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_rope(self._h, x.handle, int(position), config.heads, config.dim, float(config.theta),
                           config.rotary, int(config.interleaved), C.byref(h)))
        return self._tensor(h)

    def attention(self, q: Tensor, k: Tensor, v: Tensor, cache: tuple[Tensor, Tensor], position: int,
                  config: AttentionConfig) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_attention(self._h, q.handle, k.handle, v.handle, cache[0].handle, cache[1].handle,
                                int(position), config.qheads, config.kvheads, config.dim, float(config.scale),
                                C.byref(h)))
        return self._tensor(h)

    def gated(self, gate: Tensor, up: Tensor, kind: int) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_gated(self._h, gate.handle, up.handle, int(kind), C.byref(h)))
        return self._tensor(h)

    def combine(self, x: Tensor, y: Tensor, factor: float) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_combine(self._h, x.handle, y.handle, float(factor), C.byref(h)))
        return self._tensor(h)

    def rotate(self, hidden: Tensor, u: Tensor, v: Tensor, a: float, b: float) -> Tensor:
        h = C.c_void_p()
        check(lib.lsx_rotate(self._h, hidden.handle, u.handle, v.handle, float(a), float(b), C.byref(h)))
        return self._tensor(h)


__all__ = ["Gpu", "Tensor", "NormConfig", "RopeConfig", "AttentionConfig", "F32", "F16", "BF16", "_lib"]
