"""ctypes binding of liblsx.so (include/lsx.h).

The native library is the product: if it is missing or cannot be loaded, importing
this module raises -- there is no Python or CPU substitute for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "liblsx.so"

F32, F16, BF16 = 0, 1, 2

OK = 0
E_ARGUMENT, E_MEMORY, E_CUDA, E_NONFINITE, E_IO, E_FORMAT, E_UNSUPPORTED, E_STATE = range(1, 9)


class LsxError(RuntimeError):
    """A liblsx call failed; `status` is the lsx_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


class ModelInfo(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_uint64), ("vocab_size", C.c_uint64), ("layers", C.c_uint64),
        ("capacity", C.c_uint64), ("position", C.c_uint64), ("query_heads", C.c_uint64),
        ("kv_heads", C.c_uint64), ("head_dim", C.c_uint64), ("intermediate_size", C.c_uint64),
        ("rotary_dim", C.c_uint64), ("parameters", C.c_uint64), ("tensors", C.c_uint64),
        ("eos_count", C.c_uint64), ("eos_token_ids", C.c_uint32 * 8), ("fused", C.c_uint64),
        ("graph", C.c_uint64), ("kernels_per_step", C.c_uint64), ("persistent", C.c_uint64),
    ]


P = C.c_void_p
PP = C.POINTER(C.c_void_p)
SZ = C.c_size_t
I = C.c_int
U32 = C.c_uint32
U64 = C.c_uint64
F = C.c_float
D = C.c_double
FP = C.POINTER(C.c_float)
DP = C.POINTER(C.c_double)
UP = C.POINTER(C.c_uint32)

# name -> (restype, argtypes).  Every function declared in include/lsx.h appears here.
SIGNATURES = {
    "lsx_last_error": (C.c_char_p, []),
    "lsx_version": (C.c_char_p, []),
    "lsx_ctx_create": (I, [I, PP]),
    "lsx_ctx_destroy": (I, [P]),
    "lsx_ctx_synchronize": (I, [P]),
    "lsx_ctx_name": (I, [P, C.c_char_p, SZ]),
    "lsx_ctx_architecture": (I, [P, C.POINTER(I)]),
    "lsx_ctx_stream": (I, [P, PP]),
    "lsx_upload_raw": (I, [P, P, SZ, I, PP]),
    "lsx_upload_f32": (I, [P, FP, SZ, PP]),
    "lsx_zeros": (I, [P, SZ, PP]),
    "lsx_read": (I, [P, P, FP, SZ]),
    "lsx_tensor_free": (I, [P]),
    "lsx_tensor_len": (SZ, [P]),
    "lsx_tensor_dtype": (I, [P]),
    "lsx_tensor_data": (P, [P]),
    "lsx_tensor_wrap": (I, [P, P, SZ, I, PP]),
    "lsx_embedding": (I, [P, P, SZ, SZ, PP]),
    "lsx_linear": (I, [P, P, P, P, SZ, SZ, PP]),
    "lsx_linear_into": (I, [P, P, P, P, SZ, SZ, P]),
    "lsx_norm": (I, [P, P, P, P, SZ, SZ, F, I, PP]),
    "lsx_rope": (I, [P, P, SZ, SZ, SZ, F, SZ, I, PP]),
    "lsx_attention": (I, [P, P, P, P, P, P, SZ, SZ, SZ, SZ, F, PP]),
    "lsx_gated": (I, [P, P, P, U32, PP]),
    "lsx_combine": (I, [P, P, P, F, PP]),
    "lsx_rotate": (I, [P, P, P, P, F, F, PP]),
    "lsx_rotation_plane": (I, [P, DP, DP, D, SZ, PP]),
    "lsx_rotation_joint": (I, [P, DP, DP, SZ, SZ, PP]),
    "lsx_rotation_apply": (I, [P, P, P, PP]),
    "lsx_rotation_free": (I, [P]),
    "lsx_model_load": (I, [P, C.c_char_p, SZ, PP]),
    "lsx_model_free": (I, [P]),
    "lsx_model_info_get": (I, [P, C.POINTER(ModelInfo)]),
    "lsx_model_fused": (I, [P]),
    "lsx_model_reset": (I, [P]),
    "lsx_model_rewind": (I, [P, SZ]),
    "lsx_model_advance": (I, [P, U32, P, FP, FP, UP]),
    "lsx_model_inject": (I, [P, FP, P, FP, FP, UP]),
    "lsx_model_embedding_vector": (I, [P, U32, FP]),
    "lsx_model_readout": (I, [P, FP, P, FP]),
    "lsx_model_head_image": (I, [P, DP, FP]),
    "lsx_model_head_row": (I, [P, U32, FP]),
    "lsx_model_head_images": (I, [P, DP, SZ, FP]),
    "lsx_model_head": (I, [P, PP, PP]),
    "lsx_model_generate": (I, [P, UP, SZ, SZ, UP, SZ, P, UP, C.POINTER(SZ), C.POINTER(I), FP, FP]),
    "lsx_model_score": (I, [P, UP, SZ, UP, SZ, P, DP, UP, FP, FP]),
    "lsx_model_generate_batch": (I, [P, UP, SZ, SZ, SZ, UP]),
    "lsx_model_score_batch": (I, [P, UP, SZ, SZ, UP, SZ, P, DP, UP, DP, FP]),
    "lsx_readout_margin": (I, [P, P, P, SZ, SZ, P, I, SZ, UP, P, DP, UP, FP]),
    "lsx_readout_margin_device": (I, [P, P, P, SZ, SZ, P, I, SZ, P, P, P, P, P, P, SZ]),
    "lsx_readout_workspace_bytes": (SZ, [SZ, SZ, SZ, P]),
    "lsx_readout_status": (I, [P, P]),
    "lsx_readout_margin_fixed": (I, [P, P, P, SZ, SZ, P, I, SZ, P, P, P, P]),
    "lsx_compact_margin": (I, [P, P, P, SZ, SZ, SZ, FP, UP, DP, UP, UP]),
    "lsx_readout_shard_device": (I, [P, P, P, SZ, SZ, SZ, P, I, SZ, P, P, P, P, P, SZ]),
    "lsx_readout_merge_device": (I, [P, P, P, P, SZ, P, P, P]),
    "lsx_readout_partials_device": (I, [P, P, P, SZ, SZ, SZ, P, I, SZ, P, P, P, P, SZ]),
    "lsx_readout_partials_merge_device": (I, [P, P, P, SZ, P, P, P]),
    "lsx_feasible_create": (I, [D, PP]),
    "lsx_feasible_free": (I, [P]),
    "lsx_feasible_constrain": (I, [P, D, D, D]),
    "lsx_feasible_is_empty": (I, [P]),
    "lsx_feasible_nearest": (I, [P, DP, C.POINTER(I)]),
    "lsx_feasible_intervals": (SZ, [P, DP, SZ]),
    "lsx_feasible_work": (I, [P, C.POINTER(C.c_uint64)]),
    "lsx_plane_feasible": (I, [P, P, FP, FP, SZ, FP, UP, DP, DP, SZ, D, D]),
    "lsx_integrated_credits": (I, [P, P, P, UP, DP, SZ, SZ, SZ, DP, UP, SZ, DP, DP]),
    "lsx_synth_normal": (I, [U64, U64, U64, SZ, D, I, P]),
    "lsx_synth_uniform_u32": (I, [U64, U64, U64, SZ, U32, UP]),
}


def _load() -> C.CDLL:
    path = os.environ.get("LSX_LIBRARY", str(LIBRARY))
    if not Path(path).exists():
        raise ImportError(
            f"liblsx.so not found at {path}; build it with `python laplacesscissors_b200/build.py` "
            "(the CUDA library is required: there is no fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int) -> None:
    if status != OK:
        raise LsxError(status, lib.lsx_last_error().decode(errors="replace"))


def library_path() -> str:
    return os.environ.get("LSX_LIBRARY", str(LIBRARY))
