"""laplacesscissors_b200: B200-native decode and readout-validation path of
LaplacesScissors (CUDA sm_100a kernels behind the C ABI of include/lsx.h).

Importing the package loads liblsx.so and raises if it is missing: no entry point
has a Python or CPU substitute.
"""
from . import _lib
from ._lib import LsxError, library_path
from .gpu import AttentionConfig, Gpu, NormConfig, RopeConfig, Tensor
from .model import DeviceRotation, Frame, Model
from .rotation import ReadoutRotation, SubspaceRotation, random_subspace_rotation

__version__ = "0.1.0"

__all__ = [
    "Gpu", "Tensor", "NormConfig", "RopeConfig", "AttentionConfig", "Model", "DeviceRotation", "Frame",
    "ReadoutRotation", "SubspaceRotation", "random_subspace_rotation", "LsxError", "library_path",
]
