"""serron_b200: B200-native (sm_100a) grayscale mathematical morphology for PyTorch.

A drop-in for the public API of Serron (vhrabar/serron 0.6.0, packages/serron/torch-ext/serron/__init__.py):
the same functions, layers, enums and structuring-element builders, and the same ``torch.ops.serron``
operator schemas, computed by hand-written CUDA kernels for sm_100a behind a C ABI
(``include/serron_b200.h``).  Results are bit-identical to the reference's CPU implementation.
"""

from __future__ import annotations

from importlib.metadata import PackageNotFoundError
from importlib.metadata import version as _version

from . import functional, structuring_element
from ._autotune import autotune, calibrate
from .enums import BorderMode, Operation
from .functional import (
    black_hat,
    closing,
    dilation,
    erosion,
    gradient,
    opening,
    reconstruction_by_dilation,
    reconstruction_by_erosion,
    top_hat,
)
from .modules import Closing2d, Dilation2d, Erosion2d, Opening2d

try:
    __version__ = _version("serron_b200")
except PackageNotFoundError:
    __version__ = "0.1.0"

__all__ = [
    "BorderMode",
    "Closing2d",
    "Dilation2d",
    "Erosion2d",
    "Opening2d",
    "Operation",
    "__version__",
    "autotune",
    "black_hat",
    "calibrate",
    "closing",
    "dilation",
    "erosion",
    "functional",
    "gradient",
    "opening",
    "reconstruction_by_dilation",
    "reconstruction_by_erosion",
    "structuring_element",
    "top_hat",
]
