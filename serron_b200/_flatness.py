"""Whether a structuring element is flat (every entry zero), remembered per tensor version.

Mirrors packages/serron/torch-ext/serron/_flatness.py:14-40: the answer is cached per tensor and
re-measured (one device-to-host read) only when the tensor's version counter moves.
"""

from __future__ import annotations

import torch
from torch.utils.weak import WeakTensorKeyDictionary

_cache: WeakTensorKeyDictionary = WeakTensorKeyDictionary()


def is_flat(kernel: torch.Tensor) -> bool:
    """``True`` when every entry of ``kernel`` is ``0``."""
    version = kernel._version
    cached = _cache.get(kernel)
    if cached is not None and cached[0] == version:
        return cached[1]
    flat = bool(kernel.eq(0).all().item())
    _cache[kernel] = (version, flat)
    return flat


def mark(kernel: torch.Tensor, flat: bool) -> torch.Tensor:
    """Record the flatness of ``kernel`` so its first use need not measure it; returns ``kernel``."""
    _cache[kernel] = (kernel._version, flat)
    return kernel
