"""Structuring-element builders.

Same builders, shapes, values and errors as packages/serron/torch-ext/serron/structuring_element.py:
``square`` is all zeros and marked flat; ``cross``, ``disk`` and ``diamond`` are 0 inside the shape and
-inf outside, and are marked not flat (they run on the 2-D path).
"""

from __future__ import annotations

import torch

from . import _flatness

_OUTSIDE = float("-inf")


def _checked_dtype(dtype: torch.dtype) -> torch.dtype:
    if not dtype.is_floating_point:
        raise ValueError(f"structuring elements must use a floating dtype, got {dtype}")
    return dtype


def _mask_se(inside: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """0 where ``inside``, -inf elsewhere; recorded as not flat without inspecting it."""
    return _flatness.mark(torch.where(inside, 0.0, _OUTSIDE).to(dtype), False)


def _offsets(size: int, device: torch.device | str | None) -> tuple[torch.Tensor, torch.Tensor]:
    axis = torch.arange(size, device=device) - (size - 1) // 2
    return torch.meshgrid(axis, axis, indexing="ij")


def square(size: int, *, dtype: torch.dtype = torch.float32, device: torch.device | str | None = None) -> torch.Tensor:
    """Flat ``(size, size)`` square (all zeros)."""
    if size < 1:
        raise ValueError(f"size must be >= 1, got {size}")
    return _flatness.mark(torch.zeros(size, size, dtype=_checked_dtype(dtype), device=device), True)


def cross(size: int, *, dtype: torch.dtype = torch.float32, device: torch.device | str | None = None) -> torch.Tensor:
    """``(size, size)`` cross: the centre row and column."""
    if size < 1:
        raise ValueError(f"size must be >= 1, got {size}")
    dy, dx = _offsets(size, device)
    return _mask_se((dy == 0) | (dx == 0), _checked_dtype(dtype))


def disk(radius: int, *, dtype: torch.dtype = torch.float32, device: torch.device | str | None = None) -> torch.Tensor:
    """``(2r+1, 2r+1)`` disk: offsets with dx^2 + dy^2 <= r^2."""
    if radius < 0:
        raise ValueError(f"radius must be >= 0, got {radius}")
    dy, dx = _offsets(2 * radius + 1, device)
    return _mask_se(dx * dx + dy * dy <= radius * radius, _checked_dtype(dtype))


def diamond(radius: int, *, dtype: torch.dtype = torch.float32, device: torch.device | str | None = None) -> torch.Tensor:
    """``(2r+1, 2r+1)`` diamond: offsets with |dx| + |dy| <= r."""
    if radius < 0:
        raise ValueError(f"radius must be >= 0, got {radius}")
    dy, dx = _offsets(2 * radius + 1, device)
    return _mask_se(dx.abs() + dy.abs() <= radius, _checked_dtype(dtype))


def from_tensor(weights: torch.Tensor, *, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """An arbitrary 2-D tensor of weights as a grayscale structuring element."""
    if weights.dim() != 2:
        raise ValueError(f"expected a 2-D (kh, kw) tensor, got shape {tuple(weights.shape)}")
    return weights.to(_checked_dtype(dtype))
