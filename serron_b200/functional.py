"""Stateless morphology on CUDA tensors.

Same functions, signatures, defaults and errors as packages/serron/torch-ext/serron/functional.py.
``erosion`` / ``dilation`` go through the autograd functions.  The derived operations run in one launch
(``serron_derived_forward``: both extremes from one staged tile for the gradient, the intermediate image
in shared memory for the others) when the input and the structuring element share a dtype, autocast is
off and the window is at most 7 a side; otherwise they are the reference's compositions.  Both give the
same bits.  The reconstructions run on the library's fixed-point solver instead of a Python loop.
"""

from __future__ import annotations

import torch

from . import _flatness, _ops
from ._autotune import ensure_loaded
from .autograd import _DerivedFunction, _DilateFunction, _ErodeFunction
from .enums import BORDER_TO_INT, BorderMode


def erosion(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Grayscale erosion (sliding minimum of ``input - kernel``)."""
    return _ErodeFunction.apply(input_, kernel, BORDER_TO_INT[border])


def dilation(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Grayscale dilation (sliding maximum of ``input + kernel``)."""
    return _DilateFunction.apply(input_, kernel, BORDER_TO_INT[border])


def _fused(mode: int, input_: torch.Tensor, kernel: torch.Tensor) -> bool:
    """Whether derived operation ``mode`` runs in one launch for these arguments (same bits either way)."""
    return (isinstance(input_, torch.Tensor) and isinstance(kernel, torch.Tensor) and input_.is_cuda
            and not torch.is_autocast_enabled("cuda") and _ops.derived_supported(mode, input_, kernel))


def opening(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Erosion followed by dilation."""
    if _fused(_ops.DERIVED_OPENING, input_, kernel):
        return _DerivedFunction.apply(input_, kernel, BORDER_TO_INT[border], _ops.DERIVED_OPENING)
    return dilation(erosion(input_, kernel, border=border), kernel, border=border)


def closing(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Dilation followed by erosion."""
    if _fused(_ops.DERIVED_CLOSING, input_, kernel):
        return _DerivedFunction.apply(input_, kernel, BORDER_TO_INT[border], _ops.DERIVED_CLOSING)
    return erosion(dilation(input_, kernel, border=border), kernel, border=border)


def gradient(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Morphological gradient ``dilation(input) - erosion(input)``."""
    if _fused(_ops.DERIVED_GRADIENT, input_, kernel):
        return _DerivedFunction.apply(input_, kernel, BORDER_TO_INT[border], _ops.DERIVED_GRADIENT)
    return dilation(input_, kernel, border=border) - erosion(input_, kernel, border=border)


def top_hat(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """White top-hat ``input - opening(input)``."""
    if _fused(_ops.DERIVED_TOP_HAT, input_, kernel):
        return _DerivedFunction.apply(input_, kernel, BORDER_TO_INT[border], _ops.DERIVED_TOP_HAT)
    return input_ - opening(input_, kernel, border=border)


def black_hat(input_: torch.Tensor, kernel: torch.Tensor, *, border: BorderMode = BorderMode.REPLICATE) -> torch.Tensor:
    """Black top-hat ``closing(input) - input``."""
    if _fused(_ops.DERIVED_BLACK_HAT, input_, kernel):
        return _DerivedFunction.apply(input_, kernel, BORDER_TO_INT[border], _ops.DERIVED_BLACK_HAT)
    return closing(input_, kernel, border=border) - input_


_DEFAULT_CHECK_EVERY = 16


def _align_inputs(marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, name: str
                  ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, bool]:
    """Validate a reconstruction's three tensors and bring them to their common dtype."""
    if marker.shape != mask.shape:
        raise ValueError(f"{name}: marker and mask must share a shape, got {tuple(marker.shape)} and {tuple(mask.shape)}")
    if marker.device != mask.device or marker.device != kernel.device:
        raise ValueError(
            f"{name}: marker, mask and kernel must be on one device, got {marker.device}, {mask.device} and {kernel.device}"
        )
    if torch.is_grad_enabled() and (marker.requires_grad or mask.requires_grad or kernel.requires_grad):
        raise RuntimeError(f"{name}: reconstruction has no backward pass yet; run it under torch.no_grad() or detach its inputs")
    dtype = torch.promote_types(torch.promote_types(marker.dtype, mask.dtype), kernel.dtype)
    flat = _flatness.is_flat(kernel)
    return marker.to(dtype), mask.to(dtype), _flatness.mark(kernel.to(dtype), flat), flat


def _require_nonnegative_anchor(kernel: torch.Tensor, name: str) -> None:
    """A negative (or NaN) anchor tap would make the geodesic step non-monotone."""
    ah, aw = kernel.shape[-2] // 2, kernel.shape[-1] // 2
    if not bool((kernel[..., ah, aw] >= 0).all().item()):
        raise ValueError(
            f"{name}: the structuring element's anchor tap kernel[..., {ah}, {aw}] must be >= 0, "
            f"otherwise the geodesic iteration is not monotone and need not converge"
        )


def _reconstruct(marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, border: BorderMode, *,
                 dilate: bool, max_iter: int | None, check_every: int, name: str) -> torch.Tensor:
    if check_every < 1:
        raise ValueError(f"{name}: check_every must be >= 1, got {check_every}")
    if max_iter is not None and max_iter < 1:
        raise ValueError(f"{name}: max_iter must be >= 1 or None, got {max_iter}")
    marker, mask, kernel, flat = _align_inputs(marker, mask, kernel, name)
    if not flat:
        _require_nonnegative_anchor(kernel, name)
    ensure_loaded(marker.device)
    with torch.no_grad():
        return _ops.reconstruct(dilate, marker, mask, kernel, BORDER_TO_INT[border], max_iter, check_every)


def reconstruction_by_dilation(marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, *,
                               border: BorderMode = BorderMode.CONSTANT, max_iter: int | None = None,
                               check_every: int = _DEFAULT_CHECK_EVERY) -> torch.Tensor:
    """Fixed point of ``min(dilation(y), mask)`` from ``y = min(marker, mask)``.

    ``max_iter`` bounds the reference's Jacobi iteration count: with it set the reference's schedule is
    replayed and the call raises exactly when the reference would; without it the fixed point is found
    by tile-local relaxation, which reaches the same (unique) fixed point far sooner.
    """
    return _reconstruct(marker, mask, kernel, border, dilate=True, max_iter=max_iter, check_every=check_every,
                        name="serron.reconstruction_by_dilation")


def reconstruction_by_erosion(marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, *,
                              border: BorderMode = BorderMode.CONSTANT, max_iter: int | None = None,
                              check_every: int = _DEFAULT_CHECK_EVERY) -> torch.Tensor:
    """Fixed point of ``max(erosion(y), mask)`` from ``y = max(marker, mask)`` (the dual)."""
    return _reconstruct(marker, mask, kernel, border, dilate=False, max_iter=max_iter, check_every=check_every,
                        name="serron.reconstruction_by_erosion")
