"""Autograd functions over the compiled operators.

Contract as packages/serron/torch-ext/serron/autograd.py:32-123: the input and the structuring
element are promoted to their common dtype and saved; the backward casts ``grad_output`` to that dtype
and returns grads only for the inputs that want them.

B200 difference: the forward also writes one winner record per output, and the backward gathers
straight from those records instead of searching every window again.  Without autocast the records come
from the forward itself.  Under CUDA autocast the value is computed on float16 casts while the backward
works in the promoted dtype, exactly like the reference; for odd square windows of 3 to 15 with a
float32 structuring element one kernel computes the float16 value and the promoted (float32) winners in
the same pass (so the promoted copy of the input is never made); other autocast calls keep no records
and the backward searches the windows itself.
"""

from __future__ import annotations

import torch

from . import _flatness, _lib, _ops
from ._autotune import ensure_loaded, select_algorithm
from ._ops import add_op_namespace_prefix, ops
from .enums import Algorithm

__all__ = ["_DilateFunction", "_ErodeFunction", "add_op_namespace_prefix", "ops"]


def _match_dtype(input_: torch.Tensor, kernel: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``(input_, kernel)`` cast to ``torch.promote_types`` of their dtypes."""
    dtype = torch.promote_types(input_.dtype, kernel.dtype)
    return input_.to(dtype), kernel.to(dtype)


def _autocast_cast(t: torch.Tensor) -> torch.Tensor:
    """The cast CUDA autocast applies to serron::erode/dilate arguments (float16; float64 untouched)."""
    if t.is_cuda and t.is_floating_point() and t.dtype is not torch.float64:
        return t.to(torch.float16)
    return t


def _forward(ctx, op: int, input_: torch.Tensor, kernel: torch.Tensor, border: int, algo: int) -> torch.Tensor:
    ensure_loaded(input_.device)
    flat = _flatness.is_flat(kernel)
    ctx.border = border
    ctx.flat = flat
    ctx.algo = int(algo)
    ctx.op = op
    ctx.winners = None
    ctx.winners_format = 0
    # grad mode is off inside Function.forward; needs_input_grad says whether a backward can follow
    wants_grad = any(ctx.needs_input_grad[:2])
    ctx.dtype = torch.promote_types(input_.dtype, kernel.dtype)
    if (wants_grad and int(algo) == 0 and input_.is_cuda and torch.is_autocast_enabled("cuda")
            and ctx.dtype == torch.float32 and _ops.autocast_fused_ok(input_, kernel.to(ctx.dtype))):
        kernel = kernel.to(ctx.dtype)
        ctx.save_for_backward(kernel)
        y, ctx.winners, ctx.winners_format = _ops.forward_autocast(op, input_, kernel, border)
        return y
    input_, kernel = _match_dtype(input_, kernel)
    ctx.save_for_backward(kernel, input_)
    algo = int(algo) or select_algorithm(input_, kernel, flat, backward=False)
    x, k = input_, kernel
    if input_.is_cuda and torch.is_autocast_enabled("cuda"):
        x, k = _autocast_cast(input_), _autocast_cast(kernel)
    if wants_grad and x.dtype == input_.dtype and input_.is_cuda and kernel.is_cuda:
        y, ctx.winners, ctx.winners_format = _ops.forward_with_winners(op, x, k, border, flat, algo)
        return y
    return _ops.forward(op, x, k, border, flat, algo)


def _backward(ctx, grad_output: torch.Tensor):
    needs_input, needs_kernel = ctx.needs_input_grad[:2]
    if not (needs_input or needs_kernel):
        return None, None, None, None
    kernel = ctx.saved_tensors[0]
    grad_output = grad_output.to(ctx.dtype).contiguous()
    if ctx.winners is not None:
        grad_input, grad_kernel = _ops.backward_from_winners(ctx.op, grad_output, ctx.winners, ctx.winners_format,
                                                             kernel, ctx.border, needs_kernel)
    else:
        input_ = ctx.saved_tensors[1]
        algo = ctx.algo or select_algorithm(input_, kernel, ctx.flat, backward=True)
        grad_input, grad_kernel = _ops.backward(ctx.op, grad_output, input_, kernel, ctx.border, ctx.flat,
                                                needs_kernel, algo)
    return (grad_input if needs_input else None), (grad_kernel if needs_kernel else None), None, None


class _ErodeFunction(torch.autograd.Function):
    """Autograd binding of ``serron::erode`` / ``serron::erode_backward``."""

    @staticmethod
    def forward(ctx, input_: torch.Tensor, kernel: torch.Tensor, border: int, algo: int = Algorithm.AUTO):
        return _forward(ctx, _lib.ERODE, input_, kernel, border, algo)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        return _backward(ctx, grad_output)


class _DilateFunction(torch.autograd.Function):
    """Autograd binding of ``serron::dilate`` / ``serron::dilate_backward``."""

    @staticmethod
    def forward(ctx, input_: torch.Tensor, kernel: torch.Tensor, border: int, algo: int = Algorithm.AUTO):
        return _forward(ctx, _lib.DILATE, input_, kernel, border, algo)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        return _backward(ctx, grad_output)
