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
and the backward searches the windows itself.  After the autocast forward the backward reads the float16
``grad_output`` and writes ``grad_input`` in the input's dtype directly (float32 sums in between), which
gives the values of the reference's casts up and down without making the copies.
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
    ctx.widened = False
    ctx.input_dtype = input_.dtype
    # grad mode is off inside Function.forward; needs_input_grad says whether a backward can follow
    wants_grad = any(ctx.needs_input_grad[:2])
    ctx.dtype = torch.promote_types(input_.dtype, kernel.dtype)
    if (wants_grad and int(algo) == 0 and input_.is_cuda and torch.is_autocast_enabled("cuda")
            and ctx.dtype == torch.float32 and _ops.autocast_fused_ok(input_, kernel.to(ctx.dtype))):
        kernel = kernel.to(ctx.dtype)
        ctx.save_for_backward(kernel)
        y, ctx.winners, ctx.winners_format = _ops.forward_autocast(op, input_, kernel, border)
        ctx.widened = True
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
    if ctx.widened and grad_output.dtype in (torch.float16, torch.bfloat16, torch.float32):
        # the casts of grad_output up to float32 and of grad_input down to the input's dtype happen inside
        # the gather (the same values, without the two copies)
        grad_input, grad_kernel = _ops.backward_from_winners_widened(
            ctx.op, grad_output, ctx.winners, ctx.winners_format, kernel, ctx.border, needs_kernel, ctx.input_dtype)
        return (grad_input if needs_input else None), (grad_kernel if needs_kernel else None), None, None
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


class _DerivedFunction(torch.autograd.Function):
    """A derived operation in one launch (``serron_derived_forward``), with the backward of the reference's
    composition (packages/serron/torch-ext/serron/functional.py:40-92) from the two stages' records:

    * gradient ``D(x) - E(x)``: grad_x = D'(go) - E'(go), grad_w = Dw(go) - Ew(go);
    * opening ``D(E(x))``: h = D'(go) over the intermediate, grad_x = E'(h), grad_w = Dw(go) + Ew(h);
    * closing ``E(D(x))``: the same with the operations swapped;
    * top_hat ``x - opening(x)``: grad_x = go - E'(D'(go)), grad_w = -(Dw(go) + Ew(h));
    * black_hat ``closing(x) - x``: grad_x = D'(E'(go)) - go, grad_w = Ew(go) + Dw(h).

    A gather of -g is the negated gather of g bit for bit (each sum is negated exactly), so these are the
    reference's autograd results: its sums of two gradient contributions are the same two values, and a
    sum of two values does not depend on their order.
    """

    @staticmethod
    def forward(ctx, input_: torch.Tensor, kernel: torch.Tensor, border: int, mode: int):
        y, win_a, win_b, fmt = _ops.derived_forward(mode, input_, kernel, border)
        ctx.save_for_backward(kernel)
        ctx.records = (win_a, win_b, fmt)
        ctx.border = border
        ctx.mode = mode
        return y

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        needs_input, needs_kernel = ctx.needs_input_grad[:2]
        if not (needs_input or needs_kernel):
            return None, None, None, None
        (kernel,) = ctx.saved_tensors
        win_a, win_b, fmt = ctx.records
        go = grad_output.to(kernel.dtype).contiguous()
        mode, border = ctx.mode, ctx.border

        def gather(op, g, records):
            return _ops.backward_from_winners(op, g, records, fmt, kernel, border, needs_kernel)

        if mode == _ops.DERIVED_GRADIENT:
            g_d, k_d = gather(_lib.DILATE, go, win_a)
            g_e, k_e = gather(_lib.ERODE, go, win_b)
            grad_input, grad_kernel = g_d - g_e, k_d - k_e
        else:
            first = _lib.ERODE if mode in (_ops.DERIVED_OPENING, _ops.DERIVED_TOP_HAT) else _lib.DILATE
            second = _lib.DILATE if first == _lib.ERODE else _lib.ERODE
            h, k_2 = gather(second, go, win_b)
            g_1, k_1 = gather(first, h, win_a)
            if mode == _ops.DERIVED_TOP_HAT:
                grad_input, grad_kernel = go - g_1, -(k_2 + k_1)
            elif mode == _ops.DERIVED_BLACK_HAT:
                grad_input, grad_kernel = g_1 - go, k_2 + k_1
            else:
                grad_input, grad_kernel = g_1, k_2 + k_1
        return (grad_input if needs_input else None), (grad_kernel if needs_kernel else None), None, None
