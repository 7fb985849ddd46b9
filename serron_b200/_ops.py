"""The operator boundary: ``torch.ops.serron.*`` with the reference's schemas, backed by the C ABI.

The reference registers eight operators under ``serron::`` (packages/serron/csrc/bindings.cpp:8-19) and
an autocast rule for the two forwards (packages/serron/torch-ext/serron/_cmake_ops.py:175-189).  This
module registers the same schemas, implements them for CUDA by calling ``libserron_b200.so`` through
:mod:`serron_b200._lib`, and registers the same autocast rule.  The CPU key raises: this library has no
CPU path.

The functions below the registrations are what the autograd layer calls directly: they allocate
outputs, winner records and workspaces with torch's caching allocator and pass raw pointers on torch's
current stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_NAMESPACE = "serron"


# ------------------------------------------------------------------------------------------------
# validation the C ABI cannot do (it sees pointers, not devices or dtypes)
# ------------------------------------------------------------------------------------------------
def _check_tensors(name: str, input_: torch.Tensor, kernel: torch.Tensor, grad_output: torch.Tensor | None = None,
                   *, same_dtype: bool = True) -> None:
    if grad_output is not None and not grad_output.is_cuda:
        raise RuntimeError(f"{name}: grad_output must be a CUDA tensor")
    if not input_.is_cuda:
        raise RuntimeError(f"{name}: input must be a CUDA tensor")
    if not kernel.is_cuda:
        raise RuntimeError(f"{name}: kernel must be a CUDA tensor")
    if input_.dim() != 4:
        raise RuntimeError(f"{name}: input must be 4-D (N, C, H, W), got {input_.dim()}-D")
    if grad_output is not None and grad_output.dim() != 4:
        raise RuntimeError(f"{name}: grad_output must be 4-D (N, C, H, W), got {grad_output.dim()}-D")
    if kernel.dim() not in (2, 3):
        raise RuntimeError(f"{name}: kernel must be 2-D (kH, kW) or 3-D (C, kH, kW), got {kernel.dim()}-D")
    if same_dtype and input_.dtype != kernel.dtype:
        raise RuntimeError(f"{name}: input and kernel must share a dtype")
    if grad_output is not None and grad_output.dtype != input_.dtype:
        raise RuntimeError(f"{name}: grad_output and input must share a dtype")
    if input_.dtype not in _lib.DTYPE_CODE:
        raise RuntimeError(f"{name}: unsupported dtype {input_.dtype}")
    if input_.device != kernel.device or (grad_output is not None and grad_output.device != input_.device):
        raise RuntimeError(f"{name}: all tensors must be on one device")


def _flat_code(flat: bool | None) -> int:
    return -1 if flat is None else int(bool(flat))


# ------------------------------------------------------------------------------------------------
# calls
# ------------------------------------------------------------------------------------------------
def forward(op: int, input_: torch.Tensor, kernel: torch.Tensor, border: int, flat: bool | None = None,
            algo: int = 0) -> torch.Tensor:
    """serron::erode (op=0) / serron::dilate (op=1)."""
    name = "serron::erode" if op == _lib.ERODE else "serron::dilate"
    _check_tensors(name, input_, kernel)
    x = input_.contiguous()
    k = kernel.contiguous()
    out = torch.empty_like(x)
    xs, xd = _lib.sizes(x.shape)
    ks, kd = _lib.sizes(k.shape)
    fn = _lib.load().serron_erode if op == _lib.ERODE else _lib.load().serron_dilate
    rc = fn(x.data_ptr(), xs, xd, k.data_ptr(), ks, kd, _lib.DTYPE_CODE[x.dtype], int(border), _flat_code(flat),
            int(algo), out.data_ptr(), x.device.index, _lib.stream_of(x))
    _lib.raise_for(rc)
    return out


def plan(input_: torch.Tensor, kernel: torch.Tensor, flat: bool | None, algo: int, backward: bool) -> _lib.Plan:
    """How the library will run a call (resolved algorithm, winner format, backward workspace)."""
    k = kernel.contiguous()
    xs, xd = _lib.sizes(input_.shape)
    ks, kd = _lib.sizes(k.shape)
    p = _lib.Plan()
    rc = _lib.load().serron_plan(xs, xd, k.data_ptr(), ks, kd, _lib.DTYPE_CODE[input_.dtype], _flat_code(flat),
                                 int(algo), int(backward), input_.device.index, _lib.stream_of(input_),
                                 ctypes.byref(p))
    _lib.raise_for(rc)
    return p


def forward_with_winners(op: int, input_: torch.Tensor, kernel: torch.Tensor, border: int, flat: bool | None,
                         algo: int = 0) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Forward plus one winner record per output, for a later :func:`backward_from_winners`."""
    name = "serron::erode" if op == _lib.ERODE else "serron::dilate"
    _check_tensors(name, input_, kernel)
    x = input_.contiguous()
    k = kernel.contiguous()
    p = plan(x, k, flat, algo, backward=False)
    out = torch.empty_like(x)
    xs, xd = _lib.sizes(x.shape)
    if p.winners_format & _lib.WINNERS_MAP:
        # one byte buffer: the records, then the gather's target map
        nbytes = _lib.load().serron_winners_bytes(xs, xd, p.winners_format)
        if nbytes < 0:
            _lib.raise_for(_lib.ERR_INVALID)
        winners = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    else:
        winners = torch.empty(x.shape, dtype=_lib.WINNERS_TORCH_DTYPE[p.winners_format], device=x.device)
    ks, kd = _lib.sizes(k.shape)
    # the plan resolved the algorithm; a forced separable launch needs the flatness it was resolved with
    rc = _lib.load().serron_forward(op, x.data_ptr(), xs, xd, k.data_ptr(), ks, kd, _lib.DTYPE_CODE[x.dtype],
                                    int(border), 1 if p.algo == 3 else _flat_code(flat), p.algo, out.data_ptr(),
                                    winners.data_ptr(), p.winners_format, x.device.index, _lib.stream_of(x))
    _lib.raise_for(rc)
    return out, winners, p.winners_format


# the direct one-byte record format with the gather's target map (what the tiled algorithm plans for
# windows of up to 255 taps)
_WINNERS_DIRECT_U8_MAP = 1 | 0x10


def autocast_fused_ok(input_: torch.Tensor, kernel: torch.Tensor) -> bool:
    """The autocast forward with float32 winners (:func:`forward_autocast`) takes this call."""
    if input_.dim() != 4 or kernel.dim() not in (2, 3) or not (input_.is_cuda and kernel.is_cuda):
        return False
    if input_.dtype not in (torch.float32, torch.float16, torch.bfloat16) or kernel.dtype != torch.float32:
        return False
    kh, kw = kernel.shape[-2:]
    if kh != kw or kh % 2 == 0 or not 3 <= kh <= 15:
        return False
    return kernel.dim() == 2 or kernel.shape[0] == input_.shape[1]


def forward_autocast(op: int, input_: torch.Tensor, kernel: torch.Tensor, border: int
                     ) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Forward on float16 casts of ``input_`` and ``kernel`` (CUDA autocast) with the records of the float32
    winners, for a float32 :func:`backward_from_winners`."""
    name = "serron::erode" if op == _lib.ERODE else "serron::dilate"
    # the input and the float32 structuring element differ in dtype by design
    _check_tensors(name, input_, kernel, same_dtype=False)
    x = input_.contiguous()
    k = kernel.contiguous()
    out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    xs, xd = _lib.sizes(x.shape)
    lib = _lib.load()
    nbytes = lib.serron_winners_bytes(xs, xd, _WINNERS_DIRECT_U8_MAP)
    if nbytes < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    winners = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    ks, kd = _lib.sizes(k.shape)
    rc = lib.serron_forward_autocast(op, x.data_ptr(), xs, xd, _lib.DTYPE_CODE[x.dtype], k.data_ptr(), ks, kd,
                                     _lib.DTYPE_CODE[k.dtype], int(border), out.data_ptr(), winners.data_ptr(),
                                     _WINNERS_DIRECT_U8_MAP, x.device.index, _lib.stream_of(x))
    _lib.raise_for(rc)
    return out, winners, _WINNERS_DIRECT_U8_MAP


# derived operations in one launch (serron_derived_forward): the mode codes of the C ABI
DERIVED_GRADIENT, DERIVED_OPENING, DERIVED_CLOSING, DERIVED_TOP_HAT, DERIVED_BLACK_HAT = range(5)


def derived_supported(mode: int, input_: torch.Tensor, kernel: torch.Tensor) -> bool:
    """The one-launch form of derived operation ``mode`` takes this call (CUDA tensors of one dtype, a
    4-D input, a 2-D or per-channel 3-D kernel, windows up to 7 a side)."""
    if not (input_.is_cuda and kernel.is_cuda) or input_.dtype != kernel.dtype or input_.device != kernel.device:
        return False
    if input_.dtype not in _lib.DTYPE_CODE or input_.dim() != 4 or input_.numel() == 0:
        return False
    if kernel.dim() == 3 and kernel.shape[0] != input_.shape[1] or kernel.dim() not in (2, 3):
        return False
    xs, xd = _lib.sizes(input_.shape)
    ks, kd = _lib.sizes(kernel.shape)
    return bool(_lib.load().serron_derived_supported(mode, xs, xd, ks, kd))


def derived_forward(mode: int, input_: torch.Tensor, kernel: torch.Tensor, border: int
                    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Derived operation ``mode`` in one launch: the output and the records (with target maps) of its two
    primitive operations (gradient: dilation, erosion; others: first, second stage)."""
    x = input_.contiguous()
    k = kernel.contiguous()
    out = torch.empty_like(x)
    xs, xd = _lib.sizes(x.shape)
    ks, kd = _lib.sizes(k.shape)
    lib = _lib.load()
    nbytes = lib.serron_winners_bytes(xs, xd, _WINNERS_DIRECT_U8_MAP)
    if nbytes < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    win_a = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    win_b = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    rc = lib.serron_derived_forward(mode, x.data_ptr(), xs, xd, k.data_ptr(), ks, kd, _lib.DTYPE_CODE[x.dtype],
                                    int(border), out.data_ptr(), win_a.data_ptr(), win_b.data_ptr(),
                                    _WINNERS_DIRECT_U8_MAP, x.device.index, _lib.stream_of(x))
    _lib.raise_for(rc)
    return out, win_a, win_b, _WINNERS_DIRECT_U8_MAP


def backward(op: int, grad_output: torch.Tensor, input_: torch.Tensor, kernel: torch.Tensor, border: int,
             flat: bool | None = None, need_kernel_grad: bool = True, algo: int = 0
             ) -> tuple[torch.Tensor, torch.Tensor]:
    """serron::erode_backward (op=0) / serron::dilate_backward (op=1)."""
    name = "serron::erode_backward" if op == _lib.ERODE else "serron::dilate_backward"
    _check_tensors(name, input_, kernel, grad_output)
    go = grad_output.contiguous()
    x = input_.contiguous()
    k = kernel.contiguous()
    if go.shape != x.shape:
        raise RuntimeError(f"{name}: grad_output shape must match input")
    grad_input = torch.empty_like(x)
    grad_kernel = torch.empty_like(k)
    xs, xd = _lib.sizes(x.shape)
    ks, kd = _lib.sizes(k.shape)
    lib = _lib.load()
    ws_bytes = 0
    if x.numel() > 0:
        ws_bytes = plan(x, k, flat, algo, backward=True).workspace_bytes
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    fn = lib.serron_erode_backward if op == _lib.ERODE else lib.serron_dilate_backward
    rc = fn(go.data_ptr(), xs, xd, x.data_ptr(), xs, xd, k.data_ptr(), ks, kd, _lib.DTYPE_CODE[x.dtype], int(border),
            _flat_code(flat), int(bool(need_kernel_grad)), int(algo), grad_input.data_ptr(), grad_kernel.data_ptr(),
            workspace.data_ptr(), ws_bytes, x.device.index, _lib.stream_of(x))
    _lib.raise_for(rc)
    return grad_input, grad_kernel


def backward_from_winners(op: int, grad_output: torch.Tensor, winners: torch.Tensor, winners_format: int,
                          kernel: torch.Tensor, border: int, need_kernel_grad: bool
                          ) -> tuple[torch.Tensor, torch.Tensor]:
    """Backward from the records of :func:`forward_with_winners`; no winner search."""
    go = grad_output.contiguous()
    k = kernel.contiguous()
    grad_input = torch.empty_like(go)
    grad_kernel = torch.empty_like(k)
    xs, xd = _lib.sizes(go.shape)
    ks, kd = _lib.sizes(k.shape)
    lib = _lib.load()
    ws_bytes = lib.serron_backward_workspace_bytes(xs, xd, ks, kd, int(bool(need_kernel_grad)), winners_format, 1)
    if ws_bytes < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=go.device)
    rc = lib.serron_backward_from_winners(op, go.data_ptr(), xs, xd, ks, kd, _lib.DTYPE_CODE[go.dtype], int(border),
                                          int(bool(need_kernel_grad)), winners.data_ptr(), winners_format,
                                          grad_input.data_ptr(), grad_kernel.data_ptr(), workspace.data_ptr(),
                                          ws_bytes, go.device.index, _lib.stream_of(go))
    _lib.raise_for(rc)
    return grad_input, grad_kernel


def backward_from_winners_widened(op: int, grad_output: torch.Tensor, winners: torch.Tensor, winners_format: int,
                                  kernel: torch.Tensor, border: int, need_kernel_grad: bool,
                                  grad_input_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`backward_from_winners` in float32 arithmetic straight from a float16 / bfloat16 / float32
    ``grad_output``, with ``grad_input`` rounded to ``grad_input_dtype``: the same values as widening
    ``grad_output``, gathering in float32 and casting the result (``serron_backward_from_winners_widened``)."""
    go = grad_output.contiguous()
    k = kernel.contiguous()
    grad_input = torch.empty(go.shape, dtype=grad_input_dtype, device=go.device)
    grad_kernel = torch.empty_like(k)
    xs, xd = _lib.sizes(go.shape)
    ks, kd = _lib.sizes(k.shape)
    lib = _lib.load()
    ws_bytes = lib.serron_backward_workspace_bytes(xs, xd, ks, kd, int(bool(need_kernel_grad)), winners_format, 1)
    if ws_bytes < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=go.device)
    rc = lib.serron_backward_from_winners_widened(op, go.data_ptr(), _lib.DTYPE_CODE[go.dtype], xs, xd, ks, kd,
                                                  int(border), int(bool(need_kernel_grad)), winners.data_ptr(),
                                                  winners_format, grad_input.data_ptr(),
                                                  _lib.DTYPE_CODE[grad_input_dtype], grad_kernel.data_ptr(),
                                                  workspace.data_ptr(), ws_bytes, go.device.index, _lib.stream_of(go))
    _lib.raise_for(rc)
    return grad_input, grad_kernel


def reconstruct(dilate: bool, marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, border: int,
                max_iter: int | None, check_every: int, seed_rows: tuple[int, int] | None = None) -> torch.Tensor:
    """Geodesic reconstruction on CUDA tensors that already share a dtype and a device.

    ``seed_rows=(top, bottom)``: the marker is already at the fixed point except within ``top`` rows of the
    top edge and ``bottom`` rows of the bottom edge (``serron_reconstruct_from_edges``; fixed-point mode only).
    """
    name = "serron.reconstruction_by_dilation" if dilate else "serron.reconstruction_by_erosion"
    _check_tensors(name, marker, kernel)
    m = marker.contiguous()
    mk = mask.contiguous()
    k = kernel.contiguous()
    out = torch.empty_like(m)
    xs, xd = _lib.sizes(m.shape)
    ks, kd = _lib.sizes(k.shape)
    lib = _lib.load()
    mi = 0 if max_iter is None else int(max_iter)
    ws_bytes = lib.serron_reconstruct_workspace_bytes(xs, xd, _lib.DTYPE_CODE[m.dtype], mi)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=m.device)
    steps = ctypes.c_int64(0)
    if seed_rows is None:
        rc = lib.serron_reconstruct(int(dilate), m.data_ptr(), mk.data_ptr(), xs, xd, k.data_ptr(), ks, kd,
                                    _lib.DTYPE_CODE[m.dtype], int(border), mi, int(check_every), out.data_ptr(),
                                    workspace.data_ptr(), ws_bytes, m.device.index, _lib.stream_of(m),
                                    ctypes.byref(steps))
    else:
        if mi > 0:
            raise RuntimeError(f"{name}: an edge-seeded reconstruction runs to the fixed point (max_iter=None)")
        rc = lib.serron_reconstruct_from_edges(int(dilate), m.data_ptr(), mk.data_ptr(), xs, xd, k.data_ptr(), ks,
                                               kd, _lib.DTYPE_CODE[m.dtype], int(border), int(seed_rows[0]),
                                               int(seed_rows[1]), out.data_ptr(), workspace.data_ptr(), ws_bytes,
                                               m.device.index, _lib.stream_of(m), ctypes.byref(steps))
    _lib.raise_for(rc)
    return out


def _flat_of(kernel: torch.Tensor, flat: bool | None) -> int:
    if flat is None:
        return int(bool(kernel.eq(0).all().item()))
    return int(bool(flat))


def feasible_algos(input_: torch.Tensor, kernel: torch.Tensor, flat: bool | None = None, backward: bool = False) -> int:
    _check_selection("serron::feasible_algos", input_, kernel)
    ks, kd = _lib.sizes(kernel.shape)
    v = _lib.load().serron_feasible_algos(ks, kd, _lib.DTYPE_CODE[input_.dtype], _flat_of(kernel, flat),
                                          int(backward), input_.device.index)
    if v < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    return int(v)


def heuristic_algo(input_: torch.Tensor, kernel: torch.Tensor, flat: bool | None = None, backward: bool = False) -> int:
    _check_selection("serron::heuristic_algo", input_, kernel)
    ks, kd = _lib.sizes(kernel.shape)
    v = _lib.load().serron_heuristic_algo(ks, kd, _lib.DTYPE_CODE[input_.dtype], _flat_of(kernel, flat),
                                          int(backward), input_.device.index)
    if v < 0:
        _lib.raise_for(_lib.ERR_INVALID)
    return int(v)


def set_separable_min_k(like: torch.Tensor, backward: bool, min_k: int) -> int:
    if not like.is_cuda:
        raise RuntimeError("serron::set_separable_min_k: like must be a CUDA tensor")
    return int(_lib.load().serron_set_separable_min_k(like.device.index, _lib.DTYPE_CODE[like.dtype], int(backward),
                                                      int(min_k)))


def get_separable_min_k(like: torch.Tensor, backward: bool) -> int:
    if not like.is_cuda:
        raise RuntimeError("serron::get_separable_min_k: like must be a CUDA tensor")
    return int(_lib.load().serron_get_separable_min_k(like.device.index, _lib.DTYPE_CODE[like.dtype], int(backward)))


def _check_selection(name: str, input_: torch.Tensor, kernel: torch.Tensor) -> None:
    if not input_.is_cuda:
        raise RuntimeError(f"{name}: input must be a CUDA tensor")
    if not kernel.is_cuda:
        raise RuntimeError(f"{name}: kernel must be a CUDA tensor")
    if kernel.dim() not in (2, 3):
        raise RuntimeError(f"{name}: kernel must be 2-D (kH, kW) or 3-D (C, kH, kW), got {kernel.dim()}-D")


# ------------------------------------------------------------------------------------------------
# torch.ops.serron registration (schemas: packages/serron/csrc/bindings.cpp:8-19)
# ------------------------------------------------------------------------------------------------
_SCHEMAS = {
    "erode": "erode(Tensor input, Tensor kernel, int border, bool? flat=None, int algo=0) -> Tensor",
    "dilate": "dilate(Tensor input, Tensor kernel, int border, bool? flat=None, int algo=0) -> Tensor",
    "erode_backward": "erode_backward(Tensor grad_output, Tensor input, Tensor kernel, int border, bool? flat=None, "
                      "bool need_kernel_grad=True, int algo=0) -> (Tensor, Tensor)",
    "dilate_backward": "dilate_backward(Tensor grad_output, Tensor input, Tensor kernel, int border, bool? flat=None, "
                       "bool need_kernel_grad=True, int algo=0) -> (Tensor, Tensor)",
    "feasible_algos": "feasible_algos(Tensor input, Tensor kernel, bool? flat=None, bool backward=False) -> int",
    "heuristic_algo": "heuristic_algo(Tensor input, Tensor kernel, bool? flat=None, bool backward=False) -> int",
    "set_separable_min_k": "set_separable_min_k(Tensor like, bool backward, int min_k) -> int",
    "get_separable_min_k": "get_separable_min_k(Tensor like, bool backward) -> int",
}

_IMPLS = {
    "erode": lambda input, kernel, border, flat=None, algo=0: forward(_lib.ERODE, input, kernel, border, flat, algo),
    "dilate": lambda input, kernel, border, flat=None, algo=0: forward(_lib.DILATE, input, kernel, border, flat, algo),
    "erode_backward": lambda grad_output, input, kernel, border, flat=None, need_kernel_grad=True, algo=0: backward(
        _lib.ERODE, grad_output, input, kernel, border, flat, need_kernel_grad, algo),
    "dilate_backward": lambda grad_output, input, kernel, border, flat=None, need_kernel_grad=True, algo=0: backward(
        _lib.DILATE, grad_output, input, kernel, border, flat, need_kernel_grad, algo),
    "feasible_algos": feasible_algos,
    "heuristic_algo": heuristic_algo,
    "set_separable_min_k": set_separable_min_k,
    "get_separable_min_k": get_separable_min_k,
}


def _cpu_reject(name: str):
    def reject(*args, **kwargs):
        raise RuntimeError(f"serron::{name}: input must be a CUDA tensor (serron_b200 has no CPU path)")

    return reject


def _register() -> torch.library.Library | None:
    try:
        lib = torch.library.Library(_NAMESPACE, "DEF")
    except RuntimeError as exc:  # another library already owns serron:: in this process
        raise ImportError(f"serron_b200: cannot register the serron:: operators: {exc}") from exc
    for name, schema in _SCHEMAS.items():
        lib.define(schema)
        lib.impl(name, _IMPLS[name], "CUDA")
        lib.impl(name, _cpu_reject(name), "CPU")
    for name in ("erode", "dilate"):
        torch.library.register_autocast(f"{_NAMESPACE}::{name}", "cuda", torch.float16, lib=lib)
        torch.library.register_autocast(f"{_NAMESPACE}::{name}", "cpu", torch.bfloat16, lib=lib)
    return lib


_LIBRARY = _register()
ops = getattr(torch.ops, _NAMESPACE)


def add_op_namespace_prefix(op_name: str) -> str:
    return f"{_NAMESPACE}::{op_name}"
