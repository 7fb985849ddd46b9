"""ORACLE -- test infrastructure only.

A CPU restatement of the reference's grayscale morphology (vhrabar/serron 0.6.0,
``packages/serron/csrc/cpu/morphology/*`` and ``torch-ext/serron/functional.py``),
compiled from ``oracle/morph_oracle.c`` into ``oracle/liboracle.so``.

It checks the CUDA product path.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` may import it, and only as the checker or the timed
CPU baseline; the product never calls it.

Parity of the restatement is pinned against golden vectors that the reference itself
produced (``tests/golden/make_golden.py``), and, where the reference sources are
present, against the reference's own CPU operators compiled from those sources
(``make -C oracle ref`` -> ``oracle/_ref/serron_ref_C.so``, namespace ``serron_ref``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(_HERE, "_ref", "serron_ref_C.so")

ERODE, DILATE = 0, 1
_DTYPE_CODE = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}

_lib: ctypes.CDLL | None = None


def build() -> None:
    """Compile ``liboracle.so`` (and nothing else)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        i64, vp, ci = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        lib.oracle_forward.argtypes = [ci, ci, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, ci, ci]
        lib.oracle_forward.restype = ci
        lib.oracle_winners.argtypes = [ci, ci, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, ci, ci]
        lib.oracle_winners.restype = ci
        lib.oracle_backward.argtypes = [ci, ci, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, ci, ci, ci]
        lib.oracle_backward.restype = ci
        lib.oracle_reconstruct.argtypes = [ci, ci, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, ci, ci, i64, i64]
        lib.oracle_reconstruct.restype = i64
        lib.oracle_reconstruct_flood.argtypes = [ci, ci, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, ci]
        lib.oracle_reconstruct_flood.restype = ci
        _lib = lib
    return _lib


def _geometry(x: torch.Tensor, w: torch.Tensor) -> tuple[int, int, int, int, int, int, int]:
    if x.dim() != 4 or w.dim() not in (2, 3):
        raise ValueError("oracle: x must be (N, C, H, W) and w (kH, kW) or (C, kH, kW)")
    N, C, H, W = x.shape
    kH, kW = w.shape[-2:]
    kcs = kH * kW if w.dim() == 3 else 0
    return N, C, H, W, kH, kW, kcs


def _prep(*tensors: torch.Tensor) -> list[torch.Tensor]:
    out = [t.detach().to("cpu").contiguous() for t in tensors]
    dtypes = {t.dtype for t in out}
    if len(dtypes) != 1 or out[0].dtype not in _DTYPE_CODE:
        raise ValueError(f"oracle: tensors must share one of {list(_DTYPE_CODE)}, got {dtypes}")
    return out


def is_flat(w: torch.Tensor) -> bool:
    """Every entry is zero (torch-ext/serron/_flatness.py:14-28)."""
    return bool(w.eq(0).all().item())


def forward(op: int, x: torch.Tensor, w: torch.Tensor, border: int, *, separable: bool = False) -> torch.Tensor:
    """erode (op=0) / dilate (op=1).  ``separable`` runs the line passes (flat SE only)."""
    x, w = _prep(x, w)
    if separable and not is_flat(w):
        raise ValueError("oracle: the separable passes need a flat structuring element")
    y = torch.empty_like(x)
    rc = _load().oracle_forward(op, _DTYPE_CODE[x.dtype], x.data_ptr(), w.data_ptr(), y.data_ptr(),
                                *_geometry(x, w), border, int(separable))
    if rc:
        raise ValueError(f"oracle_forward: bad argument ({rc})")
    return y


def winners(op: int, x: torch.Tensor, w: torch.Tensor, border: int, *, separable: bool = False
            ) -> tuple[torch.Tensor, torch.Tensor]:
    """Flat offsets of the winning input pixel and SE cell per output (-1: none)."""
    x, w = _prep(x, w)
    bi = torch.empty(x.shape, dtype=torch.int64)
    bk = torch.empty(x.shape, dtype=torch.int64)
    rc = _load().oracle_winners(op, _DTYPE_CODE[x.dtype], x.data_ptr(), w.data_ptr(), bi.data_ptr(), bk.data_ptr(),
                                *_geometry(x, w), border, int(separable))
    if rc:
        raise ValueError(f"oracle_winners: bad argument ({rc})")
    return bi, bk


def backward(op: int, go: torch.Tensor, x: torch.Tensor, w: torch.Tensor, border: int, *,
             separable: bool = False, need_kernel_grad: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(grad_input, grad_kernel) with the reference's serial raster-order scatter."""
    go, x, w = _prep(go, x, w)
    if go.shape != x.shape:
        raise ValueError("oracle: grad_output shape must match input")
    gi = torch.empty_like(x)
    gk = torch.empty_like(w)
    rc = _load().oracle_backward(op, _DTYPE_CODE[x.dtype], go.data_ptr(), x.data_ptr(), w.data_ptr(), gi.data_ptr(),
                                 gk.data_ptr(), *_geometry(x, w), border, int(separable), int(need_kernel_grad))
    if rc:
        raise ValueError(f"oracle_backward: bad argument ({rc})")
    return gi, gk


def grad_kernel_wide(op: int, go: torch.Tensor, x: torch.Tensor, w: torch.Tensor, border: int, *,
                     separable: bool = False) -> torch.Tensor:
    """grad_kernel summed in float64 and rounded once to the storage type.

    The reference's CPU backward rounds half/bfloat16 sums to the storage type after every add
    (csrc/cpu/morphology/backward.cpp:250-263), so its grad_kernel drifts with the number of terms;
    its CUDA backward accumulates in float and rounds once (csrc/gpu/morphology/backward.cpp:196-203).
    This is that single-rounding semantics, on the oracle's (bit-exact) winners.
    """
    go_c, x_c, w_c = _prep(go, x, w)
    _, bk = winners(op, x_c, w_c, border, separable=separable)
    sign = -1.0 if op == ERODE else 1.0
    flat_go = go_c.reshape(-1).double()
    flat_bk = bk.reshape(-1)
    keep = flat_bk >= 0
    acc = torch.zeros(w_c.numel(), dtype=torch.float64)
    acc.index_add_(0, flat_bk[keep], flat_go[keep])
    return (sign * acc).reshape(w_c.shape).to(w_c.dtype)


def reconstruct(dilate: bool, marker: torch.Tensor, mask: torch.Tensor, w: torch.Tensor, border: int, *,
                max_iter: int | None = None, check_every: int = 16) -> tuple[torch.Tensor, int]:
    """Geodesic reconstruction; returns (result, steps).  Raises when max_iter runs out."""
    marker, mask, w = _prep(marker, mask, w)
    out = torch.empty_like(marker)
    steps = _load().oracle_reconstruct(int(dilate), _DTYPE_CODE[marker.dtype], marker.data_ptr(), mask.data_ptr(),
                                       w.data_ptr(), out.data_ptr(), *_geometry(marker, w), border, int(is_flat(w)),
                                       max_iter or 0, check_every)
    if steps == -2:
        raise ValueError("oracle_reconstruct: bad argument")
    if steps < 0:
        raise RuntimeError(f"oracle: no fixed point after {max_iter} iterations")
    return out, int(steps)


def reconstruct_flood(dilate: bool, marker: torch.Tensor, mask: torch.Tensor, w: torch.Tensor, border: int
                      ) -> torch.Tensor:
    """The fixed point ``reconstruct`` reaches, found by a max-heap flood (exact, O(n log n)).

    Only for structuring elements whose finite taps weigh zero and include the anchor (cross, square,
    diamond, disk masks) under the CONSTANT border, and inputs without NaN; it then equals the
    reference's loop bit for bit and finishes images far too large for that loop on a CPU.
    """
    marker, mask, w = _prep(marker, mask, w)
    out = torch.empty_like(marker)
    rc = _load().oracle_reconstruct_flood(int(dilate), _DTYPE_CODE[marker.dtype], marker.data_ptr(), mask.data_ptr(),
                                          w.data_ptr(), out.data_ptr(), *_geometry(marker, w), border)
    if rc:
        raise ValueError("oracle_reconstruct_flood: needs zero-weight finite taps with the anchor, CONSTANT, no NaN")
    return out


def blob_mask(n: int, *, blobs: int = 64, seeds: int = 32, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """(marker, mask) of the large-image reconstruction workload, built on the CPU.

    mask: ``blobs`` separable Gaussians (centres uniform over the image, sigma 20 + 180 * U, amplitude U)
    summed in float64, rounded to float32, plus 0.05 * U noise; marker: zeros with ``seeds`` pixels copied
    from the mask.  All draws from ``torch.Generator().manual_seed(seed)`` in that order.
    """
    cg = torch.Generator().manual_seed(seed)
    cy, cx = torch.rand(blobs, generator=cg) * n, torch.rand(blobs, generator=cg) * n
    sigma, amp = 20 + 180 * torch.rand(blobs, generator=cg), torch.rand(blobs, generator=cg)
    ax = torch.arange(n, dtype=torch.float64)
    gy = torch.exp(-((ax[None, :] - cy[:, None].double()) ** 2) / (2 * sigma[:, None].double() ** 2))
    gx = torch.exp(-((ax[None, :] - cx[:, None].double()) ** 2) / (2 * sigma[:, None].double() ** 2))
    mask = torch.einsum("k,ky,kx->yx", amp.double(), gy, gx).float().view(1, 1, n, n)
    mask += 0.05 * torch.rand(1, 1, n, n, generator=cg)
    marker = torch.zeros_like(mask)
    idx = torch.randperm(n * n, generator=cg)[:seeds]
    marker.view(-1)[idx] = mask.view(-1)[idx]
    return marker, mask


def reference_ops():
    """The reference's own CPU operators (``torch.ops.serron_ref``), or None if not built here."""
    if not os.path.exists(REF_LIB_PATH):
        return None
    if not hasattr(torch.ops, "serron_ref") or not hasattr(torch.ops.serron_ref, "erode"):
        torch.ops.load_library(REF_LIB_PATH)
    return torch.ops.serron_ref
