"""ctypes binding of the C ABI in ``include/serron_b200.h`` (``libserron_b200.so``, sm_100a).

This is the only place Python touches the compiled library.  There is no fallback: a missing or
unloadable library raises ``ImportError`` on first use, and every failed call raises
``RuntimeError`` with the library's message.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libserron_b200.so")

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_NOT_CONVERGED = 3
ERR_WORKSPACE = 4
ERR_TIMEOUT = 5

ERODE, DILATE = 0, 1

DTYPE_CODE = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}

WINNERS_NONE = 0
WINNERS_MAP = 0x10  # flag: the record buffer also carries the gather's target map
WINNERS_BYTES = {1: 1, 2: 2, 3: 4, 4: 1, 5: 2, 6: 4}
WINNERS_TORCH_DTYPE = {1: torch.uint8, 2: torch.uint16, 3: torch.uint32, 4: torch.uint8, 5: torch.uint16,
                       6: torch.uint32}

# every symbol include/serron_b200.h declares
EXPORTED = (
    "serron_last_error",
    "serron_abi_version",
    "serron_erode",
    "serron_dilate",
    "serron_plan",
    "serron_forward",
    "serron_erode_backward",
    "serron_dilate_backward",
    "serron_backward_from_winners",
    "serron_backward_workspace_bytes",
    "serron_feasible_algos",
    "serron_heuristic_algo",
    "serron_set_separable_min_k",
    "serron_get_separable_min_k",
    "serron_reconstruct",
    "serron_reconstruct_workspace_bytes",
    "serron_backward_static_scratch",
    "serron_winners_bytes",
    "serron_forward_autocast",
    "serron_reconstruct_from_edges",
    "serron_backward_from_winners_widened",
    "serron_derived_supported",
    "serron_derived_forward",
)


class Plan(ctypes.Structure):
    _fields_ = [
        ("algo", ctypes.c_int32),
        ("winners_format", ctypes.c_int32),
        ("winners_bytes", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
    ]


_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """The loaded library (loaded once)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"serron_b200: the compiled library {LIB_PATH} is missing; build it with "
                f"`make -C serron_b200/csrc` (or __graft_entry__.build()). There is no CPU fallback."
            )
        lib = ctypes.CDLL(LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        p64 = ctypes.POINTER(ctypes.c_int64)
        lib.serron_last_error.argtypes = []
        lib.serron_last_error.restype = ctypes.c_char_p
        lib.serron_abi_version.argtypes = []
        lib.serron_abi_version.restype = i32
        fwd = [vp, p64, i64, vp, p64, i64, i32, i64, i32, i64, vp, i32, vp]
        for name in ("serron_erode", "serron_dilate"):
            getattr(lib, name).argtypes = fwd
            getattr(lib, name).restype = ctypes.c_int
        lib.serron_plan.argtypes = [p64, i64, vp, p64, i64, i32, i32, i64, i32, i32, vp, ctypes.POINTER(Plan)]
        lib.serron_plan.restype = ctypes.c_int
        lib.serron_forward.argtypes = [i32, vp, p64, i64, vp, p64, i64, i32, i64, i32, i64, vp, vp, i32, i32, vp]
        lib.serron_forward.restype = ctypes.c_int
        bwd = [vp, p64, i64, vp, p64, i64, vp, p64, i64, i32, i64, i32, i32, i64, vp, vp, vp, i64, i32, vp]
        for name in ("serron_erode_backward", "serron_dilate_backward"):
            getattr(lib, name).argtypes = bwd
            getattr(lib, name).restype = ctypes.c_int
        lib.serron_backward_from_winners.argtypes = [i32, vp, p64, i64, p64, i64, i32, i64, i32, vp, i32, vp, vp, vp,
                                                     i64, i32, vp]
        lib.serron_backward_from_winners.restype = ctypes.c_int
        lib.serron_backward_from_winners_widened.argtypes = [i32, vp, i32, p64, i64, p64, i64, i64, i32, vp, i32, vp,
                                                             i32, vp, vp, i64, i32, vp]
        lib.serron_backward_from_winners_widened.restype = ctypes.c_int
        lib.serron_derived_supported.argtypes = [i32, p64, i64, p64, i64]
        lib.serron_derived_supported.restype = ctypes.c_int
        lib.serron_derived_forward.argtypes = [i32, vp, p64, i64, vp, p64, i64, i32, i64, vp, vp, vp, i32, i32, vp]
        lib.serron_derived_forward.restype = ctypes.c_int
        lib.serron_backward_workspace_bytes.argtypes = [p64, i64, p64, i64, i32, i32, i32]
        lib.serron_backward_workspace_bytes.restype = i64
        for name in ("serron_feasible_algos", "serron_heuristic_algo"):
            getattr(lib, name).argtypes = [p64, i64, i32, i32, i32, i32]
            getattr(lib, name).restype = i64
        lib.serron_set_separable_min_k.argtypes = [i32, i32, i32, i64]
        lib.serron_set_separable_min_k.restype = i64
        lib.serron_get_separable_min_k.argtypes = [i32, i32, i32]
        lib.serron_get_separable_min_k.restype = i64
        lib.serron_reconstruct.argtypes = [i32, vp, vp, p64, i64, vp, p64, i64, i32, i64, i64, i64, vp, vp, i64, i32,
                                           vp, p64]
        lib.serron_reconstruct.restype = ctypes.c_int
        lib.serron_reconstruct_from_edges.argtypes = [i32, vp, vp, p64, i64, vp, p64, i64, i32, i64, i64, i64, vp, vp,
                                                      i64, i32, vp, p64]
        lib.serron_reconstruct_from_edges.restype = ctypes.c_int
        lib.serron_reconstruct_workspace_bytes.argtypes = [p64, i64, i32, i64]
        lib.serron_reconstruct_workspace_bytes.restype = i64
        lib.serron_backward_static_scratch.argtypes = [i32] + bwd[:14] + [vp, vp, i32, vp]
        lib.serron_backward_static_scratch.restype = ctypes.c_int
        lib.serron_forward_autocast.argtypes = [i32, vp, p64, i64, i32, vp, p64, i64, i32, i64, vp, vp, i32, i32, vp]
        lib.serron_forward_autocast.restype = ctypes.c_int
        lib.serron_winners_bytes.argtypes = [p64, i64, i32]
        lib.serron_winners_bytes.restype = i64
        _lib = lib
        return lib


def abi_version() -> int:
    """Version of the C ABI the loaded library implements."""
    return int(load().serron_abi_version())


def sizes(shape) -> tuple[ctypes.Array, int]:
    """(int64 array, ndim) for a shape."""
    n = len(shape)
    return (ctypes.c_int64 * max(n, 1))(*shape), n


def raise_for(rc: int) -> None:
    """Turn a non-zero status into the exception the reference raises for it."""
    if rc == OK:
        return
    message = load().serron_last_error().decode("utf-8", "replace")
    raise RuntimeError(message)


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream
