"""Algorithm tuning (the public ``calibrate`` / ``autotune`` of packages/serron/torch-ext/serron/_autotune.py).

The reference keeps a per-machine JSON cache and seeds per architecture; this library keeps tuning
results for the process only, on top of its built-in window-length threshold for the separable path
(3, measured on a B200: the separable sweep beat the tiled kernel at every square window from 3x3 on).  :func:`calibrate` re-measures the separable crossover on the current GPU; :func:`autotune`
times every feasible algorithm on given problems and makes the autograd path force the winner.
"""

from __future__ import annotations

import threading
from collections.abc import Iterable, Sequence

import torch

from ._ops import ops
from .enums import Algorithm

__all__ = ["DEFAULT_DTYPES", "DEFAULT_KS", "HYSTERESIS", "autotune", "calibrate", "ensure_loaded",
           "select_algorithm", "shape_key"]

HYSTERESIS = 0.05
"""A tuned algorithm replaces the heuristic only when it is at least this fraction faster."""
DEFAULT_KS = (3, 5, 7, 9, 11, 13, 15, 21, 31, 63)
DEFAULT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_REFERENCE_SHAPE = (1, 3, 512, 512)
_BORDER = 1  # replicate

_shape_table: dict[str, int] = {}
_lock = threading.Lock()


def ensure_loaded(device: torch.device) -> None:
    """Nothing is persisted, so there is nothing to load; kept for API parity."""
    return None


def shape_key(dtype: torch.dtype, *, backward: bool, flat: bool, k_h: int, k_w: int, numel: int) -> str:
    return f"shape:{str(dtype).removeprefix('torch.')}|{'bwd' if backward else 'fwd'}|{int(flat)}|{k_h}x{k_w}|{numel}"


def select_algorithm(input_: torch.Tensor, kernel: torch.Tensor, flat: bool, *, backward: bool) -> int:
    """The algorithm :func:`autotune` chose for this problem, or 0 (let the library choose)."""
    if not _shape_table or not input_.is_cuda:
        return 0
    key = shape_key(input_.dtype, backward=backward, flat=flat, k_h=kernel.shape[-2], k_w=kernel.shape[-1],
                    numel=input_.numel())
    return _shape_table.get(f"{input_.device.index}|{key}", 0)


def _time_ms(fn, reps: int) -> float:
    for _ in range(2):
        fn()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(reps):
        start.record()
        fn()
        stop.record()
        stop.synchronize()
        times.append(start.elapsed_time(stop))
    times.sort()
    return times[len(times) // 2]


def _runner(x: torch.Tensor, go: torch.Tensor, kernel: torch.Tensor, flat: bool, backward: bool, algo: int):
    if backward:
        return lambda: ops.erode_backward(go, x, kernel, _BORDER, flat, True, algo)
    return lambda: ops.erode(x, kernel, _BORDER, flat, algo)


def calibrate(device: torch.device | int | None = None, *, dtypes: Sequence[torch.dtype] = DEFAULT_DTYPES,
              ks: Sequence[int] = DEFAULT_KS, reps: int = 10) -> dict[str, int]:
    """Measure, per dtype and pass, the window length from which the separable path wins, and use it.

    :returns: ``{"<dtype>|<fwd|bwd>": min_k}`` as set for this process.
    """
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    found: dict[str, int] = {}
    for dtype in dtypes:
        x = torch.rand(_REFERENCE_SHAPE, device=dev, dtype=dtype)
        go = torch.randn_like(x)
        for backward in (False, True):
            wins = []
            for k in ks:
                kernel = torch.zeros(k, k, device=dev, dtype=dtype)
                t_sep = _time_ms(_runner(x, go, kernel, True, backward, int(Algorithm.SEPARABLE)), reps)
                t_tile = _time_ms(_runner(x, go, kernel, True, backward, int(Algorithm.TILED)), reps)
                wins.append(t_sep < t_tile)
            min_k = max(ks) + 1
            for i in range(len(ks)):
                if all(wins[i:]):
                    min_k = ks[i]
                    break
            ops.set_separable_min_k(x, backward, min_k)
            found[f"{str(dtype).removeprefix('torch.')}|{'bwd' if backward else 'fwd'}"] = min_k
    return found


def autotune(problems: Iterable[tuple[tuple[int, int, int, int], torch.dtype, int, int, bool]], *,
             device: torch.device | int | None = None, reps: int = 10) -> dict[str, int]:
    """Time every feasible algorithm on each ``(shape, dtype, k_h, k_w, flat)`` problem, both passes.

    The winner is forced for matching calls through the autograd path when it beats the heuristic by
    :data:`HYSTERESIS`.  :returns: the chosen algorithm per problem key.
    """
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    chosen: dict[str, int] = {}
    for shape, dtype, k_h, k_w, flat in problems:
        x = torch.rand(shape, device=dev, dtype=dtype)
        go = torch.randn_like(x)
        kernel = torch.zeros(k_h, k_w, device=dev, dtype=dtype) if flat else torch.randn(k_h, k_w, device=dev,
                                                                                        dtype=dtype) * 0.1
        for backward in (False, True):
            mask = int(ops.feasible_algos(x, kernel, flat, backward))
            heuristic = int(ops.heuristic_algo(x, kernel, flat, backward))
            times = {a: _time_ms(_runner(x, go, kernel, flat, backward, a), reps) for a in (1, 2, 3) if mask >> a & 1}
            best = min(times, key=times.get)
            pick = best if times[best] < (1.0 - HYSTERESIS) * times[heuristic] else heuristic
            key = shape_key(dtype, backward=backward, flat=flat, k_h=k_h, k_w=k_w, numel=x.numel())
            with _lock:
                _shape_table[f"{dev.index}|{key}"] = pick
            chosen[key] = pick
    return chosen
