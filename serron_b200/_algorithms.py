"""Algorithm selection as the compiled operators see it (packages/serron/torch-ext/serron/_algorithms.py)."""

from __future__ import annotations

from importlib.metadata import PackageNotFoundError
from importlib.metadata import version as _version
from typing import NotRequired, TypedDict

import torch

from . import _flatness
from ._ops import ops
from .enums import Algorithm

__all__ = [
    "DeviceFingerprint",
    "device_fingerprint",
    "feasible_algorithms",
    "get_separable_min_k",
    "heuristic_algorithm",
    "set_separable_min_k",
]


class DeviceFingerprint(TypedDict):
    """What a tuning result depends on besides the problem."""

    name: str
    capability: str
    sm_count: int
    max_optin_smem: int
    serron: str
    cuda: NotRequired[str]


def _flat(kernel: torch.Tensor, flat: bool | None) -> bool:
    return _flatness.is_flat(kernel) if flat is None else flat


def feasible_algorithms(input_: torch.Tensor, kernel: torch.Tensor, *, flat: bool | None = None,
                        backward: bool = False) -> tuple[Algorithm, ...]:
    """Algorithms that can run a call, ascending; forcing one outside this set raises."""
    mask = int(ops.feasible_algos(input_, kernel, _flat(kernel, flat), backward))
    return tuple(a for a in Algorithm if a is not Algorithm.AUTO and mask >> a & 1)


def heuristic_algorithm(input_: torch.Tensor, kernel: torch.Tensor, *, flat: bool | None = None,
                        backward: bool = False) -> Algorithm:
    """The algorithm ``algo=0`` resolves to."""
    return Algorithm(int(ops.heuristic_algo(input_, kernel, _flat(kernel, flat), backward)))


def get_separable_min_k(like: torch.Tensor, *, backward: bool = False) -> int:
    """Window length from which the separable path is preferred (``SERRON_SEPARABLE_MIN_K`` overrides)."""
    return int(ops.get_separable_min_k(like, backward))


def set_separable_min_k(like: torch.Tensor, min_k: int, *, backward: bool = False) -> int:
    """Set that window length for one device, dtype and pass (``<= 0`` restores the default)."""
    return int(ops.set_separable_min_k(like, backward, min_k))


def device_fingerprint(device: torch.device | int | None = None) -> DeviceFingerprint:
    """The GPU, toolkit and library version a tuning result belongs to."""
    if not torch.cuda.is_available():
        raise RuntimeError("serron: device_fingerprint needs a GPU")
    props = torch.cuda.get_device_properties(device)
    try:
        lib_version = _version("serron_b200")
    except PackageNotFoundError:
        lib_version = "unknown"
    return DeviceFingerprint(
        name=props.name,
        capability=f"{props.major}.{props.minor}",
        sm_count=props.multi_processor_count,
        max_optin_smem=int(getattr(props, "shared_memory_per_block_optin")),  # noqa: B009
        serron=lib_version,
        cuda=torch.version.cuda or "unknown",
    )
