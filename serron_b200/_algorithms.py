"""Algorithm selection as the compiled operators see it (packages/serron/torch-ext/serron/_algorithms.py)."""

from __future__ import annotations

from typing import NotRequired, TypedDict

import torch

from . import _flatness, _lib
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
    """Where a measured algorithm choice is valid: this GPU model and SM count, its per-CTA shared
    memory limit, the library build (package version and C-ABI version) and the CUDA toolkit."""
    if isinstance(device, int):
        device = torch.device("cuda", device)
    if device is None or device.index is None:
        if not torch.cuda.is_available():
            raise RuntimeError("serron: a fingerprint describes a CUDA device, and none is visible")
        device = torch.device("cuda", torch.cuda.current_device())
    major, minor = torch.cuda.get_device_capability(device)
    props = torch.cuda.get_device_properties(device)
    from . import __version__

    return DeviceFingerprint(name=torch.cuda.get_device_name(device), capability=f"{major}.{minor}",
                             sm_count=props.multi_processor_count,
                             max_optin_smem=props.shared_memory_per_block_optin,
                             serron=f"{__version__}+abi{_lib.abi_version()}", cuda=str(torch.version.cuda))
