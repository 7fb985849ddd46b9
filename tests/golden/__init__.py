"""Golden fixtures produced by the reference itself (see make_golden.py)."""

from __future__ import annotations

import functools
import math
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


@functools.lru_cache(maxsize=None)
def load(name: str) -> dict[str, torch.Tensor]:
    """The fixture ``name`` as a ``{key: tensor}`` dict."""
    packed = torch.load(HERE / f"{name}.pt", weights_only=True)
    out: dict[str, torch.Tensor] = {}
    for key, (dname, offset, shape) in packed["index"].items():
        n = math.prod(shape)
        out[key] = packed["buffers"][dname][offset:offset + n].reshape(shape)
    return out
