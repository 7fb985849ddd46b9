"""The flood reconstruction oracle against the reference's own schedule (CPU).

``oracle.reconstruct_flood`` finds the reconstruction's fixed point by a max-heap flood; it is the
checker of the large-image workload (8192^2), where the reference's Jacobi loop
(torch-ext/serron/functional.py:144-202, restated by ``oracle.reconstruct``) takes thousands of full
steps.  Here it must equal that loop bit for bit on every dtype, both reconstructions, the zero-weight
structuring elements it accepts, several planes with per-channel elements, and a 1024^2 image of the
workload's own kind (Gaussian blobs plus noise, a few seeded marker pixels).
"""

from __future__ import annotations

import pytest
import torch

import oracle

NINF = float("-inf")
CONSTANT = 2


def _se(kind: str) -> torch.Tensor:
    if kind == "cross3":
        w = [[NINF, 0, NINF], [0, 0, 0], [NINF, 0, NINF]]
    elif kind == "square3":
        w = [[0.0] * 3] * 3
    elif kind == "diamond2":
        w = [[0 if abs(i - 2) + abs(j - 2) <= 2 else NINF for j in range(5)] for i in range(5)]
    elif kind == "hline5":
        w = [[0.0] * 5]
    else:
        raise KeyError(kind)
    return torch.tensor(w, dtype=torch.float64)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("kind", ["cross3", "square3", "diamond2", "hline5"])
def test_flood_equals_reference_schedule(dtype, kind):
    marker, mask = oracle.blob_mask(96, blobs=5, seeds=3, seed=7)
    marker, mask = marker.to(dtype), mask.to(dtype)
    w = _se(kind).to(dtype)
    want, _ = oracle.reconstruct(True, marker, mask, w, CONSTANT)
    assert torch.equal(oracle.reconstruct_flood(True, marker, mask, w, CONSTANT), want)
    # the dual: start above the mask and erode down to it
    marker_e = (mask + 0.5 * (mask.max() - mask) * (marker == 0)).to(dtype)
    want, _ = oracle.reconstruct(False, marker_e, mask, w, CONSTANT)
    assert torch.equal(oracle.reconstruct_flood(False, marker_e, mask, w, CONSTANT), want)


def test_flood_per_channel_planes():
    g = torch.Generator().manual_seed(3)
    mask = torch.rand(2, 3, 40, 52, generator=g)
    marker = torch.where(torch.rand(2, 3, 40, 52, generator=g) < 0.01, mask, torch.zeros_like(mask))
    w = torch.stack([_se("cross3"), _se("square3"), _se("cross3")]).float()
    want, _ = oracle.reconstruct(True, marker, mask, w, CONSTANT)
    assert torch.equal(oracle.reconstruct_flood(True, marker, mask, w, CONSTANT), want)


def test_flood_workload_kind_1024():
    marker, mask = oracle.blob_mask(1024, seed=1)
    w = _se("cross3").float()
    want, steps = oracle.reconstruct(True, marker, mask, w, CONSTANT)
    assert steps > 100  # fronts travel far: a real test of the schedule-independence
    assert torch.equal(oracle.reconstruct_flood(True, marker, mask, w, CONSTANT), want)


def test_flood_rejects_what_it_cannot_solve():
    marker, mask = oracle.blob_mask(32, blobs=2, seeds=2)
    with pytest.raises(ValueError):
        oracle.reconstruct_flood(True, marker, mask, _se("cross3").float(), 1)  # REPLICATE
    weighted = _se("cross3").float()
    weighted[0, 1] = -0.25
    with pytest.raises(ValueError):
        oracle.reconstruct_flood(True, marker, mask, weighted, CONSTANT)
