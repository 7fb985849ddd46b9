"""Reconstruction to convergence (max_iter=None) on the directional-scan path against the reference's
own Jacobi schedule (max_iter set, recon_step_kernel) and against the oracle.

Flat structuring elements within the 3x3 neighbourhood take the worklist of scan tiles (row and column
scans plus a diagonal pass), others the full-step tiles after global scan rounds; the result must
equal the Jacobi fixed point bit for bit on every dtype, border and shape, including rows longer than
one scan chunk (8192 columns), columns split unevenly into runs, single rows and single columns.
"""

from __future__ import annotations

import zlib

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

NINF = float("-inf")


@pytest.fixture(scope="module")
def serron():
    import serron_b200

    return serron_b200


def _se(kind: str, dtype) -> torch.Tensor:
    if kind == "cross3":
        w = [[NINF, 0, NINF], [0, 0, 0], [NINF, 0, NINF]]
    elif kind == "square3":
        w = [[0, 0, 0], [0, 0, 0], [0, 0, 0]]
    elif kind == "hline3":
        w = [[0, 0, 0]]
    elif kind == "vline3":
        w = [[0], [0], [0]]
    elif kind == "hline5":
        w = [[0, 0, 0, 0, 0]]
    elif kind == "left2":  # anchor and left neighbour only
        w = [[0, 0, NINF]]
    elif kind == "down2":  # anchor and lower neighbour only
        w = [[NINF], [0], [0]]
    elif kind == "x3":  # anchor and the four diagonals (the diagonal pass alone)
        w = [[0, NINF, 0], [NINF, 0, NINF], [0, NINF, 0]]
    elif kind == "diag2":  # anchor, upper-left and lower-right: folds need taps it lacks except under CONSTANT
        w = [[0, NINF, NINF], [NINF, 0, NINF], [NINF, NINF, 0]]
    elif kind == "nonflat3":  # weights: the tile relaxation alone
        w = [[NINF, -0.25, NINF], [-0.25, 0, -0.25], [NINF, -0.25, NINF]]
    else:
        raise ValueError(kind)
    return torch.tensor(w, dtype=torch.float64).to(dtype)


def _smooth_mask(shape, gen) -> torch.Tensor:
    """A mask with long ridges (so fronts travel far and turn) plus noise."""
    n, c, h, w = shape
    yy = torch.linspace(0, 6.28 * 3, h, dtype=torch.float64)[:, None]
    xx = torch.linspace(0, 6.28 * 5, w, dtype=torch.float64)[None, :]
    base = 0.5 + 0.25 * torch.sin(yy + 0.7 * torch.cos(xx)) + 0.2 * torch.cos(xx * 0.5 + yy * 0.3)
    return (base.expand(n, c, h, w) + 0.05 * torch.rand(shape, generator=gen, dtype=torch.float64)).contiguous()


def _marker(mask: torch.Tensor, gen, seeds: int = 3) -> torch.Tensor:
    marker = torch.zeros_like(mask)
    flat = marker.view(-1)
    idx = torch.randint(0, flat.numel(), (seeds,), generator=gen)
    flat[idx] = mask.reshape(-1)[idx]
    return marker


def _pair(serron, dilate, marker, mask, k, border, dtype):
    fn = serron.reconstruction_by_dilation if dilate else serron.reconstruction_by_erosion
    if not dilate:
        marker = torch.where(marker == 0, torch.full_like(marker, 2.0), marker)
    mk, ms, kk = marker.to(dtype).cuda(), mask.to(dtype).cuda(), k.cuda()
    got = fn(mk, ms, kk, border=border)
    want = fn(mk, ms, kk, border=border, max_iter=1_000_000, check_every=64)
    return got, want


SHAPES = [(2, 3, 37, 61), (1, 1, 33, 8200), (1, 2, 200, 40), (1, 1, 1, 70), (1, 1, 70, 1), (1, 1, 150, 300)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("kind", ["cross3", "square3", "hline3", "vline3", "hline5", "left2", "down2", "x3", "diag2",
                                  "nonflat3"])
def test_scan_path_equals_jacobi_fixed_point(serron, shape, kind):
    gen = torch.Generator().manual_seed(zlib.crc32(repr((shape, kind)).encode()))
    mask = _smooth_mask(shape, gen)
    marker = _marker(mask, gen)
    B = serron.BorderMode
    for dtype in (torch.float32, torch.float64, torch.float16, torch.bfloat16):
        k = _se(kind, dtype)
        for border in (B.CONSTANT, B.REFLECT, B.REPLICATE):
            for dilate in (True, False):
                got, want = _pair(serron, dilate, marker, mask, k, border, dtype)
                assert torch.equal(got, want), (kind, dtype, border, dilate)


@pytest.mark.parametrize("kind", ["cross3", "square3", "hline5", "x3", "nonflat3"])
def test_scan_path_equals_oracle(serron, kind):
    gen = torch.Generator().manual_seed(11)
    shape = (1, 2, 23, 29)
    mask = _smooth_mask(shape, gen)
    marker = _marker(mask, gen, seeds=2)
    k = _se(kind, torch.float64)
    B = serron.BorderMode
    for border, code in ((B.CONSTANT, 2), (B.REFLECT, 0), (B.REPLICATE, 1)):
        got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), k.cuda(), border=border)
        want, _ = oracle.reconstruct(True, marker, mask, k, code)
        assert torch.equal(got.cpu(), want), (kind, border)


def test_scan_path_flood_across_long_row(serron):
    """A single seed at one end of a 1 x 20000 corridor: one left-to-right scan carries it through
    three row chunks; the Jacobi schedule needs ~20000 steps for the same answer."""
    w = 20000
    mask = torch.linspace(1.0, 0.5, w, dtype=torch.float32).view(1, 1, 1, w)
    marker = torch.zeros_like(mask)
    marker[..., 0] = 1.0
    k = _se("hline3", torch.float32)
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), k.cuda(), border=serron.BorderMode.CONSTANT)
    assert torch.equal(got.cpu(), mask)
    marker = torch.zeros_like(mask)
    marker[..., -1] = 0.5
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), k.cuda(), border=serron.BorderMode.CONSTANT)
    assert torch.equal(got.cpu(), torch.full_like(mask, 0.5))
