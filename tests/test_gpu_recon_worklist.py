"""The persistent reconstruction worklist: bounded waits and its result at scale (GPU).

Without ``max_iter`` the fixed point is found in one persistent launch whose CTAs pop 64x64 tiles from
a device queue; every wait for a tile is bounded by a wall-clock budget (``SERRON_RECON_WAIT_NS``,
default two seconds), after which the kernel records a status the host turns into an error instead of
holding the GPU.  A budget of one nanosecond makes the first wait of a multi-tile call run out: the call
must fail with that error, and the next call on the same context must still give the exact result.
"""

from __future__ import annotations

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

CONSTANT = 2


@pytest.fixture(scope="module")
def serron():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import serron_b200

    return serron_b200


def test_wait_budget_runs_out_and_the_context_survives(serron, monkeypatch):
    marker, mask = oracle.blob_mask(2048, blobs=8, seeds=1, seed=5)
    cross = serron.structuring_element.cross(3)
    want = oracle.reconstruct_flood(True, marker, mask, cross, CONSTANT)
    md, kd, cd = marker.cuda(), mask.cuda(), cross.cuda()
    monkeypatch.setenv("SERRON_RECON_WAIT_NS", "1")
    with pytest.raises(RuntimeError, match="ran out"):
        serron.reconstruction_by_dilation(md, kd, cd, border=serron.BorderMode.CONSTANT)
    monkeypatch.delenv("SERRON_RECON_WAIT_NS")
    torch.cuda.synchronize()
    got = serron.reconstruction_by_dilation(md, kd, cd, border=serron.BorderMode.CONSTANT)
    assert torch.equal(got.cpu(), want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
def test_many_planes_one_launch(serron, dtype):
    """Tiles of several planes share one queue; each plane reaches its own fixed point."""
    g = torch.Generator().manual_seed(11)
    mask = torch.rand(3, 2, 200, 300, generator=g).to(dtype)
    marker = torch.where(torch.rand(3, 2, 200, 300, generator=g) < 0.002, mask, torch.zeros_like(mask))
    for kind in ("cross", "square"):
        w = getattr(serron.structuring_element, kind)(3, dtype=dtype)
        want = oracle.reconstruct_flood(True, marker, mask, w, CONSTANT)
        got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), w.cuda(), border=serron.BorderMode.CONSTANT)
        assert torch.equal(got.cpu(), want), kind


def test_full_step_tiles_with_a_wide_window(serron):
    """An SE the scans do not cover (diamond(2), 5x5) runs full-step tiles through the same worklist."""
    marker, mask = oracle.blob_mask(700, blobs=10, seeds=6, seed=9)
    w = serron.structuring_element.diamond(2)
    want = oracle.reconstruct_flood(True, marker, mask, w, CONSTANT)
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), w.cuda(), border=serron.BorderMode.CONSTANT)
    assert torch.equal(got.cpu(), want)


@pytest.mark.parametrize("n", [600, 577])  # 577: a last tile row of one pixel row, the seed rows reach the one above
@pytest.mark.parametrize("kind", ["cross", "square", "diamond"])
@pytest.mark.parametrize("dilate", [True, False])
def test_edge_seeded_continuation(serron, kind, dilate, n):
    """``serron_reconstruct_from_edges``: a marker already at its fixed point except near the top and
    bottom edges reaches the full reconstruction's result with only the edge tiles queued at first."""
    from serron_b200 import _ops

    g = torch.Generator().manual_seed(21 + int(dilate))
    marker, mask = oracle.blob_mask(n, blobs=9, seeds=4, seed=13)
    if not dilate:  # the dual: marker above the mask, fronts that lower it
        mask, marker = 1.0 - mask, 1.0 - marker
    w = getattr(serron.structuring_element, kind)(2 if kind == "diamond" else 3).cuda()  # 5x5, 3x3, 3x3
    kh = w.shape[-2]
    # the fixed point of the marker without its edge seeds, then new seeds in the top and bottom 8 rows
    inner = marker.clone()
    inner[:, :, :8] = marker.min() if dilate else marker.max()
    inner[:, :, -8:] = marker.min() if dilate else marker.max()
    settled = _ops.reconstruct(dilate, inner.cuda(), mask.cuda(), w, 2, None, 16)
    edge_seeds = torch.rand(1, 1, n, n, generator=g) < 0.02
    edge_seeds[:, :, 8:-8] = False
    start = torch.where(edge_seeds.cuda(), mask.cuda(), settled)
    want = _ops.reconstruct(dilate, start, mask.cuda(), w, 2, None, 16)
    got = _ops.reconstruct(dilate, start, mask.cuda(), w, 2, None, 16, seed_rows=(8 + kh, 8 + kh))
    assert torch.equal(got, want)
    # nothing seeded: the marker is taken as the fixed point it is
    same = _ops.reconstruct(dilate, want, mask.cuda(), w, 2, None, 16, seed_rows=(0, 0))
    assert torch.equal(same, want)
