"""Parity at the benchmark workloads' own shapes and launch geometry (GPU).

* The flat separable sweep forward with several steps per row segment: the row results carried from
  one step to the next, the next step's rows prefetched into the other staging buffer, and the staging
  buffer's padding restored after the winner queues used it.  Small images give every segment one
  step, so these run on (2, 150, 150, 70), 600 strip CTAs (one segment of 3-5 steps), and on the
  headline batch itself, (32, 64, 512, 512) float32 square(15) REFLECT (12 steps per segment), whose
  first and last images are checked against the reference's own CPU operators compiled from its
  sources (``oracle/_ref``; skipped where that library was not built).
* One image of the learnable-layer workload, Opening2d(32, 7) under CUDA autocast on bfloat16 input,
  through the reference's dtype flow (float16 forward, float32 backward of the promoted tensors).
* One image of the derived-ops workload, gradient / top_hat / black_hat on (1, 3, 1024, 1024) float16
  with disk(15) under CONSTANT.
* The large reconstruction, (1, 1, 8192, 8192) blob mask with cross(3) under CONSTANT, against the
  flood oracle (pinned to the reference's schedule in tests/test_oracle_flood.py), and a 1024^2 image of
  the same kind against the reference's schedule itself.

Forward values and grad_input are bit-exact; grad_kernel within rtol/atol 1e-5 (float32) or 1e-2
(16-bit) of the float64 sum over the oracle's winners.
"""

from __future__ import annotations

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

REFLECT, REPLICATE, CONSTANT = 0, 1, 2
GK_TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


@pytest.fixture(scope="module")
def serron():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import serron_b200

    return serron_b200


def _eq(got: torch.Tensor, want: torch.Tensor) -> bool:
    got = got.detach().cpu()
    if got.dtype != want.dtype or got.shape != want.shape:
        return False
    nan = want.isnan()
    return bool(torch.equal(got.isnan(), nan) and torch.equal(got[~nan], want[~nan]))


def _mismatch(got: torch.Tensor, want: torch.Tensor) -> str:
    got = got.detach().cpu()
    bad = (got != want) & ~(got.isnan() & want.isnan())
    idx = bad.nonzero()
    return f"{int(bad.sum())} of {want.numel()} differ, first at {idx[0].tolist() if len(idx) else None}"


# ------------------------------------------------------------------------------------------------
# the sweep forward through several steps per segment
# ------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("K", [3, 15, 31])
@pytest.mark.parametrize("border", [REFLECT, REPLICATE, CONSTANT])
def test_sweep_multi_step_segments(serron, dtype, K, border):
    from serron_b200.autograd import _DilateFunction, _ErodeFunction

    g = torch.Generator().manual_seed(K * 10 + border)
    shape = (2, 150, 150, 70)  # 300 planes x 2 strips = 600 CTAs: one segment per strip, 3-5 steps
    x = torch.rand(*shape, generator=g)
    if K == 15:
        x = (x * 8).floor()  # ties everywhere: the first-extremum rule across steps
    x = x.to(dtype)
    go = torch.randn(*shape, generator=g).to(dtype)
    w = torch.zeros(K, K, dtype=dtype)
    dev = torch.device("cuda")
    xd, wd, god = x.to(dev), w.to(dev), go.to(dev)
    for op, name, fn in ((oracle.ERODE, "erode", _ErodeFunction), (oracle.DILATE, "dilate", _DilateFunction)):
        y_ref = oracle.forward(op, x, w, border, separable=True)
        gi_ref, _ = oracle.backward(op, go, x, w, border, separable=True, need_kernel_grad=False)
        gk_wide = oracle.grad_kernel_wide(op, go, x, w, border, separable=True)
        # value-only forward, and the backward's own index-only forward with the target map
        y = getattr(torch.ops.serron, name)(xd, wd, border, True, 3)
        assert _eq(y, y_ref), (name, "forward", _mismatch(y, y_ref))
        gi, gk = getattr(torch.ops.serron, name + "_backward")(god, xd, wd, border, True, True, 3)
        assert _eq(gi, gi_ref), (name, "backward", _mismatch(gi, gi_ref))
        tol = GK_TOL[dtype]
        torch.testing.assert_close(gk.cpu().double(), gk_wide.double(), rtol=tol, atol=tol)
        # autograd: the forward writes values, records and the map in one sweep; the gather reads them
        xa = xd.clone().requires_grad_(True)
        ya = fn.apply(xa, wd, border, 3)
        ya.backward(god)
        assert _eq(ya, y_ref), (name, "autograd forward", _mismatch(ya, y_ref))
        assert _eq(xa.grad, gi_ref), (name, "autograd grad_input", _mismatch(xa.grad, gi_ref))


def test_headline_batch_against_reference_library(serron):
    """The headline step exactly as benchmarked (batch 32, 12 steps per segment), images 0 and 31 checked
    against the reference's own CPU operators."""
    ref = oracle.reference_ops()
    if ref is None:
        pytest.skip("the reference's CPU library (oracle/_ref) was not built")
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(1000)  # the benchmark's rank-0 inputs
    x = torch.rand(32, 64, 512, 512, device=dev, generator=gen)
    go = torch.randn(32, 64, 512, 512, device=dev, generator=gen)
    k = serron.structuring_element.square(15, device=dev)
    xa = x.requires_grad_(True)
    results = {}
    for name, fn in (("dilate", serron.dilation), ("erode", serron.erosion)):
        y = fn(xa, k, border=serron.BorderMode.REFLECT)
        (gx,) = torch.autograd.grad(y, xa, go)
        results[name] = (y.detach()[[0, 31]].cpu(), gx[[0, 31]].cpu())
        del y, gx
    w = torch.zeros(15, 15)
    for i, n in enumerate((0, 31)):
        xi, goi = x.detach()[n:n + 1].cpu(), go[n:n + 1].cpu()
        for name in ("dilate", "erode"):
            y_ref = getattr(ref, name)(xi, w, REFLECT, True, 0)
            gi_ref, _ = getattr(ref, name + "_backward")(goi, xi, w, REFLECT, True, False, 0)
            y, gi = results[name]
            assert _eq(y[i:i + 1], y_ref), (name, n, "forward", _mismatch(y[i:i + 1], y_ref))
            assert _eq(gi[i:i + 1], gi_ref), (name, n, "grad_input", _mismatch(gi[i:i + 1], gi_ref))


# ------------------------------------------------------------------------------------------------
# one image of the learnable-layer and derived-ops workloads
# ------------------------------------------------------------------------------------------------
def test_opening_layer_autocast_one_image(serron):
    """Opening2d(32, 7) under CUDA autocast on one bfloat16 image of (64, 32, 256, 256), REPLICATE.

    The reference's dtype flow: each primitive promotes (bfloat16 input, float32 weight) to float32 and
    saves that; autocast runs the forward on float16 casts; the backward runs in float32 on the saved
    tensors, and autograd casts each input's gradient to that input's dtype."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x_all = torch.rand(64, 32, 256, 256, device=dev, generator=g).to(torch.bfloat16)
    W = torch.randn(32, 7, 7, device=dev, generator=g) * 0.1
    go = torch.randn(64, 32, 256, 256, device=dev, generator=g).to(torch.float16)[:1].clone()
    x = x_all[:1].clone()
    del x_all

    layer = serron.Opening2d(32, 7).to(dev)
    with torch.no_grad():
        layer.weight.copy_(W)
    xg = x.clone().requires_grad_(True)
    with torch.autocast("cuda"):
        y = layer(xg)
    assert y.dtype == torch.float16
    y.backward(go)

    # the same flow on the oracle
    xc, Wc, goc = x.cpu().float(), W.cpu(), go.cpu()
    y1 = oracle.forward(oracle.ERODE, xc.half(), Wc.half(), REPLICATE)                 # erosion, float16
    y_ref = oracle.forward(oracle.DILATE, y1, Wc.half(), REPLICATE)                   # dilation, float16
    g1, gw1 = oracle.backward(oracle.DILATE, goc.float(), y1.float(), Wc, REPLICATE)  # float32
    g0, gw0 = oracle.backward(oracle.ERODE, g1.half().float(), xc, Wc, REPLICATE)
    gw_wide = (oracle.grad_kernel_wide(oracle.DILATE, goc.float(), y1.float(), Wc, REPLICATE).double() +
               oracle.grad_kernel_wide(oracle.ERODE, g1.half().float(), xc, Wc, REPLICATE).double())
    assert _eq(y, y_ref), _mismatch(y, y_ref)
    assert _eq(xg.grad, g0.to(torch.bfloat16)), _mismatch(xg.grad, g0.to(torch.bfloat16))
    torch.testing.assert_close(layer.weight.grad.cpu().double(), gw_wide, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(layer.weight.grad.cpu(), gw1 + gw0, rtol=1e-3, atol=1e-3)


def test_derived_ops_one_image(serron):
    """gradient, top_hat and black_hat forward + backward on one float16 image of (8, 3, 1024, 1024),
    disk(15) under CONSTANT (neutral padding), each op's grad_input through autograd."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.rand(8, 3, 1024, 1024, device=dev, generator=g).to(torch.float16)[:1].clone()
    gos = [torch.randn(8, 3, 1024, 1024, device=dev, generator=g).to(torch.float16)[:1].clone() for _ in range(3)]
    k = serron.structuring_element.disk(15, dtype=torch.float16, device=dev)
    xc, kc = x.cpu(), k.cpu()

    def fwd(op, t):
        return oracle.forward(op, t, kc, CONSTANT)

    def bwd(op, go, t):
        return oracle.backward(op, go, t, kc, CONSTANT, need_kernel_grad=False)[0]

    d, e = fwd(oracle.DILATE, xc), fwd(oracle.ERODE, xc)
    for name, go in zip(("gradient", "top_hat", "black_hat"), gos):
        xa = x.clone().requires_grad_(True)
        y = getattr(serron, name)(xa, k, border=serron.BorderMode.CONSTANT)
        (gx,) = torch.autograd.grad(y, xa, go)
        goc = go.cpu()
        if name == "gradient":
            y_ref = d - e
            gx_ref = bwd(oracle.DILATE, goc, xc) + bwd(oracle.ERODE, -goc, xc)
        elif name == "top_hat":
            y_ref = xc - fwd(oracle.DILATE, e)
            gx_ref = goc + bwd(oracle.ERODE, bwd(oracle.DILATE, -goc, e), xc)
        else:
            y_ref = fwd(oracle.ERODE, d) - xc
            gx_ref = bwd(oracle.DILATE, bwd(oracle.ERODE, goc, d), xc) + (-goc)
        assert _eq(y, y_ref), (name, _mismatch(y, y_ref))
        assert _eq(gx, gx_ref), (name, _mismatch(gx, gx_ref))


# ------------------------------------------------------------------------------------------------
# reconstruction at full size
# ------------------------------------------------------------------------------------------------
def test_reconstruction_8192_blob_mask(serron):
    marker, mask = oracle.blob_mask(8192)
    cross = serron.structuring_element.cross(3)
    want = oracle.reconstruct_flood(True, marker, mask, cross, CONSTANT)
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), cross.cuda(),
                                            border=serron.BorderMode.CONSTANT)
    assert _eq(got, want), _mismatch(got, want)


@pytest.mark.parametrize("kind", ["cross", "square"])
def test_reconstruction_2048_both_variants(serron, kind):
    marker, mask = oracle.blob_mask(2048, seed=2)
    se = serron.structuring_element
    w = se.cross(3) if kind == "cross" else se.square(3)
    want = oracle.reconstruct_flood(True, marker, mask, w, CONSTANT)
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), w.cuda(), border=serron.BorderMode.CONSTANT)
    assert _eq(got, want), _mismatch(got, want)
    top = (mask + 0.5 * (1.0 - mask) * (marker == 0)).float()
    want = oracle.reconstruct_flood(False, top, mask, w, CONSTANT)
    got = serron.reconstruction_by_erosion(top.cuda(), mask.cuda(), w.cuda(), border=serron.BorderMode.CONSTANT)
    assert _eq(got, want), _mismatch(got, want)


def test_reconstruction_1024_against_reference_schedule(serron):
    """A multi-tile image whose fronts requeue tiles many times, against the reference's own loop."""
    marker, mask = oracle.blob_mask(1024, seed=1)
    cross = serron.structuring_element.cross(3)
    want, steps = oracle.reconstruct(True, marker, mask, cross, CONSTANT)
    assert steps > 100
    got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), cross.cuda(),
                                            border=serron.BorderMode.CONSTANT)
    assert _eq(got, want), _mismatch(got, want)
