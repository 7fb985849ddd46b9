"""Derived operations in one launch against the reference's compositions (GPU).

``serron.functional.gradient / opening / closing / top_hat / black_hat`` run as one kernel
(``serron_derived_forward``) for windows up to 7 a side; the composition of the primitive operations
(the reference's functional.py:40-92, which these functions fall back to otherwise) is the oracle
here: forward values, grad_input and grad_kernel must be the same bits.  The primitives themselves
are pinned to the reference elsewhere; the golden composite cases of test_gpu_parity.py also run
through the one-launch form.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

OPS = ("gradient", "opening", "closing", "top_hat", "black_hat")
DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)


@pytest.fixture(scope="module")
def serron():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import serron_b200

    return serron_b200


def _composed(serron, name, x, k, border):
    f = serron.functional
    if name == "gradient":
        return f.dilation(x, k, border=border) - f.erosion(x, k, border=border)
    if name == "opening":
        return f.dilation(f.erosion(x, k, border=border), k, border=border)
    if name == "closing":
        return f.erosion(f.dilation(x, k, border=border), k, border=border)
    if name == "top_hat":
        return x - f.dilation(f.erosion(x, k, border=border), k, border=border)
    return f.erosion(f.dilation(x, k, border=border), k, border=border) - x


def _kernels(serron, dtype, channels, gen):
    se = serron.structuring_element
    return {
        "square3": se.square(3, dtype=dtype),
        "disk3": se.disk(3, dtype=dtype),                                    # 7x7 mask, 0 / -inf
        "perch5": (torch.randn(channels, 5, 5, generator=gen) * 0.1).to(dtype),  # per channel, non-flat
        "even4x2": (torch.randn(4, 2, generator=gen) * 0.1).to(dtype),       # even sides: anchor k // 2
        "row1x7": torch.zeros(1, 7, dtype=dtype),
    }


def _check(serron, name, x0, k0, border, go):
    from serron_b200 import _ops

    dev = torch.device("cuda")
    x = x0.clone().to(dev).requires_grad_(True)
    k = k0.clone().to(dev).requires_grad_(True)
    mode = getattr(_ops, "DERIVED_" + name.upper())
    assert _ops.derived_supported(mode, x, k), "the one-launch form should take this call"
    y = getattr(serron.functional, name)(x, k, border=border)
    y.backward(go)
    xr = x0.clone().to(dev).requires_grad_(True)
    kr = k0.clone().to(dev).requires_grad_(True)
    yr = _composed(serron, name, xr, kr, border)
    yr.backward(go)
    tag = f"{name} {tuple(x0.shape)} {tuple(k0.shape)} {x0.dtype} {border}"
    assert torch.equal(y, yr), tag
    assert torch.equal(x.grad, xr.grad), tag
    assert torch.equal(k.grad, kr.grad), tag


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d).split(".")[-1])
@pytest.mark.parametrize("name", OPS)
def test_one_launch_equals_composition(serron, name, dtype):
    gen = torch.Generator().manual_seed(7)
    x0 = torch.rand(2, 3, 45, 70, generator=gen).to(dtype)
    go = torch.randn(2, 3, 45, 70, generator=gen).to(dtype).cuda()
    for kname, k0 in _kernels(serron, dtype, 3, gen).items():
        for border in (serron.BorderMode.REFLECT, serron.BorderMode.REPLICATE, serron.BorderMode.CONSTANT):
            _check(serron, name, x0, k0, border, go)


@pytest.mark.parametrize("name", OPS)
def test_one_launch_edges(serron, name):
    """Images exactly the window's size, one-row tiles past a multiple of 32, ties (a quantised image),
    and NaN inputs."""
    gen = torch.Generator().manual_seed(11)
    k = serron.structuring_element.disk(3)  # 7 x 7
    cases = [torch.rand(1, 2, 7, 7, generator=gen), torch.rand(1, 1, 33, 65, generator=gen),
             (torch.rand(2, 2, 40, 40, generator=gen) * 4).floor() / 4]
    nan = torch.rand(1, 1, 37, 41, generator=gen)
    nan[0, 0, 5:9, 10:13] = float("nan")
    cases.append(nan)
    for x0 in cases:
        go = torch.randn(x0.shape, generator=gen).cuda()
        for border in (serron.BorderMode.REFLECT, serron.BorderMode.REPLICATE, serron.BorderMode.CONSTANT):
            dev = torch.device("cuda")
            x = x0.clone().to(dev).requires_grad_(True)
            y = getattr(serron.functional, name)(x, k.to(dev), border=border)
            y.backward(go)
            xr = x0.clone().to(dev).requires_grad_(True)
            yr = _composed(serron, name, xr, k.to(dev), border)
            yr.backward(go)
            tag = f"{name} {tuple(x0.shape)} {border}"
            assert torch.equal(y.nan_to_num(nan=7.0), yr.nan_to_num(nan=7.0)), tag
            assert torch.equal(x.grad.nan_to_num(nan=7.0), xr.grad.nan_to_num(nan=7.0)), tag


def test_one_launch_not_taken(serron):
    """Wider windows, an image smaller than the window (two-stage forms), mixed dtypes and autocast keep
    the composition."""
    from serron_b200 import _ops

    dev = torch.device("cuda")
    x = torch.rand(1, 1, 40, 40, device=dev)
    assert not _ops.derived_supported(_ops.DERIVED_GRADIENT, x, torch.zeros(9, 9, device=dev))
    small = torch.rand(1, 1, 5, 40, device=dev)
    assert _ops.derived_supported(_ops.DERIVED_GRADIENT, small, torch.zeros(7, 7, device=dev))
    assert not _ops.derived_supported(_ops.DERIVED_OPENING, small, torch.zeros(7, 7, device=dev))
    assert not _ops.derived_supported(_ops.DERIVED_OPENING, x.half(), torch.zeros(3, 3, device=dev))
    # still the composition's results
    y = serron.functional.opening(small, torch.zeros(7, 7, device=dev))
    yr = _composed(serron, "opening", small, torch.zeros(7, 7, device=dev), serron.BorderMode.REPLICATE)
    assert torch.equal(y, yr)
