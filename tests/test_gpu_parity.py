"""Parity of the CUDA path with the reference, on the GPU.

Forward outputs and grad_input must be bit-exact with the reference's CPU implementation (golden
fixtures generated from the reference, and the pinned oracle on fresh seeded inputs).  grad_kernel is
a deterministic reduction in a different order: rtol/atol 1e-5 for float32, 1e-9 for float64, 1e-2
for float16/bfloat16.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from tests.golden import load

pytestmark = pytest.mark.gpu

BORDERS = {"reflect": 0, "replicate": 1, "constant": 2}
GK_TOL = {torch.float64: 1e-9, torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


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


def _gk_close(got: torch.Tensor, want: torch.Tensor, wide: torch.Tensor | None = None) -> None:
    """grad_kernel check.

    The library sums grad_kernel in float64 and rounds once.  `wide` is the same sum over the oracle's
    (bit-exact) winners; it is checked at GK_TOL.  `want` is the reference's own result: a sequential
    sum in the storage type, whose rounding error grows with the number of terms (for float16 and
    bfloat16 it rounds after every add), so it is only checked loosely, and for float32/float64 only.
    """
    got = got.detach().cpu().double()
    if wide is not None:
        tol = GK_TOL[wide.dtype]
        torch.testing.assert_close(got, wide.double(), rtol=tol, atol=tol)
    if want.dtype == torch.float64:
        torch.testing.assert_close(got, want.double(), rtol=1e-9, atol=1e-9)
    elif want.dtype == torch.float32:
        torch.testing.assert_close(got, want.double(), rtol=1e-3, atol=1e-3)


def _primitive_cases():
    data = load("primitives")
    return sorted({tuple(k.split(".")[:5]) for k in data if k.endswith(".y")})


@pytest.mark.parametrize("case", _primitive_cases(), ids=lambda c: ".".join(c))
def test_golden_primitives_all_algorithms(serron, case):
    dname, xname, sname, bname, opname = case
    data = load("primitives")
    dev = torch.device("cuda")
    x = data[f"{dname}.{xname}.x"].to(dev)
    go = data[f"{dname}.{xname}.go"].to(dev)
    w = data[f"{dname}.{xname}.{sname}.w"].to(dev)
    key = f"{dname}.{xname}.{sname}.{bname}.{opname}"
    flat = bool(w.eq(0).all())
    ops = torch.ops.serron
    code = oracle.ERODE if opname == "erode" else oracle.DILATE
    wide = oracle.grad_kernel_wide(code, go, x, w, BORDERS[bname])
    mask = ops.feasible_algos(x, w, flat, False)
    algos = [0] + [a for a in (1, 2, 3) if mask >> a & 1]
    for algo in algos:
        y = getattr(ops, opname)(x, w, BORDERS[bname], flat, algo)
        assert _eq(y, data[key + ".y"]), f"forward algo={algo}"
        gi, gk = getattr(ops, opname + "_backward")(go, x, w, BORDERS[bname], flat, True, algo)
        assert _eq(gi, data[key + ".gi"]), f"grad_input algo={algo}"
        _gk_close(gk, data[key + ".gk"], wide)


@pytest.mark.parametrize("dname", ["float64", "float32"])
def test_golden_composites_through_autograd(serron, dname):
    data = load("composites")
    dev = torch.device("cuda")
    x0 = data[f"{dname}.x"]
    modes = {"reflect": serron.BorderMode.REFLECT, "replicate": serron.BorderMode.REPLICATE,
             "constant": serron.BorderMode.CONSTANT}
    for kname in ("perch", "flat5"):
        k0 = data[f"{dname}.{kname}.w"]
        for bname, border in modes.items():
            for name in ("erosion", "dilation", "opening", "closing", "gradient", "top_hat", "black_hat"):
                key = f"{dname}.{kname}.{bname}.{name}"
                x = x0.clone().to(dev).requires_grad_(True)
                k = k0.clone().to(dev).requires_grad_(True)
                y = getattr(serron.functional, name)(x, k, border=border)
                y.backward(data[key + ".go"].to(dev))
                assert _eq(y, data[key + ".y"]), key
                # a composite sums per-op grads in autograd; every op's grad is bit-exact, so is the sum
                assert _eq(x.grad, data[key + ".gx"]), key
                _gk_close(k.grad, data[key + ".gk"])


def test_golden_tie_break(serron):
    data = load("tie_break")
    for op in ("erosion", "dilation"):
        for k in (3, 21):
            x = torch.full((1, 1, 9, 10), 2.5, dtype=torch.float64, device="cuda", requires_grad=True)
            kernel = torch.zeros(k, k, dtype=torch.float64, device="cuda")
            getattr(serron, op)(x, kernel, border=serron.BorderMode.REPLICATE).sum().backward()
            assert _eq(x.grad, data[f"{op}.{k}.grad"])


def test_golden_separable_cases(serron):
    data = load("separable")
    from tests.golden.make_golden import SEPARABLE_CASES

    modes = {"reflect": serron.BorderMode.REFLECT, "replicate": serron.BorderMode.REPLICATE,
             "constant": serron.BorderMode.CONSTANT}
    for i, (op, border, shape, ksize) in enumerate(SEPARABLE_CASES):
        x = data[f"{i}.x"].cuda().requires_grad_(True)
        kernel = torch.zeros(shape[1], *ksize, dtype=torch.float64, device="cuda", requires_grad=True)
        y = getattr(serron.functional, op)(x, kernel, border=modes[border])
        y.backward(data[f"{i}.go"].cuda())
        assert _eq(y, data[f"{i}.forward"]), i
        assert _eq(x.grad, data[f"{i}.grad_input"]), i
        _gk_close(kernel.grad, data[f"{i}.grad_kernel"])


def test_golden_config1(serron):
    data = load("config1")
    x = data["x"].cuda()
    k = serron.structuring_element.disk(3, device="cuda")
    y = serron.dilation(serron.erosion(x, k), k)
    assert _eq(y, data["y"])


def test_golden_autocast_opening(serron):
    d = load("autocast_opening")
    layer = serron.Opening2d(4, 7).cuda()
    with torch.no_grad():
        layer.weight.copy_(d["w"])
    x = d["x"].cuda().requires_grad_(True)
    with torch.autocast("cuda"):
        y = layer(x)
    assert y.dtype == torch.float16
    y.backward(d["go"].cuda())
    assert _eq(y, d["y"])
    assert _eq(x.grad, d["gx"])
    _gk_close(layer.weight.grad, d["gw"])


@pytest.mark.parametrize("dname", ["float64", "float32"])
def test_golden_reconstruction(serron, dname):
    data = load("reconstruction")
    mask = data[f"{dname}.mask"].cuda()
    offset = data[f"{dname}.offset"].cuda()
    modes = {"reflect": serron.BorderMode.REFLECT, "replicate": serron.BorderMode.REPLICATE,
             "constant": serron.BorderMode.CONSTANT}
    for kname in ("square3", "cross3", "diamond2", "per_channel"):
        w = data[f"{dname}.{kname}.w"].cuda()
        for bname, border in modes.items():
            got = serron.reconstruction_by_dilation(mask - 4.0 * offset, mask, w, border=border)
            assert _eq(got, data[f"{dname}.{kname}.{bname}.by_dilation"]), (kname, bname)
            got = serron.reconstruction_by_erosion(mask + 4.0 * offset, mask, w, border=border)
            assert _eq(got, data[f"{dname}.{kname}.{bname}.by_erosion"]), (kname, bname)
            # the reference's own schedule, replayed with a generous budget, gives the same answer
            got = serron.reconstruction_by_dilation(mask - 4.0 * offset, mask, w, border=border, max_iter=10_000)
            assert _eq(got, data[f"{dname}.{kname}.{bname}.by_dilation"]), (kname, bname, "jacobi")


def test_golden_reconstruction_fixtures(serron):
    data = load("reconstruction")
    cross = serron.structuring_element.cross(3, dtype=torch.float64, device="cuda")
    mask = data["corridor.mask"].cuda()
    marker = torch.zeros_like(mask)
    marker[0, 0, 0, 0] = 1.0
    for check_every in (1, 16, 256):
        assert _eq(serron.reconstruction_by_dilation(marker, mask, cross, check_every=check_every),
                   data["corridor.flood"])
        assert _eq(serron.reconstruction_by_dilation(marker, mask, cross, check_every=check_every,
                                                     max_iter=100_000), data["corridor.flood"])
    marker = torch.zeros_like(mask)
    marker[0, 0, 1, 6] = 1.0
    assert _eq(serron.reconstruction_by_dilation(marker, mask, cross), data["corridor.walled"])
    profile = data["profile.mask"].cuda()
    marker = torch.zeros_like(profile)
    marker[0, 0, 0, 0] = 1.0
    assert _eq(serron.reconstruction_by_dilation(marker, profile, cross), data["profile.flood"])


def test_reconstruction_budget_matches_reference_schedule(serron):
    """max_iter set: the reference's Jacobi loop and check schedule are replayed, so the call returns or
    raises exactly as the reference does (oracle replay), including the reference's behaviour of
    returning the unconverged state when max_iter is a multiple of check_every."""
    data = load("reconstruction")
    mask = data["corridor.mask"]
    marker = torch.zeros_like(mask)
    marker[0, 0, 0, 0] = 1.0
    cross = serron.structuring_element.cross(3, dtype=torch.float64)
    _, steps = oracle.reconstruct(True, marker, mask, cross, 2, check_every=4)
    for max_iter in (1, 3, 4, steps - 5, steps - 4, steps - 3, steps - 1, steps, steps + 7):
        try:
            want, _ = oracle.reconstruct(True, marker, mask, cross, 2, check_every=4, max_iter=max_iter)
        except RuntimeError:
            with pytest.raises(RuntimeError, match="no fixed point"):
                serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), cross.cuda(), check_every=4,
                                                  max_iter=max_iter)
            continue
        got = serron.reconstruction_by_dilation(marker.cuda(), mask.cuda(), cross.cuda(), check_every=4,
                                                max_iter=max_iter)
        assert _eq(got, want), max_iter


# ------------------------------------------------------------------------------------------------
# fresh seeded inputs against the oracle, larger than the fixtures (multiple tiles, ragged edges)
# ------------------------------------------------------------------------------------------------
def _se(kind: str, C: int, dtype: torch.dtype, g: torch.Generator) -> torch.Tensor:
    if kind == "rand7_perch":
        return (torch.randn(C, 7, 7, generator=g) * 0.1).to(dtype)
    if kind == "rand4x6":
        return (torch.randn(4, 6, generator=g) * 0.2).to(dtype)
    if kind == "flat15":
        return torch.zeros(15, 15, dtype=dtype)
    if kind == "flat_5x17_perch":
        return torch.zeros(C, 5, 17, dtype=dtype)
    if kind == "disk3":
        yy, xx = torch.meshgrid(torch.arange(7) - 3, torch.arange(7) - 3, indexing="ij")
        return torch.where(yy * yy + xx * xx <= 9, 0.0, float("-inf")).to(dtype)
    if kind == "flat1":
        return torch.zeros(1, 1, dtype=dtype)
    if kind == "disk15":  # 31x31 flat disk: every row one span of zeros (wide kernel, shared cores)
        yy, xx = torch.meshgrid(torch.arange(31) - 15, torch.arange(31) - 15, indexing="ij")
        return torch.where(yy * yy + xx * xx <= 225, 0.0, float("-inf")).to(dtype)
    if kind == "rand9x11":  # wide kernel, per-tap weights
        return (torch.randn(9, 11, generator=g) * 0.1).to(dtype)
    if kind == "ring9_neg0":  # rows with holes (walked tap by tap) and rows of -0.0 weights
        w = torch.full((9, 13), -0.0)
        w[3:6, 4:9] = float("-inf")
        return w.to(dtype)
    if kind == "diamond6":  # 13x13 diamond: centered flat rows of every radius (radius decomposition)
        yy, xx = torch.meshgrid(torch.arange(13) - 6, torch.arange(13) - 6, indexing="ij")
        return torch.where(yy.abs() + xx.abs() <= 6, 0.0, float("-inf")).to(dtype)
    if kind == "cross9_mixed0":  # centered rows, the long one of -0.0 weights and the rest +0.0
        w = torch.full((9, 9), float("-inf"))
        w[:, 4] = 0.0
        w[4, :] = -0.0
        return w.to(dtype)
    if kind == "ell10x9":  # even height, empty rows, centered rows of radii 0..4 out of order
        w = torch.full((10, 9), float("-inf"))
        for di, r in ((1, 2), (2, 4), (3, 0), (5, 3), (6, 1), (8, 4), (9, 2)):
            w[di, 4 - r:5 + r] = 0.0
        return w.to(dtype)
    if kind == "disk5_shifted":  # one row off center: the whole SE walks tap by tap
        yy, xx = torch.meshgrid(torch.arange(11) - 5, torch.arange(11) - 5, indexing="ij")
        w = torch.where(yy * yy + xx * xx <= 25, 0.0, float("-inf"))
        w[2] = torch.roll(w[2], 1)
        return w.to(dtype)
    if kind == "row3x71":  # flat, wider than the 16-bit keyed form takes (128 staged columns)
        return torch.zeros(3, 71, dtype=dtype)
    if kind == "rand17x17":  # two-byte records (289 taps), per-tap weights: the hashed gather walk
        return (torch.randn(17, 17, generator=g) * 0.1).to(dtype)
    if kind == "disk11":  # 23x23 mask, two-byte records, ties
        yy, xx = torch.meshgrid(torch.arange(23) - 11, torch.arange(23) - 11, indexing="ij")
        return torch.where(yy * yy + xx * xx <= 121, 0.0, float("-inf")).to(dtype)
    if kind == "even16x18":  # even sides: the box reaches one output past the window through a fold
        return torch.zeros(16, 18, dtype=dtype)
    raise KeyError(kind)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("kind", ["rand7_perch", "rand4x6", "flat15", "flat_5x17_perch", "disk3", "flat1", "disk15",
                                  "rand9x11", "ring9_neg0", "diamond6", "cross9_mixed0", "ell10x9", "disk5_shifted", "row3x71",
                                  "rand17x17", "disk11", "even16x18"])
@pytest.mark.parametrize("border", [0, 1, 2])
def test_oracle_parity_multi_tile(serron, dtype, kind, border):
    g = torch.Generator().manual_seed(hash((str(dtype), kind, border)) % (2**31))
    shape = (2, 3, 70, 133)
    x = torch.rand(*shape, generator=g).to(dtype)
    if kind in ("flat15", "disk15", "ring9_neg0", "diamond6", "cross9_mixed0", "ell10x9", "disk5_shifted", "row3x71",
                "disk11", "even16x18"):
        x = (x * 8).floor().to(dtype)  # many ties
    if kind in ("ell10x9", "disk5_shifted"):
        x[:, 1, 20:26, 40:47] = float("nan")  # NaN samples never win
        x[0, 2, 0:3, :] = -x[0, 2, 0:3, :]  # signed zeros among the ties
    go = torch.randn(*shape, generator=g).to(dtype)
    w = _se(kind, shape[1], dtype, g)
    flat = bool(w.eq(0).all())
    sep = flat and max(w.shape[-2:]) >= 5
    dev = torch.device("cuda")
    for op, name in ((oracle.ERODE, "erode"), (oracle.DILATE, "dilate")):
        y_ref = oracle.forward(op, x, w, border, separable=sep)
        gi_ref, gk_ref = oracle.backward(op, go, x, w, border, separable=sep)
        gk_wide = oracle.grad_kernel_wide(op, go, x, w, border)
        xd, wd, god = x.to(dev), w.to(dev), go.to(dev)
        mask = torch.ops.serron.feasible_algos(xd, wd, flat, False)
        for algo in [0] + [a for a in (1, 2, 3) if mask >> a & 1]:
            y = getattr(torch.ops.serron, name)(xd, wd, border, flat, algo)
            assert _eq(y, y_ref), (name, algo)
            gi, gk = getattr(torch.ops.serron, name + "_backward")(god, xd, wd, border, flat, True, algo)
            assert _eq(gi, gi_ref), (name, algo)
            _gk_close(gk, gk_ref, gk_wide)
        # autograd path: forward records winners, backward gathers from them
        xa = xd.clone().requires_grad_(True)
        wa = wd.clone().requires_grad_(True)
        fn = serron.erosion if op == oracle.ERODE else serron.dilation
        border_mode = [serron.BorderMode.REFLECT, serron.BorderMode.REPLICATE, serron.BorderMode.CONSTANT][border]
        ya = fn(xa, wa, border=border_mode)
        ya.backward(god)
        assert _eq(ya, y_ref)
        assert _eq(xa.grad, gi_ref)
        _gk_close(wa.grad, gk_ref, gk_wide)


def test_empty_inputs(serron):
    w = torch.zeros(3, 3, device="cuda")
    for shape in ((0, 1, 5, 5), (1, 0, 5, 5), (1, 1, 0, 5)):
        x = torch.rand(*shape, device="cuda", requires_grad=True)
        y = serron.erosion(x, w)
        assert y.shape == x.shape
        y.sum().backward()
        assert x.grad.shape == x.shape


def test_noncontiguous_input(serron):
    g = torch.Generator().manual_seed(5)
    x = torch.rand(2, 3, 20, 30, generator=g)
    w = torch.randn(3, 3, generator=g) * 0.1
    xt = x.transpose(2, 3)
    y = serron.dilation(xt.cuda(), w.cuda())
    assert _eq(y, oracle.forward(oracle.DILATE, xt.contiguous(), w, 1))


def test_validation_messages(serron):
    x = torch.rand(1, 1, 6, 6, device="cuda", dtype=torch.float64)
    with pytest.raises(RuntimeError, match="4-D"):
        serron.erosion(torch.rand(5, 5, device="cuda"), torch.zeros(3, device="cuda"))
    with pytest.raises(RuntimeError, match="must be 2-D"):
        serron.erosion(x, torch.zeros(3, dtype=torch.float64, device="cuda"))
    with pytest.raises(RuntimeError, match="share a dtype"):
        torch.ops.serron.erode(x.float(), torch.zeros(3, 3, dtype=torch.float64, device="cuda"), 0)
    with pytest.raises(RuntimeError, match="channel"):
        serron.erosion(torch.rand(1, 3, 6, 6, device="cuda"), torch.zeros(2, 3, 3, device="cuda"))
    with pytest.raises(RuntimeError, match="positive"):
        serron.erosion(x, torch.zeros(0, 3, dtype=torch.float64, device="cuda"))
    for border in (-1, 3, 99):
        with pytest.raises(RuntimeError, match="border"):
            torch.ops.serron.erode(x, torch.zeros(3, 3, dtype=torch.float64, device="cuda"), border)
    with pytest.raises(RuntimeError, match="grad_output"):
        torch.ops.serron.erode_backward(torch.rand(1, 1, 4, 4, dtype=torch.float64, device="cuda"), x,
                                        torch.zeros(3, 3, dtype=torch.float64, device="cuda"), 1)
    with pytest.raises(RuntimeError, match="invalid algo"):
        torch.ops.serron.erode(x, torch.zeros(3, 3, dtype=torch.float64, device="cuda"), 1, True, 7)
    with pytest.raises(RuntimeError, match="needs a flat structuring element"):
        torch.ops.serron.erode(x, torch.ones(3, 3, dtype=torch.float64, device="cuda"), 1, False, 3)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        torch.ops.serron.erode(x, torch.zeros(3, 3, dtype=torch.float64), 1)


def test_cuda_graph_capture(serron):
    """With the flatness passed in, a forward+backward is capturable (no host syncs)."""
    x = torch.rand(2, 3, 64, 64, device="cuda")
    w = torch.zeros(5, 5, device="cuda")
    go = torch.randn_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            torch.ops.serron.erode(x, w, 1, True, 0)
            torch.ops.serron.erode_backward(go, x, w, 1, True, True, 0)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = torch.ops.serron.erode(x, w, 1, True, 0)
        gi, gk = torch.ops.serron.erode_backward(go, x, w, 1, True, True, 0)
    x.copy_(torch.rand_like(x))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), oracle.forward(oracle.ERODE, x.cpu(), w.cpu(), 1, separable=True))
    assert torch.equal(gi.cpu(), oracle.backward(oracle.ERODE, go.cpu(), x.cpu(), w.cpu(), 1, separable=True)[0])
