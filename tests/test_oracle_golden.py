"""Pin the oracle (oracle/morph_oracle.c) to golden vectors the reference produced.

The fixtures under tests/golden/ are outputs of the reference's own CPU operators and
Python API (tests/golden/make_golden.py).  Every comparison here is bit-exact.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from tests.golden import load

BORDERS = {"reflect": 0, "replicate": 1, "constant": 2}
OPS = {"erode": oracle.ERODE, "dilate": oracle.DILATE}


def _primitive_cases():
    data = load("primitives")
    seen = set()
    for key in data:
        if key.endswith(".y"):
            dname, xname, sname, bname, opname, _ = key.split(".")
            seen.add((dname, xname, sname, bname, opname))
    return sorted(seen)


@pytest.mark.parametrize("case", _primitive_cases(), ids=lambda c: ".".join(c))
def test_primitives(case):
    dname, xname, sname, bname, opname = case
    data = load("primitives")
    x = data[f"{dname}.{xname}.x"]
    go = data[f"{dname}.{xname}.go"]
    w = data[f"{dname}.{xname}.{sname}.w"]
    key = f"{dname}.{xname}.{sname}.{bname}.{opname}"
    flat = oracle.is_flat(w)
    for separable in ([False, True] if flat else [False]):
        y = oracle.forward(OPS[opname], x, w, BORDERS[bname], separable=separable)
        assert torch.equal(y, data[key + ".y"]), f"forward separable={separable}"
        gi, gk = oracle.backward(OPS[opname], go, x, w, BORDERS[bname], separable=separable)
        assert torch.equal(gi, data[key + ".gi"]), f"grad_input separable={separable}"
        assert torch.equal(gk, data[key + ".gk"]), f"grad_kernel separable={separable}"


def test_tie_break_kat():
    data = load("tie_break")
    for op, code in (("erosion", oracle.ERODE), ("dilation", oracle.DILATE)):
        for k in (3, 21):
            x = torch.full((1, 1, 9, 10), 2.5, dtype=torch.float64)
            w = torch.zeros(k, k, dtype=torch.float64)
            gi, _ = oracle.backward(code, torch.ones_like(x), x, w, 1, separable=k >= 5)
            assert torch.equal(gi, data[f"{op}.{k}.grad"])


def test_separable_worker_cases():
    data = load("separable")
    from tests.golden.make_golden import SEPARABLE_CASES

    for i, (op, border, shape, ksize) in enumerate(SEPARABLE_CASES):
        x, go = data[f"{i}.x"], data[f"{i}.go"]
        w = torch.zeros(shape[1], *ksize, dtype=torch.float64)
        code = oracle.ERODE if op == "erosion" else oracle.DILATE
        for separable in (False, True):
            y = oracle.forward(code, x, w, BORDERS[border], separable=separable)
            gi, gk = oracle.backward(code, go, x, w, BORDERS[border], separable=separable)
            assert torch.equal(y, data[f"{i}.forward"])
            assert torch.equal(gi, data[f"{i}.grad_input"])
            assert torch.equal(gk, data[f"{i}.grad_kernel"])


def test_config1_forward():
    data = load("config1")
    from tests.golden.make_golden import DTYPES  # noqa: F401  (fixture provenance)

    x = data["x"]
    k = torch.full((7, 7), float("-inf"))
    yy, xx = torch.meshgrid(torch.arange(7) - 3, torch.arange(7) - 3, indexing="ij")
    k[yy * yy + xx * xx <= 9] = 0.0
    y = oracle.forward(oracle.DILATE, oracle.forward(oracle.ERODE, x, k, 1), k, 1)
    assert torch.equal(y, data["y"])


@pytest.mark.parametrize("dname", ["float64", "float32"])
def test_reconstruction(dname):
    data = load("reconstruction")
    mask, offset = data[f"{dname}.mask"], data[f"{dname}.offset"]
    for kname in ("square3", "cross3", "diamond2", "per_channel"):
        w = data[f"{dname}.{kname}.w"]
        for bname, border in BORDERS.items():
            got, _ = oracle.reconstruct(True, mask - 4.0 * offset, mask, w, border)
            assert torch.equal(got, data[f"{dname}.{kname}.{bname}.by_dilation"])
            got, _ = oracle.reconstruct(False, mask + 4.0 * offset, mask, w, border)
            assert torch.equal(got, data[f"{dname}.{kname}.{bname}.by_erosion"])


def test_reconstruction_fixtures():
    data = load("reconstruction")
    cross = torch.full((3, 3), float("-inf"), dtype=torch.float64)
    cross[1, :] = 0.0
    cross[:, 1] = 0.0
    mask = data["corridor.mask"]
    marker = torch.zeros_like(mask)
    marker[0, 0, 0, 0] = 1.0
    for check_every in (1, 16, 256):
        got, _ = oracle.reconstruct(True, marker, mask, cross, 2, check_every=check_every)
        assert torch.equal(got, data["corridor.flood"])
    marker = torch.zeros_like(mask)
    marker[0, 0, 1, 6] = 1.0
    assert torch.equal(oracle.reconstruct(True, marker, mask, cross, 2)[0], data["corridor.walled"])
    profile = data["profile.mask"]
    marker = torch.zeros_like(profile)
    marker[0, 0, 0, 0] = 1.0
    assert torch.equal(oracle.reconstruct(True, marker, profile, cross, 2)[0], data["profile.flood"])


def test_reconstruction_budget():
    data = load("reconstruction")
    cross = torch.full((3, 3), float("-inf"), dtype=torch.float64)
    cross[1, :] = 0.0
    cross[:, 1] = 0.0
    mask = data["corridor.mask"]
    marker = torch.zeros_like(mask)
    marker[0, 0, 0, 0] = 1.0
    with pytest.raises(RuntimeError, match="no fixed point"):
        oracle.reconstruct(True, marker, mask, cross, 2, max_iter=3)


def test_autocast_opening_flow():
    """The CUDA-autocast dtype flow of Opening2d, replayed on the oracle's raw ops."""
    d = load("autocast_opening")
    x, w, go = d["x"], d["w"], d["go"]
    x32, w32 = x.float(), w
    y1 = oracle.forward(oracle.ERODE, x32.half(), w32.half(), 1)
    y1_32 = y1.float()
    y2 = oracle.forward(oracle.DILATE, y1_32.half(), w32.half(), 1)
    assert torch.equal(y2, d["y"])
    g1, gw_a = oracle.backward(oracle.DILATE, go.float(), y1_32, w32, 1)
    gx32, gw_b = oracle.backward(oracle.ERODE, g1.half().float(), x32, w32, 1)
    assert torch.equal(gx32.to(torch.bfloat16), d["gx"])
    torch.testing.assert_close(gw_a + gw_b, d["gw"], rtol=0, atol=0)


def test_half_conversions_round_to_nearest_even():
    vals = torch.randn(100000, dtype=torch.float32) * 1000
    vals = torch.cat([vals, torch.tensor([65504.0, 65519.9, 65520.0, 6e-8, 3e-8, 2.9e-8, -0.0, float("inf")])])
    lib = oracle._load()
    import ctypes

    lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
    lib.oracle_f32_to_f16.restype = ctypes.c_uint16
    lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
    lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
    h = torch.tensor([lib.oracle_f32_to_f16(float(v)) for v in vals[:5000].tolist() + vals[-8:].tolist()],
                     dtype=torch.int32).to(torch.int16)
    ref = torch.cat([vals[:5000], vals[-8:]]).half().view(torch.int16)
    assert torch.equal(h, ref)
    b = torch.tensor([lib.oracle_f32_to_bf16(float(v)) for v in vals[:5000].tolist()], dtype=torch.int32).to(torch.int16)
    assert torch.equal(b, vals[:5000].bfloat16().view(torch.int16))
