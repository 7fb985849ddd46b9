"""Host-side checks of the C ABI that need no GPU: the library loads, exports every declared symbol,
and rejects bad arguments with the reference's messages before touching a device."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from serron_b200 import _lib

    return _lib.load()


def _declared_symbols() -> set[str]:
    text = open(os.path.join(REPO, "include", "serron_b200.h")).read()
    return set(re.findall(r"SERRON_API\s+[\w\s\*]+?\b(serron_\w+)\s*\(", text))


def test_exports_every_declared_symbol(lib):
    from serron_b200 import _lib

    declared = _declared_symbols()
    assert declared == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.serron_abi_version() == 1


def _call_forward(lib, in_shape, k_shape, border=1, algo=0, dtype=0):
    from serron_b200 import _lib

    xs, xd = _lib.sizes(in_shape)
    ks, kd = _lib.sizes(k_shape)
    rc = lib.serron_erode(None, xs, xd, None, ks, kd, dtype, border, 1, algo, None, 0, None)
    return rc, lib.serron_last_error().decode()


@pytest.mark.parametrize("in_shape,k_shape,border,algo,pattern", [
    ((5, 5), (3, 3), 1, 0, r"serron::erode: input must be 4-D \(N, C, H, W\), got 2-D"),
    ((1, 1, 6, 6), (3,), 1, 0, r"kernel must be 2-D \(kH, kW\) or 3-D \(C, kH, kW\), got 1-D"),
    ((1, 3, 6, 6), (2, 3, 3), 1, 0, r"kernel channel dim \(2\) must match input channels \(3\)"),
    ((1, 1, 6, 6), (0, 3), 1, 0, r"kernel spatial dims must be positive"),
    ((1, 1, 6, 6), (3, 3), 3, 0, r"invalid border mode 3"),
    ((1, 1, 6, 6), (3, 3), -1, 0, r"invalid border mode -1"),
    ((1, 1, 6, 6), (3, 3), 1, 4, r"invalid algo 4"),
])
def test_validation_before_any_device_work(lib, in_shape, k_shape, border, algo, pattern):
    rc, msg = _call_forward(lib, in_shape, k_shape, border, algo)
    assert rc == 1
    assert re.search(pattern, msg), msg


def test_empty_input_needs_no_device(lib):
    rc, _ = _call_forward(lib, (0, 3, 5, 5), (3, 3))
    assert rc == 0


def test_backward_shape_mismatch_message(lib):
    from serron_b200 import _lib

    xs, xd = _lib.sizes((1, 1, 6, 6))
    gs, gd = _lib.sizes((1, 1, 4, 4))
    ks, kd = _lib.sizes((3, 3))
    rc = lib.serron_erode_backward(None, gs, gd, None, xs, xd, None, ks, kd, 0, 1, 1, 1, 0, None, None, None, 0, 0,
                                   None)
    assert rc == 1
    assert "grad_output shape must match input" in lib.serron_last_error().decode()


def test_workspace_sizes_are_deterministic(lib):
    from serron_b200 import _lib

    xs, xd = _lib.sizes((32, 64, 512, 512))
    ks, kd = _lib.sizes((15, 15))
    with_w = lib.serron_backward_workspace_bytes(xs, xd, ks, kd, 0, 4, 1)
    without = lib.serron_backward_workspace_bytes(xs, xd, ks, kd, 0, 4, 0)
    target_map = 32 * 64 * 512 * (512 // 32) * 4  # one bit per pixel
    assert with_w == target_map
    assert without == 32 * 64 * 512 * 512 + target_map  # and one byte per output for the u8 record
    # relaxation: a state word per 64x64 tile and the worklist ring (8 bytes per cell, four cells per tile
    # plus four per CTA of the largest grid); the Jacobi schedule: a second image
    tiles = 32 * 64 * 8 * 8

    def align256(v):
        return (v + 255) // 256 * 256

    assert lib.serron_reconstruct_workspace_bytes(xs, xd, 0, 0) == 256 + align256(4 * tiles) + align256(
        8 * (4 * tiles + 4 * 4096 + 64))
    assert lib.serron_reconstruct_workspace_bytes(xs, xd, 0, 5) == 256 + 32 * 64 * 512 * 512 * 4


def test_thresholds_table(lib):
    # the B200-measured default (the reference's is 11)
    assert lib.serron_get_separable_min_k(0, 0, 0) == 3
    assert lib.serron_set_separable_min_k(0, 0, 0, 7) == 7
    assert lib.serron_get_separable_min_k(0, 0, 1) == 3
    assert lib.serron_set_separable_min_k(0, 0, 0, 0) == 3


def test_public_api_surface():
    import serron_b200

    expected = ["BorderMode", "Closing2d", "Dilation2d", "Erosion2d", "Opening2d", "Operation", "__version__",
                "autotune", "black_hat", "calibrate", "closing", "dilation", "erosion", "functional", "gradient",
                "opening", "reconstruction_by_dilation", "reconstruction_by_erosion", "structuring_element",
                "top_hat"]
    assert serron_b200.__all__ == expected
    for name in expected:
        assert hasattr(serron_b200, name)
    for op in ("erode", "dilate", "erode_backward", "dilate_backward", "feasible_algos", "heuristic_algo",
               "set_separable_min_k", "get_separable_min_k"):
        assert hasattr(torch.ops.serron, op), op


def test_no_cpu_path():
    import serron_b200

    x = torch.rand(1, 1, 8, 8)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        serron_b200.erosion(x, serron_b200.structuring_element.square(3))
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        torch.ops.serron.erode(x, torch.zeros(3, 3), 1)


def test_structuring_elements_match_reference_fixtures():
    import serron_b200.structuring_element as se
    from tests.golden import load

    data = load("primitives")
    for dname, dtype in (("float32", torch.float32), ("float16", torch.float16)):
        assert torch.equal(data[f"{dname}.randn.disk2.w"], se.disk(2, dtype=dtype))
        assert torch.equal(data[f"{dname}.randn.cross3.w"], se.cross(3, dtype=dtype))
        assert torch.equal(data[f"{dname}.randn.diamond2.w"], se.diamond(2, dtype=dtype))
        assert torch.equal(data[f"{dname}.randn.square3.w"], se.square(3, dtype=dtype))
    with pytest.raises(ValueError, match="floating dtype"):
        se.square(3, dtype=torch.int32)
    with pytest.raises(ValueError, match="size must be >= 1"):
        se.cross(0)
    with pytest.raises(ValueError, match="radius must be >= 0"):
        se.disk(-1)


def test_flatness_cache():
    from serron_b200 import _flatness, structuring_element as se

    k = torch.zeros(3, 3)
    assert _flatness.is_flat(k)
    k[0, 0] = 1.0
    assert not _flatness.is_flat(k)  # the version counter moved
    assert not _flatness.is_flat(se.disk(2))
    assert _flatness.is_flat(se.square(4))


def test_modules_init_and_state_dict():
    import serron_b200

    layer = serron_b200.Opening2d(4, 7)
    assert layer.weight.shape == (4, 7, 7)
    assert torch.equal(layer.weight, torch.zeros(4, 7, 7))
    sd = layer.state_dict()
    assert list(sd) == ["weight"]
    other = serron_b200.Closing2d(4, 7)
    other.load_state_dict(sd)


def test_reconstruction_validation():
    import serron_b200

    mask = torch.rand(1, 1, 6, 6)
    k = serron_b200.structuring_element.square(3)
    with pytest.raises(ValueError, match="share a shape"):
        serron_b200.reconstruction_by_dilation(torch.rand(1, 1, 6, 7), mask, k)
    with pytest.raises(ValueError, match="check_every must be >= 1"):
        serron_b200.reconstruction_by_dilation(mask, mask, k, check_every=0)
    with pytest.raises(ValueError, match="max_iter must be >= 1"):
        serron_b200.reconstruction_by_dilation(mask, mask, k, max_iter=0)
    with pytest.raises(RuntimeError, match="no backward pass"):
        serron_b200.reconstruction_by_dilation(mask.clone().requires_grad_(True), mask, k)
    bad = torch.full((3, 3), float("-inf"))
    bad[1, 1] = -1.0
    with pytest.raises(ValueError, match="anchor tap"):
        serron_b200.reconstruction_by_dilation(mask, mask, bad)


def _sizes(shape):
    return (ctypes.c_int64 * len(shape))(*shape), len(shape)


def test_derived_supported_bounds(lib):
    """The one-launch derived operations take windows up to 7 a side, and (modes 1-4) images at least as
    large as the window; host only."""
    cases = [
        (0, (1, 1, 40, 40), (7, 7), 1), (0, (1, 1, 40, 40), (8, 3), 0), (0, (1, 1, 3, 3), (7, 7), 1),
        (1, (1, 1, 40, 40), (7, 7), 1), (1, (1, 1, 6, 40), (7, 7), 0), (3, (2, 3, 7, 7), (3, 7, 7), 1),
        (4, (1, 1, 40, 40), (1, 7), 1), (5, (1, 1, 40, 40), (3, 3), 0), (2, (1, 1, 40), (3, 3), 0),
    ]
    for mode, xshape, kshape, want in cases:
        xs, xd = _sizes(xshape)
        ks, kd = _sizes(kshape)
        assert lib.serron_derived_supported(mode, xs, xd, ks, kd) == want, (mode, xshape, kshape)


def test_new_entry_points_validate_before_device_work(lib):
    from serron_b200 import _lib

    xs, xd = _sizes((1, 1, 40, 40))
    ks, kd = _sizes((9, 9))
    rc = lib.serron_derived_forward(1, None, xs, xd, None, ks, kd, 0, 1, None, None, None, 0x11, 0, None)
    assert rc == _lib.ERR_INVALID and b"no one-launch form" in lib.serron_last_error()
    ks3, kd3 = _sizes((3, 3))
    rc = lib.serron_derived_forward(1, None, xs, xd, None, ks3, kd3, 0, 1, None, None, None, 0x12, 0, None)
    assert rc == _lib.ERR_INVALID and b"winner format" in lib.serron_last_error()
    rc = lib.serron_backward_from_winners_widened(0, None, 1, xs, xd, ks3, kd3, 1, 0, None, 0x11, None, 2, None,
                                                  None, 0, 0, None)
    assert rc == _lib.ERR_INVALID and b"float32, float16 or bfloat16" in lib.serron_last_error()
    rc = lib.serron_backward_from_winners_widened(0, None, 2, xs, xd, ks3, kd3, 1, 0, None, 0x4, None, 3, None,
                                                  None, 0, 0, None)
    assert rc == _lib.ERR_INVALID and b"direct one- or two-byte records" in lib.serron_last_error()
    steps = ctypes.c_int64(0)
    rc = lib.serron_reconstruct_from_edges(1, None, None, xs, xd, None, ks3, kd3, 0, 2, -1, 0, None, None, 0, 0, None,
                                           ctypes.byref(steps))
    assert rc == _lib.ERR_INVALID and b"seed_top and seed_bottom" in lib.serron_last_error()
