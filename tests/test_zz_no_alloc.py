"""serron_backward_static_scratch (the backward that allocates nothing) against serron_erode_backward /
serron_dilate_backward with a caller workspace, both through the C ABI.

Named to be collected last, so it also runs after every other test has used the library; it passes
alone in a fresh process too.  Each case runs twice in a row with different data, so a result that
leaned on scratch left over from the previous call would show.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

INF = float("inf")


def _call(lib, static, op, go, x, se, need_kg, flat):
    from serron_b200 import _lib

    gi = torch.full_like(x, float("nan"))
    gk = torch.full_like(se, float("nan"))
    gs, gd = _lib.sizes(go.shape)
    xs, xd = _lib.sizes(x.shape)
    ks, kd = _lib.sizes(se.shape)
    dtype = _lib.DTYPE_CODE[x.dtype]
    dev = x.device.index
    stream = _lib.stream_of(x)
    common = (go.data_ptr(), gs, gd, x.data_ptr(), xs, xd, se.data_ptr(), ks, kd, dtype, 0, flat, need_kg, 0)
    if static:
        rc = lib.serron_backward_static_scratch(op, *common, gi.data_ptr(), gk.data_ptr(), dev, stream)
    else:
        plan = _lib.Plan()
        _lib.raise_for(lib.serron_plan(xs, xd, se.data_ptr(), ks, kd, dtype, flat, 0, 1, dev, stream,
                                       ctypes.byref(plan)))
        ws = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=x.device)
        fn = lib.serron_erode_backward if op == _lib.ERODE else lib.serron_dilate_backward
        rc = fn(*common, gi.data_ptr(), gk.data_ptr(), ws.data_ptr(), plan.workspace_bytes, dev, stream)
    _lib.raise_for(rc)
    torch.cuda.synchronize()
    return gi, gk


def _se(kind: str, dtype, gen):
    if kind == "flat15":
        return torch.zeros(15, 15, dtype=dtype)
    if kind == "nonflat5":
        return (torch.rand(5, 5, generator=gen) * 0.2).to(dtype)
    if kind == "cross3":
        return torch.tensor([[-INF, 0.0, -INF], [0.0, 0.0, 0.0], [-INF, 0.0, -INF]], dtype=dtype)
    raise ValueError(kind)


CASES = [
    ("flat15", torch.float32, (2, 3, 96, 130), 1),
    ("nonflat5", torch.float32, (2, 3, 67, 45), 0),
    ("cross3", torch.float64, (1, 2, 40, 33), -1),
    ("nonflat5", torch.float16, (1, 4, 50, 70), 0),
    ("flat15", torch.bfloat16, (1, 2, 64, 64), 1),
]


@pytest.mark.parametrize("kind,dtype,shape,flat", CASES)
@pytest.mark.parametrize("op", [0, 1])
@pytest.mark.parametrize("need_kg", [1, 0])
def test_static_scratch_matches_workspace_backward(kind, dtype, shape, flat, op, need_kg):
    from serron_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    for call in range(2):
        gen = torch.Generator().manual_seed(1000 * call + 7)
        x = torch.rand(shape, generator=gen).to(dtype).to(dev)
        go = torch.randn(shape, generator=gen).to(dtype).to(dev)
        se = _se(kind, dtype, gen).to(dev)
        want_gi, want_gk = _call(lib, False, op, go, x, se, need_kg, flat)
        got_gi, got_gk = _call(lib, True, op, go, x, se, need_kg, flat)
        assert torch.equal(got_gi, want_gi), (call, kind, dtype)
        assert torch.equal(got_gk, want_gk), (call, kind, dtype)


def test_static_scratch_rejects_a_call_beyond_its_size():
    from serron_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    # 5x5 non-flat: one byte of winner record per output; 40 Mi outputs need more than 32 MiB
    shape = (1, 1, 4096, 10240)
    x = torch.zeros(shape, device=dev)
    go = torch.zeros(shape, device=dev)
    se = torch.full((5, 5), 0.5, device=dev)
    gi = torch.zeros_like(x)
    gk = torch.full_like(se, 3.0)
    gs, gd = _lib.sizes(go.shape)
    ks, kd = _lib.sizes(se.shape)
    rc = lib.serron_backward_static_scratch(0, go.data_ptr(), gs, gd, x.data_ptr(), gs, gd, se.data_ptr(), ks, kd, 0,
                                            0, 0, 1, 0, gi.data_ptr(), gk.data_ptr(), 0, _lib.stream_of(x))
    assert rc == _lib.ERR_WORKSPACE
    msg = lib.serron_last_error().decode()
    assert "static array" in msg and str(32 << 20) in msg
    torch.cuda.synchronize()
    assert torch.equal(gk, torch.full_like(se, 3.0))  # nothing ran
    assert not gi.any()
