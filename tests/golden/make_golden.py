"""Generate the golden fixtures under ``tests/golden/`` from the reference itself.

This script imports the reference's own Python package (vhrabar/serron 0.6.0,
``packages/serron/torch-ext/serron``) on top of the reference's own CPU operators,
compiled from the reference sources by ``make -C oracle ref`` into
``oracle/_ref/serron_ref_C.so`` (ops namespace ``serron_ref``).  Every tensor in
the fixtures is an output of that code; nothing is written by hand.

The reference loads its compiled library through ``_cmake_ops``; here a stand-in
module with the same attribute names points it at ``torch.ops.serron_ref``
instead, so the rest of the reference's Python code (functional, autograd,
modules, structuring_element, _flatness) runs unmodified.

CUDA autocast casts ``serron::erode/dilate`` inputs to float16
(``torch-ext/serron/_cmake_ops.py:175-189``).  To record that dtype flow on a
CPU-only machine, the same registration is made for the CPU key with float16
and the reference runs under ``torch.autocast("cpu", dtype=torch.float16)``.

Usage::

    make -C oracle ref
    python tests/golden/make_golden.py [--reference /path/to/packages/serron]

The fixtures are small (a few hundred KB in total) and committed.
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
# the reference's package sources: SERRON_REFERENCE_SOURCES, else a `reference` checkout beside this repository
DEFAULT_REFERENCE = os.environ.get("SERRON_REFERENCE_SOURCES") or str(REPO.parent / "reference" / "packages" / "serron")

BORDERS = {"reflect": 0, "replicate": 1, "constant": 2}
DTYPES = {"float64": torch.float64, "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def load_reference(reference: str) -> types.ModuleType:
    """Import the reference's Python package as ``refserron`` over the serron_ref ops."""
    lib = REPO / "oracle" / "_ref" / "serron_ref_C.so"
    if not lib.exists():
        raise SystemExit(f"{lib} is missing: run `make -C oracle ref` first")
    torch.ops.load_library(str(lib))

    fake = types.ModuleType("refserron._cmake_ops")
    fake._NAMESPACE = "serron_ref"
    fake.ops = torch.ops.serron_ref
    fake.add_op_namespace_prefix = lambda name: f"serron_ref::{name}"
    fake._gpu_backend = lambda: None
    fake._rocm_version = lambda: ""

    pkg_dir = os.path.join(reference, "torch-ext", "serron")
    spec = importlib.util.spec_from_file_location("refserron", os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    module = importlib.util.module_from_spec(spec)
    sys.modules["refserron"] = module
    sys.modules["refserron._cmake_ops"] = fake
    spec.loader.exec_module(module)
    for op in ("erode", "dilate"):
        torch.library.register_autocast(f"serron_ref::{op}", "cpu", torch.float16)
    return module


def gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


def se_cases(ref: types.ModuleType, channels: int, dtype: torch.dtype, g: torch.Generator) -> dict[str, torch.Tensor]:
    se = ref.structuring_element
    return {
        "rand3_shared": (torch.randn(3, 3, generator=g, dtype=torch.float64) * 0.5).to(dtype),
        "rand3_perch": (torch.randn(channels, 3, 3, generator=g, dtype=torch.float64) * 0.5).to(dtype),
        "rand_even_2x4": (torch.randn(channels, 2, 4, generator=g, dtype=torch.float64) * 0.5).to(dtype),
        "rand5x3_shared": (torch.randn(5, 3, generator=g, dtype=torch.float64) * 0.5).to(dtype),
        "square3": se.square(3, dtype=dtype),
        "square5_perch": torch.zeros(channels, 5, 5, dtype=dtype),
        "flat21": se.square(21, dtype=dtype),
        "flat_3x11": torch.zeros(3, 11, dtype=dtype),
        "disk2": se.disk(2, dtype=dtype),
        "cross3": se.cross(3, dtype=dtype),
        "diamond2": se.diamond(2, dtype=dtype),
    }


def primitives(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    """Raw serron_ref::erode/dilate(+_backward) over dtypes x borders x structuring elements."""
    ops = torch.ops.serron_ref
    out: dict[str, torch.Tensor] = {}
    for dname, dtype in DTYPES.items():
        g = gen(0x5E770)
        for xname, shape in (("randn", (2, 3, 9, 11)), ("quant", (1, 2, 16, 18))):
            x = torch.randn(*shape, generator=g, dtype=torch.float64)
            if xname == "quant":
                x = (x * 2).round()
            x = x.to(dtype)
            go = torch.randn(*shape, generator=g, dtype=torch.float64).to(dtype)
            out[f"{dname}.{xname}.x"] = x
            out[f"{dname}.{xname}.go"] = go
            for sname, w in se_cases(ref, shape[1], dtype, g).items():
                out[f"{dname}.{xname}.{sname}.w"] = w
                flat = bool(w.eq(0).all())
                for bname, border in BORDERS.items():
                    for opname in ("erode", "dilate"):
                        key = f"{dname}.{xname}.{sname}.{bname}.{opname}"
                        out[key + ".y"] = getattr(ops, opname)(x, w, border, flat, 0)
                        gi, gk = getattr(ops, opname + "_backward")(go, x, w, border, flat, True, 0)
                        out[key + ".gi"] = gi
                        out[key + ".gk"] = gk
    return out


def composites(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    """The public functional API, forward and autograd grads, for every op."""
    out: dict[str, torch.Tensor] = {}
    ops_names = ["erosion", "dilation", "opening", "closing", "gradient", "top_hat", "black_hat"]
    for dname in ("float64", "float32"):
        dtype = DTYPES[dname]
        g = gen(0x5E771)
        x0 = torch.randn(2, 3, 9, 11, generator=g, dtype=torch.float64).to(dtype)
        out[f"{dname}.x"] = x0
        kernels = {
            "perch": (torch.randn(3, 3, 3, generator=g, dtype=torch.float64) * 0.5).to(dtype),
            "flat5": torch.zeros(5, 5, dtype=dtype),
        }
        for kname, k0 in kernels.items():
            out[f"{dname}.{kname}.w"] = k0
            for bname, border in (("reflect", ref.BorderMode.REFLECT), ("replicate", ref.BorderMode.REPLICATE),
                                  ("constant", ref.BorderMode.CONSTANT)):
                for name in ops_names:
                    x = x0.clone().requires_grad_(True)
                    k = k0.clone().requires_grad_(True)
                    y = getattr(ref.functional, name)(x, k, border=border)
                    go = torch.randn(y.shape, generator=gen(len(name) * 31 + border.value.__len__()),
                                     dtype=torch.float64).to(dtype)
                    y.backward(go)
                    key = f"{dname}.{kname}.{bname}.{name}"
                    out[key + ".y"] = y.detach()
                    out[key + ".go"] = go
                    out[key + ".gx"] = x.grad
                    out[key + ".gk"] = k.grad
    return out


def tie_break(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    """Constant image: every window ties (tests/test_autograd.py:172-192)."""
    out: dict[str, torch.Tensor] = {}
    for op in ("erosion", "dilation"):
        for ksize in (3, 21):
            x = torch.full((1, 1, 9, 10), 2.5, dtype=torch.float64, requires_grad=True)
            kernel = torch.zeros(ksize, ksize, dtype=torch.float64)
            getattr(ref, op)(x, kernel, border=ref.BorderMode.REPLICATE).sum().backward()
            out[f"{op}.{ksize}.grad"] = x.grad
    return out


SEPARABLE_CASES = [
    # the fixed cases of the reference's tests/_separable_worker.py:15-26
    ("erosion", "reflect", (1, 2, 12, 14), (21, 21)),
    ("erosion", "replicate", (1, 2, 12, 14), (21, 21)),
    ("erosion", "constant", (1, 2, 12, 14), (21, 21)),
    ("dilation", "reflect", (1, 2, 12, 14), (21, 21)),
    ("dilation", "replicate", (1, 2, 12, 14), (21, 21)),
    ("dilation", "constant", (1, 2, 12, 14), (21, 21)),
    ("erosion", "replicate", (2, 3, 17, 23), (21, 3)),
    ("dilation", "reflect", (2, 3, 17, 23), (3, 21)),
    ("erosion", "constant", (1, 1, 5, 7), (31, 31)),
    ("dilation", "replicate", (1, 1, 5, 7), (31, 31)),
]


def separable(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    modes = {"reflect": ref.BorderMode.REFLECT, "replicate": ref.BorderMode.REPLICATE,
             "constant": ref.BorderMode.CONSTANT}
    for i, (op, border, shape, ksize) in enumerate(SEPARABLE_CASES):
        g = gen(0x5E770 + i)
        x = torch.randn(*shape, generator=g, dtype=torch.float64).requires_grad_(True)
        kernel = torch.zeros(shape[1], *ksize, dtype=torch.float64).requires_grad_(True)
        go = torch.randn(*shape, generator=g, dtype=torch.float64)
        y = getattr(ref.functional, op)(x, kernel, border=modes[border])
        y.backward(go)
        out[f"{i}.x"] = x.detach()
        out[f"{i}.go"] = go
        out[f"{i}.forward"] = y.detach()
        out[f"{i}.grad_input"] = x.grad
        out[f"{i}.grad_kernel"] = kernel.grad
    return out


def corridor() -> torch.Tensor:
    """A serpentine of open rows in a 13x13 frame (tests/test_reconstruction.py:184-200)."""
    grid = torch.zeros(13, 13, dtype=torch.float64)
    for row in range(0, 13, 2):
        grid[row, :] = 1.0
        if row + 1 < 13:
            grid[row + 1, 12 if (row // 2) % 2 == 0 else 0] = 1.0
    return grid.reshape(1, 1, 13, 13)


def reconstruction(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    se = ref.structuring_element
    for dname in ("float64", "float32"):
        dtype = DTYPES[dname]
        g = gen(0x5E772)
        mask = torch.randn(2, 3, 9, 11, generator=g, dtype=torch.float64).to(dtype)
        offset = torch.rand(mask.shape, generator=g, dtype=torch.float64).to(dtype)
        out[f"{dname}.mask"] = mask
        out[f"{dname}.offset"] = offset
        kernels = {
            "square3": se.square(3, dtype=dtype),
            "cross3": se.cross(3, dtype=dtype),
            "diamond2": se.diamond(2, dtype=dtype),
            "per_channel": torch.zeros(3, 3, 3, dtype=dtype),
        }
        for kname, k in kernels.items():
            out[f"{dname}.{kname}.w"] = k
            for bname, border in (("reflect", ref.BorderMode.REFLECT), ("replicate", ref.BorderMode.REPLICATE),
                                  ("constant", ref.BorderMode.CONSTANT)):
                out[f"{dname}.{kname}.{bname}.by_dilation"] = ref.reconstruction_by_dilation(
                    mask - 4.0 * offset, mask, k, border=border)
                out[f"{dname}.{kname}.{bname}.by_erosion"] = ref.reconstruction_by_erosion(
                    mask + 4.0 * offset, mask, k, border=border)
    mask = corridor()
    marker = torch.zeros_like(mask)
    marker[0, 0, 0, 0] = 1.0
    out["corridor.mask"] = mask
    out["corridor.flood"] = ref.reconstruction_by_dilation(marker, mask, se.cross(3, dtype=torch.float64))
    marker = torch.zeros_like(mask)
    marker[0, 0, 1, 6] = 1.0
    out["corridor.walled"] = ref.reconstruction_by_dilation(marker, mask, se.cross(3, dtype=torch.float64))
    profile = torch.tensor([[[[1.0, 2.0, 3.0], [0.0, 0.0, 4.0], [9.0, 0.0, 5.0]]]], dtype=torch.float64)
    marker = torch.zeros_like(profile)
    marker[0, 0, 0, 0] = 1.0
    out["profile.mask"] = profile
    out["profile.flood"] = ref.reconstruction_by_dilation(marker, profile, se.cross(3, dtype=torch.float64))
    return out


def config1(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    """erosion then dilation of rand(1,1,256,256) (CPU seed 0) by disk(3), REPLICATE, forward."""
    torch.manual_seed(0)
    x = torch.rand(1, 1, 256, 256)
    k = ref.structuring_element.disk(3)
    y = ref.dilation(ref.erosion(x, k, border=ref.BorderMode.REPLICATE), k, border=ref.BorderMode.REPLICATE)
    return {"x": x, "y": y}


def autocast_opening(ref: types.ModuleType) -> dict[str, torch.Tensor]:
    """Opening2d with a non-flat fp32 SE on a bf16 image under (CUDA-style, float16) autocast."""
    out: dict[str, torch.Tensor] = {}
    g = gen(0)
    x0 = torch.rand(2, 4, 16, 16, generator=g).to(torch.bfloat16)
    w0 = torch.randn(4, 7, 7, generator=g) * 0.1
    layer = ref.Opening2d(4, 7)
    with torch.no_grad():
        layer.weight.copy_(w0)
    x = x0.clone().requires_grad_(True)
    with torch.autocast("cpu", dtype=torch.float16):
        y = layer(x)
    go = torch.randn(y.shape, generator=g).to(y.dtype)
    y.backward(go)
    out.update({"x": x0, "w": w0, "y": y.detach(), "go": go, "gx": x.grad, "gw": layer.weight.grad})
    return out


def pack(tensors: dict[str, torch.Tensor]) -> dict[str, object]:
    """Concatenate same-dtype tensors into one flat buffer each, with an index (see tests/golden/__init__.py)."""
    buffers: dict[str, list[torch.Tensor]] = {}
    index: dict[str, tuple[str, int, list[int]]] = {}
    offsets: dict[str, int] = {}
    for key, t in tensors.items():
        dname = str(t.dtype).removeprefix("torch.")
        flat = t.detach().contiguous().reshape(-1)
        index[key] = (dname, offsets.get(dname, 0), list(t.shape))
        offsets[dname] = offsets.get(dname, 0) + flat.numel()
        buffers.setdefault(dname, []).append(flat)
    return {"index": index, "buffers": {d: torch.cat(b) for d, b in buffers.items()}}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=DEFAULT_REFERENCE)
    args = parser.parse_args()
    ref = load_reference(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fixtures = {
        "primitives": primitives(ref),
        "composites": composites(ref),
        "tie_break": tie_break(ref),
        "separable": separable(ref),
        "reconstruction": reconstruction(ref),
        "config1": config1(ref),
        "autocast_opening": autocast_opening(ref),
    }
    for name, tensors in fixtures.items():
        path = HERE / f"{name}.pt"
        torch.save(pack(tensors), path)
        print(f"{path.relative_to(REPO)}: {len(tensors)} tensors, {path.stat().st_size / 1024:.0f} KB")


if __name__ == "__main__":
    main()
