"""Benchmark: erode + dilate forward + backward throughput on B200.

Workload (the separable flat-rectangle configuration the headline metric is quoted on):
x = rand(32, 64, 512, 512) float32, grad_output = randn_like(x), flat square(15) structuring element,
REFLECT border; one step = dilation(x) and erosion(x), each forward + backward, through the public
API (``serron_b200.dilation`` / ``erosion`` + autograd).  Inputs (2.1 GB each) are far larger than L2,
so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1: one process per GPU (torchrun); every rank runs the same per-GPU workload with its own seed
(weak scaling, no collective on the data path); time = max over ranks of CUDA-event time.
``--impl reference`` times the reference's own CPU implementation (compiled from its sources into
``oracle/_ref``; the oracle port when that library is absent) on a bounded slice of the workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

SHAPE = (32, 64, 512, 512)
K = 15
BORDER_NAME = "reflect"
METRIC = "output Gpix/s erode+dilate fwd+bwd per GPU at 1/2/4/8 B200; % of HBM/min-max roofline"
WORKLOAD = "flat separable: dilation+erosion of x(32,64,512,512) fp32 uniform[0,1), square(15), REFLECT, fwd+bwd"
PRIMS = 2  # primitive calls per step
# algorithmic HBM bytes per output pixel of each timed stage (fp32 value 4 B, winner record 1 B):
# "forward" is one launch of the separable sweep forward (records and target map included), "gather"
# the backward's launch of the winners' sums
FWD_BYTES_PER_PX = 4 + 4 + 1  # read x, write y, write winners
BWD_BYTES_PER_PX = 4 + 1 + 4  # read grad_output, read winners, write grad_input
# per-call DRAM traffic of each stage at the full workload: dram__bytes_read + dram__bytes_write of an
# ncu capture of the batch-4 workload (1/8 of the pixels), times 8
NCU_TRAFFIC_BYTES = {"forward": 4.63e9, "gather": 4.64e9}
LAUNCHES_PER_STEP = 2 * (1 + 1)  # per op: the forward, then the gather's sum kernel
CPU_SAMPLE = (1, 64, 512, 512)  # one image of the batch: the slice the CPU baseline times (scaled by pixels)
CPU_MIN_SECONDS = 10.0  # the baseline in our arm's line times at least this much CPU work


def _peaks() -> tuple[float, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.reader = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.reader is not None:
            self.reader.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist() -> tuple[int, int, int]:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _cpu_baseline(steps: int | None = None, warmup: int = 1) -> dict:
    """The reference's CPU path on a slice, all host threads; Gpix/s scaled by pixels.  With `steps`
    None it times whole steps until CPU_MIN_SECONDS have passed (at least 3)."""
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    x = torch.rand(*CPU_SAMPLE, generator=g)
    go = torch.randn(*CPU_SAMPLE, generator=g)
    w = torch.zeros(K, K)
    ref = oracle.reference_ops()
    kind = "reference" if ref is not None else "port"

    def step() -> None:
        if ref is not None:
            for fwd, bwd in ((ref.dilate, ref.dilate_backward), (ref.erode, ref.erode_backward)):
                fwd(x, w, 0, True, 0)
                bwd(go, x, w, 0, True, False, 0)
        else:
            for op in (oracle.DILATE, oracle.ERODE):
                oracle.forward(op, x, w, 0, separable=True)
                oracle.backward(op, go, x, w, 0, separable=True, need_kernel_grad=False)

    for _ in range(max(1, warmup)):
        step()
    n = 0
    t0 = time.perf_counter()
    while True:
        step()
        n += 1
        if (steps is not None and n >= steps) or (
                steps is None and n >= 3 and time.perf_counter() - t0 >= CPU_MIN_SECONDS):
            break
    dt = (time.perf_counter() - t0) / n
    px = CPU_SAMPLE[0] * CPU_SAMPLE[1] * CPU_SAMPLE[2] * CPU_SAMPLE[3]
    return {"value": px * PRIMS / dt / 1e9, "unit": "Gpix/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"x{CPU_SAMPLE} (one image of the 32x64x512x512 batch), dilation+erosion fwd+bwd with the "
                      f"reference's CPU operators, {n} step(s) after {max(1, warmup)} warm-up, {dt:.2f} s/step; "
                      f"Gpix/s scales linearly in pixels",
            "ms_per_step_sample": dt * 1e3}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    steps, warmup = max(1, args.steps), max(1, args.warmup)
    base = _cpu_baseline(steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "Gpix/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": base["ms_per_step_sample"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": list(CPU_SAMPLE)},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "Gpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_cuda(args) -> None:
    """The reference's own CUDA kernels (sm_100, compiled from its sources into oracle/_ref by
    ``make -C oracle ref_cuda``) on this arm's workload and timing rules: each step is dilation and erosion,
    each forward + backward, through the reference's operator API (its own bindings, loaded as
    ``torch.ops.serron_ref``).  One small call is checked against the reference's CPU operators first."""
    world, rank, local = _dist()
    lib_dir = os.path.join(REPO, "oracle", "_ref")
    cpu_lib, cuda_lib = os.path.join(lib_dir, "serron_ref_C.so"), os.path.join(lib_dir, "serron_ref_C_cuda.so")
    if not (os.path.exists(cpu_lib) and os.path.exists(cuda_lib)):
        if rank == 0:
            print(json.dumps({"impl": "reference_cuda", "unavailable": "the reference's CUDA library was not built "
                              "(make -C oracle ref_cuda)"}), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    torch.ops.load_library(cpu_lib)
    torch.ops.load_library(cuda_lib)
    ref = torch.ops.serron_ref
    w = torch.zeros(K, K, device=dev)
    small = torch.rand(1, 2, 40, 48, generator=torch.Generator().manual_seed(1))
    got = ref.dilate(small.to(dev), w, 0, True, 0).cpu()
    if not torch.equal(got, ref.dilate(small, w.cpu(), 0, True, 0)):
        raise SystemExit("bench.py: the reference's CUDA forward disagrees with its CPU forward")
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    shape = (args.batch,) + SHAPE[1:]
    x = torch.rand(*shape, device=dev, generator=gen)
    go = torch.randn(*shape, device=dev, generator=gen)
    px = shape[0] * shape[1] * shape[2] * shape[3]

    def step() -> None:
        for fwd, bwd in ((ref.dilate, ref.dilate_backward), (ref.erode, ref.erode_backward)):
            fwd(x, w, 0, True, 0)
            bwd(go, x, w, 0, True, False, 0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({"impl": "reference_cuda", "metric": METRIC, "value": px * PRIMS * world / (ms * 1e-3) / 1e9,
                          "unit": "Gpix/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "dtype": "f32",
                          "data": "synthetic", "config": {"workload": WORKLOAD, "per_gpu_batch": list(shape)},
                          "note": "the reference's own sm_100 kernels (element/line passes, atomic scatter backward) "
                                  "through its operator API"}), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_ours(args) -> None:
    world, rank, local = _dist()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import serron_b200 as serron
    from serron_b200 import _lib

    _lib.load()
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    shape = (args.batch,) + SHAPE[1:]
    x = torch.rand(*shape, device=dev, generator=gen).requires_grad_(True)
    go = torch.randn(*shape, device=dev, generator=gen)
    k = serron.structuring_element.square(K, device=dev)
    border = serron.BorderMode.REFLECT
    px = shape[0] * shape[1] * shape[2] * shape[3]

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    kernel_ms = {"forward": [], "gather": []}

    def step(record: bool) -> None:
        i = 0
        for fn in (serron.dilation, serron.erosion):
            if record:
                ev[i].record()
            y = fn(x, k, border=border)
            if record:
                ev[i + 1].record()
            (gx,) = torch.autograd.grad(y, x, go)
            i += 2
        if record:
            ev[4].record()

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step(True)
        torch.cuda.synchronize()
        kernel_ms["forward"] += [ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])]
        kernel_ms["gather"] += [ev[1].elapsed_time(ev[2]), ev[3].elapsed_time(ev[4])]
    stop.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop() if clocks else None
    elapsed = start.elapsed_time(stop)
    t = torch.tensor([elapsed], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms_per_step = float(t.item()) / args.steps
    value = px * PRIMS * world / (ms_per_step * 1e-3) / 1e9

    # end to end through the public API with host buffers: H2D of the step's inputs from pinned memory,
    # both ops forward + backward, D2H of both outputs and both input gradients.  The batch goes through
    # in chunks on three streams (copies in, compute, copies out) so that both copy directions overlap
    # the compute and each other, as a user streaming host data through the API would run it.
    x_host = x.detach().cpu().pin_memory()
    go_host = go.cpu().pin_memory()
    outs = [torch.empty(shape, dtype=torch.float32).pin_memory() for _ in range(4)]
    nch = min(8, shape[0])
    bounds = [(i * shape[0] // nch, (i + 1) * shape[0] // nch) for i in range(nch)]
    cshape = (max(e - b for b, e in bounds),) + shape[1:]
    slots = [{"x": torch.empty(cshape, device=dev), "go": torch.empty(cshape, device=dev),
              "out": [torch.empty(cshape, device=dev) for _ in range(4)]} for _ in range(2)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))

    def e2e_step() -> None:
        ev_in = [torch.cuda.Event() for _ in bounds]
        ev_cmp = [torch.cuda.Event() for _ in bounds]
        ev_out = [torch.cuda.Event() for _ in bounds]
        main = torch.cuda.current_stream(dev)
        for st in (s_in, s_cmp, s_out):
            st.wait_stream(main)
        for i, (b0, b1) in enumerate(bounds):
            sl, n = slots[i % 2], b1 - b0
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_cmp[i - 2])  # the slot's inputs are consumed
                sl["x"][:n].copy_(x_host[b0:b1], non_blocking=True)
                sl["go"][:n].copy_(go_host[b0:b1], non_blocking=True)
                ev_in[i].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[i])
                if i >= 2:
                    s_cmp.wait_event(ev_out[i - 2])  # the slot's results are read back
                xd = sl["x"][:n].detach().requires_grad_(True)
                god = sl["go"][:n]
                j = 0
                for fn in (serron.dilation, serron.erosion):
                    y = fn(xd, k, border=border)
                    (gx,) = torch.autograd.grad(y, xd, god)
                    sl["out"][j][:n].copy_(y.detach())
                    sl["out"][j + 1][:n].copy_(gx)
                    j += 2
                ev_cmp[i].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[i])
                for j in range(4):
                    outs[j][b0:b1].copy_(sl["out"][j][:n], non_blocking=True)
                ev_out[i].record(s_out)
        for st in (s_in, s_cmp, s_out):
            main.wait_stream(st)

    e2e_steps = max(1, min(args.steps, 3))
    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = px * PRIMS * world / (float(te.item()) * 1e-3) / 1e9

    if rank == 0:
        peak, peak_kind = _peaks()
        kernels = {}
        for name, per_px in (("forward", FWD_BYTES_PER_PX), ("gather", BWD_BYTES_PER_PX)):
            avg = statistics.mean(kernel_ms[name])
            achieved = px * per_px / (avg * 1e-3) / 1e9
            traffic = NCU_TRAFFIC_BYTES[name]
            kernels[name] = {"ms": avg, "achieved": achieved, "algorithmic_bytes": px * per_px,
                             "frac": achieved / peak, "traffic": traffic}
        dominant = max(kernels, key=lambda n: kernels[n]["ms"])
        dk = kernels[dominant]
        line = {
            "metric": METRIC, "value": value, "value_per_gpu": value / world,
            "value_note": "value is the whole job's output pixels per second over all GPUs; value_per_gpu divides it "
                          "by n_gpus (the metric's per-GPU figure)",
            "unit": "Gpix/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD if shape == SHAPE else f"{WORKLOAD} (batch {shape[0]} instead of 32)",
                       "per_gpu_batch": list(shape), "se": "square(15) flat",
                       "border": BORDER_NAME, "l2": "inputs 2.1 GB >> 126 MB L2, no flush needed"},
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": dk["achieved"], "peak": peak,
                         "unit": "GB/s", "frac": dk["frac"], "traffic": dk["traffic"], "peak_source": peak_kind},
            "kernels": kernels,
            "e2e": {"value": e2e_value, "unit": "Gpix/s", "h2d_bytes_per_step": 2 * px * 4,
                    "d2h_bytes_per_step": 4 * px * 4},
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "clocks": clock_info,
        }
        if world == 1:
            line["cpu_baseline"] = {k_: v for k_, v in _cpu_baseline().items() if k_ != "ms_per_step_sample"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _config_inputs(cfg: int, dev: torch.device, images: int | None = None):
    """Synthetic inputs of the other workloads (shapes, distributions and seeds of their definitions).
    ``images`` shrinks the batch of workloads 3 and 4 (for profiling captures of a few hundred MB)."""
    import serron_b200 as serron

    se = serron.structuring_element
    g = torch.Generator(device=dev).manual_seed(0)
    if cfg == 1:
        x = torch.rand(1, 1, 256, 256, generator=torch.Generator().manual_seed(0)).to(dev)
        return {"x": x, "k": se.disk(3, device=dev)}
    if cfg == 3:
        x = torch.rand(images or 64, 32, 256, 256, device=dev, generator=g).to(torch.bfloat16)
        w = torch.randn(32, 7, 7, device=dev, generator=g) * 0.1
        return {"x": x, "w": w, "g": g}
    if cfg == 4:
        n = images or 8
        x = torch.rand(n, 3, 1024, 1024, device=dev, generator=g).to(torch.float16)
        go = [torch.randn(n, 3, 1024, 1024, device=dev, generator=g).to(torch.float16) for _ in range(3)]
        return {"x": x, "go": go, "k": se.disk(15, dtype=torch.float16, device=dev)}
    # cfg 5: the smooth mask (64 separable Gaussians plus noise) and a 32-point marker, built on the CPU
    cg = torch.Generator().manual_seed(0)
    n = 8192
    cy, cx = torch.rand(64, generator=cg) * n, torch.rand(64, generator=cg) * n
    sigma, amp = 20 + 180 * torch.rand(64, generator=cg), torch.rand(64, generator=cg)
    ax = torch.arange(n, dtype=torch.float64)
    gy = torch.exp(-((ax[None, :] - cy[:, None].double()) ** 2) / (2 * sigma[:, None].double() ** 2))
    gx = torch.exp(-((ax[None, :] - cx[:, None].double()) ** 2) / (2 * sigma[:, None].double() ** 2))
    mask = torch.einsum("k,ky,kx->yx", amp.double(), gy, gx).float().view(1, 1, n, n)
    mask += 0.05 * torch.rand(1, 1, n, n, generator=cg)
    marker = torch.zeros_like(mask)
    idx = torch.randperm(n * n, generator=cg)[:32]
    marker.view(-1)[idx] = mask.view(-1)[idx]
    return {"marker": marker.to(dev), "mask": mask.to(dev), "k": se.cross(3, device=dev)}


def run_config(args) -> None:
    """The other workloads, device time per step (reported in the design notes, not by the driver).

    Under torchrun (N > 1): the learnable-layer workload (3) shards its batch of 64 along N and all-reduces
    the structuring-element gradients (NCCL, rank-ordered sum) inside every timed step; the derived-ops
    workload (4) shards its batch of 8; the reconstruction (5) shards the 8192 rows along H with a halo
    exchange per round; the tiny workload (1) runs a replica per rank.  Time = max over ranks.
    """
    import datetime

    import serron_b200 as serron

    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    from serron_b200 import _lib
    from serron_b200.distributed import allreduce_se_grads, reconstruction_sharded, shard_bounds

    _lib.load()
    cfg = args.config
    d = _config_inputs(cfg, dev, args.images)
    B = serron.BorderMode
    if cfg == 1:
        x, k = d["x"], d["k"]
        prims, px, bytes_px = 2, x.numel() * world, 8

        def step():
            serron.dilation(serron.erosion(x, k, border=B.REPLICATE), k, border=B.REPLICATE)
    elif cfg == 3:
        layer = serron.Opening2d(32, 7).to(dev)
        with torch.no_grad():
            layer.weight.copy_(d["w"])
        lo, hi = shard_bounds(d["x"].shape[0], rank, world)
        x = d["x"][lo:hi].contiguous().requires_grad_(True)
        go = torch.randn(d["x"].shape, device=dev, generator=d["g"]).to(torch.float16)[lo:hi].contiguous()
        prims, px, bytes_px = 2, d["x"].numel(), 10

        def step():
            layer.weight.grad = None
            with torch.autocast("cuda"):
                y = layer(x)
            y.backward(go)
            if world > 1:
                allreduce_se_grads(layer.parameters())
    elif cfg == 4:
        lo, hi = shard_bounds(d["x"].shape[0], rank, world)
        x, k, gos = d["x"][lo:hi].contiguous().requires_grad_(True), d["k"], [g[lo:hi].contiguous() for g in d["go"]]
        prims, px, bytes_px = 6, d["x"].numel(), 12

        def step():
            for fn, go in zip((serron.gradient, serron.top_hat, serron.black_hat), gos):
                y = fn(x, k, border=B.CONSTANT)
                torch.autograd.grad(y, x, go)
    else:
        marker, mask, k = d["marker"], d["mask"], d["k"]
        prims, px, bytes_px = 1, mask.numel(), 12
        if world > 1:
            lo, hi = shard_bounds(mask.shape[2], rank, world)
            marker, mask = marker[:, :, lo:hi].contiguous(), mask[:, :, lo:hi].contiguous()

            def step():
                reconstruction_sharded(marker, mask, k, border=B.CONSTANT)
        else:
            def step():
                serron.reconstruction_by_dilation(marker, mask, k, border=B.CONSTANT)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        peak, peak_kind = _peaks()
        line = {"config": cfg, "n_gpus": world, "metric": "output Gpix/s" if cfg != 5 else "ms to the fixed point",
                "value": px * prims / (ms * 1e-3) / 1e9 if cfg != 5 else ms, "ms_per_step": ms,
                "steps": args.steps, "warmup": args.warmup, "pixels": px, "primitive_calls": prims,
                "scaling": "replicas" if cfg == 1 else "strong",
                "collective": {3: "SE-grad all-gather + rank-ordered sum per step", 5: "halo send/recv + flag "
                               "all-reduce per round"}.get(cfg) if world > 1 else None,
                "hbm_frac_of_algorithmic": (px * prims * bytes_px / (ms * 1e-3) / 1e9) / (peak * world)
                if cfg != 5 else None,
                "peak_gbs": peak, "peak_source": peak_kind}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_minmax_rate() -> None:
    """Measured element min/max rate of the GPU: the compute roofline of the compare-select work."""
    import ctypes

    lib = ctypes.CDLL(os.path.join(REPO, "serron_b200", "libserron_minmax_rate.so"))
    lib.serron_measure_minmax_rate.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
    out = {}
    for kind, name in ((0, "fp32"), (1, "half2"), (2, "bfloat162")):
        v = ctypes.c_double()
        rc = lib.serron_measure_minmax_rate(kind, 0, ctypes.byref(v))
        if rc:
            raise RuntimeError(f"min/max rate measurement failed ({rc})")
        out[name] = v.value / 1e12
    print(json.dumps({"metric": "element min/max per second", "unit": "T/s", **out}), flush=True)


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference", "reference_cuda"], default="ours")
    # a smaller leading dimension, for profiling captures that must stay within a few GB of device memory
    p.add_argument("--batch", type=int, default=SHAPE[0])
    # the other workloads (1, 3, 4, 5) for the design notes; the default run is workload 2
    p.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=2)
    # a smaller batch for workloads 3 and 4, for profiling captures that must stay small
    p.add_argument("--images", type=int, default=None)
    p.add_argument("--minmax-rate", action="store_true", help="measure the min/max issue rate and exit")
    args = p.parse_args()
    if args.minmax_rate:
        run_minmax_rate()
    elif args.config != 2:
        run_config(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference_cuda":
        run_reference_cuda(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
