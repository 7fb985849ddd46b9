"""Multi-process host logic of serron_b200.distributed on CPU ranks (gloo, world size 2 and 3).

The local fixed-point solver is injected: the oracle stands in for the CUDA kernel, so the sharding,
halo exchange, convergence test and rank-ordered reductions are checked without a GPU.  Failure
detection is exercised on the host: a rank that leaves before a collective turns into an error on the
other rank within the process group's timeout, not a hang.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_solver(dilate, marker, mask, kernel, border):
    import oracle

    out, _ = oracle.reconstruct(dilate, marker, mask, kernel, border)
    return out


def _problem(seed: int = 3):
    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(1, 2, 23, 17, generator=g, dtype=torch.float64)
    marker = torch.zeros_like(mask)
    idx = torch.randperm(mask.numel(), generator=g)[:6]
    marker.view(-1)[idx] = mask.view(-1)[idx]
    return marker, mask


KERNELS = {
    "cross3": [[float("-inf"), 0.0, float("-inf")], [0.0, 0.0, 0.0], [float("-inf"), 0.0, float("-inf")]],
    "square5": [[0.0] * 5 for _ in range(5)],
    "even2x4": [[0.0] * 4 for _ in range(2)],
}
CASES = [(k, border, dilate) for k in KERNELS for border in (0, 1, 2) for dilate in (True, False)]


def _case_inputs(dilate: bool):
    marker, mask = _problem()
    if not dilate:
        marker, mask = -marker + 1.0, -mask + 1.0
    return marker, mask


def _recon_worker(rank: int, world: int, port: int, q) -> None:
    _init(rank, world, port)
    from serron_b200 import distributed as sd
    from serron_b200.enums import BorderMode

    results = []
    for kname, border, dilate in CASES:
        marker, mask = _case_inputs(dilate)
        kernel = torch.tensor(KERNELS[kname], dtype=torch.float64)
        start, end = sd.shard_bounds(mask.shape[2], rank, world)
        mode = [BorderMode.REFLECT, BorderMode.REPLICATE, BorderMode.CONSTANT][border]
        results.append(sd.reconstruction_sharded(marker[:, :, start:end].contiguous(),
                                                 mask[:, :, start:end].contiguous(), kernel, dilate=dilate,
                                                 border=mode, solver=_oracle_solver))
    q.put((rank, [r.numpy() for r in results]))  # numpy pickles by value: safe after exit
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_reconstruction_equals_single_image(world):
    """Every (structuring element, border, variant) case: the row-sharded fixed point equals the oracle's
    single-image reconstruction bit for bit."""
    import oracle

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_recon_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    parts = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for i, (kname, border, dilate) in enumerate(CASES):
        got = torch.cat([torch.from_numpy(parts[r][i]) for r in range(world)], dim=2)
        marker, mask = _case_inputs(dilate)
        want, _ = oracle.reconstruct(dilate, marker, mask, torch.tensor(KERNELS[kname], dtype=torch.float64), border)
        assert torch.equal(got, want), (kname, border, dilate)


def _grad_worker(rank: int, world: int, port: int, q) -> None:
    _init(rank, world, port)
    from serron_b200 import distributed as sd

    p = torch.nn.Parameter(torch.zeros(3, 5, 5))
    g = torch.Generator().manual_seed(100 + rank)
    p.grad = torch.randn(3, 5, 5, generator=g)
    other = torch.nn.Parameter(torch.zeros(4))  # no grad on this rank's side
    sd.allreduce_se_grads([p, other])
    q.put((rank, p.grad.clone(), other.grad.clone()))
    dist.barrier()
    dist.destroy_process_group()


def test_se_grad_allreduce_is_rank_ordered_and_identical():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = dict((r, (a, b)) for r, a, b in (q.get(timeout=120) for _ in range(world)))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    want = torch.zeros(3, 5, 5, dtype=torch.float64)
    for r in range(world):
        want += torch.randn(3, 5, 5, generator=torch.Generator().manual_seed(100 + r)).double()
    for r in range(world):
        assert torch.equal(res[r][0], want.float())
        assert torch.equal(res[r][1], torch.zeros(4))


def test_shard_bounds_cover_the_batch():
    from serron_b200.distributed import shard_bounds

    for total in (0, 1, 7, 32):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def _dropout_worker(rank: int, world: int, port: int, q) -> None:
    _init(rank, world, port, timeout_s=5.0)
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)  # leaves between steps, before the collective
    t = torch.ones(1)
    try:
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as exc:  # the surviving rank sees the failure instead of hanging
        q.put((rank, f"error: {type(exc).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_a_rank_that_leaves_is_detected_not_hung():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error")
