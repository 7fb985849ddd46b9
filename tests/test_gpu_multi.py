"""Multi-GPU paths on NCCL: two processes, one GPU each (skipped with fewer than two GPUs).

* The H-sharded reconstruction (neighbour halo exchange by point-to-point NCCL sends, change flag
  all-reduced on the device) equals the single-GPU reconstruction bit for bit, on the large-image
  workload's kind of mask.
* The learnable-layer workload sharded along N: every rank's structuring-element gradient after
  ``allreduce_se_grads`` is identical, and equals the rank-ordered sum of the per-shard gradients that
  one process computes alone.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, port: int):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    return dist


def _sharded_reconstruction(rank: int, port: int) -> None:
    import oracle
    import serron_b200 as serron
    from serron_b200.distributed import reconstruction_sharded, shard_bounds

    dist = _init(rank, port)
    try:
        dev = torch.device("cuda", rank)
        marker, mask = oracle.blob_mask(2048, seed=4)
        cross = serron.structuring_element.cross(3, device=dev)
        full = serron.reconstruction_by_dilation(marker.to(dev), mask.to(dev), cross)
        r0, r1 = shard_bounds(2048, rank, WORLD)
        block = reconstruction_sharded(marker[:, :, r0:r1].to(dev), mask[:, :, r0:r1].to(dev), cross)
        torch.cuda.synchronize()
        assert torch.equal(block, full[:, :, r0:r1]), f"rank {rank}: sharded block differs"
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _layer_grads(rank: int, port: int) -> None:
    import serron_b200 as serron
    from serron_b200.distributed import allreduce_se_grads, shard_bounds

    dist = _init(rank, port)
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.rand(8, 4, 64, 64, device=dev, generator=g).to(torch.bfloat16)
        w = torch.randn(4, 7, 7, device=dev, generator=g) * 0.1
        go = torch.randn(8, 4, 64, 64, device=dev, generator=g).half()

        def shard_grad(lo: int, hi: int) -> torch.Tensor:
            layer = serron.Opening2d(4, 7).to(dev)
            with torch.no_grad():
                layer.weight.copy_(w)
            with torch.autocast("cuda"):
                y = layer(x[lo:hi])
            y.backward(go[lo:hi])
            return layer.weight.grad.clone()

        lo, hi = shard_bounds(8, rank, WORLD)
        layer = serron.Opening2d(4, 7).to(dev)
        with torch.no_grad():
            layer.weight.copy_(w)
        with torch.autocast("cuda"):
            y = layer(x[lo:hi])
        y.backward(go[lo:hi])
        allreduce_se_grads(layer.parameters())
        mine = layer.weight.grad
        everyone = [torch.empty_like(mine) for _ in range(WORLD)]
        dist.all_gather(everyone, mine)
        for r in range(1, WORLD):
            assert torch.equal(everyone[r], everyone[0]), "ranks disagree on the reduced gradient"
        # the same reduction in one process: per-shard gradients in float64, summed in rank order
        total = None
        for r in range(WORLD):
            part = shard_grad(*shard_bounds(8, r, WORLD)).double()
            total = part if total is None else total + part
        assert torch.equal(mine, total.to(mine.dtype)), "reduced gradient differs from the rank-ordered sum"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")


@pytest.mark.parametrize("body", [_sharded_reconstruction, _layer_grads], ids=["reconstruction", "layer_grads"])
def test_two_ranks_nccl(two_gpus, body):
    mp.start_processes(body, args=(_free_port(),), nprocs=WORLD, join=True, start_method="spawn")
