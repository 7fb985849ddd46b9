"""Multi-GPU execution: one process per GPU, torch.distributed (NCCL over NVLink) for the plumbing.

The reference is single-process; this module adds the two ways the morphology path shards:

* **Batch (N) sharding** — images are independent, so a batch is split into contiguous N-slices, one
  per rank, with no collective on the data path.  Learnable structuring elements are the only shared
  state: :func:`allreduce_se_grads` sums their gradients in rank order, so every rank gets the same,
  run-to-run identical result (all-gather of the per-rank gradients, then a fixed-order local sum).
* **Row (H) sharding of one reconstruction** — :func:`reconstruction_sharded` keeps each rank's block
  of rows plus a halo of ``kH // 2`` rows above and ``kH - 1 - kH // 2`` below.  Each round every rank
  receives its halo rows from its two neighbours only (point-to-point sends into local buffers), solves
  its block to a local fixed point with the halo frozen at those values (their marker and mask are both
  set to them, so the clipped step cannot move them), and the ranks all-reduce a "changed" flag that is
  computed on the device (one host read per round).  After the first round a block is already at its
  fixed point for the previous halos, so the library's solver continues from it with its tile worklist
  seeded only next to the halo rows (``serron_reconstruct_from_edges``).  A round in which no rank
  changed anything ends the loop: every block then satisfies the fixed-point equation against its
  neighbours' final rows, so the union is the global fixed point, bit-identical to the single-GPU
  result (the step is monotone; every schedule converges to the same least fixed point).

Every collective is issued by every rank in the same order.  The process group's timeout bounds every
wait: a rank that dies or never joins turns into an error on the others, not a hang.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable

import torch
import torch.distributed as dist

from .enums import BORDER_TO_INT, BorderMode

__all__ = ["allreduce_se_grads", "reconstruction_sharded", "shard_bounds", "shard_batch"]


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of ``total`` items (the first ``total % world`` get one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(x: torch.Tensor, rank: int | None = None, world: int | None = None) -> torch.Tensor:
    """This rank's contiguous N-slice of an (N, C, H, W) batch (a view)."""
    rank = dist.get_rank() if rank is None else rank
    world = dist.get_world_size() if world is None else world
    start, end = shard_bounds(x.shape[0], rank, world)
    return x[start:end]


def allreduce_se_grads(params: Iterable[torch.nn.Parameter], *, average: bool = False,
                       group: dist.ProcessGroup | None = None) -> None:
    """Sum (or average) the gradients of ``params`` over all ranks, in rank order, in place.

    The gradients are flattened into one buffer, all-gathered, and summed rank 0 first, so the result
    is identical on every rank and from run to run (a ring all-reduce adds in a topology-dependent
    order).  Parameters without a gradient contribute zeros.
    """
    params = [p for p in params]
    if not params:
        return
    world = dist.get_world_size(group)
    flats = [(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in params]
    local = torch.cat(flats).to(torch.float64)
    gathered = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gathered, local, group=group)
    total = gathered.view(world, -1)[0].clone()
    for r in range(1, world):
        total += gathered.view(world, -1)[r]
    if average:
        total /= world
    offset = 0
    for p, f in zip(params, flats):
        n = f.numel()
        g = total[offset:offset + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g
        else:
            p.grad.copy_(g)
        offset += n


LocalSolver = Callable[[bool, torch.Tensor, torch.Tensor, torch.Tensor, int], torch.Tensor]


def _default_solver(dilate: bool, marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, border: int,
                    seed_rows: tuple[int, int] | None = None) -> torch.Tensor:
    from . import _ops

    return _ops.reconstruct(dilate, marker, mask, kernel, border, None, 16, seed_rows=seed_rows)


def reconstruction_sharded(marker: torch.Tensor, mask: torch.Tensor, kernel: torch.Tensor, *, dilate: bool = True,
                           border: BorderMode = BorderMode.CONSTANT, group: dist.ProcessGroup | None = None,
                           max_rounds: int | None = None, solver: LocalSolver | None = None) -> torch.Tensor:
    """Geodesic reconstruction of an image whose rows are split across the ranks of ``group``.

    :param marker: this rank's block of rows, (N, C, H_rank, W); rank r holds the r-th block from the top.
    :param mask: same shape as ``marker``.
    :param kernel: structuring element (kH, kW) or (C, kH, kW), anchor tap >= 0, same dtype.
    :param dilate: reconstruction by dilation (True) or by erosion.
    :param max_rounds: bound on exchange rounds (None: until the fixed point).
    :param solver: local fixed-point solver ``(dilate, marker, mask, kernel, border) -> result``; the
        library's CUDA reconstruction by default.
    :returns: this rank's block of the reconstruction.
    :raises RuntimeError: when ``max_rounds`` runs out.
    """
    library_solver = solver is None  # the library's solver can continue from the previous round's result
    solver = solver or _default_solver
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    kh = kernel.shape[-2]
    top_h, bot_h = kh // 2, kh - 1 - kh // 2  # halo rows needed above / below
    border_int = BORDER_TO_INT[border]
    clip = torch.minimum if dilate else torch.maximum
    current = clip(marker, mask).contiguous()
    n, c, h, w = current.shape
    if (rank > 0 and h < bot_h) or (rank < world - 1 and h < top_h):
        raise ValueError("reconstruction_sharded: each block needs at least as many rows as the halo")
    up = rank - 1 if rank > 0 else None          # the rank holding the rows above
    down = rank + 1 if rank < world - 1 else None  # the rows below
    peer = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    top = top_h if up is not None else 0
    bot = bot_h if down is not None else 0
    halo_above = current.new_empty((n, c, top, w))
    halo_below = current.new_empty((n, c, bot, w))
    # the block with its halo rows: marker and mask both hold the neighbours' values there (frozen: the
    # clipped step cannot move them)
    ext_marker = current.new_empty((n, c, top + h + bot, w))
    ext_mask = torch.empty_like(ext_marker)
    ext_marker[:, :, top:top + h] = current
    ext_mask[:, :, top:top + h] = mask

    rounds = 0
    while True:
        # halo rows from the two neighbours only, into local buffers: my first bot_h rows go up (they are
        # the rows below the rank above), my last top_h rows go down
        ops = []
        if up is not None:
            ops.append(dist.P2POp(dist.irecv, halo_above, peer(up), group))
            ops.append(dist.P2POp(dist.isend, current[:, :, :bot_h].contiguous(), peer(up), group))
        if down is not None:
            ops.append(dist.P2POp(dist.irecv, halo_below, peer(down), group))
            ops.append(dist.P2POp(dist.isend, current[:, :, h - top_h:].contiguous(), peer(down), group))
        ops = [op for op in ops if op.tensor.numel() > 0]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        if top:
            ext_marker[:, :, :top] = halo_above
            ext_mask[:, :, :top] = halo_above
        if bot:
            ext_marker[:, :, top + h:] = halo_below
            ext_mask[:, :, top + h:] = halo_below
        if rounds > 0 and library_solver:
            # the block is at its fixed point for the previous halos: only tiles within reach of the halo
            # rows can move, and the worklist starts there
            solved = _default_solver(dilate, ext_marker, ext_mask, kernel, border_int,
                                     seed_rows=(top + kh if top else 0, bot + kh if bot else 0))
        else:
            solved = solver(dilate, ext_marker, ext_mask, kernel, border_int)
        new = solved[:, :, top:top + h]
        # the change flag stays on the device until the one read per round, after the all-reduce
        changed = (new != current).any().to(torch.int32).reshape(1)
        dist.all_reduce(changed, op=dist.ReduceOp.MAX, group=group)
        current = new.contiguous()
        ext_marker = solved
        rounds += 1
        if int(changed.item()) == 0:
            return current
        if max_rounds is not None and rounds >= max_rounds:
            raise RuntimeError(f"reconstruction_sharded: no fixed point after {rounds} exchange rounds")
