"""Row-sharded execution over one process per GPU (torch.distributed).

Every op of this backend is independent per row, so a batch splits into
contiguous row blocks with no communication on the data path. These helpers
cover what comes after the sharded compute:

* ``shard_rows(M, rank, world)`` — the row block [first, last) of a rank;
* ``gather_rows(y_local, group)`` — every rank's output block concatenated in
  rank order (one all_gather; blocks of unequal length are padded);
* ``cross_entropy_mean(loss, labels, ignored_index, group)`` — the mean loss
  over all ranks' non-ignored rows from one all_reduce of (sum, count), the
  reduction the reference applies to cross_entropy_fwd's per-row losses.

With NCCL the tensors stay on the GPU (the collectives run over NVLink /
NVSwitch); with gloo they are CPU tensors. None of this is timed in bench.py.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .workloads import shard_rows  # noqa: F401  (re-exported)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def gather_rows(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate the ranks' row blocks (dim 0) in rank order, on every rank."""
    world, _ = _world(group)
    if world == 1:
        return y_local
    n = torch.tensor([y_local.shape[0]], dtype=torch.int64, device=y_local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    top = max(sizes)
    pad = y_local
    if y_local.shape[0] < top:
        pad = torch.zeros((top,) + tuple(y_local.shape[1:]), dtype=y_local.dtype, device=y_local.device)
        pad[: y_local.shape[0]] = y_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)


def cross_entropy_mean(loss: torch.Tensor, labels: torch.Tensor, ignored_index: int = -100, group=None) -> float:
    """Mean of the per-row losses over all ranks, leaving out ignored rows.

    `loss` is this rank's cross_entropy_fwd loss output (one column block:
    row r's loss at flat index r), `labels` its labels."""
    n = labels.shape[0]
    keep = labels != ignored_index
    per_row = loss.reshape(-1)[:n]
    stats = torch.stack([per_row[keep].double().sum(), keep.sum().double()])
    world, _ = _world(group) if dist.is_initialized() else (1, 0)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=group)
    return float(stats[0] / stats[1]) if stats[1] > 0 else float("nan")
