"""Row-sharded execution across ranks, on CPU with the gloo backend.

Each of two ranks builds only its row block of a configuration (the same
generator the multi-GPU bench uses), runs the oracle on it, and the blocks are
gathered; the result must equal the unsharded run bit for bit. The timing
reduction (max over ranks) is checked the way bench.py does it.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dslperfgap_b200 import workloads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, rows, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle
        oracle.set_threads(2)
        r0, r1 = workloads.shard_rows(rows, rank, world)
        wl = workloads.make(name, seed=0, rows=(r0, r1))
        y = getattr(oracle, wl.fn_name)(*wl.args, **wl.kwargs)
        parts = [torch.empty(0)] * world
        dist.all_gather_object(parts, y)
        t = torch.tensor([float(rank + 1) * 1.5], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out_q.put((torch.cat(parts), float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["layer_norm_bf16_sharded", "logsumexp_bf16"])
def test_two_rank_shards_match_unsharded(name):
    rows = 64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, rows, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle
    wl = workloads.make(name, seed=0, rows=(0, rows))
    ref = getattr(oracle, wl.fn_name)(*wl.args, **wl.kwargs)
    assert torch.equal(gathered.view(torch.int16), ref.view(torch.int16))
    assert tmax == 3.0


def test_shard_rows_cover_exactly():
    for M in (1, 7, 131072):
        for world in (1, 2, 4, 8):
            blocks = [workloads.shard_rows(M, r, world) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
    with pytest.raises(ValueError):
        workloads.shard_rows(10, 2, 2)


def test_generator_rows_are_position_independent():
    full = workloads.make("softmax_fp16", rows=(0, 5000)).args[0]
    part = workloads.make("softmax_fp16", rows=(4000, 4100)).args[0]
    assert torch.equal(full[4000:4100].view(torch.int16), part.view(torch.int16))


def _gather_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dslperfgap_b200 import sharded
        from oracle import oracle
        M = 13  # uneven blocks: 4 / 4 / 5
        r0, r1 = sharded.shard_rows(M, rank, world)
        wl = workloads.make("cross_entropy_bf16", seed=0, rows=(0, M))
        logits, labels = wl.args[0][r0:r1], wl.args[1][r0:r1].clone()
        if rank == 1:
            labels[0] = -100
        loss, _, _ = oracle.cross_entropy_fwd(logits, labels, **wl.kwargs, valid_only=True)
        full = sharded.gather_rows(loss, None)
        lab_full = sharded.gather_rows(labels, None)
        mean = sharded.cross_entropy_mean(loss, labels, -100, None)
        if rank == 0:
            out_q.put((full, lab_full, mean))
    finally:
        dist.destroy_process_group()


def test_three_rank_gather_and_mean_loss():
    from oracle import oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    full, lab_full, mean = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    wl = workloads.make("cross_entropy_bf16", seed=0, rows=(0, 13))
    labels = wl.args[1].clone()
    labels[4] = -100  # rank 1's first row
    ref, _, _ = oracle.cross_entropy_fwd(wl.args[0], labels, **wl.kwargs, valid_only=True)
    assert torch.equal(full, ref)
    assert torch.equal(lab_full, labels)
    keep = labels != -100
    assert abs(mean - ref[keep].double().mean().item()) < 1e-12
