"""Row-sharded execution on 2, 4 and 8 GPUs over NCCL: each rank runs the
CUDA kernels on its row block of a configuration (device buffers, and host
buffers through layer_norm_host as the bench's e2e leg does), the blocks are
gathered over NVLink and compared with the oracle on the whole batch. A world
size larger than the box's GPU count is skipped."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import dslperfgap_b200 as B
        from dslperfgap_b200 import sharded, workloads
        rows = 1024
        r0, r1 = sharded.shard_rows(rows, rank, world)
        wl = workloads.make("layer_norm_bf16_sharded", seed=0, rows=(r0, r1)).to("cuda")
        y = B.layer_norm(*wl.args, **wl.kwargs)
        x, w, b = wl.args
        y_host = B.layer_norm_host(x.cpu().pin_memory(), w, b)
        host_ok = torch.tensor([int(torch.equal(y_host.cuda(), y))], device="cuda")
        dist.all_reduce(host_ok, op=dist.ReduceOp.MIN)
        full = sharded.gather_rows(y)
        ce = workloads.make("cross_entropy_bf16", seed=0, rows=sharded.shard_rows(64, rank, world)).to("cuda")
        loss, _, _ = B.cross_entropy_fwd(*ce.args, **ce.kwargs)
        mean = sharded.cross_entropy_mean(loss, ce.args[1], -100)
        if rank == 0:
            out_q.put((full.cpu(), mean, bool(host_ok.item())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_layer_norm_and_mean_loss(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import parity
    from oracle import oracle
    from dslperfgap_b200 import workloads
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        full, mean, host_ok = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():  # a rank that never finished: end it (host side only)
                p.terminate()
                p.join(timeout=10)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    wl = workloads.make("layer_norm_bf16_sharded", seed=0, rows=(0, 1024))
    assert host_ok, "layer_norm_host differs from the device path on some rank"
    ok, msg = parity.compare(full, oracle.layer_norm(*wl.args, **wl.kwargs), torch.bfloat16, normalised=True)
    assert ok, msg
    ce = workloads.make("cross_entropy_bf16", seed=0, rows=(0, 64))
    ref, _, _ = oracle.cross_entropy_fwd(*ce.args, **ce.kwargs, valid_only=True)
    keep = ce.args[1] != -100
    assert abs(mean - ref[keep].double().mean().item()) <= 1e-5 * abs(mean)
