"""rms_norm and layer_norm on host buffers (dslpg_rms_norm_fwd_host,
dslpg_layer_norm_fwd_host): the chunked
upload / kernel / download pipeline gives the device path's result exactly,
for one chunk, many chunks with a ragged last one, pinned and pageable
memory, and repeated calls that reuse the per-device copy streams."""
import pytest
import torch

import dslperfgap_b200 as B

pytestmark = pytest.mark.gpu

DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def inputs(m, n, dt, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, n, generator=g).to(DT[dt])
    w = (torch.randn(n, generator=g) * 0.1 + 1).to(DT[dt])
    return x, w


@pytest.mark.parametrize("dt", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("m,n", [(1, 8), (3, 1000), (300, 4096), (1037, 8192), (70000, 96)])
def test_host_pipeline_matches_device_path(m, n, dt):
    x, w = inputs(m, n, dt, m + n)
    wd = w.cuda()
    ref = B.rms_norm(x.cuda(), (n,), wd, eps=1e-6).cpu()
    out = B.rms_norm_host(x.pin_memory(), (n,), wd, eps=1e-6)
    assert out.is_pinned() and out.dtype == x.dtype and out.shape == x.shape
    assert torch.equal(out, ref)


def test_host_pipeline_pageable_memory_and_out_argument():
    x, w = inputs(2500, 2048, "bf16", 5)  # about 10 MiB: three chunks
    wd = w.cuda()
    ref = B.rms_norm(x.cuda(), (2048,), wd).cpu()
    out = torch.full_like(x, float("nan"))  # pageable, pre-filled
    got = B.rms_norm_host(x, (2048,), wd, out=out)
    assert got is out
    assert torch.equal(out, ref)


def test_host_pipeline_repeated_calls_and_3d_input():
    x, w = inputs(4 * 600, 1536, "fp16", 9)
    x = x.view(4, 600, 1536)
    wd = w.cuda()
    ref = B.rms_norm(x.cuda(), (1536,), wd).cpu()
    xp = x.pin_memory()
    out = torch.empty_like(xp).pin_memory()
    for _ in range(3):
        out.zero_()
        B.rms_norm_host(xp, (1536,), wd, out=out)
        assert torch.equal(out, ref)


def test_host_pipeline_rejects_bad_arguments():
    x, w = inputs(4, 64, "fp32", 1)
    with pytest.raises(ValueError):
        B.rms_norm_host(x.cuda(), (64,), w.cuda())  # device input
    with pytest.raises(ValueError):
        B.rms_norm_host(x, (64,), w)  # host weight
    with pytest.raises(ValueError):
        B.rms_norm_host(x, (64,), w.cuda(), out=torch.empty(4, 32))


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
@pytest.mark.parametrize("m,n", [(1, 8), (3, 1000), (1037, 8192), (70000, 96)])
def test_layer_norm_host_matches_device_path_and_oracle(m, n, dt):
    import parity
    from oracle import oracle
    x, w = inputs(m, n, dt, 7 * m + n)
    b = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.1).to(DT[dt])
    wd, bd = w.cuda(), b.cuda()
    ref = B.layer_norm(x.cuda(), wd, bd).cpu()
    out = B.layer_norm_host(x.pin_memory(), wd, bd)
    assert out.is_pinned() and out.dtype == x.dtype and out.shape == x.shape
    assert torch.equal(out, ref)
    if m * n <= 1 << 20:
        ok, msg = parity.compare(out, oracle.layer_norm(x, w, b), DT[dt], normalised=True)
        assert ok, msg
    # no bias, pageable memory
    ref_nb = B.layer_norm(x.cuda(), wd, None).cpu()
    assert torch.equal(B.layer_norm_host(x, wd, None), ref_nb)


def test_layer_norm_host_sharded_rows_equal_the_whole():
    """A row block of the box-scale configuration through the host path gives
    the device path's rows exactly (what each rank of the sharded bench does)."""
    from dslperfgap_b200 import workloads
    wl = workloads.make("layer_norm_bf16_sharded", seed=0, rows=(4096, 4096 + 3000))
    x, w, b = wl.args
    ref = B.layer_norm(x.cuda(), w.cuda(), b.cuda()).cpu()
    assert torch.equal(B.layer_norm_host(x.pin_memory(), w.cuda(), b.cuda()), ref)


def test_layer_norm_host_rejects_bad_arguments():
    x, w = inputs(4, 64, "fp32", 1)
    with pytest.raises(ValueError):
        B.layer_norm_host(x, w.cuda(), None, eps=1e-6)  # the reference's eps rule
    with pytest.raises(ValueError):
        B.layer_norm_host(x.cuda(), w.cuda(), None)
    with pytest.raises(ValueError):
        B.layer_norm_host(x, w, None)
    with pytest.raises(ValueError):
        B.layer_norm_host(x, w.cuda(), None, out=torch.empty(4, 32))
