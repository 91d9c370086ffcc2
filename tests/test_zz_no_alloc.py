"""dslpg_kernel_ff_static: the kernel_ff entry point that allocates nothing
(xs and a_norm in a static device scratch) against dslpg_kernel_ff with a
torch-allocated workspace, on two calls in a row in one process.

This file is collected last so that it runs both alone and after every other
test (the scratch set-up happens on whichever call comes first)."""
import ctypes

import pytest
import torch

import parity
from dslperfgap_b200 import _lib

pytestmark = pytest.mark.gpu

LIMIT = 16 * 1024 * 1024 + 64 * 1024  # DSLPG_KERNEL_FF_STATIC_SCRATCH_BYTES
ERR_TOO_LARGE = -6


def inputs(seed, m, k, n):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).half().cuda()
    w1 = (torch.randn(n, k, generator=g) * k ** -0.5).half().cuda()
    w3 = (torch.randn(n, k, generator=g) * k ** -0.5).half().cuda()
    rw = (torch.randn(k, generator=g) * 0.1 + 1).half().cuda()
    return x, w1, w3, rw


def with_workspace(lib, x, w1, w3, rw):
    m, k = x.shape
    n = w1.shape[0]
    need = ctypes.c_int64(0)
    _lib.check(lib.dslpg_kernel_ff_workspace_bytes(m, k, ctypes.byref(need)), "workspace_bytes")
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    out = torch.empty(m, n, dtype=torch.float16, device="cuda")
    _lib.check(lib.dslpg_kernel_ff(x.data_ptr(), w1.data_ptr(), w3.data_ptr(), rw.data_ptr(), out.data_ptr(), m, n, k,
                                   ws.data_ptr(), need.value, _lib.stream_handle(x.device)), "dslpg_kernel_ff")
    return out


def static(lib, x, w1, w3, rw, out=None):
    m, k = x.shape
    n = w1.shape[0]
    out = torch.empty(m, n, dtype=torch.float16, device="cuda") if out is None else out
    rc = lib.dslpg_kernel_ff_static(x.data_ptr(), w1.data_ptr(), w3.data_ptr(), rw.data_ptr(), out.data_ptr(), m, n, k,
                                    _lib.stream_handle(x.device))
    return rc, out


def check_close(out, ref):
    ok, msg = parity.compare(out.cpu(), ref.cpu(), torch.float16,
                             abs_slack=parity.GEMM_SLACK * ref.float().abs().max().item())
    assert ok, msg


def test_static_scratch_matches_workspace_entry_on_two_calls():
    lib = _lib.load()
    # first call: a large problem; second call: a smaller one whose xs covers
    # only part of what the first call left in the scratch
    # then decode-like rows (the weight-streaming kernel, a_norm placed right
    # after a tiny xs) over what the larger calls left behind
    for seed, (m, k, n) in [(11, (1000, 2048, 1536)), (12, (333, 320, 1000)), (15, (1, 4096, 1000)),
                            (16, (3, 4096, 1000))]:
        args = inputs(seed, m, k, n)
        ref = with_workspace(lib, *args)
        rc, out = static(lib, *args)
        _lib.check(rc, "dslpg_kernel_ff_static")
        torch.cuda.synchronize()
        check_close(out, ref)
    assert _lib.take_wait_timeouts() == 0


def test_static_scratch_allocates_nothing_after_set_up():
    lib = _lib.load()
    args = inputs(13, 256, 512, 384)
    out = torch.empty(256, 384, dtype=torch.float16, device="cuda")
    _lib.check(static(lib, *args, out=out)[0], "dslpg_kernel_ff_static")  # set-up happens at the latest here
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        _lib.check(static(lib, *args, out=out)[0], "dslpg_kernel_ff_static")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    check_close(out, with_workspace(lib, *args))


def test_static_scratch_limit():
    lib = _lib.load()
    need = ctypes.c_int64(0)
    lib.dslpg_kernel_ff_workspace_bytes(2048, 4096, ctypes.byref(need))
    assert need.value <= LIMIT  # the benchmark shape fits
    lib.dslpg_kernel_ff_workspace_bytes(2056, 4096, ctypes.byref(need))
    assert need.value > LIMIT  # 2056 x 4096 fp16 alone fills the scratch; a_norm does not fit
    args = inputs(14, 2056, 4096, 128)
    rc, _ = static(lib, *args)
    assert rc == ERR_TOO_LARGE
    assert "static scratch" in lib.dslpg_error_string(rc).decode()
    huge = lib.dslpg_kernel_ff_static(args[0].data_ptr(), args[1].data_ptr(), args[2].data_ptr(), args[3].data_ptr(),
                                      args[0].data_ptr(), 1 << 30, 128, 1 << 30, _lib.stream_handle(args[0].device))
    assert huge == ERR_TOO_LARGE  # rejected before M * K is formed
