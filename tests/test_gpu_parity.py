"""CUDA backend vs the CPU oracle on seeded inputs.

* every kernel shape the dispatcher can pick (warp-per-row, CTA-per-row with
  1/2/4/8 vectors per thread, the two-pass stream kernel, the scalar path for
  odd lengths and misaligned pointers, the strided log_softmax);
* the benchmark configurations at their full sizes;
* guard bytes around every output (no out-of-bounds writes) and bit-for-bit
  repeatability.
"""
import ctypes

import pytest
import torch

import parity
from oracle import oracle
import dslperfgap_b200 as B
from dslperfgap_b200 import _lib

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
PATHS = ["auto", "resident", "tma", "stream", "cluster"]


@pytest.fixture(params=PATHS)
def path(request):
    """Run the test under each kernel shape (shapes a path cannot take fall back)."""
    with _lib.kernel_path(request.param):
        yield request.param


LENGTHS = [1, 7, 32, 64, 100, 128, 256, 512, 1000, 1024, 2048, 4096, 5120, 8192, 12288, 16384, 32768,
           40000, 65536, 131072, 262144, 1048576]


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn(shape, dtype, g, std=1.0, mean=0.0):
    return (torch.randn(*shape, generator=g) * std + mean).to(dtype)


def rows_for(n):
    return max(1, min(64, (1 << 22) // max(n, 1)))


def assert_parity(out, ref, dtype, normalised=False):
    ok, msg = parity.compare(out, ref, dtype, normalised=normalised)
    assert ok, msg


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", LENGTHS)
def test_layer_norm_lengths(n, dt, path):
    g = gen(n)
    dtype = DT[dt]
    x = randn((rows_for(n), n), dtype, g)
    w = randn((n,), dtype, g, std=0.1, mean=1.0)
    b = randn((n,), dtype, g, std=0.1)
    out = B.layer_norm(x.cuda(), w.cuda(), b.cuda())
    assert out.dtype == dtype and out.shape == x.shape
    assert_parity(out, oracle.layer_norm(x, w, b), dtype, normalised=True)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", LENGTHS)
def test_rms_norm_lengths(n, dt, path):
    g = gen(n + 1)
    dtype = DT[dt]
    x = randn((rows_for(n), n), dtype, g)
    w = randn((n,), dtype, g, std=0.1, mean=1.0)
    out = B.rms_norm(x.cuda(), (n,), w.cuda(), eps=1e-6)
    assert_parity(out, oracle.rms_norm(x, (n,), w, eps=1e-6), dtype, normalised=True)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", LENGTHS)
def test_softmax_lengths(n, dt, path):
    g = gen(n + 2)
    dtype = DT[dt]
    x = randn((rows_for(n), n), dtype, g, std=3.0)
    out = B.softmax(x.cuda())
    assert_parity(out, oracle.softmax(x), dtype)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", LENGTHS)
def test_log_softmax_lengths(n, dt, path):
    g = gen(n + 3)
    dtype = DT[dt]
    x = randn((rows_for(n), n), dtype, g, std=3.0)
    out = B.log_softmax(x.cuda(), dim=-1)
    assert_parity(out, oracle.log_softmax(x, dim=-1), dtype)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", LENGTHS + [128256])
def test_logsumexp_lengths(n, dt, path):
    g = gen(n + 4)
    dtype = DT[dt]
    x = randn((rows_for(n), n), dtype, g, std=2.0)
    out = B.logsumexp(x.cuda())
    assert_parity(out, oracle.logsumexp(x), dtype)


@pytest.mark.parametrize("din,dout", [(a, b) for a in DT for b in DT])
@pytest.mark.parametrize("n", [64, 1000, 4096, 40000])
def test_log_softmax_dtype_kwarg(din, dout, n):
    g = gen(n + 5)
    x = randn((8, n), DT[din], g, std=3.0)
    out = B.log_softmax(x.cuda(), dim=-1, dtype=DT[dout])
    assert out.dtype == DT[dout]
    assert_parity(out, oracle.log_softmax(x, dim=-1, dtype=DT[dout]), DT[dout])


@pytest.mark.parametrize("shape,dim", [((4, 16, 8), 1), ((8, 5), 0), ((3, 4, 5, 6), 2), ((2, 300, 3), 1),
                                       ((7, 33), -2)])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_log_softmax_other_dims(shape, dim, dt):
    x = randn(shape, DT[dt], gen(len(shape)), std=2.0)
    out = B.log_softmax(x.cuda(), dim=dim)
    assert_parity(out, oracle.log_softmax(x, dim=dim), DT[dt])


@pytest.mark.parametrize("bs", [1, 5, 64, 1000, 4096, 131072])
@pytest.mark.parametrize("smooth,split", [(False, False), (True, False), (True, True), (False, True)])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_cross_entropy_blocks(bs, smooth, split, dt, path):
    g = gen(bs)
    r, c = 16, 40000
    lg = randn((r, c), DT[dt], g, std=2.0)
    lb = torch.randint(0, c, (r,), generator=g, dtype=torch.int64)
    lb[3] = -100
    lb[5] = c + 7  # out of range: in no block
    kw = dict(smoothing=0.1 if smooth else 0.0, logit_scale=0.9, lse_square_scale=1e-3, ignored_index=-100,
              total_classes=c, class_start_idx=0, BLOCK_SIZE=bs, HAS_SMOOTHING=smooth, SPLIT=split)
    out = B.cross_entropy_fwd(lg.cuda(), lb.cuda(), **kw)
    ref = oracle.cross_entropy_fwd(lg, lb, **kw)
    nv = ((c + bs - 1) // bs) * r
    for i, (o, rr) in enumerate(zip(out, ref)):
        if split and i == 2:
            continue
        assert_parity(o.reshape(-1)[:nv], rr.reshape(-1)[:nv], torch.float32)


def test_cross_entropy_int32_labels_and_row_stride():
    g = gen(7)
    full = randn((8, 3000), torch.bfloat16, g)
    lg = full[:, :2500]  # row stride 3000 > n_cols: passed through, not copied
    lb = torch.randint(0, 2500, (8,), generator=g, dtype=torch.int32)
    kw = dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100, total_classes=2500,
              class_start_idx=0, BLOCK_SIZE=4096, HAS_SMOOTHING=False, SPLIT=False)
    out = B.cross_entropy_fwd(full.cuda()[:, :2500], lb.cuda(), **kw)
    ref = oracle.cross_entropy_fwd(lg.contiguous(), lb, **kw)
    for o, rr in zip(out, ref):
        assert_parity(o.reshape(-1)[:8], rr.reshape(-1)[:8], torch.float32)


# ---------------------------------------------------------------- scalar path
def _c_call_misaligned(op, x, n, dtype):
    """Call the C ABI with x and y offset by one element (not 16-byte aligned)."""
    lib = _lib.load()
    code = _lib.FLOAT_CODES[dtype]
    m = x.shape[0]
    xb = torch.empty(m * n + 1, dtype=dtype, device="cuda")
    xb[1:].copy_(x.reshape(-1).cuda())
    yb = torch.empty(m * n + 1, dtype=dtype, device="cuda")
    xp, yp = xb[1:].data_ptr(), yb[1:].data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    if op == "softmax":
        rc = lib.dslpg_softmax_fwd(xp, yp, m, n, code, s)
    elif op == "log_softmax":
        rc = lib.dslpg_log_softmax_fwd(xp, yp, m, n, 1, code, code, s)
    assert rc == 0
    return yb[1:].reshape(m, n).cpu()


@pytest.mark.parametrize("op", ["softmax", "log_softmax"])
@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
def test_misaligned_pointers_use_scalar_path(op, dt):
    x = randn((6, 4096), DT[dt], gen(9), std=2.0)
    out = _c_call_misaligned(op, x, 4096, DT[dt])
    ref = oracle.softmax(x) if op == "softmax" else oracle.log_softmax(x)
    assert_parity(out, ref, DT[dt])


def test_layer_norm_mixed_weight_dtype():
    g = gen(11)
    x = randn((16, 4096), torch.bfloat16, g)
    w = randn((4096,), torch.float32, g, mean=1.0, std=0.1)
    b = randn((4096,), torch.float32, g, std=0.1)
    out = B.layer_norm(x.cuda(), w.cuda(), b.cuda())
    assert_parity(out, oracle.layer_norm(x, w, b), torch.bfloat16, normalised=True)


def test_layer_norm_no_bias():
    g = gen(12)
    x = randn((16, 1024), torch.float32, g)
    w = randn((1024,), torch.float32, g)
    out = B.layer_norm(x.cuda(), w.cuda(), None)
    assert_parity(out, oracle.layer_norm(x, w, None), torch.float32)


# ------------------------------------------------------- guard bytes / repeats
GUARD = 4096


def _guarded(numel, dtype):
    buf = torch.full((numel + 2 * GUARD,), 7.0, dtype=dtype, device="cuda")
    return buf, buf[GUARD:GUARD + numel]


def _guards_intact(buf, numel):
    return bool((buf[:GUARD] == 7.0).all()) and bool((buf[GUARD + numel:] == 7.0).all())


@pytest.mark.parametrize("n", [33, 1024, 5120, 40000])
def test_no_writes_outside_outputs(n):
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    m = 37
    x = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    for name, call in [
        ("softmax", lambda y: lib.dslpg_softmax_fwd(x.data_ptr(), y.data_ptr(), m, n, _lib.BF16, s)),
        ("log_softmax", lambda y: lib.dslpg_log_softmax_fwd(x.data_ptr(), y.data_ptr(), m, n, 1, _lib.BF16,
                                                            _lib.BF16, s)),
        ("rms_norm", lambda y: lib.dslpg_rms_norm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, _lib.BF16,
                                                      _lib.BF16, 1e-5, s)),
        ("layer_norm", lambda y: lib.dslpg_layer_norm_fwd(x.data_ptr(), w.data_ptr(), w.data_ptr(), y.data_ptr(),
                                                          m, n, _lib.BF16, _lib.BF16, 1e-5, s)),
    ]:
        buf, y = _guarded(m * n, torch.bfloat16)
        assert call(y) == 0, name
        torch.cuda.synchronize()
        assert _guards_intact(buf, m * n), name
    buf, y = _guarded(m, torch.bfloat16)
    assert lib.dslpg_logsumexp_fwd(x.data_ptr(), y.data_ptr(), m, n, _lib.BF16, s) == 0
    torch.cuda.synchronize()
    assert _guards_intact(buf, m)


def test_cross_entropy_writes_only_valid_prefix():
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    r, c, bs = 9, 1000, 300
    nb = (c + bs - 1) // bs
    lg = torch.randn(r, c, device="cuda")
    lb = torch.randint(0, c, (r,), device="cuda")
    bufs = [torch.full((r * c + GUARD,), 7.0, device="cuda") for _ in range(3)]
    rc = lib.dslpg_cross_entropy_fwd(lg.data_ptr(), lb.data_ptr(), bufs[0].data_ptr(), bufs[1].data_ptr(),
                                     bufs[2].data_ptr(), r, c, c, _lib.F32, _lib.I64, 0.0, 1.0, 0.0, -100, float(c),
                                     0, bs, 0, 0, s)
    assert rc == 0
    torch.cuda.synchronize()
    for bf in bufs:
        assert bool((bf[nb * r:] == 7.0).all())


def test_repeatable_bit_for_bit():
    x = torch.randn(300, 8192, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(8192, device="cuda", dtype=torch.bfloat16)
    for f in (lambda: B.rms_norm(x, (8192,), w), lambda: B.layer_norm(x, w, w), lambda: B.softmax(x),
              lambda: B.logsumexp(x)):
        a, b = f(), f()
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_empty_inputs():
    x = torch.empty(0, 64, device="cuda")
    assert B.softmax(x).shape == (0, 64)
    assert B.logsumexp(x).shape == (0,)
    assert B.layer_norm(x, torch.ones(64, device="cuda"), torch.zeros(64, device="cuda")).shape == (0, 64)
    e = B.logsumexp(torch.empty(3, 0, device="cuda"))
    assert torch.equal(e.cpu(), torch.full((3,), float("-inf")))


def test_current_stream_is_used():
    s = torch.cuda.Stream()
    x = torch.randn(512, 4096, device="cuda")
    with torch.cuda.stream(s):
        y = B.softmax(x)
    s.synchronize()
    assert_parity(y, oracle.softmax(x.cpu()), torch.float32)


def test_no_pipeline_wait_ran_out():
    """Run last in this file: no bounded device wait expired in any test above."""
    torch.cuda.synchronize()
    assert _lib.take_wait_timeouts() == 0


# ---------------------------------------------------------- cross_entropy_bwd
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [8, 37, 1000, 4096, 40000, 128256])
@pytest.mark.parametrize("smooth", [False, True])
def test_cross_entropy_bwd(n, dt, smooth):
    g = gen(n + 17)
    r = 12
    lg = randn((r, n), DT[dt], g, std=2.0)
    lb = torch.randint(0, n, (r,), generator=g, dtype=torch.int64)
    lb[1] = -100
    lb[2] = n + 3          # in no column
    lb[3] = n - 1          # last column
    lb[4] = 0
    dloss = torch.rand(r, generator=g) + 0.5
    lse = torch.logsumexp(lg.float() * 0.8, dim=-1)
    kw = dict(smoothing=0.1 if smooth else 0.0, logit_scale=0.8, lse_square_scale=1e-3, ignored_index=-100,
              total_classes=n, class_start_idx=0, BLOCK_SIZE=4096, HAS_SMOOTHING=smooth)
    out = B.cross_entropy_bwd(dloss.cuda(), lg.cuda(), lse.cuda(), lb.cuda(), **kw)
    assert out.dtype == DT[dt] and out.shape == lg.shape
    ref = oracle.cross_entropy_bwd(dloss, lg, lse, lb, **kw)
    slack = None
    if smooth:  # p - smoothing/total_classes cancels: allow the fp32 rounding of the terms
        k1 = (dloss * kw["logit_scale"]).abs().max().item()
        slack = 2.0 ** -21 * (ref.float().abs() + 2 * k1 * kw["smoothing"] / kw["total_classes"])
    ok, msg = parity.compare(out, ref, DT[dt], abs_slack=slack)
    assert ok, msg


def test_cross_entropy_bwd_strided_and_int32_labels():
    g = gen(99)
    full = randn((6, 3000), torch.bfloat16, g)
    lb = torch.tensor([5, 2499, -100, 0, 7, 100], dtype=torch.int32)
    dloss_full = torch.rand(12, generator=g) + 0.5
    dloss = dloss_full[::2]  # stride 2
    lse = torch.logsumexp(full[:, :2500].float(), dim=-1)
    kw = dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100, total_classes=2500,
              class_start_idx=2, BLOCK_SIZE=1024, HAS_SMOOTHING=False)
    out = B.cross_entropy_bwd(dloss_full.cuda()[::2], full.cuda()[:, :2500], lse.cuda(), lb.cuda(), **kw)
    ref = oracle.cross_entropy_bwd(dloss.contiguous(), full[:, :2500].contiguous(), lse, lb, **kw)
    assert_parity(out, ref, torch.bfloat16)


# --------------------------------------------- mean_reduction / max / argmax
RED_LENGTHS = [1, 7, 33, 64, 1000, 4096, 32768, 100000]


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", RED_LENGTHS)
def test_reductions_rows(n, dt):
    g = gen(n + 31)
    x = randn((rows_for(n), n), DT[dt], g)
    if n >= 8:
        x[0, n // 3] = float("nan")
        x[0, n // 2] = float("nan")
        x[1, :] = 1.0                 # all ties: index 0
        x[2, n - 1] = 100.0           # maximum in the last column
        x[3, :] = float("-inf")
    xc = x.cuda()
    assert_parity(B.mean_reduction(xc, 1), oracle.mean_reduction(x, 1), DT[dt])
    v, i = B.max_reduction(xc, 1)
    rv, ri = oracle.max_reduction(x, 1)
    assert_parity(v, rv, DT[dt])
    assert torch.equal(i.cpu(), ri)
    assert torch.equal(B.argmax(xc, 1).cpu(), oracle.argmax(x, 1))


@pytest.mark.parametrize("shape,dim,keepdim", [((64, 128), 0, False), ((8, 16, 32), 1, True), ((2, 3, 4, 5), [1, 2], False),
                                               ((3, 4, 5, 6), [0, 2], True), ((7, 9), -1, False), ((300, 5), 0, True)])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_reductions_dims(shape, dim, keepdim, dt):
    x = randn(shape, DT[dt], gen(len(shape) + 40))
    xc = x.cuda()
    out = B.mean_reduction(xc, dim, keepdim=keepdim)
    ref = oracle.mean_reduction(x, dim, keepdim=keepdim)
    assert out.shape == ref.shape
    assert_parity(out, ref, DT[dt])
    if isinstance(dim, int):
        v, i = B.max_reduction(xc, dim, keepdim)
        rv, ri = oracle.max_reduction(x, dim, keepdim)
        assert v.shape == rv.shape and torch.equal(i.cpu(), ri)
        assert_parity(v, rv, DT[dt])
        assert torch.equal(B.argmax(xc, dim, keepdim).cpu(), oracle.argmax(x, dim, keepdim))


@pytest.mark.parametrize("din,dout", [("bf16", "f32"), ("f32", "bf16"), ("f16", "f32"), ("f32", "f16")])
def test_mean_dtype_kwarg(din, dout):
    x = randn((16, 5000), DT[din], gen(77))
    out = B.mean_reduction(x.cuda(), 1, dtype=DT[dout])
    assert out.dtype == DT[dout]
    assert_parity(out, oracle.mean_reduction(x, 1, dtype=DT[dout]), DT[dout])


def test_argmax_flatten():
    x = randn((37, 91), torch.float16, gen(5))
    assert torch.equal(B.argmax(x.cuda(), None).cpu(), oracle.argmax(x, None))


@pytest.mark.parametrize("bs", [131072, 65536, 300000])
@pytest.mark.parametrize("smooth", [False, True])
def test_cross_entropy_few_long_rows(bs, smooth):
    """Few rows of long column blocks: the cluster-split path of the forward."""
    g = gen(bs + 3)
    r, c = 6, 300000
    lg = randn((r, c), torch.bfloat16, g, std=2.0)
    lb = torch.randint(0, c, (r,), generator=g, dtype=torch.int64)
    lb[1] = -100
    kw = dict(smoothing=0.1 if smooth else 0.0, logit_scale=1.0, lse_square_scale=1e-4, ignored_index=-100,
              total_classes=c, class_start_idx=0, BLOCK_SIZE=bs, HAS_SMOOTHING=smooth, SPLIT=False)
    out = B.cross_entropy_fwd(lg.cuda(), lb.cuda(), **kw)
    ref = oracle.cross_entropy_fwd(lg, lb, **kw, valid_only=True)
    nv = ref[0].numel()
    for o, rr in zip(out, ref):
        assert_parity(o.reshape(-1)[:nv], rr, torch.float32)


# ------------------------------------------------ linear_activation.kernel_ff
# path: "auto" (the weight-streaming kernel for M <= 3, one CTA per tile up to
# M = 128, CTA pairs above), "stream" (force the weight-streaming kernel for
# M <= 8), "resident" (force one CTA per 128x128 tile), "cluster" (force CTA
# pairs on 256x128 tiles)
@pytest.mark.parametrize("path", ["auto", "stream", "resident", "cluster"])
@pytest.mark.parametrize("b,s,d,n", [(1, 128, 64, 128), (1, 128, 128, 256), (2, 100, 512, 200), (1, 256, 1024, 512),
                                     (1, 300, 2048, 640), (3, 7, 72, 40), (1, 1000, 320, 1000), (4, 700, 256, 2176),
                                     (1, 1, 64, 128), (1, 1, 4096, 1000), (1, 2, 1032, 300), (1, 3, 256, 129),
                                     (2, 2, 4096, 2048), (1, 5, 520, 77), (1, 8, 4096, 4096), (8, 1, 6144, 512)])
def test_kernel_ff(b, s, d, n, path):
    g = gen(d + n)
    x = randn((b, s, d), torch.float16, g)
    w1 = randn((n, d), torch.float16, g, std=d ** -0.5)
    w3 = randn((n, d), torch.float16, g, std=d ** -0.5)
    rw = randn((d,), torch.float16, g, mean=1.0, std=0.1)
    with _lib.kernel_path(path):
        out = B.kernel_ff(x.cuda(), w1.cuda(), w3.cuda(), rw.cuda())
    ref = oracle.kernel_ff(x, w1, w3, rw)
    assert _lib.take_wait_timeouts() == 0
    assert out.shape == ref.shape and out.dtype == torch.float16
    ok, msg = parity.compare(out, ref, torch.float16, abs_slack=parity.gemm_slack(x, w1, w3, rw))
    assert ok, msg


def test_kernel_ff_misaligned_views():
    """A contiguous view at an odd offset (rms_w sliced from a flat fp16
    parameter buffer) is accepted, as the reference accepts it."""
    g = gen(77)
    d, n = 512, 384
    x = randn((1, 64, d), torch.float16, g)
    w1 = randn((n, d), torch.float16, g, std=d ** -0.5)
    w3 = randn((n, d), torch.float16, g, std=d ** -0.5)
    rw = randn((d,), torch.float16, g, mean=1.0, std=0.1)
    flat = torch.empty(d + 3, dtype=torch.float16, device="cuda")
    flat[3:] = rw.cuda()
    rw_view = flat[3:]
    assert rw_view.data_ptr() % 16 != 0 and rw_view.is_contiguous()
    out = B.kernel_ff(x.cuda(), w1.cuda(), w3.cuda(), rw_view)
    ok, msg = parity.compare(out, oracle.kernel_ff(x, w1, w3, rw), torch.float16,
                             abs_slack=parity.gemm_slack(x, w1, w3, rw))
    assert ok, msg
