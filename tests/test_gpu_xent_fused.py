"""cross_entropy_fwd_bwd (one pass over the logits) against the oracle's
forward followed by its backward, and against this backend's own
cross_entropy_fwd + cross_entropy_bwd, on seeded inputs: every dtype, short
to vocab-sized rows, smoothing, logit scale, z-loss, ignored rows, labels
outside the row, strided inputs and more rows than SMs."""
import pytest
import torch

import parity
from oracle import oracle
import dslperfgap_b200 as B
from dslperfgap_b200 import _lib

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def make(r, n, dt, seed):
    g = torch.Generator().manual_seed(seed)
    lg = (torch.randn(r, n, generator=g) * 2.0).to(DT[dt])
    lb = torch.randint(0, n, (r,), generator=g, dtype=torch.int64)
    if r >= 5:
        lb[1] = -100       # ignored
        lb[2] = n + 3      # in no column
        lb[3] = n - 1      # last column
        lb[4] = 0
    dloss = torch.rand(r, generator=g) + 0.5
    return lg, lb, dloss


def kwargs(n, smooth):
    return dict(smoothing=0.1 if smooth else 0.0, logit_scale=0.8, lse_square_scale=1e-3, ignored_index=-100,
                total_classes=n, class_start_idx=0, HAS_SMOOTHING=smooth)


def grad_slack(ref, dloss, kw):
    """The backward tests' allowance where p - smoothing/total_classes cancels."""
    if not kw["HAS_SMOOTHING"]:
        return None
    k1 = (dloss * kw["logit_scale"]).abs().max().item()
    return 2.0 ** -21 * (ref.float().abs() + 2 * k1 * kw["smoothing"] / kw["total_classes"])


def check(out, ref, dt, dloss, kw):
    for o, r in zip(out[:3], ref[:3]):
        ok, msg = parity.compare(o.cpu(), r, torch.float32)
        assert ok, msg
    ok, msg = parity.compare(out[3].cpu(), ref[3], DT[dt], abs_slack=grad_slack(ref[3], dloss, kw))
    assert ok, msg


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [8, 37, 1000, 4096, 40000, 128256])
@pytest.mark.parametrize("smooth", [False, True])
def test_fused_matches_oracle(n, dt, smooth):
    lg, lb, dloss = make(12, n, dt, n + 5)
    kw = kwargs(n, smooth)
    out = B.cross_entropy_fwd_bwd(lg.cuda(), lb.cuda(), dloss.cuda(), **kw)
    assert [t.shape for t in out] == [(12,), (12,), (12,), lg.shape]
    assert out[3].dtype == lg.dtype and out[0].dtype == torch.float32
    check(out, oracle.cross_entropy_fwd_bwd(lg, lb, dloss, **kw), dt, dloss, kw)


@pytest.mark.parametrize("smooth", [False, True])
def test_fused_matches_separate_fwd_and_bwd(smooth):
    n = 128256
    lg, lb, dloss = make(300, n, "bf16", 3)  # more rows than SMs
    kw = kwargs(n, smooth)
    lgc, lbc, dlc = lg.cuda(), lb.cuda(), dloss.cuda()
    loss, lse, z, dx = B.cross_entropy_fwd_bwd(lgc, lbc, dlc, **kw)
    f_loss, f_lse, f_z = B.cross_entropy_fwd(lgc, lbc, **kw, BLOCK_SIZE=n, SPLIT=False)
    f_dx = B.cross_entropy_bwd(dlc, lgc, f_lse.view(-1)[:300], lbc, **kw, BLOCK_SIZE=n)
    for a, b in ((loss, f_loss), (lse, f_lse), (z, f_z)):
        ok, msg = parity.compare(a.cpu(), b.view(-1)[:300].cpu(), torch.float32)
        assert ok, msg
    ok, msg = parity.compare(dx.cpu(), f_dx.cpu(), torch.bfloat16, abs_slack=grad_slack(f_dx.cpu(), dloss, kw))
    assert ok, msg
    torch.cuda.synchronize()
    assert _lib.take_wait_timeouts() == 0


def test_fused_strided_logits_dloss_and_int32_labels():
    lg_full, lb, dloss_full = make(6, 3000, "bf16", 11)
    lb = lb.to(torch.int32)
    dl2 = torch.stack([dloss_full, dloss_full], 1).reshape(-1)  # stride 2 view below
    kw = dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100, total_classes=2500,
              class_start_idx=2, HAS_SMOOTHING=False)
    out = B.cross_entropy_fwd_bwd(lg_full.cuda()[:, :2500], lb.cuda(), dl2.cuda()[::2], **kw)
    ref = oracle.cross_entropy_fwd_bwd(lg_full[:, :2500].contiguous(), lb, dloss_full, **kw)
    check(out, ref, "bf16", dloss_full, kw)


def test_fused_rejects_bad_arguments():
    lg, lb, dloss = make(4, 64, "f32", 1)
    kw = kwargs(64, False)
    with pytest.raises(ValueError):
        B.cross_entropy_fwd_bwd(lg.cuda(), lb[:3].cuda(), dloss.cuda(), **kw)
    with pytest.raises(TypeError):
        B.cross_entropy_fwd_bwd(lg.cuda(), lb.float().cuda(), dloss.cuda(), **kw)
    with pytest.raises(ValueError):
        B.cross_entropy_fwd_bwd(lg, lb, dloss, **kw)  # host tensors
