"""The benchmark configurations at their full sizes, CUDA vs the CPU oracle
on the same seeded inputs (the oracle runs on all host cores), plus
size-independent properties that hold at any size."""
import pytest
import torch

import parity
from oracle import oracle
import dslperfgap_b200 as B
from dslperfgap_b200 import workloads

pytestmark = pytest.mark.gpu


def assert_parity(out, ref, dtype, normalised=False):
    ok, msg = parity.compare(out, ref, dtype, normalised=normalised)
    assert ok, msg


@pytest.mark.parametrize("name", workloads.NAMES)
def test_full_size_config_matches_oracle(name):
    wl = workloads.make(name, seed=0)
    out = wl.cuda_fn(*wl.to("cuda").args, **wl.kwargs)
    if wl.op == "cross_entropy":
        ref = oracle.cross_entropy_fwd(*wl.args, **wl.kwargs, valid_only=True)
    else:
        ref = getattr(oracle, wl.fn_name)(*wl.args, **wl.kwargs)
    if wl.op == "cross_entropy":
        nv = wl.valid_entries
        for i, (o, r) in enumerate(zip(out, ref)):
            assert_parity(o.reshape(-1)[:nv], r.reshape(-1)[:nv], torch.float32)
    elif wl.op == "cross_entropy_fwd_bwd":  # (loss, lse, z_loss) [M] and dlogits
        for o, r in zip(out[:3], ref[:3]):
            assert_parity(o, r, torch.float32)
        assert_parity(out[3], ref[3], wl.config.dtype)
    elif isinstance(ref, tuple):  # max_reduction: (values, indices)
        assert_parity(out[0], ref[0], ref[0].dtype)
        assert torch.equal(out[1].cpu(), ref[1])
    elif not ref.dtype.is_floating_point:  # argmax
        assert torch.equal(out.cpu(), ref)
    elif wl.op == "linear_activation":  # fp32 dot products of length K before the gate
        ok, msg = parity.compare(out, ref, wl.out_dtype, abs_slack=parity.gemm_slack(*wl.args))
        assert ok, msg
        hist = parity.ulp_histogram(out, ref, wl.out_dtype)
        print(f"kernel_ff {wl.M}x{wl.config.K} @ {wl.config.N}: |out - ref| in fp16 ulps {hist}")
        within1 = hist["[0,0.5]"] + hist["(0.5,1]"]
        assert within1 >= 0.99 * out.numel(), hist  # the slack is for the cancelling few
    else:
        assert_parity(out, ref, wl.out_dtype, normalised=wl.op in parity.NORMALISED)


def test_softmax_rows_sum_to_one_full_size():
    wl = workloads.make("softmax_fp16", seed=3)
    y = B.softmax(wl.args[0].cuda()).float()
    s = y.sum(-1)
    # each of 4096 outputs is within half an fp16 ulp (<= 2^-12 relative) of its value
    assert torch.allclose(s, torch.ones_like(s), atol=4096 * 2.0 ** -12 / 64)


def test_logsumexp_shift_invariance_full_size():
    wl = workloads.make("logsumexp_bf16", seed=4)
    x = wl.args[0].cuda()
    a = B.logsumexp(x).float()
    b = B.logsumexp((x.float() + 4.0).to(torch.bfloat16)).float()
    # x + 4 is exact in bf16 only for some values; compare within 2 bf16 ulps at |lse| ~ 16
    assert torch.allclose(b - a, torch.full_like(a, 4.0), atol=0.25)


def test_cross_entropy_mean_loss_matches_oracle_full_size():
    wl = workloads.make("cross_entropy_bf16", seed=0)
    logits, labels = wl.args[0].cuda(), wl.args[1].cuda()
    loss, lse, _ = B.cross_entropy_fwd(logits, labels, **wl.kwargs)
    keep = labels != -100
    mean = loss.view(-1)[: logits.shape[0]][keep].double().mean().item()
    ref_loss, _, _ = oracle.cross_entropy_fwd(wl.args[0], wl.args[1], **wl.kwargs, valid_only=True)
    ref_mean = ref_loss.view(-1)[: logits.shape[0]][keep.cpu()].double().mean().item()
    assert abs(mean - ref_mean) <= 1e-5 * abs(ref_mean)
