"""The reference's correctness flow through the drop-in stubs: each stub is
loaded the way experiments/_harness.py:152-167 loads a backend, run on the
golden inputs (the reference's test.py shapes and the benchmark rows), and
its output compared with the reference's own output by the comparison of
ViperBench/test_utils.py (loose tolerance, as the reduction tests use)."""
import pytest
import torch

import golden_cases
import viperbench_loader as VL

pytestmark = pytest.mark.gpu

CASES = [(op, c) for op, c in golden_cases.all_cases() if op != "cross_entropy_bwd"]
KERNEL = {"cross_entropy": "cross_entropy", "linear_activation": "linear_activation"}


@pytest.mark.parametrize("op,case", CASES, ids=[f"{op}-{c['name']}" for op, c in CASES])
def test_stub_passes_reference_compare(op, case):
    mod = VL.load_impl(VL.STUBS, KERNEL.get(op, op), "cuda")
    fn = getattr(mod, golden_cases.FN_NAME[op])
    out = golden_cases.run(fn, op, case, device="cuda")
    ref = case["ref_native"]
    outs, refs = (out, ref) if isinstance(ref, tuple) else ((out,), (ref,))
    if op == "cross_entropy" and case["kwargs"]["SPLIT"]:
        outs, refs = outs[:2], refs[:2]  # z_loss is not compared under SPLIT (cross_entropy/test.py:40-44)
    for o, r in zip(outs, refs):
        if not r.dtype.is_floating_point:  # indices
            assert torch.equal(o, r)
            continue
        finite = torch.isfinite(r.float())
        assert torch.equal(torch.isfinite(o.float()), finite)
        assert torch.equal(o.float()[~finite].nan_to_num(), r.float()[~finite].nan_to_num())
        ok, err = VL.compare_tensors(r[finite].float(), o[finite].float(), r.dtype, loose=True)
        assert ok, f"max_err={err}"
