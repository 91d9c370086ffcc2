"""CUDA backend against the reference's golden vectors (tests/golden/), through
the same cuda_impl functions a ViperBench driver would import."""
import pytest

import parity
import golden_cases
import dslperfgap_b200 as B

CASES = list(golden_cases.all_cases())


@pytest.mark.gpu
@pytest.mark.parametrize("op,case", CASES, ids=golden_cases.ids())
def test_cuda_matches_reference_golden(op, case):
    fn = getattr(B, golden_cases.FN_NAME[op])
    out = golden_cases.run(fn, op, case, device="cuda")
    errs = golden_cases.check_case(op, case, out, parity)
    assert not errs, "\n".join(errs)
