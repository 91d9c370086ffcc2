"""Argument validation of the cuda_impl wrappers (mirrors the reference's
error behaviour; runs on CPU because every check happens before a launch)."""
import pytest
import torch

from dslperfgap_b200.layer_norm.cuda_impl import layer_norm
from dslperfgap_b200.rms_norm.cuda_impl import rms_norm
from dslperfgap_b200.softmax.cuda_impl import softmax
from dslperfgap_b200.log_softmax.cuda_impl import log_softmax
from dslperfgap_b200.logsumexp.cuda_impl import logsumexp
from dslperfgap_b200.cross_entropy.cuda_impl import cross_entropy_fwd


def test_layer_norm_eps_other_than_1e5_is_a_value_error():
    x = torch.randn(2, 8)
    with pytest.raises(ValueError, match="eps=1e-5"):
        layer_norm(x, torch.ones(8), torch.zeros(8), eps=1e-6)


@pytest.mark.parametrize("fn,args", [
    (layer_norm, (torch.randn(2, 8), torch.ones(8), torch.zeros(8))),
    (rms_norm, (torch.randn(2, 8), (8,), torch.ones(8))),
    (softmax, (torch.randn(2, 8),)),
    (log_softmax, (torch.randn(2, 8),)),
    (logsumexp, (torch.randn(2, 8),)),
])
def test_cpu_tensors_are_rejected(fn, args):
    # No CPU fallback: a CPU tensor is an error, never silently computed.
    with pytest.raises(ValueError, match="CUDA"):
        fn(*args)


def test_cross_entropy_cpu_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        cross_entropy_fwd(torch.randn(2, 8), torch.zeros(2, dtype=torch.int64), 0.0, 1.0, 0.0, -100, 8, 0, 8,
                          False, False)


def test_non_tensor_rejected():
    with pytest.raises(TypeError):
        softmax([1.0, 2.0])
