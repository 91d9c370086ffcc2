"""The reference's PyTorch backend restated as the torch CPU calls it makes —
TEST AND BASELINE INFRASTRUCTURE ONLY.

The reference's ``ViperBench/<kernel>/pytorch_impl.py`` files are one or a
few torch operators each. Run on CPU tensors, these functions execute exactly
those operators (torch's own CPU kernels), so ``bench.py --impl reference``
and the ``cpu_baseline`` leg can time the reference's own CPU path on the GPU
box, where the reference checkout itself is not present. Nothing on the
product path imports this module.

Each function cites the reference lines it restates.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def layer_norm(x, weight, bias, eps=1e-5):
    """ViperBench/layer_norm/pytorch_impl.py:5-12 (eps other than 1e-5 raises)."""
    if eps != 1e-5:
        raise ValueError(f"Only eps=1e-5 is supported (got {eps}).")
    return F.layer_norm(x, weight.shape, weight, bias, eps)


def rms_norm(x, normalized_shape, weight, eps=1e-5):
    """ViperBench/rms_norm/pytorch_impl.py:3-10: fp32 mean of squares over the
    trailing dims, sqrt(+eps), divide, scale by weight, cast back."""
    dims = tuple(range(x.ndim - len(normalized_shape), x.ndim))
    rms = torch.sqrt(torch.mean(x.float() ** 2, dim=dims, keepdim=True) + eps)
    return ((x.float() / rms) * weight.float()).to(x.dtype)


def softmax(x):
    """ViperBench/softmax/pytorch_impl.py:4-6."""
    return F.softmax(x, dim=-1)


def log_softmax(x, dim=-1, dtype=None):
    """ViperBench/log_softmax/pytorch_impl.py:4-8."""
    return F.log_softmax(x, dim=dim, dtype=dtype)


def logsumexp(x):
    """ViperBench/logsumexp/pytorch_impl.py:3-5."""
    return torch.logsumexp(x, dim=-1)


def mean_reduction(input_tensor, dim, keepdim=False, dtype=None):
    """ViperBench/mean_reduction/pytorch_impl.py:4-8."""
    return torch.mean(input_tensor, dim=dim, keepdim=keepdim, dtype=dtype)


def max_reduction(input, dim, keepdim=False):
    """ViperBench/max_reduction/pytorch_impl.py:4-11 (values and indices)."""
    return torch.max(input, dim=dim, keepdim=keepdim)


def argmax(input_tensor, dim, keepdim=False):
    """ViperBench/argmax/pytorch_impl.py:4-8."""
    return torch.argmax(input_tensor, dim=dim, keepdim=keepdim)


FUNCTIONS = {f.__name__: f for f in (layer_norm, rms_norm, softmax, log_softmax, logsumexp, mean_reduction,
                                     max_reduction, argmax)}


def threads() -> int:
    """Host threads torch's CPU kernels use in this process."""
    return torch.get_num_threads()
