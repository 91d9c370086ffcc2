"""CUDA (sm_100a) backend of ViperBench ``softmax``.

Same signature as ViperBench/softmax/pytorch_impl.py:4-6: ``softmax(x)`` along
the last dimension of a tensor of any rank, returning x's dtype.
"""
import torch

from .. import _lib

_fast_softmax = _lib.fast_op("softmax")


def softmax(x):
    out = _fast_softmax(x)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(x, what="softmax")
    code = _lib.float_code(x, "softmax")
    x = x.contiguous()
    y = torch.empty_like(x)
    if x.numel() == 0:
        return y
    n = x.shape[-1] if x.dim() > 0 else 1
    m = x.numel() // n
    _lib.launch(dev, "dslpg_softmax_fwd", x.data_ptr(), y.data_ptr(), m, n, code)
    return y
