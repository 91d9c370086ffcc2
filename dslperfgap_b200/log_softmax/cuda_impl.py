"""CUDA (sm_100a) backend of ViperBench ``log_softmax``.

Same signature as ViperBench/log_softmax/pytorch_impl.py:4-8:
``log_softmax(x, dim=-1, dtype=None)``. Any ``dim`` is supported (the tensor
is viewed as [M, N, K] with N the reduced axis); ``dtype`` selects the output
dtype, and x is first converted to it, as F.log_softmax does.
"""
import math

import torch

from .. import _lib

_fast_log_softmax = _lib.fast_op("log_softmax")


def log_softmax(x, dim=-1, dtype=None):
    out = _fast_log_softmax(x, dim, dtype)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(x, what="log_softmax")
    in_code = _lib.float_code(x, "log_softmax")
    out_dtype = x.dtype if dtype is None else dtype
    if out_dtype not in _lib.FLOAT_CODES:
        raise TypeError(f"log_softmax: unsupported dtype {out_dtype}")
    out_code = _lib.FLOAT_CODES[out_dtype]
    nd = max(x.dim(), 1)
    if not -nd <= dim < nd:
        raise IndexError(f"Dimension out of range (expected to be in range of [{-nd}, {nd - 1}], but got {dim})")
    dim = dim % nd
    shape = tuple(x.shape) if x.dim() > 0 else (1,)
    m = math.prod(shape[:dim])
    n = shape[dim]
    k = math.prod(shape[dim + 1:])
    x = x.contiguous()
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    if x.numel() == 0:
        return y
    _lib.launch(dev, "dslpg_log_softmax_fwd", x.data_ptr(), y.data_ptr(), m, n, k, in_code, out_code)
    return y
