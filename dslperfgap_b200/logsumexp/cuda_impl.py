"""CUDA (sm_100a) backend of ViperBench ``logsumexp``.

Same signature as ViperBench/logsumexp/pytorch_impl.py:3-5: ``logsumexp(x)``
reduces the last dimension, returning shape ``x.shape[:-1]`` in x's dtype,
with torch.logsumexp's handling of infinities (+inf in a row gives +inf, an
all -inf row gives -inf, NaN propagates).
"""
import torch

from .. import _lib

_fast_logsumexp = _lib.fast_op("logsumexp")


def logsumexp(x):
    out = _fast_logsumexp(x)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(x, what="logsumexp")
    code = _lib.float_code(x, "logsumexp")
    x = x.contiguous()
    out_shape = tuple(x.shape[:-1]) if x.dim() > 0 else ()
    n = x.shape[-1] if x.dim() > 0 else 1
    y = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    if y.numel() == 0:
        return y
    if n == 0:
        return y.fill_(float("-inf"))  # logsumexp over an empty row
    m = y.numel()
    _lib.launch(dev, "dslpg_logsumexp_fwd", x.data_ptr(), y.data_ptr(), m, n, code)
    return y
