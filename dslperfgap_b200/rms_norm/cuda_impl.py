"""CUDA (sm_100a) backend of ViperBench ``rms_norm``.

Same signature as ViperBench/rms_norm/pytorch_impl.py:3-10:
``rms_norm(x, normalized_shape, weight, eps=1e-5)`` computes
``(x.float() / sqrt(mean(x.float()**2) + eps) * weight.float()).to(x.dtype)``
over the trailing ``len(normalized_shape)`` dims, in one kernel.
"""
import math

import torch

from .. import _lib


def rms_norm(x, normalized_shape, weight, eps=1e-5):
    dev = _lib.require_cuda(x, weight, what="rms_norm")
    xc = _lib.float_code(x, "rms_norm")
    wc = _lib.float_code(weight, "rms_norm weight")
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    k = len(normalized_shape)
    if k == 0 or x.dim() < k:
        raise ValueError(f"rms_norm: normalized_shape {tuple(normalized_shape)} does not fit x {tuple(x.shape)}")
    trailing = tuple(x.shape[x.dim() - k:])
    n = math.prod(trailing)
    if weight.numel() != n or weight.dim() > k or tuple(weight.shape) != trailing[k - weight.dim():]:
        raise ValueError(f"rms_norm: weight shape {tuple(weight.shape)} does not match normalized dims {trailing}")
    m = x.numel() // n if n else 0
    x = x.contiguous()
    w = weight.contiguous()
    y = torch.empty_like(x)
    if x.numel() == 0:
        return y
    with torch.cuda.device(dev):
        rc = _lib.load().dslpg_rms_norm_fwd(
            x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, xc, wc, float(eps), _lib.stream_handle(dev))
    _lib.check(rc, "dslpg_rms_norm_fwd")
    return y
