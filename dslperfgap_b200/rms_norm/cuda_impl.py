"""CUDA (sm_100a) backend of ViperBench ``rms_norm``.

Same signature as ViperBench/rms_norm/pytorch_impl.py:3-10:
``rms_norm(x, normalized_shape, weight, eps=1e-5)`` computes
``(x.float() / sqrt(mean(x.float()**2) + eps) * weight.float()).to(x.dtype)``
over the trailing ``len(normalized_shape)`` dims, in one kernel.
"""
import math

import torch

from .. import _lib

_fast_rms_norm = _lib.fast_op("rms_norm")


def rms_norm(x, normalized_shape, weight, eps=1e-5):
    out = _fast_rms_norm(x, normalized_shape, weight, eps)
    if out is not None:  # the C++ fast path took the common case
        return out
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
    _lib.launch(dev, "dslpg_rms_norm_fwd", x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, xc, wc, float(eps))
    return y


def rms_norm_host(x, normalized_shape, weight, eps=1e-5, out=None):
    """``rms_norm`` for an input in HOST memory, returning a host tensor.

    The rows stream through the GPU of ``weight`` in chunks with the uploads,
    kernels and downloads overlapped (``dslpg_rms_norm_fwd_host``); pin ``x``
    and ``out`` (``pin_memory()``) for the copies to overlap. ``out`` (host,
    same shape and dtype as ``x``) is allocated pinned when not given. Returns
    after the current stream has finished, so the result is ready to read."""
    if not isinstance(weight, torch.Tensor) or not weight.is_cuda:
        raise ValueError("rms_norm_host: weight must be a CUDA tensor (it selects the GPU)")
    if x.is_cuda:
        raise ValueError("rms_norm_host: x must be a host tensor; use rms_norm for device tensors")
    dev = weight.device
    xc = _lib.float_code(x, "rms_norm_host")
    wc = _lib.float_code(weight, "rms_norm_host weight")
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    k = len(normalized_shape)
    if k == 0 or x.dim() < k:
        raise ValueError(f"rms_norm_host: normalized_shape {tuple(normalized_shape)} does not fit x {tuple(x.shape)}")
    trailing = tuple(x.shape[x.dim() - k:])
    n = math.prod(trailing)
    if weight.numel() != n or weight.dim() > k or tuple(weight.shape) != trailing[k - weight.dim():]:
        raise ValueError(f"rms_norm_host: weight shape {tuple(weight.shape)} does not match normalized dims {trailing}")
    m = x.numel() // n if n else 0
    x = x.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    elif out.is_cuda or out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("rms_norm_host: out must be a contiguous host tensor of x's shape and dtype")
    if x.numel() == 0:
        return out
    w = weight.contiguous()
    _lib.run_host_pipeline("dslpg_rms_norm_fwd_host", x, out, dev, m, n, xc, (w.data_ptr(),), (wc, float(eps)))
    return out
