"""CUDA (sm_100a) backend of ViperBench ``layer_norm``.

Same signature and error behaviour as ViperBench/layer_norm/pytorch_impl.py:5-12:
``layer_norm(x, weight, bias, eps=1e-5)`` normalises over ``weight.shape`` (the
trailing dims of x) and raises ``ValueError`` for any eps other than 1e-5.
Computes in fp32 and returns a new tensor of x's shape and dtype.
"""
import math

import torch

from .. import _lib

_fast_layer_norm = _lib.fast_op("layer_norm")


def layer_norm(x, weight, bias, eps=1e-5):
    out = _fast_layer_norm(x, weight, bias, eps)
    if out is not None:  # the C++ fast path took the common case
        return out
    if eps != 1e-5:
        raise ValueError(f"Only eps=1e-5 is supported (got {eps}). "
                         "The Triton kernel hardcodes eps=1e-5.")
    dev = _lib.require_cuda(x, weight, bias, what="layer_norm")
    xc = _lib.float_code(x, "layer_norm")
    wc = _lib.float_code(weight, "layer_norm weight")
    if bias is not None and bias.dtype != weight.dtype:
        raise TypeError(f"layer_norm: bias dtype {bias.dtype} differs from weight dtype {weight.dtype}")
    nshape = tuple(weight.shape)
    if len(nshape) == 0 or tuple(x.shape[x.dim() - len(nshape):]) != nshape or x.dim() < len(nshape):
        raise ValueError(f"layer_norm: weight shape {nshape} does not match the trailing dims of x {tuple(x.shape)}")
    if bias is not None and tuple(bias.shape) != nshape:
        raise ValueError(f"layer_norm: bias shape {tuple(bias.shape)} != weight shape {nshape}")
    n = math.prod(nshape)
    m = x.numel() // n if n else 0
    x = x.contiguous()
    w = weight.contiguous()
    b = bias.contiguous() if bias is not None else None
    y = torch.empty_like(x)
    if x.numel() == 0:
        return y
    _lib.launch(dev, "dslpg_layer_norm_fwd", x.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None, y.data_ptr(),
            m, n, xc, wc, float(eps))
    return y


def layer_norm_host(x, weight, bias, eps=1e-5, out=None):
    """``layer_norm`` for an input in HOST memory, returning a host tensor.

    The rows stream through the GPU that holds ``weight`` in chunks, with the
    uploads, kernels and downloads overlapped (``dslpg_layer_norm_fwd_host``);
    pin ``x`` and ``out`` (``pin_memory()``) for the copies to overlap. ``out``
    (host, x's shape and dtype) is allocated pinned when not given. Returns
    once the result is in ``out``. Same arguments, errors and result as
    ``layer_norm`` (ViperBench/layer_norm/pytorch_impl.py:5-12), row by row."""
    if eps != 1e-5:
        raise ValueError(f"Only eps=1e-5 is supported (got {eps}). "
                         "The Triton kernel hardcodes eps=1e-5.")
    if not isinstance(weight, torch.Tensor) or not weight.is_cuda:
        raise ValueError("layer_norm_host: weight must be a CUDA tensor (it selects the GPU)")
    if not isinstance(x, torch.Tensor) or x.is_cuda:
        raise ValueError("layer_norm_host: x must be a host tensor; use layer_norm for device tensors")
    dev = _lib.require_cuda(weight, bias, what="layer_norm_host")
    xc = _lib.float_code(x, "layer_norm_host")
    wc = _lib.float_code(weight, "layer_norm_host weight")
    if bias is not None and bias.dtype != weight.dtype:
        raise TypeError(f"layer_norm_host: bias dtype {bias.dtype} differs from weight dtype {weight.dtype}")
    nshape = tuple(weight.shape)
    if len(nshape) == 0 or x.dim() < len(nshape) or tuple(x.shape[x.dim() - len(nshape):]) != nshape:
        raise ValueError(f"layer_norm_host: weight shape {nshape} does not match the trailing dims of x "
                         f"{tuple(x.shape)}")
    if bias is not None and tuple(bias.shape) != nshape:
        raise ValueError(f"layer_norm_host: bias shape {tuple(bias.shape)} != weight shape {nshape}")
    n = math.prod(nshape)
    m = x.numel() // n if n else 0
    x = x.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    elif out.is_cuda or out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("layer_norm_host: out must be a contiguous host tensor of x's shape and dtype")
    if x.numel() == 0:
        return out
    w = weight.contiguous()
    b = bias.contiguous() if bias is not None else None
    _lib.run_host_pipeline("dslpg_layer_norm_fwd_host", x, out, dev, m, n, xc,
                           (w.data_ptr(), b.data_ptr() if b is not None else None), (wc, float(eps)))
    return out
