"""CUDA (sm_100a) backend of ViperBench ``argmax``.

Same signature as ViperBench/argmax/pytorch_impl.py:4-8:
``argmax(input_tensor, dim, keepdim=False)`` is
``torch.argmax(input_tensor, dim=dim, keepdim=keepdim)`` (``dim=None``
flattens). The first NaN is the maximum; equal maxima give the first index.
"""
import torch

from .. import _dims, _lib

_fast_argmax = _lib.fast_op("argmax")


def argmax(input_tensor, dim, keepdim=False):
    out = _fast_argmax(input_tensor, dim, keepdim)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(input_tensor, what="argmax")
    code = _lib.float_code(input_tensor, "argmax")
    shape = tuple(input_tensor.shape)
    if dim is None:
        x, m, n, k = input_tensor.contiguous().reshape(-1), 1, input_tensor.numel(), 1
        oshape = tuple(1 for _ in shape) if keepdim else ()
    else:
        dims = _dims.normalize_dims(dim, input_tensor.dim())
        x, m, n, k = _dims.as_mnk(input_tensor, dims)
        oshape = _dims.out_shape(shape, dims, keepdim) if shape else ()
    if n == 0:
        raise IndexError("argmax(): Expected reduction dim to have non-zero size")
    indices = torch.empty(oshape, dtype=torch.int64, device=x.device)
    if indices.numel() == 0:
        return indices
    _lib.launch(dev, "dslpg_argmax", x.data_ptr(), indices.data_ptr(), m, n, k, code)
    return indices
