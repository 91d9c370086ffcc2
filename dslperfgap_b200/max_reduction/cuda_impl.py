"""CUDA (sm_100a) backend of ViperBench ``max_reduction``.

Same signature and error behaviour as ViperBench/max_reduction/pytorch_impl.py:4-11:
``max_reduction(input, dim, keepdim=False)`` returns ``(values, indices)`` of
``torch.max(input, dim, keepdim)``; a non-tensor input raises TypeError. The
first NaN is the maximum; equal maxima give the first index.
"""
import torch

from .. import _dims, _lib

_fast_max_reduction = _lib.fast_op("max_reduction")


def max_reduction(input, dim, keepdim=False):
    out = _fast_max_reduction(input, dim, keepdim)
    if out is not None:  # the C++ fast path took the common case
        return out
    if not isinstance(input, torch.Tensor):
        raise TypeError('The input must be a torch.Tensor.')
    dev = _lib.require_cuda(input, what="max_reduction")
    code = _lib.float_code(input, "max_reduction")
    shape = tuple(input.shape)
    dims = _dims.normalize_dims(dim, input.dim())
    x, m, n, k = _dims.as_mnk(input, dims)
    if n == 0:
        raise IndexError("max(): Expected reduction dim to have non-zero size")
    oshape = _dims.out_shape(shape, dims, keepdim) if shape else ()
    values = torch.empty(oshape, dtype=input.dtype, device=x.device)
    indices = torch.empty(oshape, dtype=torch.int64, device=x.device)
    if values.numel() == 0:
        return (values, indices)
    _lib.launch(dev, "dslpg_max_reduction", x.data_ptr(), values.data_ptr(), indices.data_ptr(), m, n, k, code)
    return (values, indices)
