"""CUDA (sm_100a) backend of ViperBench ``mean_reduction``.

Same signature as ViperBench/mean_reduction/pytorch_impl.py:4-8:
``mean_reduction(input_tensor, dim, keepdim=False, dtype=None)`` is
``torch.mean(input_tensor, dim, keepdim=keepdim, dtype=dtype)``: ``dim`` an int
or a list of dims; the input is converted to ``dtype`` first; fp32 accumulation.
"""
import torch

from .. import _dims, _lib

_fast_mean_reduction = _lib.fast_op("mean_reduction")


def mean_reduction(input_tensor, dim, keepdim=False, dtype=None):
    out = _fast_mean_reduction(input_tensor, dim, keepdim, dtype)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(input_tensor, what="mean_reduction")
    in_code = _lib.float_code(input_tensor, "mean_reduction")
    out_dtype = input_tensor.dtype if dtype is None else dtype
    if out_dtype not in _lib.FLOAT_CODES:
        raise TypeError(f"mean_reduction: unsupported dtype {out_dtype}")
    shape = tuple(input_tensor.shape)
    dims = _dims.normalize_dims(dim, input_tensor.dim())
    x, m, n, k = _dims.as_mnk(input_tensor, dims)
    y = torch.empty(_dims.out_shape(shape, dims, keepdim) if shape else (), dtype=out_dtype, device=x.device)
    if y.numel() == 0:
        return y
    if n == 0:
        return y.fill_(float("nan"))  # torch: the mean of an empty set is NaN
    _lib.launch(dev, "dslpg_mean_reduction", x.data_ptr(), y.data_ptr(), m, n, k, in_code,
                                              _lib.FLOAT_CODES[out_dtype])
    return y
