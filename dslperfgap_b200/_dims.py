"""Viewing a reduction over some dims of a tensor as [M, N, K]."""
from __future__ import annotations

import math

import torch


def normalize_dims(dims, ndim: int) -> list[int]:
    if isinstance(dims, int):
        dims = [dims]
    nd = max(ndim, 1)
    out = []
    for d in dims:
        if not -nd <= d < nd:
            raise IndexError(f"Dimension out of range (expected to be in range of [{-nd}, {nd - 1}], but got {d})")
        d = d % nd
        if d in out:
            raise RuntimeError(f"dim {d} appears multiple times in the list of dims")
        out.append(d)
    return sorted(out)


def as_mnk(x: torch.Tensor, dims: list[int]):
    """Return (x', M, N, K) with x' contiguous and the reduced dims one middle
    run of extent N. Adjacent reduced dims need no copy; otherwise they are
    moved last with one contiguous copy (as the reference's wrappers do for
    layouts their kernels cannot read)."""
    shape = tuple(x.shape) if x.dim() > 0 else (1,)
    x = x.reshape(shape)
    if dims == list(range(dims[0], dims[-1] + 1)):
        m = math.prod(shape[:dims[0]])
        n = math.prod(shape[dims[0]:dims[-1] + 1])
        k = math.prod(shape[dims[-1] + 1:])
        return x.contiguous(), m, n, k
    keep = [d for d in range(len(shape)) if d not in dims]
    xp = x.permute(*keep, *dims).contiguous()
    m = math.prod(shape[d] for d in keep)
    n = math.prod(shape[d] for d in dims)
    return xp, m, n, 1


def out_shape(shape, dims: list[int], keepdim: bool):
    if keepdim:
        return tuple(1 if i in dims else s for i, s in enumerate(shape))
    return tuple(s for i, s in enumerate(shape) if i not in dims)
