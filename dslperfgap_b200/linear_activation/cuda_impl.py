"""CUDA (sm_100a) backend of ViperBench ``linear_activation``.

Same signature as ViperBench/linear_activation/pytorch_impl.py:5-54:
``kernel_ff(x, w1, w3, rms_w)`` for x [batch, seq, dim], w1 / w3 [n_out, dim],
rms_w [dim]; inputs are converted to fp16 as there, and the result is
``silu(a_norm * (x*rms_w) @ w1.T) * (a_norm * (x*rms_w) @ w3.T)`` in fp16 with
``a_norm = rsqrt(mean(x.float()**2) + 1e-6)``: a row pass computes a_norm and
x*rms_w, then a tcgen05 dual GEMM with the scale and the SiLU gate in its
epilogue.
"""
import ctypes

import torch

from .. import _lib


def _aligned16(t):
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def kernel_ff(x, w1, w3, rms_w):
    dev = _lib.require_cuda(x, w1, w3, rms_w, what="kernel_ff")
    x = x.half() if x.dtype != torch.float16 else x
    w1 = w1.half() if w1.dtype != torch.float16 else w1
    w3 = w3.half() if w3.dtype != torch.float16 else w3
    rms_w = rms_w.half() if rms_w.dtype != torch.float16 else rms_w
    if x.dim() != 3:
        raise ValueError(f"kernel_ff: x must be [batch, seq_len, dim], got {tuple(x.shape)}")
    if w1.shape != w3.shape:
        raise ValueError(f"kernel_ff: w1 {tuple(w1.shape)} and w3 {tuple(w3.shape)} differ in shape")
    batch, seq_len, dim = x.shape
    n = w1.shape[0]
    if w1.shape[1] != dim or rms_w.numel() != dim:
        raise ValueError("kernel_ff: w1/w3 must be [n_out, dim] and rms_w [dim]")
    if dim % 8 != 0:
        raise ValueError(f"kernel_ff: dim must be a multiple of 8 (16-byte rows), got {dim}")
    m = batch * seq_len
    # the kernels read 16-byte vectors and TMA tiles: a contiguous view at an odd
    # offset (e.g. sliced from a flat parameter buffer) is copied to a fresh,
    # 256-byte aligned allocation
    xf, w1c, w3c, rw = (_aligned16(t) for t in (x.reshape(m, dim), w1, w3, rms_w.reshape(dim)))
    out = torch.empty((m, n), dtype=torch.float16, device=x.device)
    if m == 0 or n == 0:
        return out.view(batch, seq_len, n)
    lib = _lib.load()
    need = ctypes.c_int64(0)
    _lib.check(lib.dslpg_kernel_ff_workspace_bytes(m, dim, ctypes.byref(need)), "dslpg_kernel_ff_workspace_bytes")
    ws = torch.empty(need.value, dtype=torch.uint8, device=x.device)
    _lib.launch(dev, "dslpg_kernel_ff", xf.data_ptr(), w1c.data_ptr(), w3c.data_ptr(), rw.data_ptr(), out.data_ptr(),
                m, n, dim, ws.data_ptr(), need.value)
    return out.view(batch, seq_len, n)
