"""CPU oracle for the row-reduction family — TEST INFRASTRUCTURE ONLY.

Python face of ``oracle.c`` (a restatement of the reference's PyTorch backend,
tingxi-li/DSLPerfGap ``ViperBench/<kernel>/pytorch_impl.py``; each C function
cites the lines it follows). Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm use it, and only as the checker
or the timed CPU implementation; the product path never imports it.

Functions take and return CPU torch tensors (used purely as typed host
buffers; no torch arithmetic is involved) with the reference signatures.
"""
from __future__ import annotations

import ctypes
import math
import subprocess
import threading
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_LABEL_CODES = {torch.int32: 3, torch.int64: 4}

_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    """Compile oracle.c into liboracle.so with the committed Makefile."""
    src = HERE / "oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        res = subprocess.run(["make", "-C", str(HERE), "-B" if force else "liboracle.so"],
                             capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                build()
                l = ctypes.CDLL(str(LIB_PATH))
                vp, i64, ci, cd = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double
                l.oracle_layer_norm.argtypes = [vp, vp, vp, vp, i64, i64, ci, ci, cd]
                l.oracle_rms_norm.argtypes = [vp, vp, vp, i64, i64, ci, ci, cd]
                l.oracle_softmax.argtypes = [vp, vp, i64, i64, ci]
                l.oracle_log_softmax.argtypes = [vp, vp, i64, i64, i64, ci, ci]
                l.oracle_logsumexp.argtypes = [vp, vp, i64, i64, ci]
                l.oracle_cross_entropy_fwd.argtypes = [vp, vp, vp, vp, vp, i64, i64, ci, ci, cd, cd, cd,
                                                       i64, cd, i64, i64, ci, ci, i64]
                l.oracle_cross_entropy_bwd.argtypes = [vp, ci, vp, vp, vp, vp, i64, i64, ci, ci, cd, cd, cd,
                                                       i64, cd, i64, ci]
                l.oracle_mean_reduction.argtypes = [vp, vp, i64, i64, i64, ci, ci]
                l.oracle_max_reduction.argtypes = [vp, vp, vp, i64, i64, i64, ci]
                l.oracle_kernel_ff.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64]
                l.oracle_set_threads.argtypes = [ci]
                l.oracle_max_threads.restype = ci
                l.oracle_half_to_float.argtypes = [ctypes.c_uint16]
                l.oracle_half_to_float.restype = ctypes.c_float
                l.oracle_float_to_half.argtypes = [ctypes.c_float]
                l.oracle_float_to_half.restype = ctypes.c_uint16
                l.oracle_float_to_bf16.argtypes = [ctypes.c_float]
                l.oracle_float_to_bf16.restype = ctypes.c_uint16
                _lib = l
    return _lib


def set_threads(n: int) -> None:
    """Host threads used per call (0: one per online CPU)."""
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_max_threads())


def _host(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu":
        t = t.cpu()
    return t.contiguous()


def _code(t: torch.Tensor) -> int:
    if t.dtype not in _CODES:
        raise TypeError(f"oracle: unsupported dtype {t.dtype}")
    return _CODES[t.dtype]


def layer_norm(x, weight, bias, eps=1e-5):
    """F.layer_norm(x, weight.shape, weight, bias, eps); ViperBench/layer_norm/pytorch_impl.py:5-12."""
    if eps != 1e-5:
        raise ValueError(f"Only eps=1e-5 is supported (got {eps}). "
                         "The Triton kernel hardcodes eps=1e-5.")
    x, w = _host(x), _host(weight)
    b = _host(bias) if bias is not None else None
    n = w.numel()
    y = torch.empty_like(x)
    lib().oracle_layer_norm(x.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None,
                            y.data_ptr(), x.numel() // n, n, _code(x), _code(w), float(eps))
    return y


def rms_norm(x, normalized_shape, weight, eps=1e-5):
    """ViperBench/rms_norm/pytorch_impl.py:3-10."""
    x, w = _host(x), _host(weight)
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    n = math.prod(x.shape[x.dim() - len(normalized_shape):])
    y = torch.empty_like(x)
    lib().oracle_rms_norm(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.numel() // n, n,
                          _code(x), _code(w), float(eps))
    return y


def softmax(x):
    """F.softmax(x, dim=-1); ViperBench/softmax/pytorch_impl.py:4-6."""
    x = _host(x)
    n = x.shape[-1] if x.dim() else 1
    y = torch.empty_like(x)
    if x.numel():
        lib().oracle_softmax(x.data_ptr(), y.data_ptr(), x.numel() // n, n, _code(x))
    return y


def log_softmax(x, dim=-1, dtype=None):
    """F.log_softmax(x, dim, dtype); ViperBench/log_softmax/pytorch_impl.py:4-8."""
    x = _host(x)
    odt = x.dtype if dtype is None else dtype
    shape = tuple(x.shape) if x.dim() else (1,)
    dim = dim % len(shape)
    m, n, k = math.prod(shape[:dim]), shape[dim], math.prod(shape[dim + 1:])
    y = torch.empty(x.shape, dtype=odt)
    if x.numel():
        lib().oracle_log_softmax(x.data_ptr(), y.data_ptr(), m, n, k, _code(x), _CODES[odt])
    return y


def logsumexp(x):
    """torch.logsumexp(x, dim=-1); ViperBench/logsumexp/pytorch_impl.py:3-5."""
    x = _host(x)
    n = x.shape[-1] if x.dim() else 1
    y = torch.empty(tuple(x.shape[:-1]) if x.dim() else (), dtype=x.dtype)
    if y.numel():
        lib().oracle_logsumexp(x.data_ptr(), y.data_ptr(), y.numel(), n, _code(x))
    return y


def cross_entropy_fwd(logits, labels, smoothing, logit_scale, lse_square_scale,
                      ignored_index, total_classes, class_start_idx, BLOCK_SIZE, HAS_SMOOTHING, SPLIT,
                      valid_only=False):
    """ViperBench/cross_entropy/pytorch_impl.py:4-90: (loss, lse, z_loss), each fp32 [R, C]
    with zeros past the valid flat prefix; with valid_only=True each output is
    just the 1-D valid prefix of ceil(C / BLOCK_SIZE) * R entries."""
    lg, lb = _host(logits), _host(labels)
    r, c = lg.shape
    shape = (r * ((c + int(BLOCK_SIZE) - 1) // int(BLOCK_SIZE)),) if valid_only else (r, c)
    loss = torch.empty(shape, dtype=torch.float32)
    lse = torch.empty(shape, dtype=torch.float32)
    z = torch.empty(shape, dtype=torch.float32)
    lib().oracle_cross_entropy_fwd(
        lg.data_ptr(), lb.data_ptr(), loss.data_ptr(), lse.data_ptr(), z.data_ptr(), r, c,
        _code(lg), _LABEL_CODES[lb.dtype], float(smoothing), float(logit_scale),
        float(lse_square_scale), int(ignored_index), float(total_classes), int(class_start_idx),
        int(BLOCK_SIZE), 1 if HAS_SMOOTHING else 0, 1 if SPLIT else 0, loss.numel())
    return loss, lse, z


def cross_entropy_bwd(dloss, logits, lse, labels, smoothing, logit_scale, lse_square_scale,
                      ignored_index, total_classes, class_start_idx, BLOCK_SIZE, HAS_SMOOTHING):
    """ViperBench/cross_entropy/pytorch_impl.py:93-141: dlogits with logits' shape and dtype."""
    dl, lg, lb = _host(dloss), _host(logits), _host(labels)
    ls = _host(lse).reshape(-1).float().contiguous()
    r, c = lg.shape
    dx = torch.empty_like(lg)
    lib().oracle_cross_entropy_bwd(
        dl.data_ptr(), _code(dl), lg.data_ptr(), ls.data_ptr(), lb.data_ptr(), dx.data_ptr(), r, c, _code(lg),
        _LABEL_CODES[lb.dtype], float(smoothing), float(logit_scale), float(lse_square_scale),
        int(ignored_index), float(total_classes), int(class_start_idx), 1 if HAS_SMOOTHING else 0)
    return dx


def cross_entropy_fwd_bwd(logits, labels, dloss, smoothing, logit_scale, lse_square_scale,
                          ignored_index, total_classes, class_start_idx, HAS_SMOOTHING):
    """cross_entropy_fwd with one block per row (BLOCK_SIZE = C, SPLIT False)
    followed by cross_entropy_bwd from that lse (the same two reference
    functions): (loss, lse, z_loss) as 1-D [R], and dlogits."""
    c = _host(logits).shape[1]
    kw = dict(smoothing=smoothing, logit_scale=logit_scale, lse_square_scale=lse_square_scale,
              ignored_index=ignored_index, total_classes=total_classes, class_start_idx=class_start_idx)
    loss, lse, z = cross_entropy_fwd(logits, labels, **kw, BLOCK_SIZE=max(c, 1), HAS_SMOOTHING=HAS_SMOOTHING,
                                     SPLIT=False, valid_only=True)
    dx = cross_entropy_bwd(dloss, logits, lse, labels, **kw, BLOCK_SIZE=max(c, 1), HAS_SMOOTHING=HAS_SMOOTHING)
    return loss, lse, z, dx


def _mnk(x, dims):
    """(contiguous x, M, N, K, output shape without keepdim) for reducing `dims`."""
    shape = tuple(x.shape) if x.dim() else (1,)
    nd = len(shape)
    dims = sorted(d % nd for d in ([dims] if isinstance(dims, int) else dims))
    keep = [d for d in range(nd) if d not in dims]
    if dims == list(range(dims[0], dims[-1] + 1)):
        m = math.prod(shape[:dims[0]])
        n = math.prod(shape[dims[0]:dims[-1] + 1])
        k = math.prod(shape[dims[-1] + 1:])
        xc = x.reshape(shape).contiguous()
    else:
        xc = x.reshape(shape).permute(*keep, *dims).contiguous()
        m, n, k = math.prod(shape[d] for d in keep), math.prod(shape[d] for d in dims), 1
    return xc, m, n, k, dims, shape


def _oshape(shape, dims, keepdim, scalar):
    if scalar:
        return ()
    if keepdim:
        return tuple(1 if i in dims else s for i, s in enumerate(shape))
    return tuple(s for i, s in enumerate(shape) if i not in dims)


def mean_reduction(input_tensor, dim, keepdim=False, dtype=None):
    """torch.mean(x, dim, keepdim, dtype); ViperBench/mean_reduction/pytorch_impl.py:4-8."""
    x = _host(input_tensor)
    odt = x.dtype if dtype is None else dtype
    xc, m, n, k, dims, shape = _mnk(x, dim)
    y = torch.empty(_oshape(shape, dims, keepdim, x.dim() == 0), dtype=odt)
    lib().oracle_mean_reduction(xc.data_ptr(), y.data_ptr(), m, n, k, _code(x), _CODES[odt])
    return y


def max_reduction(input, dim, keepdim=False):
    """torch.max(x, dim, keepdim) -> (values, indices); ViperBench/max_reduction/pytorch_impl.py:4-11."""
    if not isinstance(input, torch.Tensor):
        raise TypeError('The input must be a torch.Tensor.')
    x = _host(input)
    xc, m, n, k, dims, shape = _mnk(x, dim)
    os_ = _oshape(shape, dims, keepdim, x.dim() == 0)
    v = torch.empty(os_, dtype=x.dtype)
    i = torch.empty(os_, dtype=torch.int64)
    lib().oracle_max_reduction(xc.data_ptr(), v.data_ptr(), i.data_ptr(), m, n, k, _code(x))
    return (v, i)


def argmax(input_tensor, dim, keepdim=False):
    """torch.argmax(x, dim, keepdim); ViperBench/argmax/pytorch_impl.py:4-8."""
    x = _host(input_tensor)
    if dim is None:
        shape = tuple(x.shape)
        xc, m, n, k = x.reshape(-1).contiguous(), 1, x.numel(), 1
        os_ = tuple(1 for _ in shape) if keepdim else ()
    else:
        xc, m, n, k, dims, shape = _mnk(x, dim)
        os_ = _oshape(shape, dims, keepdim, x.dim() == 0)
    i = torch.empty(os_, dtype=torch.int64)
    lib().oracle_max_reduction(xc.data_ptr(), None, i.data_ptr(), m, n, k, _code(x))
    return i


def kernel_ff(x, w1, w3, rms_w):
    """ViperBench/linear_activation/pytorch_impl.py:5-54: fp16 [batch, seq, n_out]."""
    x, w1, w3, rms_w = (_host(t.half() if t.dtype != torch.float16 else t) for t in (x, w1, w3, rms_w))
    b, s, k = x.shape
    n = w1.shape[0]
    out = torch.empty((b, s, n), dtype=torch.float16)
    lib().oracle_kernel_ff(x.data_ptr(), w1.data_ptr(), w3.data_ptr(), rms_w.data_ptr(), out.data_ptr(), b * s, n, k)
    return out
