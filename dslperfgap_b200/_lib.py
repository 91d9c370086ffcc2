"""ctypes binding of the C ABI in ``include/dslpg_b200.h``.

This is the only place Python touches the native library. There is no CPU
implementation behind it: if ``lib/libdslpg_b200.so`` is missing, or a tensor
is not on a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

import os

# DSLPG_LIB may name another build of the same library (e.g. one compiled
# with different cache hints, for a measurement).
LIB_PATH = Path(os.environ.get("DSLPG_LIB") or Path(__file__).resolve().parent / "lib" / "libdslpg_b200.so")

F32, F16, BF16, I32, I64 = 0, 1, 2, 3, 4
FLOAT_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
LABEL_CODES = {torch.int32: I32, torch.int64: I64}

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_f32 = ctypes.c_float
_vp = ctypes.c_void_p

# name -> argtypes (every entry point returns int)
SIGNATURES = {
    "dslpg_layer_norm_fwd": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_f32, _vp],
    "dslpg_rms_norm_fwd": [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_f32, _vp],
    "dslpg_softmax_fwd": [_vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "dslpg_log_softmax_fwd": [_vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "dslpg_logsumexp_fwd": [_vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "dslpg_cross_entropy_fwd": [
        _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
        _c_f32, _c_f32, _c_f32, _c_i64, _c_f32, _c_i64, _c_i64, _c_int, _c_int, _vp,
    ],
    "dslpg_cross_entropy_bwd": [
        _vp, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
        _c_f32, _c_f32, _c_f32, _c_i64, _c_f32, _c_i64, _c_int, _vp,
    ],
    "dslpg_cross_entropy_fwd_bwd": [_vp, _vp, _vp, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                    _c_i64, _c_int, _c_int, _c_f32, _c_f32, _c_f32, _c_i64, _c_f32, _c_i64, _c_int,
                                    _vp],
    "dslpg_mean_reduction": [_vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "dslpg_max_reduction": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp],
    "dslpg_argmax": [_vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp],
    "dslpg_kernel_ff_workspace_bytes": [_c_i64, _c_i64, _vp],
    "dslpg_kernel_ff": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_i64, _vp],
    "dslpg_rms_norm_fwd_host_workspace_bytes": [_c_i64, _c_i64, _c_int, _vp],
    "dslpg_rms_norm_fwd_host": [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_f32, _vp, _c_i64, _vp],
    "dslpg_layer_norm_fwd_host_workspace_bytes": [_c_i64, _c_i64, _c_int, _vp],
    "dslpg_layer_norm_fwd_host": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_f32, _vp, _c_i64, _vp],
    "dslpg_kernel_ff_static": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp],
    "dslpg_version": [],
    "dslpg_set_kernel_path": [_c_int],
    "dslpg_get_kernel_path": [],
}

PATHS = {"auto": 0, "resident": 1, "tma": 2, "stream": 3, "cluster": 4}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the native library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"dslperfgap_b200: CUDA library {LIB_PATH} is not built; run "
                    "`python -m dslperfgap_b200.build` (there is no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            lib.dslpg_take_wait_timeouts.argtypes = []
            lib.dslpg_take_wait_timeouts.restype = ctypes.c_uint
            lib.dslpg_error_string.argtypes = [ctypes.c_int]
            lib.dslpg_error_string.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().dslpg_error_string(rc).decode()
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def float_code(t: torch.Tensor, what: str) -> int:
    code = FLOAT_CODES.get(t.dtype)
    if code is None:
        raise TypeError(f"{what}: unsupported dtype {t.dtype}; expected float32, float16 or bfloat16")
    return code


def require_cuda(*tensors, what: str) -> torch.device:
    """All tensors must live on the same CUDA device; return it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{what}: expected a torch.Tensor, got {type(t).__name__}")
        if t.device.type != "cuda":
            raise ValueError(f"{what}: tensors must be on a CUDA device (got {t.device}); "
                             "this backend has no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: tensors are on different devices ({dev} and {t.device})")
    return dev


def stream_handle(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


_get_device = torch._C._cuda_getDevice
_raw_stream = torch._C._cuda_getCurrentRawStream


_fast = None  # the _dslpg_fast extension module, or False when not used


def fast_module():
    """The METH_FASTCALL binding of the per-call entry points (built next to the
    library), or None. Not used when DSLPG_LIB selects another library build:
    the extension is linked to the default one."""
    global _fast
    if _fast is None:
        load()  # the library itself first, from LIB_PATH
        mod = False
        if not os.environ.get("DSLPG_LIB"):
            import importlib.machinery
            import importlib.util
            from .build import FAST_PATH
            if FAST_PATH.exists():
                loader = importlib.machinery.ExtensionFileLoader("_dslpg_fast", str(FAST_PATH))
                spec = importlib.util.spec_from_file_location("_dslpg_fast", str(FAST_PATH), loader=loader)
                mod = importlib.util.module_from_spec(spec)
                loader.exec_module(mod)
        _fast = mod
    return _fast or None


_torch_ops = None  # the _dslpg_torch extension module, or False when not used


def torch_ops():
    """The C++ fast path of the wrappers (csrc/torch_ops.cpp, built next to the
    library), or None. Each of its functions returns None for a case it does
    not take, and the Python wrapper then does the work. Not used when
    DSLPG_LIB selects another library build (the extension is linked to the
    default one)."""
    global _torch_ops
    if _torch_ops is None:
        load()
        mod = False
        if not os.environ.get("DSLPG_LIB"):
            import importlib.machinery
            import importlib.util
            from .build import TORCH_OPS_PATH
            if TORCH_OPS_PATH.exists():
                loader = importlib.machinery.ExtensionFileLoader("_dslpg_torch", str(TORCH_OPS_PATH))
                spec = importlib.util.spec_from_file_location("_dslpg_torch", str(TORCH_OPS_PATH), loader=loader)
                mod = importlib.util.module_from_spec(spec)
                loader.exec_module(mod)
        _torch_ops = mod
    return _torch_ops or None


def fast_op(name: str):
    """Callable taking the wrapper's arguments and returning its result, or
    None when the C++ fast path does not take the case (or is not built)."""
    state = {}

    def call(*args):
        fn = state.get("fn")
        if fn is None:
            mod = torch_ops()
            fn = state["fn"] = getattr(mod, name) if mod is not None else (lambda *a: None)
        return fn(*args)
    return call


def launch(dev: torch.device, name: str, *args) -> None:
    """Call entry point `name`(*args, stream) on `dev` with that device's current
    stream appended; raise RuntimeError on a non-zero return. The current device
    is switched (and restored) only when it is not `dev` already. Goes through
    the _dslpg_fast extension when it has the entry point, else ctypes."""
    fast = _fast if _fast is not None else fast_module()
    fn = getattr(fast, name, None) if fast else None
    if fn is None:
        fn = getattr(_lib if _lib is not None else load(), name)
    idx = dev.index if dev.index is not None else _get_device()
    if _get_device() == idx:
        rc = fn(*args, _raw_stream(idx))
    else:
        with torch.cuda.device(idx):
            rc = fn(*args, _raw_stream(idx))
    if rc != 0:
        check(rc, name)


class kernel_path:
    """Context manager forcing one kernel shape ("auto", "resident", "tma",
    "stream", "cluster") for the calls this host thread makes inside it (the
    selection is per thread; for tests and benchmarks)."""

    def __init__(self, name: str):
        self.code = PATHS[name]

    def __enter__(self):
        check(load().dslpg_set_kernel_path(self.code), "dslpg_set_kernel_path")
        return self

    def __exit__(self, *exc):
        load().dslpg_set_kernel_path(0)
        return False


def run_host_pipeline(name: str, x, out, dev: torch.device, m: int, n: int, xc: int, ptrs_before: tuple,
                      ptrs_after: tuple) -> None:
    """Shared tail of the host-buffer entry points (``dslpg_<op>_fwd_host``):
    query the chunk workspace, allocate it on `dev` with torch's caching
    allocator, launch `name`(x, *ptrs_before, out, m, n, xc, *ptrs_after,
    workspace, bytes, stream) on `dev`'s current stream and wait for that
    stream, so `out` is ready to read when this returns."""
    lib = load()
    need = ctypes.c_int64(0)
    check(getattr(lib, name + "_workspace_bytes")(m, n, xc, ctypes.byref(need)), name + "_workspace_bytes")
    with torch.cuda.device(dev):
        ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        rc = getattr(lib, name)(x.data_ptr(), *ptrs_before, out.data_ptr(), m, n, xc, *ptrs_after, ws.data_ptr(),
                                need.value, stream.cuda_stream)
        check(rc, name)
        stream.synchronize()


def take_wait_timeouts() -> int:
    """Device-side pipeline waits that ran out of time since the last call."""
    return int(load().dslpg_take_wait_timeouts())
