"""The C-ABI library: it loads, exports every entry point that
include/dslpg_b200.h declares, and rejects bad arguments before launching
anything (these calls return before any CUDA API call, so they run on CPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from dslperfgap_b200 import _lib, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "dslpg_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DSLPG_API\s+[\w\s\*]+?\b(dslpg_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_the_family():
    names = declared_symbols()
    for op in ["layer_norm", "rms_norm", "softmax", "log_softmax", "logsumexp", "cross_entropy"]:
        assert f"dslpg_{op}_fwd" in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_python_binding_covers_header():
    bound = set(_lib.SIGNATURES) | {"dslpg_error_string", "dslpg_take_wait_timeouts"}
    assert set(declared_symbols()) <= bound


def test_kernel_path_is_per_thread(lib):
    """A shape forced on one host thread does not reach another thread's calls."""
    import threading
    seen = {}
    lib.dslpg_set_kernel_path(3)
    try:
        def other():
            seen["before"] = lib.dslpg_get_kernel_path()
            lib.dslpg_set_kernel_path(1)
            seen["after"] = lib.dslpg_get_kernel_path()
        t = threading.Thread(target=other)
        t.start()
        t.join()
        assert seen == {"before": 0, "after": 1}
        assert lib.dslpg_get_kernel_path() == 3
    finally:
        lib.dslpg_set_kernel_path(0)


def test_kernel_path_validation(lib):
    assert lib.dslpg_set_kernel_path(9) == -5
    assert lib.dslpg_set_kernel_path(-1) == -5
    for code in range(5):
        assert lib.dslpg_set_kernel_path(code) == 0
    assert lib.dslpg_set_kernel_path(0) == 0


def test_version(lib):
    assert lib.dslpg_version() >= 1


@pytest.mark.parametrize("code,text", [(-1, "NULL"), (-2, "shape"), (-3, "dtype"), (-4, "eps"), (0, "success")])
def test_error_strings(lib, code, text):
    assert text in lib.dslpg_error_string(code).decode()


def test_argument_errors_return_before_launch(lib):
    # null pointers
    assert lib.dslpg_softmax_fwd(None, None, 4, 4, 0, None) == -1
    assert lib.dslpg_layer_norm_fwd(8, None, None, 8, 4, 4, 0, 0, 1e-5, None) == -1
    assert lib.dslpg_cross_entropy_fwd(8, None, 8, 8, 8, 2, 2, 2, 0, 4, 0, 1, 0, -100, 2, 0, 2, 0, 0, None) == -1
    # dtype codes
    assert lib.dslpg_softmax_fwd(8, 8, 4, 4, 7, None) == -3
    assert lib.dslpg_rms_norm_fwd(8, 8, 8, 4, 4, 0, 9, 1e-5, None) == -3
    assert lib.dslpg_log_softmax_fwd(8, 8, 4, 4, 1, 0, 3, None) == -3
    assert lib.dslpg_cross_entropy_fwd(8, 8, 8, 8, 8, 2, 2, 2, 0, 0, 0, 1, 0, -100, 2, 0, 2, 0, 0, None) == -3
    # shapes
    assert lib.dslpg_softmax_fwd(8, 8, -1, 4, 0, None) == -2
    assert lib.dslpg_log_softmax_fwd(8, 8, 4, 4, 0, 0, 0, None) == -2
    assert lib.dslpg_cross_entropy_fwd(8, 8, 8, 8, 8, 2, 4, 2, 0, 4, 0, 1, 0, -100, 2, 0, 2, 0, 0, None) == -2
    assert lib.dslpg_cross_entropy_fwd(8, 8, 8, 8, 8, 2, 4, 4, 0, 4, 0, 1, 0, -100, 2, 0, 0, 0, 0, None) == -2
    # eps
    assert lib.dslpg_layer_norm_fwd(8, 8, None, 8, 4, 4, 0, 0, float("nan"), None) == -4
    assert lib.dslpg_rms_norm_fwd(8, 8, 8, 4, 4, 0, 0, -1.0, None) == -4
    # host-buffer rms_norm: nulls, dtype, eps, a missing workspace, the workspace size query
    assert lib.dslpg_rms_norm_fwd_host(None, 8, 8, 4, 4, 2, 2, 1e-6, 8, 1 << 30, None) == -1
    assert lib.dslpg_rms_norm_fwd_host(8, 8, 8, 4, 4, 2, 5, 1e-6, 8, 1 << 30, None) == -3
    assert lib.dslpg_rms_norm_fwd_host(8, 8, 8, 4, 4, 2, 2, float("inf"), 8, 1 << 30, None) == -4
    assert lib.dslpg_rms_norm_fwd_host(8, 8, 8, 4, 4, 2, 2, 1e-6, None, 1 << 30, None) == -1
    need = ctypes.c_int64(-1)
    assert lib.dslpg_rms_norm_fwd_host_workspace_bytes(16384, 8192, 2, ctypes.byref(need)) == 0
    assert need.value == 4 * 2 * (16 << 20)  # 4 slots of a 16 MiB input chunk and its output chunk
    assert lib.dslpg_rms_norm_fwd_host_workspace_bytes(3, 5, 0, ctypes.byref(need)) == 0 and need.value == 4 * 2 * 256
    assert lib.dslpg_rms_norm_fwd_host(8, 8, 8, 4, 4, 2, 2, 1e-6, 256, need.value - 1, None) == -5  # too small
    # host-buffer layer_norm: the same checks (bias may be NULL), the same workspace rule
    assert lib.dslpg_layer_norm_fwd_host(None, 8, None, 8, 4, 4, 2, 2, 1e-5, 8, 1 << 30, None) == -1
    assert lib.dslpg_layer_norm_fwd_host(8, 8, None, 8, 4, 4, 2, 5, 1e-5, 8, 1 << 30, None) == -3
    assert lib.dslpg_layer_norm_fwd_host(8, 8, None, 8, 4, 4, 2, 2, float("nan"), 8, 1 << 30, None) == -4
    assert lib.dslpg_layer_norm_fwd_host(8, 8, 8, 8, 4, 4, 2, 2, 1e-5, None, 1 << 30, None) == -1
    need2 = ctypes.c_int64(-1)
    assert lib.dslpg_layer_norm_fwd_host_workspace_bytes(131072, 8192, 2, ctypes.byref(need2)) == 0
    assert need2.value == 4 * 2 * (16 << 20)
    assert lib.dslpg_layer_norm_fwd_host(8, 8, 8, 8, 4, 4, 2, 2, 1e-5, 256, need.value - 1, None) == -5
    # kernel_ff: K % 8, the workspace size, and the static-scratch variant's limit (checked before M * K is formed)
    assert lib.dslpg_kernel_ff(8, 8, 8, 8, 8, 4, 4, 12, 256, 1 << 20, None) == -2
    assert lib.dslpg_kernel_ff(8, 8, 8, 8, 8, 4, 4, 16, 256, 1, None) == -5
    assert lib.dslpg_kernel_ff_static(8, 8, 8, 8, 8, 1 << 30, 4, 1 << 30, None) == -6
    assert lib.dslpg_kernel_ff_static(8, 8, 8, 8, 8, 2056, 4, 4096, None) == -6
    # empty problems are a no-op success
    assert lib.dslpg_softmax_fwd(8, 8, 0, 4, 0, None) == 0
    assert lib.dslpg_logsumexp_fwd(8, 8, 0, 4, 0, None) == 0


def test_fast_binding_matches_ctypes_signatures(lib):
    """The METH_FASTCALL extension takes each entry point's arguments in the
    ctypes order: all-NULL calls come back from the C layer as
    DSLPG_ERR_NULL_POINTER (so arity and argument kinds agree)."""
    fast = _lib.fast_module()
    assert fast is not None, "the _dslpg_fast extension is not built"
    names = [n for n in dir(fast) if n.startswith("dslpg_")]
    assert len(names) >= 11
    for name in names:
        args = [0.0 if t is ctypes.c_float else 0 for t in _lib.SIGNATURES[name]]
        assert getattr(fast, name)(*args) == -1, name
        with pytest.raises(TypeError):
            getattr(fast, name)(*args[:-1])


def test_torch_fast_path_loads_and_declines_cpu_tensors(lib):
    """The C++ fast path (_dslpg_torch) is built and loads; for what it does
    not take (host tensors, dim lists, other eps) it returns None so that the
    Python wrapper raises exactly as the reference-shaped API says."""
    import torch
    mod = _lib.torch_ops()
    assert mod is not None, "the _dslpg_torch extension is not built"
    x, w = torch.randn(4, 8), torch.ones(8)
    assert mod.layer_norm(x, w, None, 1e-5) is None
    assert mod.rms_norm(x, (8,), w, 1e-5) is None
    assert mod.softmax(x) is None and mod.logsumexp(x) is None
    assert mod.log_softmax(x, -1, None) is None
    assert mod.mean_reduction(x, [0, 1], False, None) is None
    assert mod.max_reduction("not a tensor", 1, False) is None
    assert mod.argmax(x, None, False) is None
    assert mod.cross_entropy_fwd(x, torch.zeros(4, dtype=torch.long), 0.0, 1.0, 0.0, -100, 8, 0, 8, False,
                                 False) is None
