"""How the reference's drivers find a backend, restated for the tests.

`load_impl(viper_dir, kernel, impl)` follows experiments/_harness.py:152-167
(load ViperBench/<kernel>/<impl>_impl.py by file path after putting the
kernel's directory and ViperBench on sys.path); `default_compare` follows the
comparison of ViperBench/test_utils.py:21-46,197-205 (`compare_tensors` with
the dtype's tolerance, doubled when the kernel's test.py passes loose_tol, and
`compare_tuple_outputs` over tuples).
"""
from __future__ import annotations

import importlib.util
import inspect
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
STUBS = REPO / "integration" / "ViperBench"

FUNCTIONS = {
    "layer_norm": ["layer_norm"], "rms_norm": ["rms_norm"], "softmax": ["softmax"],
    "log_softmax": ["log_softmax"], "logsumexp": ["logsumexp"],
    "cross_entropy": ["cross_entropy_fwd", "cross_entropy_bwd"], "mean_reduction": ["mean_reduction"],
    "max_reduction": ["max_reduction"], "argmax": ["argmax"], "linear_activation": ["kernel_ff"],
}

_TOL = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 1e-2}


def load_impl(viper_dir: Path, kernel: str, impl: str):
    path = Path(viper_dir) / kernel / f"{impl}_impl.py"
    if not path.exists():
        raise FileNotFoundError(path)
    spec = importlib.util.spec_from_file_location(f"{kernel}_{impl}_impl", str(path))
    mod = importlib.util.module_from_spec(spec)
    for p in (str(Path(viper_dir) / kernel), str(viper_dir)):
        if p not in sys.path:
            sys.path.insert(0, p)
    spec.loader.exec_module(mod)
    return mod


def plain_signature(fn) -> str:
    """The signature without annotations (names, kinds and defaults only)."""
    sig = inspect.signature(fn)
    params = [p.replace(annotation=inspect.Parameter.empty) for p in sig.parameters.values()]
    return str(sig.replace(parameters=params, return_annotation=inspect.Signature.empty))


def compare_tensors(ref, test, dtype, loose=False):
    tol = _TOL.get(dtype, 1e-5) * (2 if loose else 1)
    ref_f, test_f = ref.float(), test.float()
    max_err = (ref_f - test_f).abs().max().item() if ref_f.numel() else 0.0
    return bool(torch.allclose(ref_f, test_f, atol=tol, rtol=tol)), max_err


def default_compare(ref_out, out, dtype, loose):
    if isinstance(ref_out, (tuple, list)):
        ok, worst = True, 0.0
        for r, o in zip(ref_out, out):
            if isinstance(r, torch.Tensor) and isinstance(o, torch.Tensor):
                p, e = compare_tensors(r, o, dtype, loose)
                ok, worst = ok and p, max(worst, e)
        return ok, worst
    return compare_tensors(ref_out, out, dtype, loose)
