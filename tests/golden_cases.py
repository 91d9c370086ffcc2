"""Loader for the committed golden fixtures (tests/golden/golden_<op>.pt)."""
from __future__ import annotations

from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
OPS = ["layer_norm", "rms_norm", "softmax", "log_softmax", "logsumexp", "cross_entropy", "cross_entropy_bwd",
       "mean_reduction", "max_reduction", "argmax", "linear_activation"]
_cache: dict = {}


def load(op: str) -> list[dict]:
    if op not in _cache:
        _cache[op] = torch.load(GOLDEN / f"golden_{op}.pt", weights_only=True)["cases"]
    return _cache[op]


def all_cases():
    for op in OPS:
        for c in load(op):
            yield op, c


def ids():
    return [f"{op}-{c['name']}" for op, c in all_cases()]


FN_NAME = {"layer_norm": "layer_norm", "rms_norm": "rms_norm", "softmax": "softmax",
           "log_softmax": "log_softmax", "logsumexp": "logsumexp", "cross_entropy": "cross_entropy_fwd",
           "cross_entropy_bwd": "cross_entropy_bwd", "mean_reduction": "mean_reduction",
           "max_reduction": "max_reduction", "argmax": "argmax", "linear_activation": "kernel_ff"}


def run(fn, op: str, case: dict, device: str = "cpu"):
    """Call `fn` (an implementation of `op` with the reference signature) on the
    case's inputs moved to `device`; cross-entropy results are cut to the
    valid flat prefix, everything is returned on the CPU."""
    def mv(a):
        return a.to(device) if isinstance(a, torch.Tensor) else a
    args = [mv(a) for a in case["args"]]
    kw = dict(case["kwargs"])
    if op in ("log_softmax", "mean_reduction") and "dtype" in kw:
        kw["dtype"] = getattr(torch, kw["dtype"])
    out = fn(*args, **kw)
    if isinstance(out, tuple):
        out = tuple(o.cpu() for o in out)
    if op == "cross_entropy":
        r, c = case["args"][0].shape
        nb = (c + kw["BLOCK_SIZE"] - 1) // kw["BLOCK_SIZE"]
        return tuple(o.reshape(-1)[: nb * r].cpu() for o in out)
    return out if isinstance(out, tuple) else out.cpu()


def check_case(op: str, case: dict, out, parity) -> list[str]:
    """Compare an implementation's output with the fixture; return failures."""
    errs = []
    multi = isinstance(case["ref_native"], tuple)
    refs32 = case["ref_f32"] if multi else (case["ref_f32"],)
    natives = case["ref_native"] if multi else (case["ref_native"],)
    outs = out if multi else (out,)
    split = op == "cross_entropy" and case["kwargs"]["SPLIT"]
    for i, (o, r32, rn) in enumerate(zip(outs, refs32, natives)):
        if split and i == 2:  # z_loss is not stored under SPLIT (cross_entropy/test.py:40-44)
            continue
        dt = rn.dtype  # the reference's own output dtype
        if o.dtype != rn.dtype or tuple(o.shape) != tuple(rn.shape):
            errs.append(f"output {i}: dtype/shape {o.dtype}{tuple(o.shape)} != {rn.dtype}{tuple(rn.shape)}")
            continue
        slack = None
        if op == "linear_activation":  # K-long dot products: fp32 accumulation-order slack per element
            slack = parity.gemm_slack(*case["args"])
        ok, msg = parity.compare(o, r32, dt, normalised=op in parity.NORMALISED, abs_slack=slack)
        if not ok:
            errs.append(f"output {i} vs fp32 reference: {msg}")
        if not parity.reference_allclose(o, rn, dt):
            errs.append(f"output {i} fails the reference's own loose tolerance vs its {rn.dtype} output")
    return errs
