"""Parity rules shared by the tests (the tolerance is written here, once).

* fp32 outputs: |out - ref| <= 1e-5 + 1e-5 * |ref| (atol = rtol = 1e-5).
* fp16 / bf16 outputs: within 1 ulp of the output dtype at the fp32-computed
  reference value; normalised outputs (layer_norm, rms_norm) may also pass
  with |out - ref| <= 2e-2.
* NaN and +/-inf must appear at exactly the reference's positions.
* `abs_slack` (optional, per element or scalar) widens the bound where the
  reference itself subtracts nearly equal fp32 terms (cross_entropy_bwd with
  smoothing: p - smoothing/total_classes): there any fp32 implementation
  differs by the fp32 rounding of the terms, 2^-21 of their magnitude.
The reference's own check (ViperBench/test_utils.py:11-35, loose=True: fp32
2e-5, fp16 2e-3, bf16 2e-2, atol = rtol) is `reference_allclose`.
"""
from __future__ import annotations

import torch

FP32_TOL = 1e-5
# kernel_ff (a K-long fp32-accumulated dot product before the gate): outputs may
# also differ by this fraction of the tensor's largest magnitude, which covers
# summation-order differences where the dot product cancels. (The tests use the
# per-element bound `gemm_slack` below; this global form is kept for the smoke.)
GEMM_SLACK = 2.0 ** -14
# per-element kernel_ff slack: this fraction of sum_k |xs_k * w_k| (the
# condition of each fp32 dot product), carried through the a_norm scale and the
# SiLU gate to the output
GEMM_REL = 2.0 ** -17
NORM_ATOL_16 = 2e-2
_P = {torch.float16: (11, -14), torch.bfloat16: (8, -126), torch.float32: (24, -126)}
_REF_TOL = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 1e-2}


def dtype_ulp(ref: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of `dtype` numbers at |ref| (ref as float64)."""
    p, emin = _P[dtype]
    a = ref.double().abs()
    e = torch.floor(torch.log2(torch.where(a > 0, a, torch.ones_like(a))))
    e = torch.clamp(e, min=emin)
    e = torch.where(a > 0, e, torch.full_like(e, emin))
    return torch.pow(2.0, e - (p - 1))


def compare(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype, normalised: bool = False,
            chunk: int = 1 << 24, abs_slack=None):
    """Return (ok, message) for the parity rule above (checked in chunks)."""
    out = out.detach().reshape(-1)
    ref = ref.detach().reshape(-1)
    if out.shape != ref.shape:
        return False, f"shape {tuple(out.shape)} != {tuple(ref.shape)}"
    if not dtype.is_floating_point:  # indices: exact
        eq = torch.equal(out.cpu(), ref.cpu().to(out.dtype))
        return eq, "exact" if eq else f"{int((out.cpu() != ref.cpu()).sum())} indices differ"
    worst = 0.0
    for s in range(0, max(out.numel(), 1), chunk):
        sl = None
        if abs_slack is not None:
            sl = (abs_slack.reshape(-1)[s:s + chunk].cpu().double() if isinstance(abs_slack, torch.Tensor)
                  else float(abs_slack))
        ok, msg, w = _compare_chunk(out[s:s + chunk].cpu().double(), ref[s:s + chunk].cpu().double(), dtype,
                                    normalised, s, sl)
        if not ok:
            return False, msg
        worst = max(worst, w)
    if dtype == torch.float32:
        return True, f"max|d|={worst:.3g}"
    return True, f"max ulps={worst:.3f}"


def _compare_chunk(out, ref, dtype, normalised, offset, slack=None):
    on, rn = torch.isnan(out), torch.isnan(ref)
    if not torch.equal(on, rn):
        return False, f"NaN pattern differs ({int(on.sum())} vs {int(rn.sum())} NaNs)", 0.0
    oi, ri = torch.isinf(out), torch.isinf(ref)
    if not torch.equal(oi, ri) or not torch.equal(out[oi], ref[ri]):
        return False, "inf pattern differs", 0.0
    fin = ~(rn | ri)
    o, r = out[fin], ref[fin]
    if isinstance(slack, torch.Tensor):
        slack = slack[fin]
    if o.numel() == 0:
        return True, "", 0.0
    d = (o - r).abs()
    if dtype == torch.float32:
        bound = FP32_TOL + FP32_TOL * r.abs()
        if slack is not None:
            bound = bound + slack
        bad = d > bound
        what = "atol=rtol=1e-5"
        worst = d.max().item()
    else:
        u = dtype_ulp(r, dtype)
        bound = u * (1 + 1e-9)
        if normalised:
            bound = torch.maximum(bound, torch.full_like(bound, NORM_ATOL_16))
        if slack is not None:
            bound = bound + slack
        bad = d > bound
        what = "1 ulp" + (" or 2e-2" if normalised else "")
        worst = (d / u).max().item()
    if bad.any():
        i = int(torch.nonzero(bad)[0])
        return False, (f"{int(bad.sum())}/{d.numel()} values outside {what} (chunk at {offset}); first: "
                       f"out={o[i].item()!r} ref={r[i].item()!r}; max|d|={d.max().item():.3g}"), worst
    return True, "", worst


def gemm_slack(x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor, rms_w: torch.Tensor) -> torch.Tensor:
    """Per-element extra bound for kernel_ff outputs [M, N] (float64, CPU).

    Each output is silu(g) * u with g = a_norm * xs.w1[n], u = a_norm * xs.w3[n]
    and xs = fp16(x * rms_w). Reordering a fp32 sum of K products changes it by
    a multiple of the unit roundoff times sum_k |xs_k w_k| (S1, S3), whatever
    the size of the sum itself; through the gate that is
        GEMM_REL * a_norm * (|silu'(g) u| S1 + |silu(g)| S3).
    Elements whose dot products cancel get a bound scaled to their own
    condition, not to the tensor's largest value."""
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    K = x.shape[-1]
    xf = x.reshape(-1, K).to(dev).float()
    an = torch.rsqrt(xf.double().pow(2).mean(-1) + 1e-6).float()
    xs = (xf.half() * rms_w.to(dev).half().reshape(K)).float()
    w1f, w3f = w1.to(dev).float(), w3.to(dev).float()
    g = (xs @ w1f.t()) * an[:, None]
    u = (xs @ w3f.t()) * an[:, None]
    s1 = (xs.abs() @ w1f.abs().t()) * an[:, None]
    s3 = (xs.abs() @ w3f.abs().t()) * an[:, None]
    sg = torch.sigmoid(g)
    dsilu = sg * (1 + g * (1 - sg))
    slack = GEMM_REL * ((dsilu * u).abs() * s1 + (g * sg).abs() * s3)
    return slack.cpu().double()


def ulp_histogram(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype, edges=(0.5, 1, 2, 4, 8, 16)) -> dict:
    """Counts of |out - ref| in units of `dtype`'s spacing at ref, binned at
    `edges` (finite values only)."""
    o, r = out.detach().reshape(-1).cpu().double(), ref.detach().reshape(-1).cpu().double()
    fin = torch.isfinite(r)
    d = ((o - r).abs() / dtype_ulp(r, dtype))[fin]
    hist, lo = {}, 0.0
    for e in edges:
        hist[f"({lo},{e}]" if lo else f"[0,{e}]"] = int(((d > lo) & (d <= e)).sum()) + (int((d == 0).sum()) if not lo else 0)
        lo = e
    hist[f">{lo}"] = int((d > lo).sum())
    hist["max_ulps"] = float(d.max()) if d.numel() else 0.0
    return hist


def reference_allclose(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype) -> bool:
    """ViperBench/test_utils.py:21-35 with loose=True, NaN positions compared equal."""
    if not dtype.is_floating_point:
        return torch.equal(out.cpu(), ref.cpu())
    tol = 2 * _REF_TOL.get(dtype, 1e-5)
    return bool(torch.allclose(ref.detach().cpu().float(), out.detach().cpu().float(),
                               atol=tol, rtol=tol, equal_nan=True))


def out_dtype(op: str, args, kwargs) -> torch.dtype:
    if op == "log_softmax" and kwargs.get("dtype"):
        return getattr(torch, kwargs["dtype"])
    if op == "cross_entropy":
        return torch.float32
    if op == "cross_entropy_bwd":
        return args[1].dtype
    return args[0].dtype


NORMALISED = {"layer_norm", "rms_norm"}


def resolve_kwargs(op: str, kwargs: dict) -> dict:
    kw = dict(kwargs)
    if op == "log_softmax" and "dtype" in kw:
        kw["dtype"] = getattr(torch, kw["dtype"])
    return kw
