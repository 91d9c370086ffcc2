"""bench.py's host-side pieces that need no GPU: the reference's eager
cross-entropy baseline against the reference's own golden outputs, the
profile.csv rows (and the reference's compute_elib.py reading them, where the
checkout is present), and the timing reductions."""
import csv
import importlib.util
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import golden_cases

ROOT = Path(__file__).resolve().parent.parent
REF = Path(os.environ.get("DSLPG_REFERENCE", "/root/reference"))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("dslpg_bench", str(ROOT / "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CE = [c for c in golden_cases.load("cross_entropy") if not c["kwargs"]["HAS_SMOOTHING"] and not c["kwargs"]["SPLIT"]]


@pytest.mark.parametrize("case", CE, ids=[c["name"] for c in CE])
def test_eager_cross_entropy_baseline_is_the_reference(bench, case):
    logits, labels = case["args"]
    kw = case["kwargs"]
    out = bench.eager_cross_entropy_fwd(logits, labels, kw["logit_scale"], kw["lse_square_scale"], kw["ignored_index"], kw["class_start_idx"],
                                        kw["BLOCK_SIZE"])
    r, c = logits.shape
    nv = ((c + kw["BLOCK_SIZE"] - 1) // kw["BLOCK_SIZE"]) * r
    for o, ref in zip(out, case["ref_native"]):
        assert torch.allclose(o.reshape(-1)[:nv], ref.reshape(-1), rtol=1e-6, atol=1e-6, equal_nan=True)


def test_profile_csv_schema_and_compute_elib(bench, tmp_path):
    shapes = {"cases": {
        "layer_norm x:(8192,8192) bf16": {"size": "large", "ms": 0.07, "peak_memory_mb": 384.0,
                                           "pytorch_impl_ms": 0.14, "pytorch_impl_peak_memory_mb": 384.0},
        "softmax x:(512,1024) fp16": {"size": "small", "ms": 0.02, "peak_memory_mb": 3.0,
                                      "pytorch_impl_ms": 0.01, "pytorch_impl_peak_memory_mb": 3.0}}}
    path = tmp_path / "profile.csv"
    bench.write_profile_csv(shapes, path)
    rows = list(csv.DictReader(open(path)))
    assert list(rows[0]) == ["kernel", "size", "impl", "input_desc", "latency_ms", "peak_memory_mb"]
    assert {(r["kernel"], r["size"], r["impl"]) for r in rows} == {
        ("layer_norm", "large", "pytorch"), ("layer_norm", "large", "cuda"),
        ("softmax", "small", "pytorch"), ("softmax", "small", "cuda")}
    script = REF / "experiments" / "compute_elib.py"
    if not script.exists():
        pytest.skip("reference checkout not present")
    out = tmp_path / "elib.csv"
    res = subprocess.run([sys.executable, str(script), str(path), "-o", str(out)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    elib = {(r["kernel"], r["size"], r["impl"]): float(r["elib_percent"]) for r in csv.DictReader(open(out))}
    assert elib[("layer_norm", "large", "cuda")] == pytest.approx(200.0)
    assert elib[("softmax", "small", "cuda")] == pytest.approx(50.0)
