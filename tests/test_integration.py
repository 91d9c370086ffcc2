"""The drop-in stubs (integration/ViperBench/<kernel>/cuda_impl.py) as the
reference's drivers load them: every stub loads by file path the way
experiments/_harness.py:152-167 does, exposes the reference's function names,
and each function's signature equals the reference pytorch_impl's (recorded
from the reference in tests/golden/reference_signatures.json). Where the
reference checkout is present, its own `_harness.load_impl` loads the stubs
too, and the signatures are compared with the live pytorch_impl files."""
import importlib.util
import json
import os
from pathlib import Path

import pytest

import viperbench_loader as VL

SIGS = json.loads((Path(__file__).resolve().parent / "golden" / "reference_signatures.json").read_text())
REF = Path(os.environ.get("DSLPG_REFERENCE", "/root/reference"))


@pytest.mark.parametrize("kernel", sorted(VL.FUNCTIONS))
def test_stub_loads_and_matches_reference_signature(kernel):
    mod = VL.load_impl(VL.STUBS, kernel, "cuda")
    import dslperfgap_b200 as B
    for fn in VL.FUNCTIONS[kernel]:
        f = getattr(mod, fn)
        assert f is getattr(B, fn), fn
        ref = SIGS[kernel][fn]
        ref_plain = ref.split(" -> ")[0].replace(": torch.Tensor", "")
        assert VL.plain_signature(f) == ref_plain, (fn, VL.plain_signature(f), ref)


def test_every_reference_kernel_of_the_family_has_a_stub():
    assert sorted(p.name for p in VL.STUBS.iterdir() if (p / "cuda_impl.py").exists()) == sorted(VL.FUNCTIONS)


def _reference_harness():
    path = REF / "experiments" / "_harness.py"
    if not path.exists():
        pytest.skip("reference checkout not present")
    spec = importlib.util.spec_from_file_location("dslpg_ref_harness", str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("kernel", sorted(VL.FUNCTIONS))
def test_reference_harness_loads_stub(kernel):
    """experiments/_harness.load_impl(kernel, "cuda") itself, pointed at the
    stub tree (its VIPER_DIR), and its pytorch_impl loaded the same way."""
    h = _reference_harness()
    viper = h.VIPER_DIR
    try:
        h.VIPER_DIR = VL.STUBS
        cuda = h.load_impl(kernel, "cuda")
    finally:
        h.VIPER_DIR = viper
    ref = h.load_impl(kernel, "pytorch")
    for fn in VL.FUNCTIONS[kernel]:
        assert VL.plain_signature(getattr(cuda, fn)) == VL.plain_signature(getattr(ref, fn)), fn


def test_reference_caller_patch_applies(tmp_path):
    """integration/reference_callers.patch (cuda in run_one_kernel.py's
    choices and ncu_counters.sh's kernel filter, a cuda row in benchmark.py,
    VIPER_IMPL=cuda in layer_norm/test.py) applies to the reference as is."""
    import shutil
    import subprocess
    files = ["experiments/run_one_kernel.py", "experiments/ncu_counters.sh", "ViperBench/benchmark.py",
             "ViperBench/layer_norm/test.py"]
    if not all((REF / f).exists() for f in files):
        pytest.skip("reference checkout not present")
    for f in files:
        (tmp_path / f).parent.mkdir(parents=True, exist_ok=True)
        shutil.copy(REF / f, tmp_path / f)
    patch = VL.REPO / "integration" / "reference_callers.patch"
    res = subprocess.run(["patch", "-p1", "-i", str(patch)], cwd=tmp_path, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert '"cuda"]' in (tmp_path / "experiments/run_one_kernel.py").read_text()
    sh = (tmp_path / "experiments/ncu_counters.sh").read_text()
    assert 'cuda)' in sh and "--clock-control none" in sh
    compile((tmp_path / "ViperBench/benchmark.py").read_text(), "benchmark.py", "exec")


def test_ncu_summary_consolidation_schema(tmp_path):
    """The package's ncu collection writes the reference's ncu_summary.csv
    columns (experiments/consolidate_ncu.py:84-90) from ncu --csv logs."""
    import csv
    from dslperfgap_b200 import ncu_counters as NC
    log = tmp_path / "rms_norm_bf16_cuda_r16384_l2dram.csv"
    log.write_text('==PROF== Connected to process 1\n'
                   '"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"\n'
                   '"0","void dslpg::resident_kernel<1>","dram__bytes_read.sum","byte","268460544"\n'
                   '"0","void dslpg::resident_kernel<1>","gpu__time_duration.sum","ns","84032"\n'
                   '"0","void dslpg::resident_kernel<1>","not_a_kept_metric","","1"\n')
    dst = NC.consolidate(tmp_path)
    rows = list(csv.DictReader(open(dst)))
    assert list(rows[0]) == ["target", "kernel", "set", "rc", "metric", "label", "value", "unit"]
    assert len(rows) == 2 and rows[0]["target"] == "rms_norm_bf16_cuda_r16384" and rows[0]["set"] == "l2dram"
    assert NC.target_rows("logsumexp_bf16") == (512 << 20) // (128256 * 2) and NC.target_rows("layer_norm_fp32") == 4096
