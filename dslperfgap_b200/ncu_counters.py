"""Nsight Compute counters of this backend's kernels, in the reference's
collection and table format.

The reference collects four metric sets per (kernel, impl, size) target with
one ncu run each, isolating ONE launch inside an NVTX range "TARGET"
(experiments/ncu_counters.sh:173-213, :263-298, single-launch harness
experiments/run_one_kernel.py), and consolidates the per-set CSVs into
``ncu_summary.csv`` with columns target, kernel, set, rc, metric, label,
value, unit (experiments/consolidate_ncu.py:22-53,84-97). With
``integration/reference_callers.patch`` applied, that script profiles
``impl=cuda`` itself. This module does the same collection where the
reference checkout is absent (the GPU box):

    python -m dslperfgap_b200.ncu_counters collect OUT_DIR [--targets a,b] [--rows R]
    python -m dslperfgap_b200.ncu_counters consolidate OUT_DIR
    python -m dslperfgap_b200.ncu_counters run WORKLOAD [--rows R]   # the one-launch target

Every ncu run passes ``--clock-control none`` (the GPU's clocks are never
locked) and captures one launch of a ``dslpg::`` kernel. Targets are the
benchmark configurations (dslperfgap_b200.workloads), cut to their first
``--rows`` rows where the whole input would be more than 512 MiB, so a
multi-pass capture stays small.
"""
from __future__ import annotations

import argparse
import csv
import os
import shutil
import subprocess
import sys
from pathlib import Path

# The four metric sets of the reference's collection (Nsight Compute metric
# names; ncu_counters.sh:173-213): A loads, B registers/occupancy, C warp
# stalls (+ the WarpStateStats section), D L2/DRAM.
METRIC_SETS = {
    "A": ("loads", "", [
        "l1tex__t_sectors_pipe_lsu_mem_global_op_ld.sum",
        "l1tex__average_t_sectors_per_request_pipe_lsu_mem_global_op_ld.ratio",
        "smsp__sass_average_data_bytes_per_sector_mem_global_op_ld.pct",
        "sm__sass_inst_executed_op_global_ld.sum"]),
    "B": ("regs", "", [
        "launch__registers_per_thread", "launch__occupancy_limit_registers",
        "l1tex__t_bytes_pipe_lsu_mem_local_op_ld.sum", "l1tex__t_bytes_pipe_lsu_mem_local_op_st.sum",
        "sm__warps_active.avg.pct_of_peak_sustained_active"]),
    "C": ("stalls", "--section WarpStateStats", [
        "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
        "smsp__average_warps_issue_stalled_short_scoreboard_per_issue_active.ratio",
        "smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio",
        "smsp__average_warps_issue_stalled_membar_per_issue_active.ratio",
        "smsp__average_warps_issue_stalled_mio_throttle_per_issue_active.ratio"]),
    "D": ("l2dram", "", [
        "lts__t_sector_hit_rate.pct", "dram__bytes_read.sum",
        "dram__throughput.avg.pct_of_peak_sustained_elapsed", "gpu__time_duration.sum",
        # not in the reference's set D: the write side, for the roofline traffic
        "dram__bytes_write.sum"]),
}

# metric -> (label, root-cause tag) of the consolidated table (consolidate_ncu.py:22-53)
LABELS = {
    "l1tex__average_t_sectors_per_request_pipe_lsu_mem_global_op_ld.ratio": ("sectors/req (↑=less vectorized)", "RC1"),
    "smsp__sass_average_data_bytes_per_sector_mem_global_op_ld.pct": ("bytes/sector load eff %", "RC1"),
    "launch__registers_per_thread": ("regs/thread", "RC3"),
    "launch__occupancy_limit_registers": ("occ limit (reg) %", "RC3"),
    "l1tex__t_bytes_pipe_lsu_mem_local_op_ld.sum": ("local-ld bytes (spill)", "RC3"),
    "l1tex__t_bytes_pipe_lsu_mem_local_op_st.sum": ("local-st bytes (spill)", "RC3"),
    "sm__warps_active.avg.pct_of_peak_sustained_active": ("achieved occ %", "RC3"),
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio": ("stall long_scoreboard", "RC0"),
    "smsp__average_warps_issue_stalled_short_scoreboard_per_issue_active.ratio": ("stall short_scoreboard", "RC0"),
    "smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio": ("stall barrier (sync)", "RC0"),
    "smsp__average_warps_issue_stalled_membar_per_issue_active.ratio": ("stall membar", "RC0"),
    "smsp__average_warps_issue_stalled_mio_throttle_per_issue_active.ratio": ("stall mio_throttle", "RC0"),
    "lts__t_sector_hit_rate.pct": ("L2 hit %", "RC2b"),
    "dram__bytes_read.sum": ("DRAM read bytes", "RC2b"),
    "dram__bytes_write.sum": ("DRAM write bytes", "RC2b"),
    "dram__throughput.avg.pct_of_peak_sustained_elapsed": ("DRAM thru %", "RC2b"),
    "gpu__time_duration.sum": ("kernel time (ns)", "ref"),
}

# the row-reduction family's benchmark configurations (the a-rows), and the
# box-scale LayerNorm's per-GPU row block
DEFAULT_TARGETS = ["layer_norm_fp32", "rms_norm_bf16", "softmax_fp16", "log_softmax_fp16", "logsumexp_bf16",
                   "cross_entropy_bf16", "layer_norm_bf16_sharded"]
MAX_INPUT_BYTES = 512 << 20


def target_rows(name: str, rows: int = 0) -> int:
    from . import workloads
    cfg = workloads.CONFIGS[name]
    if rows:
        return min(rows, cfg.M)
    es = {"fp32": 4, "fp16": 2, "bf16": 2}[workloads.config_dict(cfg)["dtype"]]
    return max(1, min(cfg.M, MAX_INPUT_BYTES // (cfg.N * es)))


def run_target(name: str, rows: int = 0, warmup: int = 5, range_name: str = "TARGET") -> int:
    """The single-launch target (the role of experiments/run_one_kernel.py):
    warm the op up, then call it once inside the NVTX range `range_name`."""
    import torch
    from . import workloads
    r = target_rows(name, rows)
    wl = workloads.make(name, seed=0, device="cuda", rows=(0, r))
    fn = wl.cuda_fn
    for _ in range(warmup):
        fn(*wl.args, **wl.kwargs)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push(range_name)
    out = fn(*wl.args, **wl.kwargs)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    first = out[0] if isinstance(out, tuple) else out
    _ = float(first.reshape(-1)[0].item()) if first.numel() else 0.0
    print(f"[ncu_counters] {name} rows [0, {r}) of {wl.config.M}: 1 launch inside '{range_name}'")
    return 0


def ncu_path() -> str:
    for cand in (os.environ.get("NCU"), shutil.which("ncu"), "/usr/local/cuda/bin/ncu"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("ncu not found: set NCU")


def collect(out_dir: Path, targets, rows: int = 0) -> int:
    """One ncu run per (target, metric set), one captured launch each."""
    out_dir.mkdir(parents=True, exist_ok=True)
    fails = 0
    for name in targets:
        r = target_rows(name, rows)
        for letter, (tag, extra, metrics) in METRIC_SETS.items():
            out = out_dir / f"{name}_cuda_r{r}_{tag}.csv"
            # the demangled name carries the namespace: only this library's kernels match
            cmd = [ncu_path(), "--clock-control", "none", "--target-processes", "all", "--nvtx", "--nvtx-include",
                   "TARGET/", "--kernel-name-base", "demangled", "--kernel-name", "regex:dslpg::", "--launch-count",
                   "1", *extra.split(), "--metrics", ",".join(metrics), "--csv", "--log-file", str(out),
                   sys.executable, "-m", "dslperfgap_b200.ncu_counters", "run", name, "--rows", str(r)]
            print("[ncu_counters]", " ".join(cmd), flush=True)
            rc = subprocess.run(cmd).returncode
            if rc == 0 and not any(r.get("Metric Name") for r in _rows(out)):
                rc = -1  # ncu exited 0 but captured no kernel
            if rc != 0:
                print(f"[ncu_counters] set {letter} of {name} exited {rc}", flush=True)
                fails += 1
    return 1 if fails else 0


def _rows(path: Path):
    if not path.exists():  # ncu stopped before writing its log
        return []
    lines = [ln for ln in path.read_text().splitlines(True) if not ln.startswith("==")]
    return list(csv.DictReader(lines)) if lines else []


def consolidate(out_dir: Path) -> Path:
    """ncu_summary.csv in the reference's tidy schema, one row per metric."""
    tidy = []
    for path in sorted(out_dir.glob("*_cuda_r*_*.csv")):
        target, tag = path.stem.rsplit("_", 1)
        for row in _rows(path):
            metric = row.get("Metric Name", "")
            if metric not in LABELS:
                continue
            label, rc = LABELS[metric]
            tidy.append(dict(target=target, kernel=row.get("Kernel Name", "?"), set=tag, rc=rc, metric=metric,
                             label=label, value=row.get("Metric Value", ""), unit=row.get("Metric Unit", "")))
    dst = out_dir / "ncu_summary.csv"
    with open(dst, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["target", "kernel", "set", "rc", "metric", "label", "value", "unit"])
        w.writeheader()
        w.writerows(tidy)
    print(f"[ncu_counters] wrote {dst} ({len(tidy)} rows)")
    return dst


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("workload")
    r.add_argument("--rows", type=int, default=0)
    r.add_argument("--warmup", type=int, default=5)
    c = sub.add_parser("collect")
    c.add_argument("out_dir", type=Path)
    c.add_argument("--targets", default=",".join(DEFAULT_TARGETS))
    c.add_argument("--rows", type=int, default=0)
    s = sub.add_parser("consolidate")
    s.add_argument("out_dir", type=Path)
    a = ap.parse_args(argv)
    if a.cmd == "run":
        return run_target(a.workload, a.rows, a.warmup)
    if a.cmd == "collect":
        rc = collect(a.out_dir, [t for t in a.targets.split(",") if t], a.rows)
        consolidate(a.out_dir)
        return rc
    consolidate(a.out_dir)
    return 0


if __name__ == "__main__":
    sys.exit(main())
