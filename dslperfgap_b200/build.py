"""Build recipe for the CUDA C-ABI library ``lib/libdslpg_b200.so``.

The library is compiled in-tree with nvcc for sm_100a only:
each ``csrc/*.cu`` becomes an object (in parallel), and the objects are linked
into one shared library against the CUDA runtime. ``csrc/pyfast.c`` then
becomes the CPython extension ``lib/_dslpg_fast*.so`` (gcc, linked to the
library through an ``$ORIGIN`` run path): the low-overhead binding of the
per-call entry points. Re-running is cheap: an
object is rebuilt only when a source or header under ``csrc/`` or ``include/``
is newer than it.

Usage: ``python -m dslperfgap_b200.build [--force] [--verbose]``
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_DIR = PKG_DIR / "lib"
LIB_NAME = "libdslpg_b200.so"
LIB_PATH = LIB_DIR / LIB_NAME
FAST_PATH = LIB_DIR / ("_dslpg_fast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
TORCH_OPS_PATH = LIB_DIR / ("_dslpg_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
CUDA_INCLUDE = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DDSLPG_BUILD",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def _newest_header_mtime() -> float:
    mt = 0.0
    for p in list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")):
        mt = max(mt, p.stat().st_mtime)
    return mt


def _compile(src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False, defines=(), out: Path | None = None,
          build_dir: Path | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link lib/libdslpg_b200.so (or
    `out`, with extra -D `defines` and objects in `build_dir`)."""
    lib_path = Path(out) if out else LIB_PATH
    bdir = Path(build_dir) if build_dir else BUILD_DIR
    bdir.mkdir(parents=True, exist_ok=True)
    lib_path.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr_mt = _newest_header_mtime()
    extra = (["-Xptxas", "-v"] if ptxas_info else []) + [f"-D{d}" for d in defines]
    todo = []
    objs = []
    for src in sources:
        obj = bdir / (src.stem + ".o")
        objs.append(obj)
        stale = force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mt)
        if stale:
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, extra, verbose or ptxas_info) for s, o in todo]
            for f in futs:
                f.result()
    relink = bool(todo) or not lib_path.exists() or any(o.stat().st_mtime > lib_path.stat().st_mtime for o in objs)
    if relink:
        tmp = lib_path.parent / (lib_path.name + ".tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart",
               "-Xlinker", f"-soname={LIB_NAME}"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib_path)
    if out is None:
        build_fast(force=relink or force)
        build_torch_ops(force=relink or force)
    return lib_path


def build_fast(force: bool = False) -> Path:
    """Compile csrc/pyfast.c into the CPython extension next to the library."""
    src = CSRC / "pyfast.c"
    if not force and FAST_PATH.exists() and FAST_PATH.stat().st_mtime >= max(
            src.stat().st_mtime, LIB_PATH.stat().st_mtime, _newest_header_mtime()):
        return FAST_PATH
    tmp = FAST_PATH.parent / (FAST_PATH.name + ".tmp")
    cmd = [os.environ.get("CC", "gcc"), "-O2", "-shared", "-fPIC", "-fvisibility=hidden",
           "-I", sysconfig.get_paths()["include"], "-I", str(INCLUDE), "-I", str(CUDA_INCLUDE),
           str(src), "-o", str(tmp), "-L", str(LIB_DIR), "-ldslpg_b200", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building {FAST_PATH.name} failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, FAST_PATH)
    return FAST_PATH


def build_torch_ops(force: bool = False) -> Path:
    """Compile csrc/torch_ops.cpp (the C++ fast path of the Python wrappers)
    against torch's headers and libraries into lib/_dslpg_torch*.so."""
    src = CSRC / "torch_ops.cpp"
    if not force and TORCH_OPS_PATH.exists() and TORCH_OPS_PATH.stat().st_mtime >= max(
            src.stat().st_mtime, LIB_PATH.stat().st_mtime, _newest_header_mtime()):
        return TORCH_OPS_PATH
    import torch
    from torch.utils import cpp_extension
    incs = [sysconfig.get_paths()["include"], str(INCLUDE), *cpp_extension.include_paths("cuda")]
    tlib = cpp_extension.library_paths("cuda")[0]
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    tmp = TORCH_OPS_PATH.parent / (TORCH_OPS_PATH.name + ".tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_dslpg_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in incs], str(src), "-o", str(tmp), "-L", tlib, "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_python", "-L", str(LIB_DIR), "-ldslpg_b200", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building {TORCH_OPS_PATH.name} failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_OPS_PATH)
    return TORCH_OPS_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill info")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
