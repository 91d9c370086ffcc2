"""ViperBench/max_reduction/cuda_impl.py: the B200 (sm_100a) CUDA backend of `max_reduction`.

A fourth backend beside pytorch_impl.py, triton_impl.py and tilelang_impl.py,
with the same function name(s) and signature(s) (ViperBench/max_reduction/pytorch_impl.py:4-11).
Copy this file to ViperBench/max_reduction/ of a reference checkout. It imports the
dslperfgap_b200 package from PYTHONPATH, else from $DSLPG_B200_ROOT, else from
the repository this file sits in.
"""
import os
import sys

try:
    import dslperfgap_b200  # noqa: F401
except ImportError:
    _here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.environ.get("DSLPG_B200_ROOT") or os.path.join(_here, "..", "..", ".."))

from dslperfgap_b200.max_reduction.cuda_impl import max_reduction  # noqa: E402,F401

__all__ = ['max_reduction']
