"""ViperBench/cross_entropy/cuda_impl.py: the B200 (sm_100a) CUDA backend of `cross_entropy`.

A fourth backend beside pytorch_impl.py, triton_impl.py and tilelang_impl.py,
with the same function name(s) and signature(s) (ViperBench/cross_entropy/pytorch_impl.py:4-90 and :93-141).
Copy this file to ViperBench/cross_entropy/ of a reference checkout. It imports the
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

from dslperfgap_b200.cross_entropy.cuda_impl import cross_entropy_fwd, cross_entropy_bwd, cross_entropy_fwd_bwd  # noqa: E402,F401

__all__ = ['cross_entropy_fwd', 'cross_entropy_bwd', 'cross_entropy_fwd_bwd']
