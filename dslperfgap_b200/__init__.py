"""B200 (sm_100a) CUDA backend for DSLPerfGap's ViperBench row-reduction family.

``dslperfgap_b200.<kernel>.cuda_impl`` mirrors ``ViperBench/<kernel>/cuda_impl.py``
of the reference suite: the same function names and signatures as its
pytorch/triton/tilelang backends, running hand-written sm_100a kernels from
``lib/libdslpg_b200.so`` through the C ABI declared in ``include/dslpg_b200.h``.
"""
from .layer_norm.cuda_impl import layer_norm, layer_norm_host
from .rms_norm.cuda_impl import rms_norm, rms_norm_host
from .softmax.cuda_impl import softmax
from .log_softmax.cuda_impl import log_softmax
from .logsumexp.cuda_impl import logsumexp
from .cross_entropy.cuda_impl import cross_entropy_fwd, cross_entropy_bwd, cross_entropy_fwd_bwd
from .mean_reduction.cuda_impl import mean_reduction
from .max_reduction.cuda_impl import max_reduction
from .argmax.cuda_impl import argmax
from .linear_activation.cuda_impl import kernel_ff

__all__ = ["layer_norm", "layer_norm_host", "rms_norm", "rms_norm_host", "softmax", "log_softmax", "logsumexp", "cross_entropy_fwd", "cross_entropy_bwd", "cross_entropy_fwd_bwd",
           "mean_reduction", "max_reduction", "argmax", "kernel_ff"]
