"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own PyTorch backend (tingxi-li/DSLPerfGap,
``ViperBench/<kernel>/pytorch_impl.py`` — the oracle its own test.py files
compare every DSL backend against) on CPU, on seeded inputs, and stores inputs
and outputs in ``golden_<op>.pt``. The reference checkout is read from
``$DSLPG_REFERENCE`` (default: a `reference` directory beside this repository);
the fixtures are committed, so nothing that runs on a GPU box needs it.

Each case records:
  args / kwargs   the exact call of the reference signature
  ref_f32         pytorch_impl on fp32 upcasts of the float inputs (the
                  "fp32-computed reference"; log_softmax with a dtype= is
                  computed on x.to(dtype).float())
  ref_native      pytorch_impl on the inputs as stored (its own dtype path)
Cross-entropy outputs are stored as the valid flat prefix
(ceil(n_cols / BLOCK_SIZE) * n_rows entries) of each [n_rows, n_cols] output.

Shapes: the reference test.py shapes (rows trimmed so the files stay small;
the row length, which selects the kernel shape, is kept), rows of every
benchmark configuration with their value distributions, odd lengths, and the
edge-case kinds of experiments/exp_correctness_edge.py:53-82.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
# the reference checkout: DSLPG_REFERENCE, else a `reference` directory beside this repository
REF = Path(os.environ.get("DSLPG_REFERENCE") or HERE.parents[2] / "reference") / "ViperBench"

OPS = ["layer_norm", "rms_norm", "softmax", "log_softmax", "logsumexp", "cross_entropy", "cross_entropy_bwd",
       "mean_reduction", "max_reduction", "argmax", "linear_activation"]


def load_ref(kernel: str):
    kernel = "cross_entropy" if kernel == "cross_entropy_bwd" else kernel
    path = REF / kernel / "pytorch_impl.py"
    spec = importlib.util.spec_from_file_location(f"ref_{kernel}_pytorch_impl", str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


GEN = torch.Generator().manual_seed(0)


def randn(*shape, dtype=torch.float32, mean=0.0, std=1.0):
    return (torch.randn(*shape, generator=GEN) * std + mean).to(dtype)


def edge(kind: str, shape, dtype):
    """Edge-case inputs (kinds of experiments/exp_correctness_edge.py:53-82)."""
    t = randn(*shape)
    if kind == "nan":
        t.view(-1)[0] = float("nan")
    elif kind == "posinf":
        t.view(-1)[0] = float("inf")
    elif kind == "neginf":
        t.view(-1)[0] = float("-inf")
    elif kind == "large_mag":
        t = t * 1e4
    elif kind == "denormal":
        tiny = 1.4e-45 if dtype == torch.float32 else 6e-8
        t = t.sign() * tiny
    elif kind == "all_equal_rows":
        t = torch.ones(shape)
    elif kind == "masked_row":  # one row entirely -inf, one row with a single finite entry
        t[0] = float("-inf")
        t[1] = float("-inf")
        t[1, 3] = 0.5
    return t.to(dtype)


def masked(shape, dtype, std=3.0, frac=0.01):
    """softmax / log_softmax benchmark distribution: N(0, std) with ~1% -inf, no fully masked row."""
    x = randn(*shape, std=std)
    mask = torch.rand(*shape, generator=GEN) < frac
    x[mask] = float("-inf")
    full = torch.isinf(x).all(dim=-1)
    x[full, 0] = 0.0
    return x.to(dtype)


EDGE_KINDS = ["nan", "posinf", "neginf", "large_mag", "denormal", "all_equal_rows"]


def upcast(v):
    if isinstance(v, torch.Tensor) and v.is_floating_point():
        return v.float()
    return v


def cases_layer_norm():
    c = []
    for name, shape in [("ref_128x1024", (32, 1024)), ("ref_256x2048", (16, 2048)),
                        ("ref_64x4096", (8, 4096)), ("ref_512x1024", (16, 1024)),
                        ("ref_3d_4x32x1024", (2, 4, 1024)), ("ref_3d_2x8x2048", (2, 2, 2048))]:
        d = shape[-1]
        c.append((name, [randn(*shape, dtype=torch.bfloat16), randn(d, dtype=torch.bfloat16),
                         randn(d, dtype=torch.bfloat16)], {}))
    c.append(("cfg_fp32_4096", [randn(8, 4096), randn(4096, mean=1.0, std=0.1), randn(4096, std=0.1)], {}))
    c.append(("cfg_bf16_8192", [randn(4, 8192, dtype=torch.bfloat16),
                                randn(8192, mean=1.0, std=0.1, dtype=torch.bfloat16),
                                randn(8192, std=0.1, dtype=torch.bfloat16)], {}))
    c.append(("fp16_512", [randn(8, 512, dtype=torch.float16), randn(512, dtype=torch.float16),
                           randn(512, dtype=torch.float16)], {}))
    c.append(("fp32_16384", [randn(2, 16384), randn(16384), randn(16384)], {}))
    for shape, dt in [((3, 31), torch.float32), ((5, 33), torch.bfloat16), ((2, 100), torch.float16),
                      ((1, 1), torch.float32)]:
        d = shape[-1]
        c.append((f"odd_{shape[0]}x{d}_{str(dt)[6:]}", [randn(*shape, dtype=dt), randn(d, dtype=dt),
                                                       randn(d, dtype=dt)], {}))
    for k in EDGE_KINDS:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32), randn(64), randn(64)], {}))
    return c


def cases_rms_norm():
    c = []
    for name, (b, f), dt in [("ref_small_fp32", (4, 64), torch.float32), ("ref_medium_fp32", (32, 128), torch.float32),
                             ("ref_large_fp32", (32, 512), torch.float32), ("ref_edge_fp32", (1, 32), torch.float32),
                             ("ref_small_fp16", (32, 128), torch.float16)]:
        c.append((name, [randn(b, f, dtype=dt), (f,), randn(f, dtype=dt)], {}))
    c.append(("cfg_bf16_8192", [randn(4, 8192, dtype=torch.bfloat16), (8192,),
                                randn(8192, mean=1.0, std=0.1, dtype=torch.bfloat16)], {"eps": 1e-6}))
    c.append(("cfg_bf16_5120_tail", [randn(4, 5120, dtype=torch.bfloat16), (5120,),
                                     randn(5120, mean=1.0, std=0.1, dtype=torch.bfloat16)], {"eps": 1e-6}))
    c.append(("two_dims_normalized", [randn(2, 4, 8, 16), (8, 16), randn(8, 16)], {}))
    c.append(("odd_3x33_bf16", [randn(3, 33, dtype=torch.bfloat16), (33,), randn(33, dtype=torch.bfloat16)], {}))
    c.append(("fp32_weight_bf16_x", [randn(4, 256, dtype=torch.bfloat16), (256,), randn(256)], {}))
    for k in EDGE_KINDS:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32), (64,), randn(64)], {}))
    return c


def cases_softmax():
    c = []
    for name, shape in [("ref_small_2d", (4, 8)), ("ref_medium_2d", (16, 512)), ("ref_large_cols", (4, 4096)),
                        ("ref_wide", (4, 2048)), ("ref_square", (10, 100)), ("ref_3d_tensor", (4, 8, 64)),
                        ("ref_4d_tensor", (2, 3, 4, 32)), ("ref_1d_tensor", (128,))]:
        c.append((name, [randn(*shape)], {}))
    c.append(("cfg_fp16_4096_masked", [masked((8, 4096), torch.float16)], {}))
    c.append(("bf16_1024", [randn(8, 1024, std=2.0, dtype=torch.bfloat16)], {}))
    c.append(("fp32_40000_stream", [randn(2, 40000)], {}))
    for shape, dt in [((3, 33), torch.float16), ((2, 31), torch.bfloat16), ((1, 1), torch.float32)]:
        c.append((f"odd_{shape[0]}x{shape[1]}_{str(dt)[6:]}", [randn(*shape, dtype=dt)], {}))
    for k in EDGE_KINDS + ["masked_row"]:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32)], {}))
    return c


def cases_log_softmax():
    c = []
    for name, shape, dt in [("ref_small_fp32", (4, 64), torch.float32), ("ref_medium_fp32", (8, 256), torch.float32),
                            ("ref_large_fp32", (8, 1024), torch.float32), ("ref_4d_fp32", (2, 2, 16, 64), torch.float32),
                            ("ref_small_fp16", (8, 256), torch.float16)]:
        c.append((name, [randn(*shape, dtype=dt)], {"dim": -1}))
    c.append(("cfg_fp16_4096_masked", [masked((8, 4096), torch.float16)], {"dim": -1}))
    c.append(("dim1_3d", [randn(4, 16, 8)], {"dim": 1}))
    c.append(("dim0_2d", [randn(8, 5)], {"dim": 0}))
    c.append(("dtype_fp16_to_fp32", [randn(4, 256, dtype=torch.float16)], {"dim": -1, "dtype": "float32"}))
    c.append(("dtype_fp32_to_bf16", [randn(4, 256)], {"dim": -1, "dtype": "bfloat16"}))
    c.append(("dtype_bf16_to_fp16_dim0", [randn(6, 40, dtype=torch.bfloat16)], {"dim": 0, "dtype": "float16"}))
    c.append(("odd_3x33_bf16", [randn(3, 33, dtype=torch.bfloat16)], {"dim": -1}))
    for k in EDGE_KINDS + ["masked_row"]:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32)], {"dim": -1}))
    return c


def cases_logsumexp():
    c = []
    for name, shape in [("ref_small_2d", (4, 64)), ("ref_medium_2d", (8, 256)), ("ref_large_2d", (8, 1024)),
                        ("ref_wide_2d", (4, 4096)), ("ref_3d_tensor", (4, 8, 64)), ("ref_4d_tensor", (2, 3, 4, 32)),
                        ("ref_1d_tensor", (128,))]:
        c.append((name, [randn(*shape)], {}))
    c.append(("cfg_bf16_vocab", [randn(2, 128256, std=2.0, dtype=torch.bfloat16)], {}))
    c.append(("fp16_1000", [randn(4, 1000, dtype=torch.float16)], {}))
    c.append(("odd_3x33_bf16", [randn(3, 33, dtype=torch.bfloat16)], {}))
    for k in EDGE_KINDS + ["masked_row"]:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32)], {}))
    return c


CE_REF_CONFIGS = [  # ViperBench/cross_entropy/test.py:61-92
    ("no_smooth_no_split_1blk", dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.1, ignored_index=-1,
                                     total_classes=10, class_start_idx=0, BLOCK_SIZE=8, HAS_SMOOTHING=False, SPLIT=False)),
    ("smooth_no_split_1blk", dict(smoothing=0.1, logit_scale=1.0, lse_square_scale=0.1, ignored_index=-1,
                                  total_classes=10, class_start_idx=0, BLOCK_SIZE=8, HAS_SMOOTHING=True, SPLIT=False)),
    ("smooth_split_1blk", dict(smoothing=0.1, logit_scale=1.0, lse_square_scale=0.1, ignored_index=-1,
                               total_classes=10, class_start_idx=0, BLOCK_SIZE=8, HAS_SMOOTHING=True, SPLIT=True)),
    ("no_smooth_no_split_2blk", dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.1, ignored_index=-1,
                                     total_classes=10, class_start_idx=0, BLOCK_SIZE=4, HAS_SMOOTHING=False, SPLIT=False)),
    ("logit_scale_2blk", dict(smoothing=0.0, logit_scale=0.5, lse_square_scale=0.05, ignored_index=-1,
                              total_classes=10, class_start_idx=0, BLOCK_SIZE=4, HAS_SMOOTHING=False, SPLIT=False)),
]


def cases_cross_entropy():
    c = []
    g42 = torch.Generator().manual_seed(42)  # the reference test's seed (test.py:13-17), CPU generator
    logits = torch.randn((4, 8), generator=g42, dtype=torch.float32)
    labels = torch.randint(0, 8, (4,), generator=g42, dtype=torch.int32)
    for name, p in CE_REF_CONFIGS:
        c.append((f"ref_{name}", [logits, labels], dict(p)))
    base = dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100,
                total_classes=128256, class_start_idx=0, BLOCK_SIZE=131072, HAS_SMOOTHING=False, SPLIT=False)
    lg = randn(4, 128256, std=2.0, dtype=torch.bfloat16)
    lb = torch.randint(0, 128256, (4,), generator=GEN, dtype=torch.int64)
    lb[2] = -100
    c.append(("cfg_bf16_vocab", [lg, lb], dict(base)))
    lg2 = randn(6, 1000, dtype=torch.bfloat16)
    lb2 = torch.randint(0, 1000, (6,), generator=GEN, dtype=torch.int64)
    lb2[0] = 999
    lb2[1] = -100
    c.append(("multiblock_smooth_scale", [lg2, lb2], dict(smoothing=0.2, logit_scale=0.7, lse_square_scale=1e-3,
                                                          ignored_index=-100, total_classes=1000, class_start_idx=0,
                                                          BLOCK_SIZE=256, HAS_SMOOTHING=True, SPLIT=False)))
    c.append(("multiblock_split", [lg2, lb2], dict(smoothing=0.2, logit_scale=1.0, lse_square_scale=1e-3,
                                                   ignored_index=-100, total_classes=1000, class_start_idx=0,
                                                   BLOCK_SIZE=256, HAS_SMOOTHING=True, SPLIT=True)))
    lg3 = randn(5, 96, dtype=torch.float16)
    lb3 = torch.tensor([5, 200, 100, -7, 50], dtype=torch.int32)
    c.append(("class_start_and_out_of_range", [lg3, lb3], dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.01,
                                                               ignored_index=-7, total_classes=96, class_start_idx=40,
                                                               BLOCK_SIZE=64, HAS_SMOOTHING=False, SPLIT=False)))
    lg4 = randn(3, 37)
    lb4 = torch.tensor([0, 36, 12], dtype=torch.int64)
    c.append(("odd_cols_fp32", [lg4, lb4], dict(smoothing=0.1, logit_scale=2.0, lse_square_scale=0.0,
                                                ignored_index=-100, total_classes=37, class_start_idx=0,
                                                BLOCK_SIZE=16, HAS_SMOOTHING=True, SPLIT=False)))
    for k in ["nan", "posinf", "neginf", "large_mag", "all_equal_rows"]:
        lgk = edge(k, (4, 64), torch.float32)
        lbk = torch.tensor([0, 5, 63, -100], dtype=torch.int64)
        c.append((f"edge_{k}", [lgk, lbk], dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0,
                                                 ignored_index=-100, total_classes=64, class_start_idx=0,
                                                 BLOCK_SIZE=64, HAS_SMOOTHING=False, SPLIT=False)))
    return c


def bwd_case(name, logits, labels, p, seedgen):
    """cross_entropy_bwd inputs: dloss ~ U(0.5, 1.5) per row and lse = the row's
    logsumexp of logits * scale (one value per row, as the forward stores it)."""
    r = logits.shape[0]
    dloss = torch.rand(r, generator=seedgen) + 0.5
    lse = torch.logsumexp(logits.float() * p["logit_scale"], dim=-1)
    kw = {k: v for k, v in p.items() if k != "SPLIT"}
    return (name, [dloss, logits, lse, labels], kw)


def cases_cross_entropy_bwd():
    c = []
    g42 = torch.Generator().manual_seed(42)  # the reference test's seed (test.py:13-17), CPU generator
    logits = torch.randn((4, 8), generator=g42, dtype=torch.float32)
    labels = torch.randint(0, 8, (4,), generator=g42, dtype=torch.int32)
    for name, p in CE_REF_CONFIGS:
        c.append(bwd_case(f"ref_{name}", logits, labels, dict(p), GEN))
    lg = randn(2, 128256, std=2.0, dtype=torch.bfloat16)
    lb = torch.tensor([5, 128255], dtype=torch.int64)
    c.append(bwd_case("cfg_bf16_vocab", lg, lb, dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0,
                                                      ignored_index=-100, total_classes=128256, class_start_idx=0,
                                                      BLOCK_SIZE=131072, HAS_SMOOTHING=False, SPLIT=False), GEN))
    lg2 = randn(6, 1000, dtype=torch.bfloat16)
    lb2 = torch.tensor([999, -100, 3, 500, 0, 1500], dtype=torch.int64)
    c.append(bwd_case("multiblock_smooth_scale", lg2, lb2, dict(smoothing=0.2, logit_scale=0.7, lse_square_scale=1e-3,
                                                                ignored_index=-100, total_classes=1000, class_start_idx=0,
                                                                BLOCK_SIZE=256, HAS_SMOOTHING=True, SPLIT=False), GEN))
    lg3 = randn(5, 96, dtype=torch.float16)
    lb3 = torch.tensor([45, 200, 100, -7, 50], dtype=torch.int32)
    c.append(bwd_case("class_start_fp16", lg3, lb3, dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.01,
                                                         ignored_index=-7, total_classes=96, class_start_idx=40,
                                                         BLOCK_SIZE=64, HAS_SMOOTHING=False, SPLIT=False), GEN))
    lg4 = randn(3, 37)
    lb4 = torch.tensor([0, 36, 12], dtype=torch.int64)
    c.append(bwd_case("odd_cols_fp32", lg4, lb4, dict(smoothing=0.1, logit_scale=2.0, lse_square_scale=0.0,
                                                      ignored_index=-100, total_classes=37, class_start_idx=0,
                                                      BLOCK_SIZE=16, HAS_SMOOTHING=True, SPLIT=False), GEN))
    return c


def cases_mean_reduction():
    c = []
    for name, shape, dim, kw in [("ref_2D_dim0", (64, 128), 0, {}), ("ref_2D_dim1_keepdim", (64, 128), 1, {"keepdim": True}),
                                 ("ref_4D_multi_dim", (2, 3, 4, 5), [1, 2], {}), ("ref_3D_dim2", (8, 16, 32), 2, {})]:
        c.append((name, [randn(*shape), dim], kw))
    c.append(("cfg_fp32_32768", [randn(4, 32768), 1], {}))
    c.append(("bf16_dtype_fp32", [randn(8, 1000, dtype=torch.bfloat16), 1], {"dtype": "float32"}))
    c.append(("fp16_rows", [randn(8, 4096, dtype=torch.float16), -1], {}))
    c.append(("fp32_to_bf16", [randn(4, 256), 1], {"dtype": "bfloat16"}))
    c.append(("non_adjacent_dims", [randn(3, 4, 5, 6), [0, 2]], {}))
    c.append(("odd_3x33", [randn(3, 33), 1], {}))
    for k in ["nan", "posinf", "large_mag", "all_equal_rows"]:
        c.append((f"edge_{k}", [edge(k, (4, 64), torch.float32), 1], {}))
    return c


def _argmax_inputs():
    c = []
    for name, shape, dim, kw in [("ref_2D_dim0", (128, 256), 0, {}), ("ref_2D_dim1", (256, 128), 1, {}),
                                 ("ref_3D_dim2", (8, 16, 128), 2, {}), ("ref_3D_dim1_keepdim", (4, 32, 64), 1, {"keepdim": True}),
                                 ("ref_3D_neg_dim", (4, 8, 64), -1, {})]:
        c.append((name, [randn(*shape), dim], kw))
    c.append(("cfg_fp16_32768", [randn(4, 32768, dtype=torch.float16), 1], {}))
    c.append(("bf16_1000", [randn(6, 1000, dtype=torch.bfloat16), 1], {}))
    ties = torch.zeros(4, 96)
    ties[0, 10] = ties[0, 50] = 3.0
    ties[1] = 1.0
    ties[2, 95] = 7.0
    ties[3, :] = float("-inf")
    c.append(("ties_and_neginf", [ties, 1], {}))
    nanrow = randn(3, 80)
    nanrow[0, 7] = float("nan")
    nanrow[0, 40] = float("nan")
    nanrow[1, 79] = float("nan")
    c.append(("nans_first_wins", [nanrow, 1], {}))
    c.append(("odd_5x33_fp16", [randn(5, 33, dtype=torch.float16), 1], {}))
    return c


def cases_max_reduction():
    return _argmax_inputs()


def cases_argmax():
    return _argmax_inputs()


def cases_linear_activation():
    c = []
    g42 = torch.Generator().manual_seed(42)  # the reference test's seed (test.py:10), CPU generator
    for b, s_, d in [(2, 4, 64), (3, 4, 64), (2, 8, 64), (1, 16, 128)]:  # test.py:21-26 (n_out = dim)
        x = torch.randn((b, s_, d), generator=g42).half()
        w1 = torch.randn((d, d), generator=g42).half()
        w3 = torch.randn((d, d), generator=g42).half()
        rw = torch.randn((d,), generator=g42).half()
        c.append((f"ref_{b}x{s_}x{d}", [x, w1, w3, rw], {}))
    for name, (b, s_, d, n) in [("ragged_1x70x256_n200", (1, 70, 256, 200)), ("multi_tile_2x96x512_n384", (2, 96, 512, 384)),
                                ("k_tail_1x130x1000_n136", (1, 130, 1000, 136))]:
        x = randn(b, s_, d, dtype=torch.float16)
        w1 = randn(n, d, std=0.05, dtype=torch.float16)
        w3 = randn(n, d, std=0.05, dtype=torch.float16)
        rw = randn(d, mean=1.0, std=0.1, dtype=torch.float16)
        c.append((name, [x, w1, w3, rw], {}))
    return c


def call(op, mod, args, kwargs):
    if op == "linear_activation":
        return mod.kernel_ff(*args)
    if op in ("mean_reduction", "max_reduction", "argmax"):
        kw = dict(kwargs)
        if "dtype" in kw:
            kw["dtype"] = getattr(torch, kw["dtype"])
        return getattr(mod, op)(*args, **kw)
    if op == "cross_entropy_bwd":
        return mod.cross_entropy_bwd(*args, **kwargs)
    if op == "layer_norm":
        return mod.layer_norm(*args, **kwargs)
    if op == "rms_norm":
        return mod.rms_norm(*args, **kwargs)
    if op == "softmax":
        return mod.softmax(*args)
    if op == "log_softmax":
        kw = dict(kwargs)
        if "dtype" in kw:
            kw["dtype"] = getattr(torch, kw["dtype"])
        return mod.log_softmax(*args, **kw)
    if op == "logsumexp":
        return mod.logsumexp(*args)
    if op == "cross_entropy":
        return mod.cross_entropy_fwd(*args, **kwargs)
    raise KeyError(op)


def valid_prefix(outs, n_rows, n_cols, bs):
    nb = (n_cols + bs - 1) // bs
    return tuple(o.reshape(-1)[: nb * n_rows].clone() for o in outs)


def main() -> int:
    builders = dict(layer_norm=cases_layer_norm, rms_norm=cases_rms_norm, softmax=cases_softmax,
                    log_softmax=cases_log_softmax, logsumexp=cases_logsumexp, cross_entropy=cases_cross_entropy,
                    cross_entropy_bwd=cases_cross_entropy_bwd, mean_reduction=cases_mean_reduction,
                    max_reduction=cases_max_reduction, argmax=cases_argmax, linear_activation=cases_linear_activation)
    total = 0
    for op in OPS:
        mod = load_ref(op)
        out = []
        for name, args, kwargs in builders[op]():
            native = call(op, mod, args, kwargs)
            if op == "mean_reduction" and "dtype" in kwargs:
                x32 = args[0].to(getattr(torch, kwargs["dtype"])).float()
                ref32 = call(op, mod, [x32, args[1]], {k: v for k, v in kwargs.items() if k != "dtype"})
            elif op == "log_softmax" and "dtype" in kwargs:
                x32 = args[0].to(getattr(torch, kwargs["dtype"])).float()
                ref32 = call(op, mod, [x32], {"dim": kwargs.get("dim", -1)})
            else:
                ref32 = call(op, mod, [upcast(a) for a in args], kwargs)
            if op == "cross_entropy":
                r, cc = args[0].shape
                native = valid_prefix(native, r, cc, kwargs["BLOCK_SIZE"])
                ref32 = valid_prefix(ref32, r, cc, kwargs["BLOCK_SIZE"])
            out.append(dict(name=name, args=args, kwargs=kwargs, ref_f32=ref32, ref_native=native))
        path = HERE / f"golden_{op}.pt"
        src = "cross_entropy" if op == "cross_entropy_bwd" else op
        torch.save(dict(op=op, source="ViperBench/%s/pytorch_impl.py (reference, CPU)" % src,
                        torch=str(torch.__version__), cases=out), path)
        total += path.stat().st_size
        print(f"{path.name}: {len(out)} cases, {path.stat().st_size / 1e6:.2f} MB")
    print(f"total {total / 1e6:.2f} MB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
