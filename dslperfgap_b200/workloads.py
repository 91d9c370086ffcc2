"""Synthetic benchmark workloads: the configurations the backend is measured
on, as seeded generators.

The reference measures on internal synthetic shapes only (no dataset), so
these generators are the whole workload. Values follow the stated
distributions; inputs are generated in fp32 and cast to the storage dtype.

Rows are generated in fixed blocks, each from its own generator seeded by
(seed, block index), so any row range — a GPU's shard, or a bounded CPU
sample — is bit-identical to the same rows of the full tensor generated on
the same device type.

Algorithmic bytes (the roofline numerator) count each input read once and
each output written once:
  layer_norm / rms_norm / softmax / log_softmax   2 * M * N * elem_size
  logsumexp                                      M * N * elem_size + M * elem_size
  cross_entropy (one block per row)              M * N * elem_size + 8 * M + 3 * 4 * M
  cross_entropy_bwd                              2 * M * N * elem_size + 8 * M + 4 * M + 4 * M
  cross_entropy_fwd_bwd                          2 * M * N * elem_size + 8 * M + 4 * M + 3 * 4 * M
  mean_reduction / max_reduction / argmax        M * N * elem_size + the M outputs
  linear_activation (kernel_ff)                  (M*K + 2*N*K + K + M*N) * 2; its roofline is
                                                 tensor-bound: 4 * M * N * K flops
(the [N] weight and bias vectors of the row ops, read once per GPU, are not counted).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

ROW_BLOCK_ELEMS = 1 << 24  # elements generated per seeded block


@dataclass(frozen=True)
class Config:
    name: str
    op: str
    fn_name: str
    M: int
    N: int
    dtype: torch.dtype
    description: str
    kwargs: dict = field(default_factory=dict)
    K: int = 0  # linear_activation: the reduction (model) dimension


CONFIGS = {
    c.name: c
    for c in [
        Config("layer_norm_fp32", "layer_norm", "layer_norm", 4096, 4096, torch.float32,
               "LayerNorm fwd fp32 x[4096,4096]~N(0,1), w~N(1,0.1), b~N(0,0.1), eps=1e-5", {"eps": 1e-5}),
        Config("rms_norm_bf16", "rms_norm", "rms_norm", 16384, 8192, torch.bfloat16,
               "RMSNorm fwd bf16 x[16384,8192]~N(0,1), w~N(1,0.1), eps=1e-6", {"eps": 1e-6}),
        Config("rms_norm_bf16_tail", "rms_norm", "rms_norm", 16384, 5120, torch.bfloat16,
               "RMSNorm fwd bf16 tail variant x[16384,5120]~N(0,1), w~N(1,0.1), eps=1e-6", {"eps": 1e-6}),
        Config("softmax_fp16", "softmax", "softmax", 32768, 4096, torch.float16,
               "softmax fwd fp16 x[32768,4096]~N(0,3), 1% -inf, no fully masked row"),
        Config("log_softmax_fp16", "log_softmax", "log_softmax", 32768, 4096, torch.float16,
               "log_softmax fwd fp16 x[32768,4096]~N(0,3), 1% -inf, no fully masked row", {"dim": -1}),
        Config("logsumexp_bf16", "logsumexp", "logsumexp", 8192, 128256, torch.bfloat16,
               "logsumexp bf16 logits[8192,128256]~N(0,2)"),
        Config("cross_entropy_bf16", "cross_entropy", "cross_entropy_fwd", 8192, 128256, torch.bfloat16,
               "cross-entropy fwd bf16 logits[8192,128256]~N(0,2), int64 targets U[0,128256), 410 rows "
               "ignore_index=-100, BLOCK_SIZE=131072, smoothing 0, scale 1, lse_sq 0, SPLIT False",
               dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100,
                    total_classes=128256, class_start_idx=0, BLOCK_SIZE=131072, HAS_SMOOTHING=False,
                    SPLIT=False)),
        Config("cross_entropy_bwd_bf16", "cross_entropy_bwd", "cross_entropy_bwd", 8192, 128256, torch.bfloat16,
               "cross-entropy bwd bf16 on the forward's configuration: logits[8192,128256]~N(0,2), int64 targets "
               "U[0,128256), 410 rows ignore_index=-100, dloss~U(0.5,1.5), lse = row logsumexp",
               dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100,
                    total_classes=128256, class_start_idx=0, BLOCK_SIZE=131072, HAS_SMOOTHING=False)),
        Config("cross_entropy_fwd_bwd_bf16", "cross_entropy_fwd_bwd", "cross_entropy_fwd_bwd", 8192, 128256,
               torch.bfloat16,
               "cross-entropy forward + backward in one pass, bf16, on the forward's configuration: "
               "logits[8192,128256]~N(0,2), int64 targets U[0,128256), 410 rows ignore_index=-100, "
               "dloss = 1/n_valid (the gradient of the mean loss)",
               dict(smoothing=0.0, logit_scale=1.0, lse_square_scale=0.0, ignored_index=-100,
                    total_classes=128256, class_start_idx=0, HAS_SMOOTHING=False)),
        Config("mean_reduction_fp32", "mean_reduction", "mean_reduction", 8192, 32768, torch.float32,
               "mean over dim 1, fp32 x[8192,32768]~N(0,1) (the reference's large shape, benchmark.py:288-290)",
               {"dim": 1}),
        Config("max_reduction_fp16", "max_reduction", "max_reduction", 8192, 32768, torch.float16,
               "max (values, indices) over dim 1, fp16 x[8192,32768]~N(0,1) (benchmark.py:278-280)", {"dim": 1}),
        Config("argmax_fp16", "argmax", "argmax", 8192, 32768, torch.float16,
               "argmax over dim 1, fp16 x[8192,32768]~N(0,1) (benchmark.py:97-99)", {"dim": 1}),
        Config("layer_norm_bf16_sharded", "layer_norm", "layer_norm", 131072, 8192, torch.bfloat16,
               "row-sharded LayerNorm bf16 x[131072,8192]~N(0,1), w~N(1,0.1), b~N(0,0.1), eps=1e-5, "
               "row blocks over 1/2/4/8 GPUs", {"eps": 1e-5}),
        Config("linear_activation_fp16", "linear_activation", "kernel_ff", 2048, 16384, torch.float16,
               "Llama FFN kernel_ff fp16: x[1,2048,4096], w1/w3[16384,4096], rms_w[4096] ~N(0,1) "
               "(the reference's large shape, benchmark.py:223-228); RMSNorm + dual GEMM + SiLU gate",
               {}, K=4096),
    ]
}
NAMES = list(CONFIGS)


@dataclass
class Workload:
    config: Config
    rows: tuple  # (first, last) row of the full configuration held here
    args: list
    kwargs: dict

    @property
    def name(self):
        return self.config.name

    @property
    def op(self):
        return self.config.op

    @property
    def fn_name(self):
        return self.config.fn_name

    @property
    def M(self):
        return self.rows[1] - self.rows[0]

    @property
    def out_dtype(self):
        if self.op == "cross_entropy":
            return torch.float32
        if self.op == "argmax":
            return torch.int64
        return self.config.dtype

    @property
    def cuda_fn(self):
        import dslperfgap_b200
        return getattr(dslperfgap_b200, self.fn_name)

    @property
    def valid_entries(self):
        bs = self.kwargs.get("BLOCK_SIZE", 1)
        return self.M * ((self.config.N + bs - 1) // bs)

    def algo_bytes(self) -> int:
        return algo_bytes(self.config, self.M)

    def to(self, device):
        args = [a.to(device) if isinstance(a, torch.Tensor) else a for a in self.args]
        return Workload(self.config, self.rows, args, dict(self.kwargs))


def algo_bytes(cfg: Config, rows: int) -> int:
    es = torch.tensor([], dtype=cfg.dtype).element_size()
    if cfg.op in ("layer_norm", "rms_norm", "softmax", "log_softmax"):
        return 2 * rows * cfg.N * es
    if cfg.op == "logsumexp":
        return rows * cfg.N * es + rows * es
    if cfg.op == "cross_entropy":
        return rows * cfg.N * es + 8 * rows + 3 * 4 * rows
    if cfg.op == "cross_entropy_bwd":
        return 2 * rows * cfg.N * es + 8 * rows + 4 * rows + 4 * rows
    if cfg.op == "cross_entropy_fwd_bwd":  # logits read once, dlogits written, labels + dloss, 3 fp32 outputs
        return 2 * rows * cfg.N * es + 8 * rows + 4 * rows + 3 * 4 * rows
    if cfg.op == "mean_reduction":
        return rows * cfg.N * es + rows * es
    if cfg.op == "max_reduction":
        return rows * cfg.N * es + rows * (es + 8)
    if cfg.op == "argmax":
        return rows * cfg.N * es + rows * 8
    if cfg.op == "linear_activation":  # x, w1, w3, rms_w read once, out written once
        return es * (rows * cfg.K + 2 * cfg.N * cfg.K + cfg.K + rows * cfg.N)
    raise KeyError(cfg.op)


def algo_flops(cfg: Config, rows: int) -> int:
    """Tensor-core work of linear_activation: two [rows, K] x [K, N] products."""
    return 4 * rows * cfg.N * cfg.K if cfg.op == "linear_activation" else 0


def shard_rows(M: int, rank: int, world: int) -> tuple:
    """Contiguous row block [first, last) of `rank` out of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad shard {rank}/{world}")
    return (M * rank // world, M * (rank + 1) // world)


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _rows(cfg: Config, r0: int, r1: int, seed: int, device, std: float, masked: bool) -> torch.Tensor:
    n = cfg.N
    block = max(1, ROW_BLOCK_ELEMS // n)
    out = torch.empty((r1 - r0, n), dtype=cfg.dtype, device=device)
    b0, b1 = r0 // block, (r1 - 1) // block if r1 > r0 else -1
    for b in range(b0, b1 + 1):
        lo, hi = b * block, min((b + 1) * block, cfg.M)
        g = _gen(device, seed * 1_000_003 + b)
        t = torch.randn((hi - lo, n), generator=g, device=device)
        if std != 1.0:
            t.mul_(std)
        if masked:
            m = torch.rand((hi - lo, n), generator=g, device=device) < 0.01
            t.masked_fill_(m, float("-inf"))
            full = torch.isinf(t).all(dim=1)
            t[full, 0] = 0.0
        s0, s1 = max(lo, r0), min(hi, r1)
        out[s0 - r0:s1 - r0].copy_(t[s0 - lo:s1 - lo])
    return out


def _vec(n, dtype, seed, device, mean, std):
    g = _gen(device, seed)
    return (torch.randn(n, generator=g, device=device) * std + mean).to(dtype)


def make(name: str, seed: int = 0, device="cpu", rows: tuple | None = None) -> Workload:
    """Build workload `name` (rows [first, last) of it; default all) on `device`."""
    cfg = CONFIGS[name]
    r0, r1 = rows if rows is not None else (0, cfg.M)
    if not 0 <= r0 <= r1 <= cfg.M:
        raise ValueError(f"rows {rows} outside [0, {cfg.M}]")
    kw = dict(cfg.kwargs)
    if cfg.op == "layer_norm":
        x = _rows(cfg, r0, r1, seed, device, 1.0, False)
        w = _vec(cfg.N, cfg.dtype, seed + 101, device, 1.0, 0.1)
        b = _vec(cfg.N, cfg.dtype, seed + 102, device, 0.0, 0.1)
        args = [x, w, b]
    elif cfg.op == "rms_norm":
        x = _rows(cfg, r0, r1, seed, device, 1.0, False)
        w = _vec(cfg.N, cfg.dtype, seed + 101, device, 1.0, 0.1)
        args = [x, (cfg.N,), w]
    elif cfg.op in ("softmax", "log_softmax"):
        args = [_rows(cfg, r0, r1, seed, device, 3.0, True)]
    elif cfg.op == "logsumexp":
        args = [_rows(cfg, r0, r1, seed, device, 2.0, False)]
    elif cfg.op == "linear_activation":
        x = _rows(Config(cfg.name, cfg.op, cfg.fn_name, cfg.M, cfg.K, cfg.dtype, ""), r0, r1, seed, device, 1.0, False)
        wcfg = Config(cfg.name, cfg.op, cfg.fn_name, cfg.N, cfg.K, cfg.dtype, "")
        w1 = _rows(wcfg, 0, cfg.N, seed + 201, device, 1.0, False)
        w3 = _rows(wcfg, 0, cfg.N, seed + 202, device, 1.0, False)
        rw = _vec(cfg.K, cfg.dtype, seed + 203, device, 0.0, 1.0)
        args = [x.reshape(1, r1 - r0, cfg.K), w1, w3, rw]
    elif cfg.op in ("mean_reduction", "max_reduction", "argmax"):
        args = [_rows(cfg, r0, r1, seed, device, 1.0, False)]
    elif cfg.op in ("cross_entropy", "cross_entropy_bwd", "cross_entropy_fwd_bwd"):
        x = _rows(cfg, r0, r1, seed, device, 2.0, False)
        g = _gen("cpu", seed + 103)
        labels = torch.randint(0, cfg.N, (cfg.M,), generator=g, dtype=torch.int64)
        n_ign = int(round(0.05 * cfg.M))
        labels[torch.randperm(cfg.M, generator=g)[:n_ign]] = -100
        labels = labels[r0:r1].to(device)
        if cfg.op == "cross_entropy":
            args = [x, labels]
        elif cfg.op == "cross_entropy_fwd_bwd":
            dloss = torch.full((r1 - r0,), 1.0 / (cfg.M - n_ign), dtype=torch.float32, device=device)
            args = [x, labels, dloss]
        else:
            dloss = (torch.rand(cfg.M, generator=g) + 0.5)[r0:r1].to(device)
            # input preparation only: the forward's per-row lse
            lse = torch.cat([torch.logsumexp(x[i:i + 256].float(), dim=-1) for i in range(0, x.shape[0], 256)])
            args = [dloss, x, lse, labels]
    else:
        raise KeyError(cfg.op)
    return Workload(cfg, (r0, r1), args, kw)


def config_dict(cfg: Config) -> dict:
    return {"workload": cfg.name, "op": cfg.op, "shape": [cfg.M, cfg.N], "dtype": {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}[cfg.dtype],
            "description": cfg.description}


def num_elements(cfg: Config) -> int:
    return math.prod((cfg.M, cfg.N))
