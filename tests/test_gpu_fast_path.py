"""The C++ fast path (_dslpg_torch) and the Python wrappers give the same
tensors bit for bit: every op is called once as shipped (the fast path takes
these common cases) and once with the fast path switched off, so the Python
wrapper does the checks, the allocation and the launch."""
import importlib

import pytest
import torch

import dslperfgap_b200 as B
from dslperfgap_b200 import _lib

pytestmark = pytest.mark.gpu

MODULES = {"layer_norm": "layer_norm", "rms_norm": "rms_norm", "softmax": "softmax", "log_softmax": "log_softmax",
           "logsumexp": "logsumexp", "mean_reduction": "mean_reduction", "max_reduction": "max_reduction",
           "argmax": "argmax", "cross_entropy_fwd": "cross_entropy"}


def _without_fast_path(monkeypatch, fn_name):
    mod = importlib.import_module(f"dslperfgap_b200.{MODULES[fn_name]}.cuda_impl")
    monkeypatch.setattr(mod, f"_fast_{fn_name}", lambda *a: None)
    return getattr(mod, fn_name)


def _same(a, b):
    if isinstance(a, tuple):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            _same(x, y)
        return
    assert a.dtype == b.dtype and a.shape == b.shape
    assert torch.equal(a.view(-1).view(torch.uint8) if a.dtype.is_floating_point else a,
                       b.view(-1).view(torch.uint8) if b.dtype.is_floating_point else b)


def _cases():
    g = torch.Generator(device="cuda").manual_seed(5)
    rn = lambda *s, dt=torch.float32: torch.randn(*s, generator=g, device="cuda").to(dt)  # noqa: E731
    x16 = rn(3, 37, 1000, dt=torch.bfloat16)
    w16, b16 = rn(1000, dt=torch.bfloat16), rn(1000, dt=torch.bfloat16)
    xh = rn(64, 4096, dt=torch.float16)
    lg = rn(40, 3000)
    lab = torch.randint(0, 3000, (40,), generator=g, device="cuda")
    lab[3] = -100
    return [
        ("layer_norm", (x16, w16, b16), {}),
        ("layer_norm", (x16, w16, None), {}),
        ("rms_norm", (x16, (1000,), w16), {"eps": 1e-6}),
        ("softmax", (xh,), {}),
        ("log_softmax", (x16,), {"dim": 1}),
        ("logsumexp", (lg,), {}),
        ("mean_reduction", (xh, 1), {"keepdim": True}),
        ("mean_reduction", (x16, 1), {"dtype": torch.float32}),
        ("max_reduction", (x16, -1), {}),
        ("argmax", (xh, 0), {}),
        ("cross_entropy_fwd", (lg, lab, 0.1, 1.0, 1e-4, -100, 3000, 0, 1024, True, False), {}),
    ]


@pytest.mark.parametrize("i", range(11))
def test_fast_path_equals_python_path(i, monkeypatch):
    assert _lib.torch_ops() is not None, "the _dslpg_torch extension is not built"
    name, args, kw = _cases()[i]
    fast = getattr(B, name)(*args, **kw)
    slow = _without_fast_path(monkeypatch, name)(*args, **kw)
    if name == "cross_entropy_fwd":  # only the valid flat prefix is written (the rest is uninitialised)
        n_rows, n_cols = args[0].shape
        nv = n_rows * -(-n_cols // args[8])
        fast = tuple(t.reshape(-1)[:nv] for t in fast)
        slow = tuple(t.reshape(-1)[:nv] for t in slow)
    _same(fast, slow)
