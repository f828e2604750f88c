"""Shared test helpers: golden loading and the parity comparison."""
from __future__ import annotations

import pathlib

import numpy as np
import torch

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"

# BASELINE tolerance on the bf16 output (stricter than the reference's 5e-2 at
# track-01/test_correctness.py:18-19)
ATOL = 2e-2
RTOL = 2e-2


def load_golden(name):
    import make_golden
    q, kv, sink, idx, scale = make_golden.make_case(name)
    z = np.load(GOLDEN / f"{name}.npz")
    assert str(z["digest"]) == make_golden.input_digest(q, kv, sink, idx, scale), \
        f"golden inputs of {name!r} no longer reproduce (generator drift)"
    o = torch.from_numpy(z["o"]).view(torch.bfloat16)
    return (q, kv, sink, idx, scale), o


def assert_close(actual, expected, atol=ATOL, rtol=RTOL, what=""):
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    assert a.shape == e.shape, (a.shape, e.shape)
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    diff = (a - e).abs()
    ok = diff <= atol + rtol * e.abs()
    if not bool(ok.all()):
        bad = (~ok).sum().item()
        raise AssertionError(f"{what}: {bad} of {ok.numel()} elements outside "
                             f"atol={atol} rtol={rtol}; max|d|={diff.max().item():.3e}")
    return diff.max().item()


def load_golden_fp8(name):
    import make_golden
    args = make_golden.make_fp8_case(name)
    z = np.load(GOLDEN / f"{name}.npz")
    assert str(z["digest"]) == make_golden.input_digest_fp8(*args), \
        f"golden inputs of {name!r} no longer reproduce (generator drift)"
    return args, torch.from_numpy(z["o"]).view(torch.bfloat16)
