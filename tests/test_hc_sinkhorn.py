"""hc_split_sinkhorn (track-02): the CPU oracle against the live reference's
golden vectors, and the CUDA kernel against both (GPU tests marked).

Tolerance: atol = 1e-5, rtol = 1e-4 on fp32 outputs, the reference's own
(track-02/test_correctness.py:17-18).
"""
import numpy as np
import pytest
import torch

import make_golden
from helpers import GOLDEN
from oracle.hc_sinkhorn_oracle import hc_split_sinkhorn_oracle

ATOL, RTOL = 1e-5, 1e-4
# track-02/workloads.py:21-26: decode and prefill shapes of the four scenarios
WORKLOAD_SHAPES = [(1, 1), (1, 16384), (16, 1), (16, 4096), (64, 1), (64, 1024)]


def load_hc_golden(name):
    args = make_golden.make_hc_case(name)
    z = np.load(GOLDEN / f"{name}.npz")
    assert str(z["digest"]) == make_golden.input_digest_hc(*args)
    return args, tuple(torch.from_numpy(z[k]) for k in ("pre", "post", "comb"))


@pytest.mark.parametrize("name", list(make_golden.HC_CASES))
def test_oracle_equals_reference_golden(name):
    args, gold = load_hc_golden(name)
    for a, e in zip(hc_split_sinkhorn_oracle(*args), gold):
        assert torch.equal(a, e)


def test_rows_and_columns_become_stochastic():
    args, _ = load_hc_golden("hc_ragged")
    _, _, comb = hc_split_sinkhorn_oracle(*args, sinkhorn_iters=60)
    assert torch.allclose(comb.sum(-1), torch.ones(comb.shape[:-1]), atol=1e-4)
    assert torch.allclose(comb.sum(-2), torch.ones(comb.shape[:-1]), atol=1e-4)


def _close(a, e, what):
    a, e = a.detach().cpu(), e.detach().cpu()
    assert a.shape == e.shape, (what, a.shape, e.shape)
    ok = (a - e).abs() <= ATOL + RTOL * e.abs()
    assert bool(ok.all()), f"{what}: max |d| = {(a - e).abs().max().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(make_golden.HC_CASES))
def test_kernel_matches_golden(name):
    from sparse_attn import hc_split_sinkhorn
    args, gold = load_hc_golden(name)
    outs = hc_split_sinkhorn(*[t.cuda() for t in args])
    for a, e, what in zip(outs, gold, ("pre", "post", "comb")):
        _close(a, e, f"{name} {what}")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", WORKLOAD_SHAPES)
def test_kernel_workload_shapes(shape):
    from sparse_attn import hc_split_sinkhorn
    g = torch.Generator().manual_seed(shape[0] * 7 + shape[1])
    mixes = torch.randn(*shape, 24, generator=g)
    sc, base = torch.randn(3, generator=g), torch.randn(24, generator=g)
    outs = hc_split_sinkhorn(mixes.cuda(), sc.cuda(), base.cuda(), 4, 20, 1e-6)
    for a, e, what in zip(outs, hc_split_sinkhorn_oracle(mixes, sc, base), ("pre", "post", "comb")):
        _close(a, e, f"{shape} {what}")


@pytest.mark.gpu
def test_kernel_strided_iters_eps_and_empty():
    from sparse_attn import hc_split_sinkhorn
    g = torch.Generator().manual_seed(3)
    big = torch.randn(5, 9, 40, generator=g)
    mixes = big[:, ::2, 8:32]  # token stride 80 elements, batch stride 360
    sc, base = torch.randn(3, generator=g), torch.randn(24, generator=g)
    for iters, eps in ((1, 1e-6), (7, 1e-3), (20, 0.0)):
        outs = hc_split_sinkhorn(big.cuda()[:, ::2, 8:32], sc.cuda(), base.cuda(), 4, iters, eps)
        ref = hc_split_sinkhorn_oracle(mixes, sc, base, 4, iters, eps)
        for a, e, what in zip(outs, ref, ("pre", "post", "comb")):
            _close(a, e, f"iters={iters} eps={eps} {what}")
    empty = hc_split_sinkhorn(torch.empty(2, 0, 24, device="cuda"), sc.cuda(), base.cuda())
    assert [tuple(t.shape) for t in empty] == [(2, 0, 4), (2, 0, 4), (2, 0, 4, 4)]


@pytest.mark.gpu
def test_dropin_and_errors():
    import importlib.util
    import pathlib
    path = pathlib.Path(__file__).resolve().parent.parent / "kernelgen-challenge_b200" / \
        "track02" / "submission.py"
    spec = importlib.util.spec_from_file_location("track02_submission", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    args, gold = load_hc_golden("hc_decode")
    outs = mod.hc_split_sinkhorn(*[t.cuda() for t in args], 4, 20, 1e-6)
    _close(outs[2], gold[2], "drop-in comb")
    with pytest.raises(AssertionError):
        mod.hc_split_sinkhorn(torch.zeros(1, 1, 15, device="cuda"), args[1].cuda(),
                              torch.zeros(15, device="cuda"), hc_mult=3)
    with pytest.raises(RuntimeError):
        mod.hc_split_sinkhorn(*args)  # CPU tensors: no CPU path
