"""The backward pass (``sa_bwd``) against autograd of the fp32 CPU oracle.

The reference has no backward; the check is the gradient of its forward.
Tolerance: |g - g_ref| <= 1e-2 * max|g_ref| + 2e-2 * |g_ref| elementwise (bf16
products and a bf16 o in the D = dO.o term, fp32 accumulation throughout).
"""
import pytest
import torch

import make_golden
from helpers import load_golden
from oracle.sparse_attn_oracle import sparse_attn_oracle_grads
from sparse_attn import sparse_attn, sparse_attn_backward
from sparse_attn.workloads import make_inputs

pytestmark = pytest.mark.gpu


def _close(a, e, what):
    a, e = a.detach().float().cpu(), e.detach().float().cpu()
    assert a.shape == e.shape, (what, a.shape, e.shape)
    assert torch.isfinite(a).all(), what
    tol = 1e-2 * e.abs().max().clamp_min(1e-6) + 2e-2 * e.abs()
    bad = (a - e).abs() > tol
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} of {bad.numel()} outside; "
                                 f"max |d| = {(a - e).abs().max():.3e}, max |ref| = {e.abs().max():.3e}")


def _check(q, kv, sink, idx, scale, seed=0, what=""):
    g = torch.Generator().manual_seed(seed)
    do = torch.randn(q.shape, generator=g).to(torch.bfloat16)
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    o = sparse_attn(qc, kvc, sc, ic, scale)
    dq, dkv, dsink = sparse_attn_backward(qc, kvc, sc, ic, scale, o, do.cuda())
    torch.cuda.synchronize()
    _, rq, rkv, rs = sparse_attn_oracle_grads(q, kv, sink, idx, scale, do)
    _close(dq, rq, f"{what} dq")
    _close(dkv, rkv, f"{what} dkv")
    _close(dsink, rs, f"{what} dsink")


@pytest.mark.parametrize("name", ["plumbing", "ragged", "replacement", "masked", "out_of_range",
                                  "short"])
def test_backward_golden_inputs(name):
    args, _ = load_golden(name)
    _check(*args, what=name)


def test_backward_decode_rows():
    q, kv, sink, idx, scale = make_inputs("decode", seed=3, b=4)
    _check(q, kv, sink, idx, scale, seed=1, what="decode b=4")


def test_backward_causal_head():
    args = make_golden.make_case("causal_head")
    _check(*args, seed=2, what="causal rows 0-39")


def test_backward_fewer_heads():
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=6)
    _check(q[:, :, :5].contiguous(), kv, sink[:5].contiguous(), idx, scale, what="h=5")


def test_autograd_through_the_op():
    """sparse_attn records for autograd when an input requires grad; the
    gradients are sa_bwd's."""
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=8)
    qc = q.cuda().requires_grad_(True)
    kvc = kv.cuda().requires_grad_(True)
    sc = sink.cuda().requires_grad_(True)
    ic = idx.cuda()
    o = sparse_attn(qc, kvc, sc, ic, scale)
    do = torch.randn(o.shape, generator=torch.Generator().manual_seed(4)).to(o.dtype).cuda()
    o.backward(do)
    dq, dkv, dsink = sparse_attn_backward(qc.detach(), kvc.detach(), sc.detach(), ic, scale,
                                          o.detach(), do)
    # dq has no atomics: identical; dkv and dsink are sums by atomics, whose
    # order varies between runs
    assert torch.equal(qc.grad, dq)
    _close(kvc.grad, dkv, "autograd dkv")
    _close(sc.grad, dsink, "autograd dsink")
