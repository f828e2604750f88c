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
from sparse_attn.op import _forward_train
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


def test_backward_touched_rows_only():
    """m * topk < kv_len: the fp32 gradient is zeroed and cast on the rows the
    valid slots name only.  Duplicated, -1 and out-of-range indices, a fully
    masked row; every row no valid slot names is exactly zero."""
    g = torch.Generator().manual_seed(7)
    b, m, kv_len, topk, scale = 3, 2, 5000, 700, 512 ** -0.5
    q = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    idx[0, 0, 10:20] = idx[0, 0, 0]   # duplicates
    idx[1, 1, 5:50] = -1
    idx[2, 0, 7] = kv_len + 3         # out of range: masked
    idx[2, 1] = -1                    # no valid slot
    assert m * topk < kv_len
    _check(q, kv, sink, idx, scale, seed=2, what="touched rows")
    do = torch.randn(q.shape, generator=g).to(torch.bfloat16).cuda()
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    _, dkv, _ = sparse_attn_backward(qc, kvc, sc, ic, scale, sparse_attn(qc, kvc, sc, ic, scale), do)
    touched = torch.zeros(b, kv_len, dtype=torch.bool)
    for bi in range(b):
        v = idx[bi].reshape(-1)
        v = v[(v >= 0) & (v < kv_len)].long()
        touched[bi, v] = True
    assert dkv.dtype == torch.bfloat16
    assert not dkv.cpu()[~touched].any()


def test_backward_causal_head():
    args = make_golden.make_case("causal_head")
    _check(*args, seed=2, what="causal rows 0-39")


def test_backward_fewer_heads():
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=6)
    _check(q[:, :, :5].contiguous(), kv, sink[:5].contiguous(), idx, scale, what="h=5")


@pytest.mark.parametrize("h", [32, 40])
def test_backward_more_heads(h):
    """h > 16: the groups of 16 heads each add into dkv; dq and dsink per head
    (h = 40 pads to 48)."""
    g = torch.Generator().manual_seed(30 + h)
    b, m, kv_len, topk = 2, 24, 500, 256
    q = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(h, generator=g)
    idx = torch.randint(-1, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    _check(q, kv, sink, idx, 512 ** -0.5, seed=h, what=f"h={h}")


def test_training_forward_more_heads_lse():
    """The training forward's lse [b, m, h] for h = 48 gives the one-pass
    backward the same gradients as the two-pass one."""
    g = torch.Generator().manual_seed(77)
    b, m, h, kv_len, topk = 1, 64, 48, 800, 512
    q = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16).cuda()
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16).cuda()
    sink = torch.randn(h, generator=g).cuda()
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32).cuda()
    do = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16).cuda()
    scale = 512 ** -0.5
    o, lse = _forward_train(q, kv, sink, idx, scale)
    assert lse.shape == (b, m, h)
    # (the inference call may merge split rows in another order: equal within
    # the parity tolerance, not bit for bit)
    from helpers import assert_close
    assert_close(o, sparse_attn(q, kv, sink, idx, scale), what="training vs inference forward")
    one = sparse_attn_backward(q, kv, sink, idx, scale, o, do, lse)
    two = sparse_attn_backward(q, kv, sink, idx, scale, o, do)
    for a, e, what in zip(one, two, ("dq", "dkv", "dsink")):
        _close(a, e, f"one-pass vs two-pass {what}")


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
    # the autograd path runs the training forward and the one-pass backward;
    # compare with the two-pass backward (bf16 rounding of dq may differ)
    dq, dkv, dsink = sparse_attn_backward(qc.detach(), kvc.detach(), sc.detach(), ic, scale,
                                          o.detach(), do)
    _close(qc.grad, dq, "autograd dq")
    _close(kvc.grad, dkv, "autograd dkv")
    _close(sc.grad, dsink, "autograd dsink")
    _, rq, rkv, rs = sparse_attn_oracle_grads(q, kv, sink, idx, scale, do.cpu())
    _close(qc.grad, rq, "autograd dq vs oracle")
    _close(kvc.grad, rkv, "autograd dkv vs oracle")
    _close(sc.grad, rs, "autograd dsink vs oracle")


def _ref_lse2(q, kv, sink, idx, scale):
    """log2 of each row's full softmax denominator (sink included), fp64 CPU."""
    b, m, h, d = q.shape
    valid = (idx >= 0) & (idx < kv.shape[1])
    safe = torch.where(valid, idx, torch.zeros_like(idx)).long()
    g = torch.gather(kv.double(), 1, safe.reshape(b, -1, 1).expand(-1, -1, d)).reshape(b, m, -1, d)
    s = torch.einsum("bmhd,bmtd->bmht", q.double(), g) * scale
    s = s.masked_fill(~valid.unsqueeze(2), float("-inf"))
    full = torch.cat([s, sink.double()[None, None, :, None].expand(b, m, h, 1)], -1)
    return torch.logsumexp(full, -1) / torch.log(torch.tensor(2.0, dtype=torch.float64))


@pytest.mark.parametrize("name", ["plumbing", "masked", "ragged"])
def test_training_forward_lse_and_one_pass_backward(name):
    """sa_fwd_train: the same o as sa_fwd and the row log-sum-exp; the
    backward given it (one pass) matches the two-pass backward."""
    from sparse_attn.op import _forward_train
    (q, kv, sink, idx, scale), _ = load_golden(name)
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    o_t, lse = _forward_train(qc, kvc, sc, ic, scale)
    o = sparse_attn(qc, kvc, sc, ic, scale)
    from helpers import assert_close
    assert_close(o_t, o, what="training vs inference forward")
    ref = _ref_lse2(q, kv, sink, idx, scale).float()
    assert torch.allclose(lse.cpu(), ref, atol=2e-3, rtol=1e-4), (lse.cpu() - ref).abs().max()
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    g1 = sparse_attn_backward(qc, kvc, sc, ic, scale, o, do, lse)
    g2 = sparse_attn_backward(qc, kvc, sc, ic, scale, o, do)
    for a, e, what in zip(g1, g2, ("dq", "dkv", "dsink")):
        _close(a, e, f"{name} one-pass vs two-pass {what}")


@pytest.mark.parametrize("b,h", [(4, 16), (8, 16), (3, 32), (70, 16)])
def test_one_pass_backward_with_split_rows(b, h):
    """Decode rows with the log-sum-exp: when the rows are fewer than half the
    SMs, each row's slots run as several parts on separate CTAs, dq added
    through an fp32 scratch (b = 70 stays unsplit).  Against autograd of the
    oracle, with masked and duplicated slots."""
    from sparse_attn.op import _forward_train
    q, kv, sink, idx, scale = make_inputs("decode", seed=11, b=b)
    if h != 16:
        q = q.repeat(1, 1, h // 16, 1).contiguous()
        sink = sink.repeat(h // 16).contiguous()
    idx[0, 0, 100:400] = -1
    idx[b - 1, 0, 5:9] = idx[b - 1, 0, 0]
    g = torch.Generator().manual_seed(4)
    do = torch.randn(q.shape, generator=g).to(torch.bfloat16)
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    o, lse = _forward_train(qc, kvc, sc, ic, scale)
    dq, dkv, dsink = sparse_attn_backward(qc, kvc, sc, ic, scale, o, do.cuda(), lse)
    torch.cuda.synchronize()
    _, rq, rkv, rs = sparse_attn_oracle_grads(q, kv, sink, idx, scale, do)
    _close(dq, rq, f"b={b} h={h} dq")
    _close(dkv, rkv, f"b={b} h={h} dkv")
    _close(dsink, rs, f"b={b} h={h} dsink")
