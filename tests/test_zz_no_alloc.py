"""The allocation-free entry point ``sa_fwd_noalloc`` (GPU).

Callers that cannot allocate device memory (a host framework that owns every
allocation, a serving loop reserved up front) use ``sa_fwd_noalloc``, which
keeps its scratch in a fixed device array inside the library instead of a
caller workspace.  These tests call it through the C ABI: twice in a row on
two inputs against the regular ``sa_fwd`` path, and on the shapes that use the
array differently -- decode (split rows merged by the combine kernel), prefill
with the row schedule (per-row counts in the array), prefill at the largest
grid (split rows merged in the kernel through the ticket words at the array's
start) and 32 heads (two head groups reusing the array one after the other)
-- against the CPU oracle.  The file is collected last and passes alone or
after the other tests.
"""
import ctypes

import pytest
import torch

from helpers import assert_close
from oracle.sparse_attn_oracle import sparse_attn_oracle
from sparse_attn import _lib, sparse_attn_out
from sparse_attn.workloads import make_inputs

pytestmark = pytest.mark.gpu

MAX_CTAS = 160  # SA_NOALLOC_MAX_CTAS


def _noalloc(q, kv, sink, idx, scale, grid=0):
    o = torch.empty_like(q)
    L = _lib.lib()
    b, m, h, d = q.shape
    rc = L.sa_fwd_noalloc(
        q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), o.data_ptr(),
        b, m, h, d, kv.shape[1], idx.shape[-1],
        _lib.i64_array(q.stride()), _lib.i64_array(kv.stride()),
        _lib.i64_array(idx.stride()), _lib.i64_array(o.stride()), float(scale),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), grid)
    return rc, o


def _cuda(args):
    return [t.cuda() if torch.is_tensor(t) else t for t in args]


def test_noalloc_matches_sa_fwd_twice():
    for seed in (0, 1):  # decode shape: rows are split across CTAs -> scratch used
        q, kv, sink, idx, scale = _cuda(make_inputs("decode", seed=seed))
        rc, o = _noalloc(q, kv, sink, idx, scale)
        torch.cuda.synchronize()
        _lib.check(rc)
        ref = torch.empty_like(q)
        sparse_attn_out(ref, q, kv, sink, idx, scale)
        torch.cuda.synchronize()
        assert_close(o, ref, what=f"noalloc seed={seed}")


@pytest.mark.parametrize("grid", [0, MAX_CTAS])
def test_noalloc_prefill_vs_oracle(grid):
    """grid 0: row schedule (per-row counts after the partials); grid 160: no
    room left for them, so split rows merge in the kernel by ticket.  Two calls
    each: the second finds the tickets the first left behind."""
    args = make_inputs("causal", seed=2, m=600)
    ref = sparse_attn_oracle(*args)
    q, kv, sink, idx, scale = _cuda(args)
    for _ in range(2):
        rc, o = _noalloc(q, kv, sink, idx, scale, grid=grid)
        torch.cuda.synchronize()
        _lib.check(rc)
        assert_close(o, ref, what=f"noalloc prefill grid={grid}")


def test_noalloc_two_head_groups_vs_oracle():
    g = torch.Generator().manual_seed(8)
    b, m, h, kv_len, topk = 8, 3, 32, 2000, 700
    q = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(h, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    idx[:, :, 650:] = -1
    ref = sparse_attn_oracle(q, kv, sink, idx, 512 ** -0.5)
    rc, o = _noalloc(*_cuda((q, kv, sink, idx, 512 ** -0.5)))
    torch.cuda.synchronize()
    _lib.check(rc)
    assert_close(o, ref, what="noalloc h=32")


def test_noalloc_rejects_grid_beyond_scratch():
    q, kv, sink, idx, scale = _cuda(make_inputs("plumbing", seed=0))
    rc, _ = _noalloc(q, kv, sink, idx, scale, grid=MAX_CTAS + 1)
    assert rc == _lib.SA_ERR_WORKSPACE
