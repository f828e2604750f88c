"""The allocation-free entry point ``sa_fwd_noalloc`` (GPU).

Callers that cannot allocate device memory (a host framework that owns every
allocation, a serving loop reserved up front) use ``sa_fwd_noalloc``, which
keeps its scratch in a fixed device array inside the library instead of a
caller workspace.  This test calls it through the C ABI twice in a row, on
two different inputs, and compares each result with the regular ``sa_fwd``
path.  It lives in its own file, collected last, and passes alone or after
the other tests.
"""
import ctypes

import pytest
import torch

from helpers import assert_close
from sparse_attn import _lib, sparse_attn_out
from sparse_attn.workloads import make_inputs

pytestmark = pytest.mark.gpu


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


def test_noalloc_matches_sa_fwd_twice():
    for seed in (0, 1):  # decode shape: rows are split across CTAs -> scratch used
        q, kv, sink, idx, scale = [t.cuda() if torch.is_tensor(t) else t
                                   for t in make_inputs("decode", seed=seed)]
        rc, o = _noalloc(q, kv, sink, idx, scale)
        torch.cuda.synchronize()
        _lib.check(rc)
        ref = torch.empty_like(q)
        sparse_attn_out(ref, q, kv, sink, idx, scale)
        torch.cuda.synchronize()
        assert_close(o, ref, what=f"noalloc seed={seed}")


def test_noalloc_rejects_grid_beyond_scratch():
    q, kv, sink, idx, scale = [t.cuda() if torch.is_tensor(t) else t
                               for t in make_inputs("plumbing", seed=0)]
    rc, _ = _noalloc(q, kv, sink, idx, scale, grid=161)
    assert rc == _lib.SA_ERR_WORKSPACE
