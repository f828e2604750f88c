"""ctypes front of the C restatement ``sa_fwd_host`` (``oracle/sa_host.c``).

TEST INFRASTRUCTURE ONLY (tests, smoke checks and bench.py's CPU legs).
``sparse_attn_host`` takes and returns CPU torch tensors with the reference's
signature (``track-01/reference/reference.py:10``).
"""
from __future__ import annotations

import ctypes
import functools

import torch

from .build_host import OUT, build_host

__all__ = ["sparse_attn_host", "host_lib"]

_I64P = ctypes.POINTER(ctypes.c_int64)


@functools.lru_cache(maxsize=1)
def host_lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build_host() if not OUT.exists() else OUT))
    lib.sa_host_version.restype = ctypes.c_int
    lib.sa_fwd_host.restype = ctypes.c_int
    lib.sa_fwd_host.argtypes = ([ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6 + [_I64P] * 4
                                + [ctypes.c_float, ctypes.c_int])
    return lib


def _strides(t: torch.Tensor):
    return (ctypes.c_int64 * t.dim())(*t.stride())


def sparse_attn_host(q, kv, attn_sink, topk_idxs, scale, num_threads: int = 0):
    """o = sa_fwd_host(...) on CPU tensors (any strides); returns bf16 [b,m,h,d]."""
    q, kv, topk_idxs = q.cpu(), kv.cpu(), topk_idxs.cpu()
    sink = attn_sink.cpu().float().contiguous()
    assert q.dtype == torch.bfloat16 and kv.dtype == torch.bfloat16
    assert topk_idxs.dtype == torch.int32
    b, m, h, d = q.shape
    o = torch.empty(b, m, h, d, dtype=torch.bfloat16)
    rc = host_lib().sa_fwd_host(q.data_ptr(), kv.data_ptr(), sink.data_ptr(),
                                topk_idxs.data_ptr(), o.data_ptr(), b, m, h, d, kv.shape[1],
                                topk_idxs.shape[-1], _strides(q), _strides(kv),
                                _strides(topk_idxs), _strides(o), float(scale), int(num_threads))
    if rc != 0:
        raise RuntimeError(f"sa_fwd_host failed: {rc}")
    return o
