"""The C-ABI library loads and exports every symbol the header declares (CPU).

No compute call is made here: only entry points that fail before touching
the GPU (argument validation) or need no GPU at all.
"""
import ctypes
import pathlib
import re

import pytest
import torch

import sparse_attn
from sparse_attn import _lib

INCLUDE = pathlib.Path(__file__).resolve().parent.parent / "include"
# headers of libsparse_attn.so (sparse_attn_host.h belongs to the oracle's library)
HEADERS = [INCLUDE / "sparse_attn.h", INCLUDE / "hc_sinkhorn.h"]


def declared_functions():
    names = set()
    for hdr in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", hdr.read_text(), flags=re.S)
        names |= set(re.findall(r"\b((?:sa|hcs)_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_builds_and_loads():
    assert _lib.LIB_PATH.exists()
    assert _lib.lib().sa_version() >= 10000


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert "sa_fwd" in names and len(names) >= 6
    h = ctypes.CDLL(str(_lib.LIB_PATH))
    for n in names:
        assert hasattr(h, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_strerror_codes():
    for code in (0, -1, -2, -3, -4):
        assert _lib.strerror(code)
    assert "unknown" in _lib.strerror(-99)


def _call(**over):
    L = _lib.lib()
    a = dict(q=16, kv=16, sink=16, idx=16, o=16, b=1, m=1, h=16, d=512, kv_len=8, topk=4)
    a.update(over)
    st = _lib.i64_array([8192, 8192, 512, 1])
    return L.sa_fwd(a["q"], a["kv"], a["sink"], a["idx"], a["o"], a["b"], a["m"], a["h"], a["d"],
                    a["kv_len"], a["topk"], st, _lib.i64_array([4096, 512, 1]),
                    _lib.i64_array([4, 4, 1]), st, 1.0, None, 0, None)


def test_validation_before_any_gpu_work():
    assert _call(b=-1) == _lib.SA_ERR_INVALID_ARG
    assert _call(h=8) == _lib.SA_ERR_UNSUPPORTED
    assert _call(d=256) == _lib.SA_ERR_UNSUPPORTED
    assert _call(b=0) == _lib.SA_OK           # empty problem: nothing to do
    assert _call(q=0) == _lib.SA_ERR_INVALID_ARG
    assert _call(q=8) == _lib.SA_ERR_INVALID_ARG  # misaligned row


def test_op_rejects_cpu_tensors_and_bad_rank():
    q = torch.zeros(1, 1, 16, 512, dtype=torch.bfloat16)
    kv = torch.zeros(1, 4, 512, dtype=torch.bfloat16)
    sink = torch.zeros(16)
    idx = torch.zeros(1, 1, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_attn.sparse_attn(q, kv, sink, idx, 0.1)
    with pytest.raises(AssertionError):
        sparse_attn.sparse_attn(q[0], kv, sink, idx, 0.1)
