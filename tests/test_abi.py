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
    assert _call(h=24) == _lib.SA_ERR_UNSUPPORTED  # more heads: multiples of 16 only
    assert _call(h=32, b=0) == _lib.SA_OK
    assert _call(h=32, q=8) == _lib.SA_ERR_INVALID_ARG  # each group is validated
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


def _i64(*v):
    return _lib.i64_array(list(v))


def test_fp8_entries_validate_before_any_gpu_work():
    L = _lib.lib()
    st = _i64(8192, 8192, 512, 1)

    def fwd8(q=16, kv8=16, ks=16, b=1, h=16, kv_strides=(2048, 512, 1)):
        return L.sa_fwd_fp8(q, kv8, ks, 16, 16, 16, b, 1, h, 512, 4, 4, st, _i64(*kv_strides),
                            _i64(4, 1), _i64(4, 4, 1), st, 1.0, None, 0, None, 0)
    assert fwd8(b=0) == _lib.SA_OK
    assert fwd8(b=-1) == _lib.SA_ERR_INVALID_ARG
    assert fwd8(h=8) == _lib.SA_ERR_UNSUPPORTED
    assert fwd8(h=40) == _lib.SA_ERR_UNSUPPORTED                   # more heads: multiples of 16
    assert fwd8(h=32, b=0) == _lib.SA_OK
    assert fwd8(h=32, kv8=8) == _lib.SA_ERR_INVALID_ARG
    assert fwd8(ks=0) == _lib.SA_ERR_INVALID_ARG
    assert fwd8(kv8=8) == _lib.SA_ERR_INVALID_ARG                  # misaligned rows
    assert fwd8(kv_strides=(2048, 520, 1)) == _lib.SA_ERR_INVALID_ARG  # row stride not 16 B

    def quant(kv=16, d=512, b=1):
        return L.sa_quantize_kv_fp8(kv, 16, 16, b, 4, d, _i64(2048, 512, 1), _i64(2048, 512, 1),
                                    _i64(4, 1), None)
    assert quant(b=0) == _lib.SA_OK
    assert quant(d=256) == _lib.SA_ERR_UNSUPPORTED
    assert quant(kv=0) == _lib.SA_ERR_INVALID_ARG


def test_backward_entry_validates_before_any_gpu_work():
    L = _lib.lib()
    st = _i64(8192, 8192, 512, 1)

    def bwd(dq=16, dkv=16, b=1, h=16, dkv_strides=(2048, 512, 1)):
        return L.sa_bwd(16, 16, 16, 16, 16, 16, None, dq, dkv, 16, b, 1, h, 512, 4, 4, st,
                        _i64(2048, 512, 1), _i64(4, 4, 1), st, _i64(*dkv_strides), 1.0, None)
    assert bwd(b=0) == _lib.SA_OK
    assert bwd(h=4) == _lib.SA_ERR_UNSUPPORTED
    assert bwd(h=24) == _lib.SA_ERR_UNSUPPORTED
    assert bwd(h=48, b=0) == _lib.SA_OK
    assert bwd(h=48, dq=0) == _lib.SA_ERR_INVALID_ARG
    assert bwd(h=48, dkv=4) == _lib.SA_ERR_INVALID_ARG
    assert bwd(dq=0) == _lib.SA_ERR_INVALID_ARG
    assert bwd(dkv=4) == _lib.SA_ERR_INVALID_ARG                   # misaligned fp32 buffer
    assert bwd(dkv_strides=(2048, 511, 1)) == _lib.SA_ERR_INVALID_ARG


def test_dkv_row_entries_validate_before_any_gpu_work():
    L = _lib.lib()
    ist, dst = _i64(8, 4, 1), _i64(2048, 512, 1)

    def zero(dkv=16, b=1, topk=4, strides=(2048, 512, 1)):
        return L.sa_dkv_zero_rows(dkv, 16, b, 1, topk, 4, ist, _i64(*strides), None)

    def cast(out=16, strides=(2048, 512, 1)):
        return L.sa_dkv_cast_rows(16, out, 16, 1, 1, 4, 4, ist, dst, _i64(*strides), None)
    assert zero(b=0) == _lib.SA_OK and zero(topk=0) == _lib.SA_OK
    assert zero(b=-1) == _lib.SA_ERR_INVALID_ARG
    assert zero(dkv=0) == _lib.SA_ERR_INVALID_ARG
    assert zero(dkv=8) == _lib.SA_ERR_INVALID_ARG                   # fp32 rows 16-byte aligned
    assert zero(strides=(2048, 510, 1)) == _lib.SA_ERR_INVALID_ARG
    assert zero(strides=(2048, 512, 2)) == _lib.SA_ERR_INVALID_ARG
    assert cast(out=0) == _lib.SA_ERR_INVALID_ARG
    assert cast(out=4) == _lib.SA_ERR_INVALID_ARG                   # bf16 rows 8-byte aligned
    assert cast(strides=(2048, 514, 1)) == _lib.SA_ERR_INVALID_ARG


def test_sinkhorn_entry_validates_before_any_gpu_work():
    L = _lib.lib()

    def hcs(n=1, hc=4, iters=20, mixes=16, stride=24, out=16):
        return L.hcs_split_sinkhorn(mixes, 16, 16, out, 16, 16, n, stride, hc, iters, 1e-6, None)
    assert hcs(n=0) == 0
    assert hcs(n=-1) == -1
    assert hcs(hc=3) == -4
    assert hcs(iters=0) == -1
    assert hcs(mixes=0) == -1
    assert hcs(stride=23) == -1
    assert hcs(out=8) == -1                                          # misaligned outputs


def test_new_ops_reject_cpu_tensors():
    q = torch.zeros(1, 1, 16, 512, dtype=torch.bfloat16)
    kv = torch.zeros(1, 4, 512, dtype=torch.bfloat16)
    sink = torch.zeros(16)
    idx = torch.zeros(1, 1, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_attn.sparse_attn_fp8(q, kv.to(torch.float8_e4m3fn), torch.ones(1, 4), sink, idx, 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_attn.quantize_kv_fp8(kv)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_attn.sparse_attn_backward(q, kv, sink, idx, 0.1, q, q)
    with pytest.raises(AssertionError):
        sparse_attn.hc_split_sinkhorn(torch.zeros(1, 1, 15), torch.zeros(3), torch.zeros(15),
                                      hc_mult=3)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_attn.hc_split_sinkhorn(torch.zeros(1, 1, 24), torch.zeros(3), torch.zeros(24))


def test_options_round_trip_on_the_host():
    """sa_set_option / sa_get_option need no GPU: every option keeps the value
    set, rejects values outside its range, and the defaults come back."""
    lib = _lib.lib()
    cases = {
        _lib.SA_OPT_ROW_SCHEDULE: (0, 2),
        _lib.SA_OPT_INDEXER_TC: (0, -1),
        _lib.SA_OPT_TEST_STALL: (1, 2),
        _lib.SA_OPT_KV_POLICY: (2, 3),
        _lib.SA_OPT_GATHER_ONLY: (1, 5),
        _lib.SA_OPT_HEAD_GROUPS: (0, 2),
    }
    for opt, (good, bad) in cases.items():
        old = lib.sa_get_option(opt)
        try:
            assert lib.sa_set_option(opt, good) == _lib.SA_OK
            assert lib.sa_get_option(opt) == good
            assert lib.sa_set_option(opt, bad) == _lib.SA_ERR_INVALID_ARG
            assert lib.sa_get_option(opt) == good
        finally:
            assert lib.sa_set_option(opt, old) == _lib.SA_OK
    assert lib.sa_get_option(_lib.SA_OPT_HEAD_GROUPS) == 1
    assert lib.sa_get_option(99) == -1
    assert lib.sa_set_option(99, 0) == _lib.SA_ERR_INVALID_ARG
