"""The C restatement ``sa_fwd_host`` (oracle/sa_host.c) against the golden
vectors of the live reference and against the torch oracle (CPU only)."""
import ctypes

import pytest
import torch

import make_golden
from helpers import load_golden
from oracle.sa_host import host_lib, sparse_attn_host
from oracle.sparse_attn_oracle import sparse_attn_oracle

# One bf16 ulp of the expected value, or 3e-5 absolute: outputs below ~1e-5
# come from cancellation in fp32 sums taken in another order (torch's einsum
# vs the C loop), where a bf16 ulp is far below the summation error.
ATOL_TINY = 3e-5


def assert_ulp_close(a, b):
    g = b.float()
    ulp = torch.exp2(torch.floor(torch.log2(g.abs().clamp_min(1e-30))) - 7)
    d = (a.float() - g).abs()
    bad = d > torch.maximum(ulp, torch.full_like(ulp, ATOL_TINY))
    assert not bool(bad.any()), f"{int(bad.sum())} elements beyond one ulp, max {d.max():.3e}"


def test_version():
    assert host_lib().sa_host_version() == 1


@pytest.mark.parametrize("name", make_golden.CASES)
def test_host_matches_golden(name):
    args, o_gold = load_golden(name)
    assert_ulp_close(sparse_attn_host(*args), o_gold)


def test_host_matches_torch_oracle_with_duplicates_and_masks():
    g = torch.Generator().manual_seed(7)
    b, m, h, d, kv_len, topk = 2, 5, 16, 512, 300, 90
    q = torch.randn(b, m, h, d, generator=g).bfloat16()
    kv = torch.randn(b, kv_len, d, generator=g).bfloat16()
    sink = torch.randn(h, generator=g)
    idx = torch.randint(-3, kv_len + 20, (b, m, topk), generator=g, dtype=torch.int32)
    idx[1, 2] = -1  # one row with no valid slot: o = 0
    o = sparse_attn_host(q, kv, sink, idx, 0.05)
    assert_ulp_close(o, sparse_attn_oracle(q, kv, sink, idx, 0.05))
    assert bool((o[1, 2] == 0).all())


def test_host_strided_inputs_and_thread_count():
    args, o_gold = load_golden("ragged")
    q, kv, sink, idx, scale = args
    qs = torch.zeros(q.shape[0], q.shape[1], q.shape[2], 2 * q.shape[3], dtype=q.dtype)
    qs[..., ::2] = q  # last-dimension stride 2
    kvt = kv.transpose(1, 2).contiguous().transpose(1, 2)  # column-major rows
    a = sparse_attn_host(qs[..., ::2], kvt, sink, idx, scale, num_threads=1)
    b = sparse_attn_host(q, kv, sink, idx, scale, num_threads=3)
    assert torch.equal(a, b)  # same per-row arithmetic whatever the layout or threads
    assert_ulp_close(a, o_gold)


def test_host_empty_and_invalid():
    lib = host_lib()
    z = (ctypes.c_int64 * 4)(0, 0, 0, 0)
    assert lib.sa_fwd_host(None, None, None, None, None, 0, 4, 16, 512, 8, 8, z, z, z, z,
                           1.0, 0) == 0
    assert lib.sa_fwd_host(None, None, None, None, None, 1, 1, 16, 512, 8, 8, z, z, z, z,
                           1.0, 0) == -1
    assert lib.sa_fwd_host(None, None, None, None, None, 1, 1, 0, 512, 8, 8, z, z, z, z,
                           1.0, 0) == -1


def test_every_host_header_symbol_is_exported():
    import pathlib
    import re
    hdr = pathlib.Path(__file__).resolve().parent.parent / "include" / "sparse_attn_host.h"
    text = re.sub(r"/\*.*?\*/", "", hdr.read_text(), flags=re.S)
    names = sorted(set(re.findall(r"\b(sa_[a-z_]+)\s*\(", text)))
    assert names == ["sa_fwd_host", "sa_host_version"]
    for n in names:
        assert hasattr(host_lib(), n), n


def test_product_library_has_no_host_path():
    """libsparse_attn.so exports no CPU compute entry: the host restatement
    lives only in the oracle's own library."""
    import ctypes as C

    from sparse_attn import _lib
    prod = C.CDLL(str(_lib.LIB_PATH))
    assert not hasattr(prod, "sa_fwd_host")
