"""The fp8 (e4m3) KV-cache path on the GPU: quantiser bit-exact against its
CPU statement, attention against the oracle on the dequantised cache and
against the live reference's golden outputs on that cache.

Tolerance: atol = rtol = 2e-2 on the bf16 output, as for the bf16 path.  The
kernel widens the e4m3 K/V to f16 in registers (exact) and runs f16 MMAs with
f16 Q (scaled per head by a power of two) and f16 P, so its error budget is at
most the bf16 kernels'.  The K/V quantisation is not an error here: the
oracle uses the same e4m3 values.
"""
import pytest
import torch

import make_golden
from helpers import assert_close, load_golden_fp8
from oracle.sparse_attn_oracle import quantize_kv_fp8_ref, sparse_attn_fp8_oracle
from sparse_attn import quantize_kv_fp8, sparse_attn_fp8, sparse_attn_fp8_out
from sparse_attn.workloads import make_inputs

pytestmark = pytest.mark.gpu


def _cuda(*ts):
    return [t.cuda() if torch.is_tensor(t) else t for t in ts]


def run_fp8(q, kv8, ks, sink, idx, scale, grid=0):
    q, kv8, ks, sink, idx = _cuda(q, kv8, ks, sink, idx)
    o = torch.empty_like(q)
    sparse_attn_fp8_out(o, q, kv8, ks, sink, idx, scale, grid=grid)
    torch.cuda.synchronize()
    return o


def _assert_same_bytes(a, b, what):
    a, b = a.view(torch.uint8), b.view(torch.uint8)
    bad = (a != b).nonzero()
    assert bad.numel() == 0, (
        f"{what}: {bad.shape[0]} bytes differ; first {bad[:5].tolist()}: "
        f"gpu {[int(a[tuple(i)]) for i in bad[:5].tolist()]} "
        f"cpu {[int(b[tuple(i)]) for i in bad[:5].tolist()]}")


def test_quantiser_bit_exact():
    g = torch.Generator().manual_seed(9)
    kv = (torch.randn(3, 257, 512, generator=g) *
          torch.logspace(-4, 4, 257).view(1, 257, 1)).to(torch.bfloat16)
    kv[2, 100] = 0
    kv[1, 5, 17] = 3.0e38  # a huge value in a row: still saturates to 448 at most
    ref8, ref_s = quantize_kv_fp8_ref(kv)
    kv8, s = quantize_kv_fp8(kv.cuda())
    torch.cuda.synchronize()
    _assert_same_bytes(kv8.cpu(), ref8, "kv8")
    _assert_same_bytes(s.cpu(), ref_s, "scales")


def test_quantiser_strided_and_out_buffers():
    g = torch.Generator().manual_seed(10)
    big = torch.randn(2, 64, 1024, generator=g).to(torch.bfloat16).cuda()
    kv = big[:, :, 256:768]  # row stride 1024 elements
    out = torch.empty(2, 64, 2048, dtype=torch.float8_e4m3fn, device="cuda")[:, :, :512]
    sc = torch.empty(64, 2, device="cuda").t()  # strided scales
    quantize_kv_fp8(kv, out=out, scale_out=sc)
    ref8, ref_s = quantize_kv_fp8_ref(kv.cpu())
    _assert_same_bytes(out.cpu().contiguous(), ref8, "strided kv8")
    _assert_same_bytes(sc.cpu().contiguous(), ref_s, "strided scales")


@pytest.mark.parametrize("name", make_golden.FP8_CASES)
@pytest.mark.parametrize("grid", [0, 1, 3, 37])
def test_fp8_golden(name, grid):
    args, o_gold = load_golden_fp8(name)
    o = run_fp8(*args, grid=grid)
    assert_close(o, o_gold, what=f"{name} grid={grid}")
    if name == "fp8_masked":
        assert torch.count_nonzero(o[0, 1]) == 0 and torch.count_nonzero(o[1, 4]) == 0


def _fp8_inputs(config, seed, rows=None):
    q, kv, sink, idx, scale = make_inputs(config, seed=seed)
    kv8, ks = quantize_kv_fp8_ref(kv)
    return q, kv8, ks, sink, idx, scale


def test_fp8_decode_full():
    q, kv8, ks, sink, idx, scale = _fp8_inputs("decode", 1)
    o = run_fp8(q, kv8, ks, sink, idx, scale)
    assert_close(o, sparse_attn_fp8_oracle(q, kv8, ks, sink, idx, scale), what="fp8 decode")


def test_fp8_causal_sampled_rows():
    q, kv8, ks, sink, idx, scale = _fp8_inputs("causal", 2)
    o = run_fp8(q, kv8, ks, sink, idx, scale)
    rows = torch.tensor([0, 1, 2, 3, 63, 64, 65, 127, 511, 1000, 2047, 2048, 3000, 4095])
    ref = sparse_attn_fp8_oracle(q[:, rows], kv8, ks, sink, idx[:, rows], scale)
    assert_close(o[:, rows.cuda()], ref, what="fp8 causal")


def test_fp8_public_op_and_gpu_quantiser_agree_with_oracle():
    """Quantise on the GPU, attend through the public op."""
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=4)
    kv8, ks = quantize_kv_fp8(kv.cuda())
    o = sparse_attn_fp8(q.cuda(), kv8, ks, sink.cuda(), idx.cuda(), scale)
    ref = sparse_attn_fp8_oracle(q, kv8.cpu(), ks.cpu(), sink, idx, scale)
    assert_close(o, ref, what="fp8 op")
    # and the fp8 result stays near the bf16 op on the original cache
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    assert_close(o, sparse_attn_oracle(q, kv, sink, idx, scale), atol=5e-2, rtol=5e-2,
                 what="fp8 vs bf16 cache")


@pytest.mark.parametrize("h", [8, 32, 72])
def test_fp8_head_counts(h):
    """Other head counts: fewer pad to 16, more run as groups of 16."""
    g = torch.Generator().manual_seed(h)
    b, m, kv_len, topk = 2, 20, 600, 320
    q = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(h, generator=g)
    idx = torch.randint(-1, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    scale = 512 ** -0.5
    kv8, ks = quantize_kv_fp8(kv.cuda())
    o = sparse_attn_fp8(q.cuda(), kv8, ks, sink.cuda(), idx.cuda(), scale)
    assert o.shape == q.shape
    ref = sparse_attn_fp8_oracle(q, kv8.cpu(), ks.cpu(), sink, idx, scale)
    assert_close(o, ref, what=f"fp8 h={h}")


@pytest.mark.parametrize("grid", [0, 3, 37])
def test_fp8_row_schedule_trailing_padding(grid):
    """Prefill shapes run whole rows per CTA up to each row's last valid slot
    (the bf16 kernel's row schedule); out-of-range indices in the skipped
    tails are still counted."""
    from sparse_attn._lib import index_faults
    g = torch.Generator().manual_seed(43)
    b, m, kv_len, topk = 2, 300, 900, 320
    q = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    length = (torch.arange(m) + 1).clamp(max=topk)[None, :, None].expand(b, m, 1)
    idx = torch.where(torch.arange(topk)[None, None, :] < length, idx, torch.full_like(idx, -1))
    idx[0, 5] = -1
    idx[1, 40, 7] = kv_len
    idx[0, 20, 200] = kv_len + 5
    kv8, ks = quantize_kv_fp8_ref(kv)
    ref = sparse_attn_fp8_oracle(q, kv8, ks, sink, idx, 512 ** -0.5)
    torch.cuda.synchronize()
    index_faults(reset=True)
    o = run_fp8(q, kv8, ks, sink, idx, 512 ** -0.5, grid=grid)
    assert index_faults(reset=True) == 2
    assert_close(o, ref, what=f"fp8 row schedule grid={grid}")
    assert torch.count_nonzero(o[0, 5]) == 0


def test_fp8_scales_spanning_decades():
    """Token scales that grow along the key order exercise the running
    scale maximum (O rescaled whenever a unit brings a larger scale)."""
    g = torch.Generator().manual_seed(12)
    b, m, kv_len, topk = 2, 3, 4096, 2048
    q = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    mag = torch.logspace(-2, 0.5, kv_len).view(1, kv_len, 1)
    kv = (torch.randn(b, kv_len, 512, generator=g) * mag).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    idx = torch.sort(torch.rand(b * m, kv_len, generator=g).topk(topk, dim=1).indices, dim=1)
    idx = idx.values.to(torch.int32).reshape(b, m, topk)
    kv8, ks = quantize_kv_fp8_ref(kv)
    scale = 512 ** -0.5
    for grid in (0, 5):
        o = run_fp8(q, kv8, ks, sink, idx, scale, grid=grid)
        assert_close(o, sparse_attn_fp8_oracle(q, kv8, ks, sink, idx, scale),
                     what=f"decades grid={grid}")


def test_fp8_zero_rows_masks_and_faults():
    from sparse_attn._lib import index_faults
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=13)
    kv[0, :100] = 0  # scale-0 rows
    kv8, ks = quantize_kv_fp8_ref(kv)
    idx[0, 0] = -1                  # whole row masked: o = 0
    idx[0, 1, :10] = kv.shape[1]    # out of range: masked and counted
    idx[0, 2, 5] = -9
    torch.cuda.synchronize()
    index_faults(reset=True)
    o = run_fp8(q, kv8, ks, sink, idx, scale)
    assert index_faults(reset=True) == 11
    assert torch.count_nonzero(o[0, 0]) == 0
    assert_close(o, sparse_attn_fp8_oracle(q, kv8, ks, sink, idx, scale), what="zero rows")


def test_fp8_strided_cache_and_determinism():
    args, o_gold = load_golden_fp8("fp8_masked")
    q, kv8, ks, sink, idx, scale = args
    big = torch.zeros(kv8.shape[0], kv8.shape[1], 1024, dtype=torch.uint8)
    big[:, :, 512:] = kv8.view(torch.uint8)
    kv8_s = big.cuda().view(torch.float8_e4m3fn)[:, :, 512:]  # row stride 1024 bytes
    ks_s = torch.zeros(ks.shape[1], ks.shape[0]).t()  # [b, kv_len], strides (1, b)
    ks_s.copy_(ks)
    o1 = run_fp8(q, kv8_s, ks_s, sink, idx, scale)
    o2 = run_fp8(q, kv8, ks, sink, idx, scale)
    assert torch.equal(o1, o2)
    assert_close(o1, o_gold, what="strided fp8 cache")


def test_fp8_no_pipeline_timeouts():
    from sparse_attn._lib import device_status
    args, _ = load_golden_fp8("fp8_plumbing")
    run_fp8(*args)
    assert device_status() == 0


def test_fp8_ticket_merge_with_a_short_workspace():
    """A workspace without room for the per-row ints (a size from an older
    formula) makes prefill-shaped grids merge split rows by ticket instead of
    running the row schedule; both give the oracle's result."""
    from sparse_attn import workspace_bytes
    args, ref = load_golden_fp8("fp8_plumbing")
    q, kv8, ks, sink, idx, scale = args
    q, kv8, ks, sink, idx = _cuda(q, kv8, ks, sink, idx)
    ws = torch.zeros(workspace_bytes(1, 64, 64, q.device), dtype=torch.uint8, device="cuda")
    short = ws[:ws.numel() - (64 * 4 + 255) // 256 * 256]
    for w in (short, ws, short):
        for grid in (3, 5, 0):
            o = torch.empty_like(q)
            sparse_attn_fp8_out(o, q, kv8, ks, sink, idx, scale, w, grid=grid)
            torch.cuda.synchronize()
            assert_close(o, ref, what=f"fp8 grid {grid}, workspace {w.numel()} B")
