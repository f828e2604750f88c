"""Parity of the CUDA path with the CPU oracle and the golden vectors (GPU).

Every call goes through the C ABI (``sparse_attn_out`` -> ``sa_fwd_ex``) or
the drop-in op (``sparse_attn`` -> ``sa_fwd``).  Tolerance: atol = rtol =
2e-2 on the bf16 output (track-01/test_correctness.py:18-19 uses 5e-2).
"""
import dataclasses

import pytest
import torch

import make_golden
from helpers import assert_close, load_golden
from oracle.sparse_attn_oracle import sparse_attn_oracle
from sparse_attn import (SA_VARIANT_MMA, SA_VARIANT_TCGEN05, SA_VARIANT_WS, SA_VARIANT_WT,
                         sparse_attn, sparse_attn_out)
from sparse_attn import _lib
from sparse_attn import lib as _salib
from sparse_attn.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu

VARIANTS = [v for v in (SA_VARIANT_MMA, SA_VARIANT_TCGEN05, SA_VARIANT_WS, SA_VARIANT_WT)
            if _salib().sa_variant_available(v)]
VARIANT_IDS = [{SA_VARIANT_MMA: "mma", SA_VARIANT_TCGEN05: "tcgen05", SA_VARIANT_WS: "ws",
                SA_VARIANT_WT: "wt"}[v] for v in VARIANTS]


def _cuda(*ts):
    return [t.cuda() if torch.is_tensor(t) else t for t in ts]


def run_gpu(q, kv, sink, idx, scale, variant=0, grid=0):
    q, kv, sink, idx = _cuda(q, kv, sink, idx)
    o = torch.empty_like(q)
    sparse_attn_out(o, q, kv, sink, idx, scale, variant=variant, grid=grid)
    torch.cuda.synchronize()
    return o


@pytest.mark.parametrize("variant", VARIANTS, ids=VARIANT_IDS)
@pytest.mark.parametrize("name", make_golden.CASES)
@pytest.mark.parametrize("grid", [0, 1, 3, 37])
def test_golden(name, variant, grid):
    args, o_gold = load_golden(name)
    o = run_gpu(*args, variant=variant, grid=grid)
    assert_close(o, o_gold, what=f"{name} variant={variant} grid={grid}")
    if name == "masked":  # whole masked rows give exactly 0
        assert torch.count_nonzero(o[0, 1]) == 0 and torch.count_nonzero(o[1, 4]) == 0


def test_dropin_op_matches_golden():
    args, o_gold = load_golden("plumbing")
    from submission import sparse_attn as drop_in  # track-01 harness import
    o = drop_in(*_cuda(*args))
    assert o.dtype == torch.bfloat16 and o.shape == o_gold.shape and o.is_cuda
    assert_close(o, o_gold, what="drop-in")


def test_strided_inputs():
    (q, kv, sink, idx, scale), o_gold = load_golden("ragged")
    b, m, h, d = q.shape
    # q: rows of a wider buffer; kv: padded row stride; idx: transposed storage;
    # o: written into a strided slice
    qb = torch.zeros(b, m + 2, h, d + 64, dtype=q.dtype)
    qb[:, 1:m + 1, :, :d] = q
    kvb = torch.zeros(b, kv.shape[1], d + 128, dtype=kv.dtype)
    kvb[:, :, :d] = kv
    idxb = idx.transpose(0, 1).contiguous()
    qb, kvb, sinkc, idxb = _cuda(qb, kvb, sink, idxb)
    qs, kvs, idxs = qb[:, 1:m + 1, :, :d], kvb[:, :, :d], idxb.transpose(0, 1)
    assert not qs.is_contiguous() and not kvs.is_contiguous() and not idxs.is_contiguous()
    ob = torch.zeros(b, m, h, d + 32, dtype=q.dtype, device="cuda")
    for variant in VARIANTS:
        sparse_attn_out(ob[..., :d], qs, kvs, sinkc, idxs, scale, variant=variant)
        torch.cuda.synchronize()
        assert_close(ob[..., :d], o_gold, what=f"strided variant={variant}")
    assert torch.count_nonzero(ob[..., d:]) == 0
    # the drop-in op accepts the same views
    assert_close(sparse_attn(qs, kvs, sinkc, idxs, scale), o_gold, what="strided op")


@pytest.mark.parametrize("variant", VARIANTS, ids=VARIANT_IDS)
def test_decode_full_vs_oracle(variant):
    args = make_inputs("decode", seed=0)
    o = run_gpu(*args, variant=variant)
    assert_close(o, sparse_attn_oracle(*args), what="decode")


def _sampled_rows(m, n=48, seed=0):
    g = torch.Generator().manual_seed(seed)
    rows = {0, 1, 2, m // 2, m - 1} | set(torch.randint(0, m, (n,), generator=g).tolist())
    if m > 2048:
        rows |= {2046, 2047, 2048}
    return sorted(r for r in rows if r < m)


def _check_rows(args, o, rows, what):
    q, kv, sink, idx, scale = args
    r = torch.tensor(rows)
    ref = sparse_attn_oracle(q[:, r], kv, sink, idx[:, r], scale)
    assert_close(o[:, r.cuda()], ref, what=what)


@pytest.mark.parametrize("variant", VARIANTS, ids=VARIANT_IDS)
def test_causal_full_size(variant):
    args = make_inputs("causal", seed=0)
    o = run_gpu(*args, variant=variant)
    _check_rows(args, o, _sampled_rows(4096), "causal")


def test_long_context_full_size():
    args = make_inputs("long", seed=0)
    o = {}
    for v in VARIANTS:
        o[v] = run_gpu(*args, variant=v)
        _check_rows(args, o[v], _sampled_rows(8192, n=24), f"long variant={v}")


def test_mtp_reduced_batch():
    cfg = dataclasses.replace(CONFIGS["mtp"], b=8)
    args = make_inputs(cfg, seed=0)
    for v in VARIANTS:
        o = run_gpu(*args, variant=v)
        _check_rows(args, o, [0, 1], f"mtp variant={v}")


@pytest.mark.parametrize("variant", VARIANTS, ids=VARIANT_IDS)
def test_properties_at_decode_size(variant):
    q, kv, sink, idx, scale = make_inputs("decode", seed=1)
    base = run_gpu(q, kv, sink, idx, scale, variant=variant)
    # deterministic: same inputs, same bits
    assert torch.equal(base, run_gpu(q, kv, sink, idx, scale, variant=variant))
    # slot order does not matter
    perm = torch.randperm(idx.shape[-1], generator=torch.Generator().manual_seed(3))
    assert_close(run_gpu(q, kv, sink, idx[..., perm], scale, variant=variant), base,
                 what="slot permutation")
    # trailing -1 padding does not matter
    pad = torch.full((*idx.shape[:2], 77), -1, dtype=idx.dtype)
    assert_close(run_gpu(q, kv, sink, torch.cat([idx, pad], -1), scale, variant=variant), base,
                 what="-1 padding")
    # grid size (how rows are split across CTAs) does not matter
    for grid in (1, 64, 200):
        assert_close(run_gpu(q, kv, sink, idx, scale, variant=variant, grid=grid), base,
                     what=f"grid {grid}")


def test_variants_agree():
    args = make_inputs("plumbing", seed=7)
    outs = [run_gpu(*args, variant=v) for v in VARIANTS]
    for o in outs[1:]:
        assert_close(o, outs[0], what="variants")


def test_no_pipeline_timeouts():
    """No bounded wait inside the tensor-core kernel gave up during this run."""
    from sparse_attn._lib import device_status
    args = make_inputs("plumbing", seed=3)
    run_gpu(*args)
    assert device_status() == 0


def test_custom_op_registration_matches():
    """torch.ops.sparse_attn_b200.fwd (for graph capture / compile users) is the
    same computation as the drop-in function."""
    args, o_gold = load_golden("ragged")
    a = _cuda(*args)
    o1 = torch.ops.sparse_attn_b200.fwd(a[0], a[1], a[2], a[3], float(a[4]))
    o2 = sparse_attn(*a)
    assert torch.equal(o1, o2)
    assert_close(o1, o_gold, what="custom op")


@pytest.mark.parametrize("h", [1, 5, 8, 16])
def test_fewer_heads_padded(h):
    """h < 16 is served by padding to 16 heads (reference: submission.py:1004)."""
    q, kv, sink, idx, scale = make_golden.make_case("ragged")
    q, sink = q[:, :, :h].contiguous(), sink[:h].contiguous()
    o = sparse_attn(*_cuda(q, kv, sink, idx, scale))
    assert o.shape == q.shape
    assert_close(o, sparse_attn_oracle(q, kv, sink, idx, scale), what=f"h={h}")


def _many_heads_case(h, seed=21, b=2, m=40, kv_len=700, topk=300):
    """Ragged rows (trailing -1 padding, interior -1, an all-masked row)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, m, h, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(h, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    length = torch.randint(0, topk + 1, (b, m, 1), generator=g)
    idx = torch.where(torch.arange(topk)[None, None, :] < length, idx, torch.full_like(idx, -1))
    idx[1, 3] = -1
    return q, kv, sink, idx, 512 ** -0.5


@pytest.mark.parametrize("h", [17, 32, 40, 64, 128])
def test_more_heads_in_groups(h):
    """h > 16 runs as groups of 16 heads (h not a multiple of 16 is padded),
    through every kernel variant."""
    q, kv, sink, idx, scale = _many_heads_case(h)
    ref = sparse_attn_oracle(q, kv, sink, idx, scale)
    o = sparse_attn(*_cuda(q, kv, sink, idx, scale))
    assert o.shape == q.shape
    assert_close(o, ref, what=f"h={h}")
    if h % 16 == 0:
        for variant in VARIANTS:
            qc, kvc, sc, ic, _ = _cuda(q, kv, sink, idx, scale)
            o = torch.empty_like(qc)
            sparse_attn_out(o, qc, kvc, sc, ic, scale, variant=variant, grid=37)
            assert_close(o, ref, what=f"h={h} variant {variant}")


def test_more_heads_strided_q_and_o():
    """Head groups step through q and o by their head stride: q a slice of a
    wider buffer, o written into a strided view."""
    h = 48
    q, kv, sink, idx, scale = _many_heads_case(h, seed=5)
    ref = sparse_attn_oracle(q, kv, sink, idx, scale)
    qc, kvc, sc, ic, _ = _cuda(q, kv, sink, idx, scale)
    wide = torch.zeros(q.shape[0], q.shape[1], h + 16, 512, dtype=q.dtype, device="cuda")
    wide[:, :, 8:8 + h] = qc
    ob = torch.zeros(q.shape[0], q.shape[1], h + 24, 512, dtype=q.dtype, device="cuda")
    sparse_attn_out(ob[:, :, 16:16 + h], wide[:, :, 8:8 + h], kvc, sc, ic, scale)
    assert_close(ob[:, :, 16:16 + h], ref, what="strided h=48")
    assert not ob[:, :, :16].any() and not ob[:, :, 16 + h:].any()


def _decode_heads_case(h, seed=3, b=6, kv_len=4096, topk=2048):
    """Decode-shaped rows with many heads: every row split over several CTAs."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, 1, h, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(h, generator=g)
    idx = torch.stack([torch.randperm(kv_len, generator=g)[:topk] for _ in range(b)])
    idx = idx.to(torch.int32).reshape(b, 1, topk)
    idx[2, 0, 1500:] = -1
    return q, kv, sink, idx, 512 ** -0.5


@pytest.mark.parametrize("shape", ["decode", "prefill"])
@pytest.mark.parametrize("h,grid", [(32, 0), (64, 0), (48, 100), (64, 5)])
def test_head_groups_one_launch_and_in_turn(shape, h, grid):
    """h > 16 on the default kernel: all head groups in one launch (the
    default) and one group after another (SA_OPT_HEAD_GROUPS = 0) both match
    the oracle, on split decode rows (combine kernel) and on prefill rows."""
    if shape == "decode":
        q, kv, sink, idx, scale = _decode_heads_case(h)
    else:
        q, kv, sink, idx, scale = _many_heads_case(h, seed=h + grid)
    ref = sparse_attn_oracle(q, kv, sink, idx, scale)
    outs = []
    for mode in (1, 0):
        old = _lib.set_option(_lib.SA_OPT_HEAD_GROUPS, mode)
        try:
            outs.append(run_gpu(q, kv, sink, idx, scale, grid=grid))
        finally:
            _lib.set_option(_lib.SA_OPT_HEAD_GROUPS, old)
        assert_close(outs[-1], ref, what=f"{shape} h={h} grid={grid} head groups mode {mode}")
    assert _lib.device_status() == 0


def _ragged_case(seed=11):
    """1200 rows (ragged schedule), rows padded with -1 to random lengths,
    interior -1 slots, and a few fully masked rows."""
    g = torch.Generator().manual_seed(seed)
    b, m, kv_len, topk = 2, 600, 300, 200
    q = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    length = torch.randint(0, topk + 1, (b, m, 1), generator=g)
    idx = torch.where(torch.arange(topk)[None, None, :] < length, idx, torch.full_like(idx, -1))
    idx = torch.where(torch.rand(b, m, topk, generator=g) < 0.1, torch.full_like(idx, -1), idx)
    idx[0, 7] = -1
    idx[1, 599] = -1
    return q, kv, sink, idx, 512 ** -0.5


@pytest.mark.parametrize("grid", [0, 5, 1000])
def test_ragged_schedule_rows_of_varying_length(grid):
    args = _ragged_case()
    ref = sparse_attn_oracle(*args)
    for v in VARIANTS:
        o = run_gpu(*args, variant=v, grid=grid)
        assert_close(o, ref, what=f"ragged variant={v} grid={grid}")
        assert torch.count_nonzero(o[0, 7]) == 0 and torch.count_nonzero(o[1, 599]) == 0


@pytest.mark.parametrize("variant", VARIANTS)
def test_index_faults_counted(variant):
    """Indices that are neither -1 nor in [0, kv_len) are masked and counted
    exactly once per slot; -1 is not counted."""
    from sparse_attn._lib import index_faults
    q, kv, sink, idx, scale = make_inputs("plumbing", seed=11)
    kv_len = kv.shape[1]
    idx[0, 0, :7] = -1                    # sentinel: masked, not counted
    idx[0, 1, 3] = -2
    idx[0, 2, 10:15] = kv_len
    idx[0, 5, 63] = kv_len + 1000
    idx[0, 9, 0] = -(2 ** 31)
    expected = 1 + 5 + 1 + 1
    torch.cuda.synchronize()
    index_faults(reset=True)
    o = run_gpu(q, kv, sink, idx, scale, variant=variant)
    torch.cuda.synchronize()
    assert index_faults(reset=True) == expected
    assert index_faults() == 0
    assert_close(o, sparse_attn_oracle(q, kv, sink, idx, scale), what="faulty indices")


@pytest.mark.parametrize("grid", [0, 3, 37])
def test_row_schedule_trailing_padding(grid):
    """Prefill shapes (rows >= 2 x grid) run whole rows per CTA, each only up
    to its last valid slot.  Rows of causal form (valid prefix, then -1), rows
    with no valid slot, interior -1, and out-of-range indices both inside the
    run part and in the skipped tail: the output matches the oracle and every
    out-of-range index is counted once."""
    from sparse_attn._lib import index_faults
    g = torch.Generator().manual_seed(41)
    b, m, kv_len, topk = 2, 300, 900, 320
    q = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    length = (torch.arange(m) + 1).clamp(max=topk)[None, :, None].expand(b, m, 1)
    idx = torch.where(torch.arange(topk)[None, None, :] < length, idx, torch.full_like(idx, -1))
    idx[0, 5] = -1                      # no valid slot
    idx[1, 250, 3] = -1                 # interior -1
    idx[1, 40, 7] = kv_len              # counted by the forward kernel (run part)
    idx[0, 20, 200] = kv_len + 5        # in the skipped tail of a 21-slot row
    idx[1, 0, 319] = -7                 # in the skipped tail of a 1-slot row
    expected = 3
    ref = sparse_attn_oracle(q, kv, sink, idx, 512 ** -0.5)
    torch.cuda.synchronize()
    index_faults(reset=True)
    o = run_gpu(q, kv, sink, idx, 512 ** -0.5, variant=SA_VARIANT_WS, grid=grid)
    assert index_faults(reset=True) == expected
    assert_close(o, ref, what=f"row schedule grid={grid}")
    assert torch.count_nonzero(o[0, 5]) == 0


def test_workspace_reuse_across_grids():
    """Split rows are merged in the kernel by the last CTA to finish them
    (per-CTA counters in the workspace, zeroed again by every call), or rows
    are not split at all (row schedule): one workspace serves calls with
    different grids and both paths back to back."""
    from sparse_attn import workspace_bytes
    q, kv, sink, idx, scale = [t.cuda() if torch.is_tensor(t) else t
                               for t in make_inputs("plumbing", seed=31)]
    ref = sparse_attn_oracle(q.cpu(), kv.cpu(), sink.cpu(), idx.cpu(), scale)
    ws = torch.zeros(workspace_bytes(1, 64, 64, q.device), dtype=torch.uint8, device="cuda")
    # without room for the per-row ints (a size from an older formula) the
    # prefill-shaped grids take the ticket merge instead of the row schedule
    short = ws[:ws.numel() - (64 * 4 + 255) // 256 * 256]
    for w in (ws, short, ws):
        for grid in (5, 37, 3, 64, 5, 0, 7):
            o = torch.empty_like(q)
            sparse_attn_out(o, q, kv, sink, idx, scale, w, variant=SA_VARIANT_WS, grid=grid)
            torch.cuda.synchronize()
            assert_close(o, ref, what=f"grid {grid} (reused workspace of {w.numel()} B)")
