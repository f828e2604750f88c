"""The CPU oracle against the golden vectors and the live reference (CPU)."""
import importlib.util
import os
import pathlib

import pytest
import torch

import make_golden
from helpers import load_golden
from oracle.sparse_attn_oracle import sparse_attn_oracle

# The live reference: $SPARSE_ATTN_REFERENCE (a checkout), else the copy that
# baseline/install_reference.sh makes under baseline/_ref; skipped if neither.
REF_ROOT = pathlib.Path(os.environ.get("SPARSE_ATTN_REFERENCE") or
                        pathlib.Path(__file__).resolve().parent.parent / "baseline" / "_ref")
HAVE_REF = (REF_ROOT / "track-01" / "reference" / "reference.py").exists()


MASKED_CASES = {"masked", "causal_head"}


@pytest.mark.parametrize("name", make_golden.CASES)
def test_oracle_matches_golden(name):
    args, o_gold = load_golden(name)
    o = sparse_attn_oracle(*args)
    if name not in MASKED_CASES:
        # no masked slot: the restatement follows reference.py op for op
        assert torch.equal(o.view(torch.int16), o_gold.view(torch.int16))
    else:
        # masked rows were evaluated by the reference on the compacted slot set
        # (different einsum shapes, different fp32 summation order): at most one
        # bf16 ulp apart
        assert_within_one_ulp(o, o_gold)


def assert_within_one_ulp(a, b):
    g = b.float()
    ulp = torch.exp2(torch.floor(torch.log2(g.abs().clamp_min(1e-30))) - 7)
    assert bool(((a.float() - g).abs() <= ulp).all())


@pytest.mark.skipif(not HAVE_REF, reason="reference checkout not present")
def test_oracle_matches_live_reference_unmasked():
    ref = make_golden._load_reference(REF_ROOT)
    q, kv, sink, idx, scale = make_golden.make_case("replacement")
    assert torch.equal(ref(q, kv, sink, idx, scale), sparse_attn_oracle(q, kv, sink, idx, scale))


def test_oracle_chunking_is_exact():
    args, _ = load_golden("ragged")
    a = sparse_attn_oracle(*args)
    b = sparse_attn_oracle(*args, rows_per_chunk=1)
    assert torch.equal(a, b)


def test_masked_slot_equals_removed_slot():
    q, kv, sink, idx, scale = make_golden.make_case("ragged")
    idx2 = idx.clone()
    idx2[:, :, 5] = -1
    full = sparse_attn_oracle(q, kv, sink, idx2, scale)
    keep = torch.cat([idx[:, :, :5], idx[:, :, 6:]], dim=-1)
    assert_within_one_ulp(full, sparse_attn_oracle(q, kv, sink, keep, scale))


def test_all_masked_row_is_zero():
    q, kv, sink, idx, scale = make_golden.make_case("ragged")
    idx = torch.full_like(idx, -1)
    o = sparse_attn_oracle(q, kv, sink, idx, scale)
    assert torch.count_nonzero(o) == 0


def test_sink_only_scales_output():
    # o = softmax-weighted mean * (1 - p_sink): a very negative sink is plain attention
    q, kv, sink, idx, scale = make_golden.make_case("ragged")
    lo = sparse_attn_oracle(q, kv, torch.full_like(sink, -1e4), idx, scale).float()
    g = torch.gather(kv, 1, idx.long().reshape(kv.shape[0], -1, 1).expand(-1, -1, 512))
    g = g.reshape(*idx.shape, 512).float()
    s = torch.einsum("bmhd,bmtd->bmht", q.float(), g) * scale
    plain = torch.einsum("bmht,bmtd->bmhd", torch.softmax(s, -1), g)
    assert torch.allclose(lo, plain, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("name", make_golden.FP8_CASES)
def test_fp8_oracle_matches_golden(name):
    """The fp8-cache oracle is the reference's algorithm on the dequantised
    cache: equal to the live reference's output on that cache."""
    from helpers import load_golden_fp8
    from oracle.sparse_attn_oracle import sparse_attn_fp8_oracle
    args, o_gold = load_golden_fp8(name)
    o = sparse_attn_fp8_oracle(*args)
    if name == "fp8_plumbing":
        assert torch.equal(o.view(torch.int16), o_gold.view(torch.int16))
    else:
        assert_within_one_ulp(o, o_gold)


def test_fp8_quantiser_statement():
    """Dequantised rows are within half an e4m3 step (2^-4 relative to the
    row's amax at most) of the bf16 rows; zero rows give scale 0."""
    from oracle.sparse_attn_oracle import dequantize_kv_fp8, quantize_kv_fp8_ref
    g = torch.Generator().manual_seed(5)
    kv = (torch.randn(2, 40, 512, generator=g) *
          torch.logspace(-3, 3, 40).view(1, 40, 1)).to(torch.bfloat16)
    kv[1, 7] = 0
    kv8, sc = quantize_kv_fp8_ref(kv)
    assert kv8.dtype == torch.float8_e4m3fn and sc.shape == (2, 40)
    x = kv.float()
    amax = x.abs().amax(-1, keepdim=True)
    err = (dequantize_kv_fp8(kv8, sc) - x).abs()
    assert bool((err <= amax * 2.0 ** -4 + 1e-30).all())
    assert float(kv8[0].float().abs().max()) == 448.0
    assert float(sc[1, 7]) == 0.0 and bool((kv8[1, 7].float() == 0).all())


def test_indexer_selection_statement():
    """select_topk: largest scores, ties to the lower index, ascending order,
    -1 padding (CPU)."""
    from oracle.indexer_oracle import select_topk
    sc = torch.tensor([[[0.5, 2.0, 2.0, -1.0, 3.0, 2.0]]])
    ln = torch.tensor([[6]], dtype=torch.int32)
    assert select_topk(sc, ln, 3).tolist() == [[[1, 2, 4]]]
    assert select_topk(sc, ln, 8).tolist() == [[[0, 1, 2, 3, 4, 5, -1, -1]]]
    assert select_topk(sc, torch.tensor([[2]], dtype=torch.int32), 3).tolist() == [[[0, 1, -1]]]
