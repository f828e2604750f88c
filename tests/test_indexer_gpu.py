"""The top-k index producer (``indexer_topk``) against its CPU oracle.

Scores: fp32 sums of bf16 products in another order than torch's einsum, so
they agree to 1e-4 of the largest score.  Selection: exactly the topk of the
GPU's own scores (ties to the lower index); against the oracle's scores, only
keys within rounding of the threshold may differ.
"""
import pytest
import torch

from oracle.indexer_oracle import indexer_scores_oracle, select_topk
from oracle.sparse_attn_oracle import sparse_attn_oracle

pytestmark = pytest.mark.gpu


def _inputs(b, m, kv_len, seed, lengths=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, m, 64, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(b, kv_len, 128, generator=g).to(torch.bfloat16)
    w = torch.rand(b, m, 64, generator=g) * 0.1
    if lengths is None:
        lengths = torch.full((b, m), kv_len, dtype=torch.int32)
    return q, k, w, lengths


def _check(q, k, w, lengths, topk, what):
    from sparse_attn import indexer_topk
    idx, sc = indexer_topk(q.cuda(), k.cuda(), w.cuda(), lengths.cuda(), topk, return_scores=True)
    torch.cuda.synchronize()
    idx, sc = idx.cpu(), sc.cpu()
    ref = indexer_scores_oracle(q, k, w, lengths)
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(sc)), f"{what}: -inf pattern"
    scale = ref[fin].abs().max() if bool(fin.any()) else torch.tensor(1.0)
    assert bool(((sc[fin] - ref[fin]).abs() <= 1e-4 * scale + 1e-6).all()), \
        f"{what}: scores, max |d| = {(sc[fin] - ref[fin]).abs().max():.3e}"
    # exactly the top-k of the GPU's own scores
    assert torch.equal(idx, select_topk(sc, lengths, topk)), f"{what}: selection"
    # against the oracle's scores: differences only at the threshold
    ro = select_topk(ref, lengths, topk)
    for bi in range(idx.shape[0]):
        for mi in range(idx.shape[1]):
            a = set(idx[bi, mi][idx[bi, mi] >= 0].tolist())
            e = set(ro[bi, mi][ro[bi, mi] >= 0].tolist())
            assert len(a) == len(e), what
            diff = a ^ e
            if diff:
                thr = ref[bi, mi][sorted(e)].min()
                gap = (ref[bi, mi][sorted(diff)] - thr).abs().max()
                assert gap <= 1e-4 * scale + 1e-6, f"{what}: selection beyond rounding ({gap:.3e})"
    return idx


def test_decode_shape():
    q, k, w, ln = _inputs(4, 1, 32768, seed=1)
    _check(q, k, w, ln, 2048, "decode")


def test_causal_lengths_and_padding():
    m, kv_len = 300, 4096
    q, k, w, _ = _inputs(1, m, kv_len, seed=2)
    ln = (torch.arange(m, dtype=torch.int32) * 13 + 1).view(1, m)  # 1 .. 3888 keys
    ln[0, 5] = 0                                                      # no candidates
    idx = _check(q, k, w, ln, 2048, "causal")
    assert bool((idx[0, 5] == -1).all())
    assert bool((idx[0, 0, 1:] == -1).all()) and int(idx[0, 0, 0]) == 0


def test_topk_larger_than_keys_and_multi_span():
    q, k, w, ln = _inputs(2, 3, 9000, seed=3)  # three 4096-key spans, the last partial
    ln[1, 2] = 9999                            # beyond kv_len: clamped
    _check(q, k, w, ln, 10000, "topk > kv_len")
    _check(q, k, w, ln, 7, "small topk")


def test_indexer_feeds_sparse_attn():
    """indexer_topk -> sparse_attn: the op on the produced indices matches the
    oracle on the same indices."""
    from sparse_attn import indexer_topk, sparse_attn
    b, m, kv_len = 2, 64, 4096
    q, k, w, _ = _inputs(b, m, kv_len, seed=4)
    ln = torch.full((b, m), kv_len, dtype=torch.int32)
    ln[:, :10] = torch.arange(1, 11, dtype=torch.int32)
    idx = indexer_topk(q.cuda(), k.cuda(), w.cuda(), ln.cuda(), 2048)
    g = torch.Generator().manual_seed(5)
    qa = torch.randn(b, m, 16, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(16, generator=g)
    o = sparse_attn(qa.cuda(), kv.cuda(), sink.cuda(), idx, 512 ** -0.5)
    ref = sparse_attn_oracle(qa, kv, sink, idx.cpu(), 512 ** -0.5)
    from helpers import assert_close
    assert_close(o, ref, what="indexer -> sparse_attn")


def test_strided_inputs_and_many_rows_per_cta():
    """q and k as slices of wider buffers (the tensor maps take the strides);
    130 rows of 700 keys put several rows and a partial last tile in every
    persistent CTA's range."""
    from sparse_attn import indexer_topk
    q, k, w, ln = _inputs(2, 65, 700, seed=7)
    ln[0, 3] = 0
    ln[1, 10] = 129
    qw = torch.zeros(2, 65, 80, 128, dtype=torch.bfloat16)
    qw[:, :, 8:72] = q
    kw = torch.zeros(2, 700, 192, dtype=torch.bfloat16)
    kw[:, :, 64:] = k
    qs, ks = qw.cuda()[:, :, 8:72], kw.cuda()[:, :, 64:]
    idx, sc = indexer_topk(qs, ks, w.cuda(), ln.cuda(), 100, return_scores=True)
    idx0, sc0 = indexer_topk(q.cuda(), k.cuda(), w.cuda(), ln.cuda(), 100, return_scores=True)
    assert torch.equal(sc, sc0) and torch.equal(idx, idx0)
    _check(q, k, w, ln, 100, "many rows per CTA")


@pytest.mark.parametrize("m", [2, 5, 9])
def test_row_groups_of_four(m):
    """m > 1 runs groups of four rows against each k tile (the last group
    partial), with different length limits inside a group."""
    q, k, w, _ = _inputs(3, m, 1000, seed=20 + m)
    ln = torch.randint(0, 1001, (3, m), generator=torch.Generator().manual_seed(m),
                       dtype=torch.int32)
    ln[0, 0] = 1000
    _check(q, k, w, ln, 64, f"groups m={m}")


def test_unaligned_weight_rows_use_the_warp_mma_scorer():
    """Weight rows whose stride is not a multiple of 16 bytes cannot be
    described by a tensor map: the same results come from the other scorer."""
    from sparse_attn import indexer_topk
    q, k, w, ln = _inputs(1, 6, 600, seed=9)
    wb = torch.zeros(1, 6, 65)
    wb[:, :, :64] = w
    idx, sc = indexer_topk(q.cuda(), k.cuda(), wb.cuda()[:, :, :64], ln.cuda(), 50,
                           return_scores=True)
    _check(q, k, w, ln, 50, "unaligned weights (reference run)")
    ref = indexer_scores_oracle(q, k, w, ln)
    assert bool(((sc.cpu() - ref).abs() <= 1e-4 * ref.abs().max() + 1e-6).all())


@pytest.mark.parametrize("m", [1, 3])
def test_negative_weights_and_tied_scores(m):
    """Signed weights give negative scores (order keys below the sign bit);
    repeated k rows give exactly tied scores, taken lowest index first."""
    q, k, w, ln = _inputs(2, m, 3000, seed=30 + m)
    w = w * 20 - 1.0                       # about half the weights negative
    k[:, 1000:1500] = k[:, 0:1].expand(-1, 500, -1)   # 501 keys with one score
    _check(q, k, w, ln, 700, f"signed weights, ties m={m}")
