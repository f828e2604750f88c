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
