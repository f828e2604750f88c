"""CPU oracle of the top-k index producer (``sparse_attn.indexer_topk``).

TEST INFRASTRUCTURE ONLY.  The reference has no indexer; this states the
published DeepSeek-V3.2 lightning-indexer score in fp32 torch
(score[b,t,s] = sum_j w[b,t,j] * ReLU(q[b,t,j,:] . k[b,s,:]) over s < len[b,t])
and selects the topk keys by (score descending, index ascending), returned in
ascending index order with -1 padding.  Parity is unpinned (no reference
vectors exist for this step).
"""
from __future__ import annotations

import torch

__all__ = ["indexer_scores_oracle", "select_topk", "indexer_topk_oracle"]


@torch.no_grad()
def indexer_scores_oracle(q_idx, k_idx, weights, lengths):
    q, k = q_idx.cpu().float(), k_idx.cpu().float()
    w, ln = weights.cpu().float(), lengths.cpu().long()
    dots = torch.einsum("bmhd,bsd->bmhs", q, k).clamp_min(0)
    score = (dots * w.unsqueeze(-1)).sum(2)
    s = torch.arange(k.shape[1]).view(1, 1, -1)
    return score.masked_fill(s >= ln.unsqueeze(-1), float("-inf"))


def select_topk(score, lengths, topk):
    """topk keys of largest score (ties: lower index) among s < lengths, in
    ascending index order, -1 padded; exact for the given scores."""
    b, m, n = score.shape
    out = torch.full((b, m, topk), -1, dtype=torch.int32)
    for bi in range(b):
        for mi in range(m):
            L = int(min(max(int(lengths[bi, mi]), 0), n))
            # stable sort: equal scores keep ascending index order
            order = torch.sort(-score[bi, mi, :L].double(), stable=True).indices[:topk]
            sel = torch.sort(order).values
            out[bi, mi, :sel.numel()] = sel.to(torch.int32)
    return out


def indexer_topk_oracle(q_idx, k_idx, weights, lengths, topk):
    score = indexer_scores_oracle(q_idx, k_idx, weights, lengths)
    return select_topk(score, lengths.cpu(), topk), score
