"""CPU oracle for ``hc_split_sinkhorn`` (track-02 of the reference project).

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` and the CPU legs of
``bench.py``, never by the product path.

Restates ``track-02/reference/reference.py:11-51`` op for op in fp32 torch on
the CPU, so its outputs equal the reference's bit for bit; pinned by the golden
vectors ``tests/golden/hc_*.npz`` made from the live reference.
"""
from __future__ import annotations

import torch

__all__ = ["hc_split_sinkhorn_oracle"]


@torch.no_grad()
def hc_split_sinkhorn_oracle(mixes, hc_scale, hc_base, hc_mult=4, sinkhorn_iters=20, eps=1e-6):
    mixes, hc_scale, hc_base = mixes.cpu().float(), hc_scale.cpu().float(), hc_base.cpu().float()
    b, s, _ = mixes.shape
    hc = hc_mult
    # reference.py:36-38: the three slices of the mixing logits
    pre_raw, post_raw = mixes[..., :hc], mixes[..., hc:2 * hc]
    comb_raw = mixes[..., 2 * hc:].reshape(b, s, hc, hc)
    # reference.py:40-42: gates, scale and bias
    pre = torch.sigmoid(pre_raw * hc_scale[0] + hc_base[:hc]) + eps
    post = 2 * torch.sigmoid(post_raw * hc_scale[1] + hc_base[hc:2 * hc])
    comb = comb_raw * hc_scale[2] + hc_base[2 * hc:].reshape(hc, hc)
    # reference.py:44-49: row softmax, one column step, then row/column steps
    comb = torch.softmax(comb, dim=-1) + eps
    comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    for _ in range(sinkhorn_iters - 1):
        comb = comb / (comb.sum(dim=-1, keepdim=True) + eps)
        comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    return pre, post, comb
