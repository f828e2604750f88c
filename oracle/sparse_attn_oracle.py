"""CPU oracle for ``sparse_attn`` (track-01 of inin-zou/kernelgen-challenge).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
(``cpu_baseline`` and ``--impl reference``) use it, and only as the checker or
as the timed CPU baseline.

What it restates
----------------
``track-01/reference/reference.py:10-40`` step for step, in fp32 on the CPU:

* gather the top-k KV rows            (reference.py:27-30)
* scores = q.float() @ kv.float()^T * scale   (reference.py:32)
* append the per-head sink as logit topk+1    (reference.py:34-35)
* softmax over topk+1, drop the sink column   (reference.py:36-38)
* o = attn @ kv.float(), cast to bf16         (reference.py:39-40)

plus the ``-1`` sentinel rule of the reference's NVIDIA-path kernel
(``track-01/submission.py:313-322``): a slot holding ``-1`` gathers a zero row
and gets score ``-inf``, so it contributes nothing.  ``reference.py`` itself
raises on ``-1`` (``torch.gather`` bounds check), so for index sets without
``-1`` this restatement is required to equal ``reference.py`` bit for bit
(pinned by ``tests/test_oracle.py`` against the live reference in the build
container and by the committed golden vectors in ``tests/golden/``).

Two documented extensions beyond the reference (both also implemented by the
CUDA path, both pinned by tests):

* any index outside ``[0, kv_len)`` is masked like ``-1`` (the reference raises
  or reads out of bounds; the product never reads out of bounds);
* a row whose slots are all masked returns ``o = 0`` (the sink takes all the
  probability mass).  The reference's universal kernel returns NaN there
  (``submission.py:328-329``: ``exp(-inf - -inf)``); ``o = 0`` is the limit of
  the softmax definition.

Work is processed in chunks of query rows so that memory stays bounded
(the reference materialises ``[b, m, topk, d]`` three times).
"""
from __future__ import annotations

import torch

__all__ = ["sparse_attn_oracle", "valid_slot_count", "quantize_kv_fp8_ref", "dequantize_kv_fp8",
           "sparse_attn_fp8_oracle", "sparse_attn_oracle_grads"]


def _chunk_rows(m: int, topk: int, d: int, budget_bytes: int = 1 << 30) -> int:
    # per query row the chunk holds topk*d of bf16 + 2 fp32 copies (10 B/elt)
    per_row = max(1, topk * d * 10)
    return max(1, min(m, budget_bytes // per_row))


@torch.no_grad()
def sparse_attn_oracle(q, kv, attn_sink, topk_idxs, scale, *, num_threads=None,
                       rows_per_chunk=None):
    """fp32 CPU oracle with the reference's semantics (see module docstring).

    Args mirror ``track-01/reference/reference.py:10`` exactly:
        q [b, m, h, d] bf16, kv [b, kv_len, d] bf16, attn_sink [h] fp32,
        topk_idxs [b, m, topk] int32, scale float.
    Returns o [b, m, h, d] with q's dtype, on the CPU.
    """
    if num_threads is not None:
        torch.set_num_threads(int(num_threads))
    q = q.cpu()
    kv = kv.cpu()
    attn_sink = attn_sink.cpu()
    topk_idxs = topk_idxs.cpu()

    b, m, h, d = q.shape
    kv_len = kv.shape[1]
    topk = topk_idxs.shape[-1]
    out = torch.empty(b, m, h, d, dtype=q.dtype)
    if b == 0 or m == 0:
        return out
    step = rows_per_chunk or _chunk_rows(m, topk, d)
    sink = attn_sink.float()
    for m0 in range(0, m, step):
        m1 = min(m, m0 + step)
        mc = m1 - m0
        idx = topk_idxs[:, m0:m1].long()                        # [b, mc, topk]
        valid = (idx >= 0) & (idx < kv_len)
        safe = torch.where(valid, idx, torch.zeros_like(idx))
        # reference.py:27-30 — one gather per batch row of the flattened indices
        flat = safe.reshape(b, mc * topk)
        g = torch.gather(kv, 1, flat.unsqueeze(-1).expand(-1, -1, d)).reshape(b, mc, topk, d)
        g = g.masked_fill(~valid.unsqueeze(-1), 0)             # submission.py:320-321
        gf = g.float()
        # reference.py:32
        scores = torch.einsum("bmhd,bmtd->bmht", q[:, m0:m1].float(), gf) * scale
        # submission.py:318-322: masked slot -> score -inf
        scores = scores.masked_fill(~valid.unsqueeze(2), float("-inf"))
        # reference.py:34-38
        s = sink[None, None, :, None].expand(b, mc, h, 1)
        attn = torch.softmax(torch.cat([scores, s], dim=-1), dim=-1)[..., :-1]
        # reference.py:39-40
        o = torch.einsum("bmht,bmtd->bmhd", attn, gf)
        out[:, m0:m1] = o.to(q.dtype)
    return out


def valid_slot_count(topk_idxs, kv_len: int) -> int:
    """Number of slots whose row is actually gathered (index in [0, kv_len))."""
    idx = topk_idxs
    return int(((idx >= 0) & (idx < kv_len)).sum().item())


# ---------------------------------------------------------------------------
# fp8 (e4m3) KV cache with one fp32 scale per token.  The reference has no fp8
# cache; its semantics here are the reference op on the dequantised cache.
# ---------------------------------------------------------------------------
E4M3_MAX = 448.0


@torch.no_grad()
def quantize_kv_fp8_ref(kv):
    """CPU statement of the quantiser: per row amax = max|x|,
    kv8 = e4m3_rn(x * (448 / amax)), scale = amax / 448 (zero rows: 0, 0)."""
    x = kv.cpu().float()
    amax = x.abs().amax(dim=-1)
    # a correctly rounded fp32 division (torch evaluates `float / tensor` as a
    # reciprocal followed by a product: two roundings)
    inv = torch.where(amax > 0, torch.full_like(amax, E4M3_MAX) / amax, torch.zeros_like(amax))
    kv8 = (x * inv.unsqueeze(-1)).to(torch.float8_e4m3fn)
    return kv8, amax / E4M3_MAX


def dequantize_kv_fp8(kv8, kv_scale):
    """fp32 cache rows: kv8[b, t, :] * kv_scale[b, t]."""
    return kv8.cpu().float() * kv_scale.cpu().float().unsqueeze(-1)


def sparse_attn_fp8_oracle(q, kv8, kv_scale, attn_sink, topk_idxs, scale, **kw):
    """The reference's algorithm (``sparse_attn_oracle``) on the dequantised
    fp32 cache; reference.py:32 widens kv to fp32 first, so an fp32 cache
    enters its arithmetic unchanged."""
    return sparse_attn_oracle(q, dequantize_kv_fp8(kv8, kv_scale), attn_sink, topk_idxs,
                              scale, **kw)


# ---------------------------------------------------------------------------
# Gradients (the reference has no backward): torch autograd through the same
# fp32 restatement, on the CPU.
# ---------------------------------------------------------------------------
def sparse_attn_oracle_grads(q, kv, attn_sink, topk_idxs, scale, do):
    """(o, dq, dkv, dsink) in fp32: autograd of the fp32 restatement of
    reference.py:24-40 with the -1 masking rule, for upstream gradient do."""
    q32 = q.detach().cpu().float().requires_grad_(True)
    kv32 = kv.detach().cpu().float().requires_grad_(True)
    s32 = attn_sink.detach().cpu().float().requires_grad_(True)
    idx = topk_idxs.cpu().long()
    b, m, h, d = q32.shape
    kv_len = kv32.shape[1]
    valid = (idx >= 0) & (idx < kv_len)
    safe = torch.where(valid, idx, torch.zeros_like(idx))
    g = torch.gather(kv32, 1, safe.reshape(b, -1).unsqueeze(-1).expand(-1, -1, d))
    g = g.reshape(b, m, -1, d) * valid.unsqueeze(-1)
    scores = torch.einsum("bmhd,bmtd->bmht", q32, g) * scale
    scores = scores.masked_fill(~valid.unsqueeze(2), float("-inf"))
    attn = torch.softmax(torch.cat([scores, s32[None, None, :, None].expand(b, m, h, 1)], -1),
                         -1)[..., :-1]
    o = torch.einsum("bmht,bmtd->bmhd", attn, g)
    o.backward(do.detach().cpu().float())
    return o.detach(), q32.grad, kv32.grad, s32.grad
