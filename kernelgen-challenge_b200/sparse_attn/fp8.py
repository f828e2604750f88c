"""``sparse_attn`` over an fp8 (e4m3) KV cache with one fp32 scale per token.

The cache layout is ``kv8 [b, kv_len, 512]`` of ``torch.float8_e4m3fn``, plus
``kv_scale [b, kv_len]`` fp32.  Row t of batch b stands for
``kv8[b, t].float() * kv_scale[b, t]``.  :func:`quantize_kv_fp8` builds this
layout from a bf16 cache on the GPU.  :func:`sparse_attn_fp8` is the bf16 op
(``track-01/submission.py:975``) applied to the dequantised cache.  It
gathers 516 bytes per slot instead of 1024 and runs both products on e4m3
tensor-core MMAs (kernel ``sa_fp8_fwd_kernel`` in ``libsparse_attn.so``).
The reference has no fp8 cache.
"""
from __future__ import annotations

import torch

from . import _lib
from .op import _cached_workspace, _pad_heads, _padded_heads, _row_ok, workspace_bytes

__all__ = ["quantize_kv_fp8", "sparse_attn_fp8", "sparse_attn_fp8_out"]

FP8 = torch.float8_e4m3fn


def quantize_kv_fp8(kv: torch.Tensor, *, out=None, scale_out=None, stream=None):
    """bf16 cache [b, kv_len, 512] -> (e4m3 cache, fp32 scales [b, kv_len]).

    Per row: ``amax = max|x|``, ``kv8 = e4m3_rn_satfinite(x * (448 / amax))``,
    ``kv_scale = amax / 448``.  An all-zero row gives zeros and scale 0.
    """
    if kv.dim() != 3 or kv.dtype != torch.bfloat16 or not kv.is_cuda:
        raise RuntimeError("quantize_kv_fp8: expected a CUDA bf16 tensor [b, kv_len, d]")
    b, kv_len, d = kv.shape
    kv_c = kv if _row_ok(kv) else kv.contiguous()
    kv8 = torch.empty(b, kv_len, d, dtype=FP8, device=kv.device) if out is None else out
    sc = torch.empty(b, kv_len, dtype=torch.float32, device=kv.device) \
        if scale_out is None else scale_out
    st = torch.cuda.current_stream(kv.device) if stream is None else stream
    with torch.cuda.device(kv.device):
        _lib.check(_lib.lib().sa_quantize_kv_fp8(
            kv_c.data_ptr(), kv8.data_ptr(), sc.data_ptr(), b, kv_len, d,
            _lib.i64_array(kv_c.stride()), _lib.i64_array(kv8.stride()),
            _lib.i64_array(sc.stride()), st.cuda_stream))
    return kv8, sc


def sparse_attn_fp8_out(o, q, kv8, kv_scale, attn_sink, topk_idxs, scale, workspace=None, *,
                        grid: int = 0, stream=None):
    """Write ``sparse_attn_fp8(...)`` into ``o`` (no copies; see ``sparse_attn_out``)."""
    b, m, h, d = q.shape
    kv_len, topk = kv8.shape[1], topk_idxs.shape[-1]
    st = torch.cuda.current_stream(q.device) if stream is None else stream
    if workspace is None:
        workspace = _cached_workspace(q.device, st, workspace_bytes(b, m, topk, q.device))
    rc = _lib.lib().sa_fwd_fp8(
        q.data_ptr(), kv8.data_ptr(), kv_scale.data_ptr(), attn_sink.data_ptr(),
        topk_idxs.data_ptr(), o.data_ptr(), b, m, h, d, kv_len, topk,
        _lib.i64_array(q.stride()), _lib.i64_array(kv8.stride()),
        _lib.i64_array(kv_scale.stride()), _lib.i64_array(topk_idxs.stride()),
        _lib.i64_array(o.stride()), float(scale), workspace.data_ptr(), workspace.numel(),
        st.cuda_stream, int(grid))
    _lib.check(rc)
    return o


def sparse_attn_fp8(q, kv8, kv_scale, attn_sink, topk_idxs, scale):
    """Top-k sparse attention with sink over an e4m3 cache.

    Args:
        q:          [b, m, h, 512] bf16 (any h; padded to a multiple of 16)
        kv8:        [b, kv_len, 512] float8_e4m3fn (K and V shared)
        kv_scale:   [b, kv_len] fp32 (dequantised row = kv8 row * scale)
        attn_sink:  [h] fp32
        topk_idxs:  [b, m, topk] int32; -1 (or any index outside [0, kv_len))
                    marks a masked slot
        scale:      float
    Returns:
        o:          [b, m, h, 512] bf16
    """
    assert q.dim() == 4
    for name, t in (("q", q), ("kv8", kv8), ("kv_scale", kv_scale), ("attn_sink", attn_sink),
                    ("topk_idxs", topk_idxs)):
        if not t.is_cuda:
            raise RuntimeError(f"sparse_attn_fp8: {name} must be a CUDA tensor (no CPU path)")
    if q.dtype != torch.bfloat16 or kv8.dtype != FP8 or kv_scale.dtype != torch.float32 \
            or attn_sink.dtype != torch.float32 or topk_idxs.dtype != torch.int32:
        raise RuntimeError("sparse_attn_fp8: expected q bf16, kv8 float8_e4m3fn, kv_scale fp32, "
                           "attn_sink fp32, topk_idxs int32")
    b, m, h, d = q.shape
    if kv8.dim() != 3 or kv8.shape[0] != b or kv8.shape[2] != d or \
            tuple(kv_scale.shape) != (b, kv8.shape[1]) or tuple(topk_idxs.shape[:2]) != (b, m) or \
            tuple(attn_sink.shape) != (h,):
        raise RuntimeError("sparse_attn_fp8: inconsistent shapes")
    hp = _padded_heads(h)
    if hp != h:
        qp, sp = _pad_heads(q, attn_sink, hp)
        return sparse_attn_fp8(qp, kv8, kv_scale, sp, topk_idxs, scale)[:, :, :h].contiguous()
    q_c = q if _row_ok(q) else q.contiguous()
    kv_c = kv8 if (kv8.stride(-1) == 1 and kv8.data_ptr() % 16 == 0 and
                   all(s % 16 == 0 for s in kv8.stride()[:-1])) else kv8.contiguous()
    o = torch.empty(b, m, h, d, dtype=q.dtype, device=q.device)
    if o.numel() == 0:
        return o
    with torch.cuda.device(q.device):
        return sparse_attn_fp8_out(o, q_c, kv_c, kv_scale, attn_sink.contiguous(), topk_idxs,
                                   float(scale))
