"""``hc_split_sinkhorn`` (track-02 of the reference project) over the C ABI.

Drop-in for ``track-02/submission.py:316`` — same name, arguments, dtypes,
shapes and return values:

    hc_split_sinkhorn(mixes[b,s,24] fp32, hc_scale[3] fp32, hc_base[24] fp32,
                      hc_mult=4, sinkhorn_iters=20, eps=1e-6)
        -> pre[b,s,4], post[b,s,4], comb[b,s,4,4]   (fp32)

Like the reference wrapper it asserts a 3-D ``mixes`` and ``hc_mult == 4``
(submission.py:340-346) and allocates the outputs; the kernel
(``hcs_split_sinkhorn`` in ``libsparse_attn.so``) runs on the current CUDA
stream.  There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["hc_split_sinkhorn"]


def hc_split_sinkhorn(mixes, hc_scale, hc_base, hc_mult: int = 4, sinkhorn_iters: int = 20,
                      eps: float = 1e-6):
    assert mixes.dim() == 3, f"mixes must be 3D, got shape {tuple(mixes.shape)}"
    assert hc_mult == 4, f"this kernel is specialized for hc_mult=4, got {hc_mult}"
    b, s, m = mixes.shape
    assert m == (2 + hc_mult) * hc_mult, f"mixes last dim must be {(2 + hc_mult) * hc_mult}, got {m}"
    for name, t in (("mixes", mixes), ("hc_scale", hc_scale), ("hc_base", hc_base)):
        if not t.is_cuda:
            raise RuntimeError(f"hc_split_sinkhorn: {name} must be a CUDA tensor (no CPU path)")
        if t.dtype != torch.float32:
            raise RuntimeError(f"hc_split_sinkhorn: {name} must be float32")
    # the tokens r = (b, s) must sit one stride apart, with a contiguous last dim
    tok = mixes.stride(0) if s == 1 else mixes.stride(1)
    uniform = (mixes.stride(2) == 1 and tok >= m and
               (s == 1 or b == 1 or mixes.stride(0) == s * mixes.stride(1)))
    mx = mixes if uniform else mixes.contiguous()
    if not uniform:
        tok = m
    scale_c, base_c = hc_scale.contiguous(), hc_base.contiguous()
    pre = torch.empty(b, s, hc_mult, dtype=torch.float32, device=mixes.device)
    post = torch.empty(b, s, hc_mult, dtype=torch.float32, device=mixes.device)
    comb = torch.empty(b, s, hc_mult, hc_mult, dtype=torch.float32, device=mixes.device)
    n = b * s
    if n == 0:
        return pre, post, comb
    with torch.cuda.device(mixes.device):
        st = torch.cuda.current_stream(mixes.device)
        rc = _lib.lib().hcs_split_sinkhorn(
            mx.data_ptr(), scale_c.data_ptr(), base_c.data_ptr(), pre.data_ptr(),
            post.data_ptr(), comb.data_ptr(), n, tok,
            int(hc_mult), int(sinkhorn_iters), float(eps), st.cuda_stream)
    if rc != 0:
        raise RuntimeError(f"hc_split_sinkhorn: status {rc}")
    return pre, post, comb
