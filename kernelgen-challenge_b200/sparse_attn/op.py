"""``sparse_attn`` over the C ABI, plus its torch custom-op registration.

Drop-in for ``track-01/submission.py:975`` — same name, arguments, dtypes,
shapes and return value:

    sparse_attn(q[b,m,h,512] bf16, kv[b,kv_len,512] bf16, attn_sink[h] fp32,
                topk_idxs[b,m,topk] int32, scale: float) -> o[b,m,h,512] bf16

for any h: the kernels run heads in groups of 16, and a head count that is
not a multiple of 16 is zero-padded up to one.

Like the reference wrapper it asserts ``q.dim() == 4`` (submission.py:989),
makes the inputs contiguous (:995-998) and allocates the output (:1000); the
launch goes to ``libsparse_attn.so`` on the current CUDA stream.  Anything the
C library rejects raises ``RuntimeError`` with the library's status text.
There is no CPU path: CPU tensors raise.

The call path is kept short (the kernels of a decode step take ~40 us, so
host overhead matters): the workspace is cached per (device, stream) and
reused by every call on that stream (stream order makes that safe; ~19 MB per
stream on a B200), and the C library is called directly.  The same function
is registered as the torch custom op ``torch.ops.sparse_attn_b200.fwd`` (with
a fake implementation) for graph capture and ``torch.compile`` users.
"""
from __future__ import annotations

import functools

import torch

from . import _lib

__all__ = ["sparse_attn", "sparse_attn_out", "sparse_attn_backward", "workspace_bytes"]


def _device_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    return device.index if device.index is not None else torch.cuda.current_device()


@functools.lru_cache(maxsize=256)
def _workspace_bytes(b: int, m: int, topk: int, dev: int) -> int:
    n = _lib.lib().sa_workspace_bytes(b, m, topk, dev)
    if n == 0:
        raise RuntimeError(f"sparse_attn: cannot size workspace on cuda:{dev}")
    return int(n)


def workspace_bytes(b: int, m: int, topk: int, device: torch.device | int | None = None) -> int:
    """Device workspace (bytes) ``sparse_attn_out`` needs for this problem."""
    return _workspace_bytes(int(b), int(m), int(topk), _device_index(device))


_ws_cache: dict = {}


def _cached_workspace(dev: torch.device, stream, nbytes: int) -> torch.Tensor:
    key = (dev.index, stream.cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        # zero-filled once: the library leaves it zero-filled after every call
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _ws_cache[key] = ws
    return ws


def _validate(q, kv, attn_sink, topk_idxs):
    assert q.dim() == 4
    if kv.dim() != 3 or attn_sink.dim() != 1 or topk_idxs.dim() != 3:
        raise RuntimeError("sparse_attn: expected kv [b,kv_len,d], attn_sink [h], "
                           "topk_idxs [b,m,topk]")
    for name, t in (("q", q), ("kv", kv), ("attn_sink", attn_sink), ("topk_idxs", topk_idxs)):
        if not t.is_cuda:
            raise RuntimeError(f"sparse_attn: {name} must be a CUDA tensor (no CPU path)")
    if q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise RuntimeError("sparse_attn: q and kv must be bfloat16")
    if attn_sink.dtype != torch.float32:
        raise RuntimeError("sparse_attn: attn_sink must be float32")
    if topk_idxs.dtype != torch.int32:
        raise RuntimeError("sparse_attn: topk_idxs must be int32")
    b, m, h, d = q.shape
    if kv.shape[0] != b or kv.shape[2] != d or topk_idxs.shape[:2] != (b, m) \
            or attn_sink.shape[0] != h:
        raise RuntimeError(f"sparse_attn: inconsistent shapes q{tuple(q.shape)} "
                           f"kv{tuple(kv.shape)} sink{tuple(attn_sink.shape)} "
                           f"idx{tuple(topk_idxs.shape)}")


def _row_ok(t: torch.Tensor) -> bool:
    return t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(
        s % 8 == 0 for s in t.stride()[:-1])


def sparse_attn_out(o, q, kv, attn_sink, topk_idxs, scale, workspace=None, *,
                    variant: int = _lib.SA_VARIANT_AUTO, grid: int = 0, stream=None):
    """Write ``sparse_attn(q, kv, attn_sink, topk_idxs, scale)`` into ``o``.

    No copies: q/kv/o need a unit last-dim stride and 16-byte aligned rows.
    ``workspace`` (uint8 CUDA tensor of at least :func:`workspace_bytes`,
    zero-filled before its first use; every call leaves its merge counters
    zero) is taken from a per-(device, stream) cache when omitted.  ``variant``/``grid`` select the kernel
    variant and persistent grid size (0 = automatic).
    """
    b, m, h, d = q.shape
    kv_len, topk = kv.shape[1], topk_idxs.shape[-1]
    st = torch.cuda.current_stream(q.device) if stream is None else stream
    if workspace is None:
        workspace = _cached_workspace(q.device, st, workspace_bytes(b, m, topk, q.device))
    L = _lib.lib()
    rc = L.sa_fwd_ex(
        q.data_ptr(), kv.data_ptr(), attn_sink.data_ptr(), topk_idxs.data_ptr(), o.data_ptr(),
        b, m, h, d, kv_len, topk,
        _lib.i64_array(q.stride()), _lib.i64_array(kv.stride()),
        _lib.i64_array(topk_idxs.stride()), _lib.i64_array(o.stride()),
        float(scale), workspace.data_ptr(), workspace.numel(), st.cuda_stream,
        int(variant), int(grid))
    _lib.check(rc)
    return o


_KERNEL_HEADS = 16


def _padded_heads(h: int) -> int:
    """The head count the kernels run: h rounded up to a multiple of 16 (the
    C library takes multiples of 16 as groups of 16; the reference pads its
    head tile to max(16, next_pow2(h)) and masks, submission.py:1004).  Heads
    are independent, so padded heads only cost their own work."""
    return -(-h // _KERNEL_HEADS) * _KERNEL_HEADS


def _pad_heads(q, attn_sink, hp):
    h = q.shape[2]
    qp = q.new_zeros(*q.shape[:2], hp, q.shape[3])
    qp[:, :, :h] = q
    sp = attn_sink.new_zeros(hp)
    sp[:h] = attn_sink
    return qp, sp


def _forward(q, kv, attn_sink, topk_idxs, scale):
    _validate(q, kv, attn_sink, topk_idxs)
    h = q.shape[2]
    hp = _padded_heads(h)
    if h != hp:
        qp, sp = _pad_heads(q, attn_sink, hp)
        return _forward(qp, kv, sp, topk_idxs, scale)[:, :, :h].contiguous()
    q_c = q if _row_ok(q) else q.contiguous()
    kv_c = kv if _row_ok(kv) else kv.contiguous()
    sink_c = attn_sink.contiguous()
    b, m, h, d = q.shape
    o = torch.empty(b, m, h, d, dtype=q.dtype, device=q.device)
    if o.numel() == 0:
        return o
    if q.device.index != torch.cuda.current_device():
        with torch.cuda.device(q.device):
            return sparse_attn_out(o, q_c, kv_c, sink_c, topk_idxs, scale)
    return sparse_attn_out(o, q_c, kv_c, sink_c, topk_idxs, scale)


@torch.library.custom_op("sparse_attn_b200::fwd", mutates_args=())
def _fwd(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
         topk_idxs: torch.Tensor, scale: float) -> torch.Tensor:
    return _forward(q, kv, attn_sink, topk_idxs, scale)


@_fwd.register_fake
def _(q, kv, attn_sink, topk_idxs, scale):
    assert q.dim() == 4
    return q.new_empty(q.shape)


def _forward_train(q, kv, attn_sink, topk_idxs, scale):
    """(o, lse): the forward through ``sa_fwd_train``, which also returns the
    per-row, per-head log2 softmax denominator (fp32 [b, m, h]) for the
    backward pass."""
    _validate(q, kv, attn_sink, topk_idxs)
    h = q.shape[2]
    hp = _padded_heads(h)
    if h != hp:
        qp, sp = _pad_heads(q, attn_sink, hp)
        o, lse = _forward_train(qp, kv, sp, topk_idxs, scale)
        return o[:, :, :h].contiguous(), lse[:, :, :h].contiguous()
    q_c = q if _row_ok(q) else q.contiguous()
    kv_c = kv if _row_ok(kv) else kv.contiguous()
    b, m, _, d = q.shape
    o = torch.empty(b, m, h, d, dtype=q.dtype, device=q.device)
    lse = torch.empty(b, m, h, dtype=torch.float32, device=q.device)
    if o.numel() == 0:
        return o, lse
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream(q.device)
        ws = _cached_workspace(q.device, st, workspace_bytes(b, m, topk_idxs.shape[-1], q.device))
        _lib.check(_lib.lib().sa_fwd_train(
            q_c.data_ptr(), kv_c.data_ptr(), attn_sink.contiguous().data_ptr(),
            topk_idxs.data_ptr(), o.data_ptr(), lse.data_ptr(), b, m, h, d, kv.shape[1],
            topk_idxs.shape[-1], _lib.i64_array(q_c.stride()), _lib.i64_array(kv_c.stride()),
            _lib.i64_array(topk_idxs.stride()), _lib.i64_array(o.stride()), float(scale),
            ws.data_ptr(), ws.numel(), st.cuda_stream))
    return o, lse


_SM_COUNTS = {}


def _sm_count(device) -> int:
    idx = torch.device(device).index
    if idx not in _SM_COUNTS:
        _SM_COUNTS[idx] = torch.cuda.get_device_properties(device).multi_processor_count
    return _SM_COUNTS[idx]


def sparse_attn_backward(q, kv, attn_sink, topk_idxs, scale, o, do, lse=None):
    """Gradients of ``sparse_attn`` (``sa_bwd`` in ``libsparse_attn.so``).

    Given the forward's inputs, its output ``o`` and the upstream gradient
    ``do``, returns ``(dq, dkv, dsink)`` with the dtypes of q, kv and
    attn_sink.  ``lse`` (from the training forward) saves the kernel its first
    pass over the gathered rows.  Masked slots contribute nothing; duplicated indices add.  The
    reference has no backward: this is the gradient of its forward
    (track-01/reference/reference.py:24-40).
    """
    _validate(q, kv, attn_sink, topk_idxs)
    h = q.shape[2]
    if h != _padded_heads(h):  # zero heads: zero gradients of their own, none into kv
        pad = _padded_heads(h) - h
        zq = q.new_zeros(*q.shape[:2], pad, q.shape[3])
        lse_p = None if lse is None else torch.cat([lse, lse.new_zeros(*lse.shape[:2], pad)], 2)
        dq, dkv, dsink = sparse_attn_backward(
            torch.cat([q, zq], 2), kv, torch.cat([attn_sink, attn_sink.new_zeros(pad)]),
            topk_idxs, scale, torch.cat([o, torch.zeros_like(zq)], 2),
            torch.cat([do, torch.zeros_like(zq)], 2), lse_p)
        return dq[:, :, :h].contiguous(), dkv, dsink[:h].contiguous()
    b, m, _, d = q.shape
    q_c = q if _row_ok(q) else q.contiguous()
    kv_c = kv if _row_ok(kv) else kv.contiguous()
    o_c, do_c = o.contiguous(), do.to(q.dtype).contiguous()
    dq = torch.empty(b, m, h, d, dtype=q.dtype, device=q.device)
    topk = topk_idxs.shape[-1]
    # Few touched rows (m * topk < kv_len: decode, MTP): the fp32 buffer is
    # zeroed, and cast to the bf16 gradient, on the rows the valid slots name
    # only; the rest of the bf16 gradient is a plain zero fill.
    rows_only = m * topk < kv.shape[1] and b * m > 0
    if rows_only:
        dkv = torch.empty(kv.shape, dtype=torch.float32, device=q.device)
    else:
        dkv = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)
    dsink = torch.zeros(h, dtype=torch.float32, device=q.device)
    if dq.numel() == 0:
        return dq, dkv.to(kv.dtype), dsink.to(attn_sink.dtype)
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream(q.device)
        lse_c = None if lse is None else lse.float().contiguous()
        ids = (b, m, topk, kv.shape[1], _lib.i64_array(topk_idxs.stride()))
        if rows_only:
            _lib.check(_lib.lib().sa_dkv_zero_rows(
                dkv.data_ptr(), topk_idxs.data_ptr(), *ids[:4], ids[4],
                _lib.i64_array(dkv.stride()), st.cuda_stream))
        # decode-shaped calls with the lse: rows split over CTAs, dq through
        # an fp32 scratch (sa_bwd_ex)
        dq_acc = None
        if lse_c is not None and 2 * b * m <= _sm_count(q.device):
            dq_acc = torch.zeros(dq.shape, dtype=torch.float32, device=q.device)
        _lib.check(_lib.lib().sa_bwd_ex(
            q_c.data_ptr(), kv_c.data_ptr(), attn_sink.contiguous().data_ptr(),
            topk_idxs.data_ptr(), o_c.data_ptr(), do_c.data_ptr(),
            None if lse_c is None else lse_c.data_ptr(), dq.data_ptr(),
            dkv.data_ptr(), dsink.data_ptr(), b, m, h, d, kv.shape[1], topk_idxs.shape[-1],
            _lib.i64_array(q_c.stride()), _lib.i64_array(kv_c.stride()),
            _lib.i64_array(topk_idxs.stride()), _lib.i64_array(o_c.stride()),
            _lib.i64_array(dkv.stride()), float(scale),
            None if dq_acc is None else dq_acc.data_ptr(), st.cuda_stream))
        if rows_only:
            out = torch.zeros(kv.shape, dtype=kv.dtype, device=q.device)
            _lib.check(_lib.lib().sa_dkv_cast_rows(
                dkv.data_ptr(), out.data_ptr(), topk_idxs.data_ptr(), *ids[:4], ids[4],
                _lib.i64_array(dkv.stride()), _lib.i64_array(out.stride()), st.cuda_stream))
            return dq, out, dsink.to(attn_sink.dtype)
    return dq, dkv.to(kv.dtype), dsink.to(attn_sink.dtype)


def _setup_context(ctx, inputs, output):
    q, kv, attn_sink, topk_idxs, scale = inputs
    ctx.save_for_backward(q, kv, attn_sink, topk_idxs, output)
    ctx.scale = scale


def _fwd_backward(ctx, grad_o):
    q, kv, attn_sink, topk_idxs, o = ctx.saved_tensors
    dq, dkv, dsink = sparse_attn_backward(q, kv, attn_sink, topk_idxs, ctx.scale, o, grad_o)
    return dq, dkv, dsink, None, None


torch.library.register_autograd("sparse_attn_b200::fwd", _fwd_backward,
                                setup_context=_setup_context)


@torch.library.custom_op("sparse_attn_b200::fwd_train", mutates_args=())
def _fwd_train(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
               topk_idxs: torch.Tensor, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    return _forward_train(q, kv, attn_sink, topk_idxs, scale)


@_fwd_train.register_fake
def _(q, kv, attn_sink, topk_idxs, scale):
    assert q.dim() == 4
    return q.new_empty(q.shape), q.new_empty(q.shape[:3], dtype=torch.float32)


def _setup_context_train(ctx, inputs, output):
    q, kv, attn_sink, topk_idxs, scale = inputs
    o, lse = output
    ctx.save_for_backward(q, kv, attn_sink, topk_idxs, o, lse)
    ctx.scale = scale


def _fwd_train_backward(ctx, grad_o, grad_lse):
    q, kv, attn_sink, topk_idxs, o, lse = ctx.saved_tensors
    dq, dkv, dsink = sparse_attn_backward(q, kv, attn_sink, topk_idxs, ctx.scale, o, grad_o, lse)
    return dq, dkv, dsink, None, None


torch.library.register_autograd("sparse_attn_b200::fwd_train", _fwd_train_backward,
                                setup_context=_setup_context_train)


def sparse_attn(q, kv, attn_sink, topk_idxs, scale):
    """Top-k sparse attention with attention sink (track-01 signature).

    Args:
        q:          [b, m, h, d]   bf16 (any h, d = 512)
        kv:         [b, kv_len, d] bf16 (K and V shared)
        attn_sink:  [h]            fp32
        topk_idxs:  [b, m, topk]   int32; -1 (or any index outside [0, kv_len))
                    marks a masked slot
        scale:      float
    Returns:
        o:          [b, m, h, d]   bf16

    Differentiable: when autograd records (an input requires grad) the call
    goes through the registered op, whose backward is ``sa_bwd``.
    """
    if torch.is_grad_enabled() and (q.requires_grad or kv.requires_grad or
                                    attn_sink.requires_grad):
        # the training forward keeps the log-sum-exp for a one-pass backward
        return torch.ops.sparse_attn_b200.fwd_train(q, kv, attn_sink, topk_idxs, float(scale))[0]
    return _forward(q, kv, attn_sink, topk_idxs, float(scale))
