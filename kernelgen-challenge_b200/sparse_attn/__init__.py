"""B200-native top-k sparse attention with attention sink.

``sparse_attn(q, kv, attn_sink, topk_idxs, scale)`` is a drop-in for
``track-01/submission.py:975`` of inin-zou/kernelgen-challenge; the work runs
in hand-written sm_100a kernels in ``libsparse_attn.so`` (C ABI:
``include/sparse_attn.h``).
"""
from ._lib import (SA_VARIANT_AUTO, SA_VARIANT_MMA, SA_VARIANT_TCGEN05,  # noqa: F401
                   SA_VARIANT_WS, SA_VARIANT_WT, LIB_PATH, lib)
from .op import sparse_attn, sparse_attn_backward, sparse_attn_out, workspace_bytes  # noqa: F401
from .fp8 import quantize_kv_fp8, sparse_attn_fp8, sparse_attn_fp8_out  # noqa: F401
from .mhc import hc_split_sinkhorn  # noqa: F401
from .indexer import indexer_topk  # noqa: F401

__all__ = ["sparse_attn", "sparse_attn_out", "sparse_attn_backward", "workspace_bytes", "lib", "LIB_PATH",
           "quantize_kv_fp8", "sparse_attn_fp8", "sparse_attn_fp8_out", "hc_split_sinkhorn",
           "indexer_topk",
           "SA_VARIANT_AUTO", "SA_VARIANT_MMA", "SA_VARIANT_TCGEN05", "SA_VARIANT_WS",
           "SA_VARIANT_WT"]
