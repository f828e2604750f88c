"""Generate the golden vectors in this directory from the LIVE reference.

Run where the reference checkout is available, with its path in
``$SPARSE_ATTN_REFERENCE`` (required):

    SPARSE_ATTN_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Each case's inputs come from a seeded CPU generator (``make_case``), so only
the outputs and a SHA-256 of the input bytes are stored; the tests rebuild the
inputs, check the hash, and compare.  Outputs are produced by
``track-01/reference/reference.py:sparse_attn`` itself, unmodified:

* cases without masked slots: one call on the whole batch;
* cases with masked slots (``-1`` / out-of-range): the reference raises on
  them (torch.gather bounds check), so each query row is evaluated by the
  reference on the row's valid slots only — which is exactly the masking
  rule of ``track-01/submission.py:313-322`` (a masked slot contributes
  nothing to numerator or denominator).  A row with no valid slot is
  evaluated with an empty slot set, where the reference's own code returns
  ``o = 0`` (softmax over the sink alone, empty P V).
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "kernelgen-challenge_b200"))
sys.path.insert(0, str(HERE.parent.parent))

from sparse_attn.workloads import SCALE, make_inputs  # noqa: E402

H, D = 16, 512


def _randn_case(b, m, kv_len, topk, seed, *, with_replacement=False, masked=0.0,
                all_masked_rows=(), out_of_range=0.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, m, H, D, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, kv_len, D, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, generator=g)
    if with_replacement:  # the reference's own generator (track-01/workloads.py:36)
        idx = torch.randint(0, kv_len, (b, m, topk), generator=g, dtype=torch.int32)
    else:
        idx = torch.rand(b * m, kv_len, generator=g).topk(topk, dim=1).indices
        idx = idx.to(torch.int32).reshape(b, m, topk)
    if masked > 0:
        sel = torch.rand(b, m, topk, generator=g) < masked
        idx = torch.where(sel, torch.full_like(idx, -1), idx)
    if out_of_range > 0:
        sel = torch.rand(b, m, topk, generator=g) < out_of_range
        bad = torch.where(torch.rand(b, m, topk, generator=g) < 0.5,
                          torch.full_like(idx, kv_len), torch.full_like(idx, -7))
        idx = torch.where(sel, bad, idx)
    for (bi, mi) in all_masked_rows:
        idx[bi, mi] = -1
    return q, kv, sink, idx, SCALE


def make_case(name):
    """Inputs of golden case ``name`` (CPU tensors)."""
    if name == "plumbing":
        return make_inputs("plumbing", seed=0)
    if name == "ragged":          # topk not a multiple of any unit size
        return _randn_case(2, 3, 300, 37, seed=1)
    if name == "replacement":     # duplicates, as the reference's generator makes
        return _randn_case(3, 2, 64, 96, seed=2, with_replacement=True)
    if name == "masked":          # -1 slots, incl. whole masked rows and units
        return _randn_case(2, 5, 700, 100, seed=3, masked=0.4,
                           all_masked_rows=((0, 1), (1, 4)))
    if name == "out_of_range":    # indices outside [0, kv_len) besides -1
        return _randn_case(1, 4, 256, 80, seed=4, out_of_range=0.25)
    if name == "short":           # topk smaller than a unit, kv_len tiny
        return _randn_case(4, 1, 5, 3, seed=5)
    if name == "causal_head":     # first rows of the causal configuration
        q, kv, sink, idx, scale = make_inputs("causal", seed=0)
        return q[:, :40].contiguous(), kv, sink, idx[:, :40].contiguous(), scale
    raise KeyError(name)


CASES = ["plumbing", "ragged", "replacement", "masked", "out_of_range", "short", "causal_head"]

# fp8 cache cases: the bf16 case's cache quantised by the quantiser's CPU
# statement (oracle/sparse_attn_oracle.py:quantize_kv_fp8_ref); the expected
# output is the reference run on the dequantised fp32 cache.
FP8_CASES = ["fp8_plumbing", "fp8_masked", "fp8_causal_head"]


def make_fp8_case(name):
    """(q, kv8, kv_scale, sink, idx, scale) of fp8 golden case ``name``."""
    from oracle.sparse_attn_oracle import quantize_kv_fp8_ref
    q, kv, sink, idx, scale = make_case(name[len("fp8_"):])
    kv8, ks = quantize_kv_fp8_ref(kv)
    return q, kv8, ks, sink, idx, scale


# hc_split_sinkhorn (track-02) cases: shapes of track-02/workloads.py:21-26
# (one decode and one prefill shape) plus a ragged one
HC_CASES = {"hc_decode": (64, 1), "hc_prefill": (4, 1024), "hc_ragged": (3, 37)}


def make_hc_case(name, seed=0):
    """(mixes, hc_scale, hc_base) of hc case ``name``: N(0,1) fp32 like
    track-02/workloads.py:32-37, from a seeded CPU generator."""
    b, s = HC_CASES[name]
    g = torch.Generator().manual_seed(100 + seed + len(name))
    mixes = torch.randn(b, s, 24, generator=g)
    hc_scale = torch.randn(3, generator=g)
    hc_base = torch.randn(24, generator=g)
    return mixes, hc_scale, hc_base


def input_digest_hc(mixes, hc_scale, hc_base) -> str:
    h = hashlib.sha256()
    for t in (mixes, hc_scale, hc_base):
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def _reference_root() -> pathlib.Path:
    root = os.environ.get("SPARSE_ATTN_REFERENCE")
    if not root:
        raise RuntimeError("set SPARSE_ATTN_REFERENCE to the reference checkout")
    return pathlib.Path(root)


def _load_hc_reference():
    root = _reference_root()
    path = root / "track-02" / "reference" / "reference.py"
    spec = importlib.util.spec_from_file_location("kernelgen_track02_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.hc_split_sinkhorn


def input_digest_fp8(q, kv8, ks, sink, idx, scale) -> str:
    h = hashlib.sha256()
    for t in (q.view(torch.int16), kv8.view(torch.uint8), ks, sink, idx):
        h.update(t.contiguous().numpy().tobytes())
    h.update(repr(float(scale)).encode())
    return h.hexdigest()


def input_digest(q, kv, sink, idx, scale) -> str:
    h = hashlib.sha256()
    for t in (q.view(torch.int16), kv.view(torch.int16), sink, idx):
        h.update(t.contiguous().numpy().tobytes())
    h.update(repr(float(scale)).encode())
    return h.hexdigest()


def _load_reference(root=None):
    root = pathlib.Path(root) if root is not None else _reference_root()
    path = root / "track-01" / "reference" / "reference.py"
    spec = importlib.util.spec_from_file_location("kernelgen_track01_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.sparse_attn


def reference_output(ref, q, kv, sink, idx, scale):
    """Run the unmodified reference; masked slots handled row by row."""
    kv_len = kv.shape[1]
    valid = (idx >= 0) & (idx < kv_len)
    if bool(valid.all()):
        return ref(q, kv, sink, idx, scale)
    b, m = idx.shape[:2]
    out = torch.empty_like(q)
    for bi in range(b):
        for mi in range(m):
            keep = idx[bi, mi][valid[bi, mi]]
            out[bi:bi + 1, mi:mi + 1] = ref(q[bi:bi + 1, mi:mi + 1], kv[bi:bi + 1], sink,
                                            keep.view(1, 1, -1), scale)
    return out


def main():
    ref = _load_reference()
    for name in CASES:
        q, kv, sink, idx, scale = make_case(name)
        o = reference_output(ref, q, kv, sink, idx, scale)
        np.savez_compressed(HERE / f"{name}.npz", o=o.view(torch.int16).numpy(),
                            digest=np.array(input_digest(q, kv, sink, idx, scale)))
        print(name, tuple(o.shape), "finite:", bool(torch.isfinite(o.float()).all()))
    from oracle.sparse_attn_oracle import dequantize_kv_fp8
    for name in FP8_CASES:
        q, kv8, ks, sink, idx, scale = make_fp8_case(name)
        o = reference_output(ref, q, dequantize_kv_fp8(kv8, ks), sink, idx, scale)
        np.savez_compressed(HERE / f"{name}.npz", o=o.view(torch.int16).numpy(),
                            digest=np.array(input_digest_fp8(q, kv8, ks, sink, idx, scale)))
        print(name, tuple(o.shape), "finite:", bool(torch.isfinite(o.float()).all()))
    hc_ref = _load_hc_reference()
    for name in HC_CASES:
        mixes, sc, base = make_hc_case(name)
        pre, post, comb = hc_ref(mixes, sc, base, 4, 20, 1e-6)
        np.savez_compressed(HERE / f"{name}.npz", pre=pre.numpy(), post=post.numpy(),
                            comb=comb.numpy(), digest=np.array(input_digest_hc(mixes, sc, base)))
        print(name, tuple(comb.shape))


if __name__ == "__main__":
    main()
