"""Profiling driver: three L2-flushed calls of one configuration.

    python -m sparse_attn.profile_case <config> [variant | fp8 | bwd]
    python -m sparse_attn.profile_case hc          (track-02 hc_split_sinkhorn)

Counterpart of the reference's ``track-01/profile.py`` (torch.profiler
timeline, :19-33); here it is the target program for ``ncu`` captures
(``-s 1 -c 1`` selects the second call).  Inputs are seeded and made on the
GPU; ``variant`` is an SA_VARIANT_* number (0 = automatic), ``fp8`` for
the e4m3 KV-cache kernel (the cache quantised on the GPU before the calls) or
``bwd`` for the backward kernel (after one forward).
"""
from __future__ import annotations

import sys

import torch

from . import (hc_split_sinkhorn, quantize_kv_fp8, sparse_attn_backward, sparse_attn_fp8_out,
               sparse_attn_out, workspace_bytes)
from .workloads import CONFIGS, D, H, SCALE, make_indices


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if argv and argv[0] == "hc":
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(0)
        mixes = torch.randn(64, 1024, 24, generator=g, device=dev)
        sc, base = torch.randn(3, generator=g, device=dev), torch.randn(24, generator=g, device=dev)
        for _ in range(3):
            out = hc_split_sinkhorn(mixes, sc, base)
        torch.cuda.synchronize()
        print(f"hc: mean comb = {out[2].mean().item():.5f}")
        return
    cfg = CONFIGS[argv[0] if argv else "decode"]
    fp8 = len(argv) > 1 and argv[1] == "fp8"
    bwd = len(argv) > 1 and argv[1] == "bwd"
    variant = int(argv[1]) if len(argv) > 1 and not (fp8 or bwd) else 0
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(cfg.b, cfg.m, H, D, generator=g, device=dev, dtype=torch.bfloat16)
    kv = torch.randn(cfg.b, cfg.kv_len, D, generator=g, device=dev, dtype=torch.bfloat16)
    sink = torch.randn(H, generator=g, device=dev)
    idx = make_indices(cfg, torch.Generator().manual_seed(0)).to(dev)
    o = torch.empty_like(q)
    ws = torch.zeros(workspace_bytes(cfg.b, cfg.m, cfg.topk, 0), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    if fp8:
        kv8, ks = quantize_kv_fp8(kv)
        del kv
    if bwd:
        sparse_attn_out(o, q, kv, sink, idx, SCALE, ws)
        do = torch.randn(q.shape, generator=g, device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            flush.zero_()
            dq, dkv, dsink = sparse_attn_backward(q, kv, sink, idx, SCALE, o, do)
        torch.cuda.synchronize()
        print(f"{cfg.name} bwd: mean |dq| = {dq.float().abs().mean().item():.5f}")
        return
    for _ in range(3):
        flush.zero_()
        if fp8:
            sparse_attn_fp8_out(o, q, kv8, ks, sink, idx, SCALE, ws)
        else:
            sparse_attn_out(o, q, kv, sink, idx, SCALE, ws, variant=variant)
    torch.cuda.synchronize()
    print(f"{cfg.name}: mean |o| = {o.float().abs().mean().item():.5f}")


if __name__ == "__main__":
    main()
