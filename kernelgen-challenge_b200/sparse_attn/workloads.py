"""Seeded, CPU-generated inputs for the ``sparse_attn`` configurations.

The reference's own generator is ``track-01/workloads.py:29-37`` (randn bf16
q/kv, randn fp32 sink, ``randint`` indices drawn WITH replacement from the
global RNG, so its indices are not reproducible).  Here every tensor comes
from one seeded CPU ``torch.Generator`` and indices are drawn WITHOUT
replacement, as the benchmark configurations specify.  Tensors are made on
the CPU first so the CPU oracle and the GPU path see identical bytes.

Configurations (``h = 16``, ``d = 512``, ``scale = 512**-0.5`` as in
``track-01/workloads.py:11``):

=========  =====================================================  ==========================
name       shape                                                  indices per (b, m) row
=========  =====================================================  ==========================
plumbing   b=1   m=64   kv_len=1024   topk=64                     64 distinct U[0, 1024)
decode     b=64  m=1    kv_len=32768  topk=2048                   2048 distinct U[0, 32768)
causal     b=1   m=4096 kv_len=4096   topk=2048                   row i: min(i+1, 2048) distinct
                                                                  from [0, i], rest -1
long       b=2   m=8192 kv_len=65536  topk=2048                   1024 distinct from the 4096
                                                                  positions before p ~ U[4096,
                                                                  65536], 1024 distinct U[0,
                                                                  65536) outside that set
mtp        b=128 m=2    kv_len=131072 topk=2048                   1536 distinct from the last
                                                                  8192 positions, 512 distinct
                                                                  U[0, 131072) outside that set
=========  =====================================================  ==========================

Slot order inside a row is random (a real indexer emits indices in score
order, not position order); the causal padding ``-1`` sits at the row end.
"""
from __future__ import annotations

import dataclasses

import torch

H = 16
D = 512
SCALE = 0.04419417382415922  # 512 ** -0.5, track-01/workloads.py:11


@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    b: int
    m: int
    kv_len: int
    topk: int
    pattern: str  # "uniform" | "causal" | "long" | "mtp"


CONFIGS = {
    "plumbing": Config("plumbing", 1, 64, 1024, 64, "uniform"),
    "decode": Config("decode", 64, 1, 32768, 2048, "uniform"),
    "causal": Config("causal", 1, 4096, 4096, 2048, "causal"),
    "long": Config("long", 2, 8192, 65536, 2048, "long"),
    "mtp": Config("mtp", 128, 2, 131072, 2048, "mtp"),
}

# The reference's own benchmark table, track-01/workloads.py:15-26, as
# (label, b, m, kv_len, topk); its inputs are randn q/kv/sink and indices drawn
# WITH replacement from [0, kv_len) (track-01/workloads.py:29-37).  Used by the
# parity tests and by ``bench.py --suite reftable``.
REFERENCE_TABLE = [
    ("prefill-64x1024-1024-128", 64, 1024, 1024, 128),
    ("prefill-64x1024-1280-384", 64, 1024, 1280, 384),
    ("prefill-16x4096-4096-128", 16, 4096, 4096, 128),
    ("prefill-1x16384-16384-128", 1, 16384, 16384, 128),
    ("prefill-1x16384-20480-640", 1, 16384, 20480, 640),
    ("decode-64x1-128-128", 64, 1, 128, 128),
    ("decode-64x1-400-392", 64, 1, 400, 392),
    ("decode-64x1-640-640", 64, 1, 640, 640),
    ("decode-16x1-1408-640", 16, 1, 1408, 640),
    ("decode-1x1-4480-640", 1, 1, 4480, 640),
]

_CHUNK_ELEMS = 1 << 25  # bound the random-key scratch to ~128 MiB


def _distinct_uniform(rows: int, n: int, k: int, g: torch.Generator,
                      exclude: torch.Tensor | None = None) -> torch.Tensor:
    """``k`` distinct ints per row, uniform over [0, n) minus ``exclude``."""
    out = torch.empty(rows, k, dtype=torch.int64)
    step = max(1, _CHUNK_ELEMS // max(n, 1))
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        keys = torch.rand(r1 - r0, n, generator=g)
        if exclude is not None:
            keys.scatter_(1, exclude[r0:r1], -1.0)
        out[r0:r1] = keys.topk(k, dim=1).indices
    return out


def _shuffle_rows(x: torch.Tensor, g: torch.Generator) -> torch.Tensor:
    perm = torch.rand(x.shape, generator=g).argsort(dim=1)
    return torch.gather(x, 1, perm)


def make_indices(cfg: Config, g: torch.Generator, m0: int = 0) -> torch.Tensor:
    """int32 ``[b, m, topk]`` index tensor for ``cfg`` (CPU).

    ``m0`` is the query position of the first row within its batch item (a
    shard of rows ``m0 : m0 + cfg.m``); only the causal pattern depends on it.
    """
    rows = cfg.b * cfg.m
    k, n = cfg.topk, cfg.kv_len
    if cfg.pattern == "uniform":
        idx = _distinct_uniform(rows, n, k, g)
    elif cfg.pattern == "causal":
        # row i (query position i within its batch) may attend [0, i]
        pos = torch.arange(m0, m0 + cfg.m).repeat(cfg.b)          # [rows]
        idx = torch.empty(rows, k, dtype=torch.int64)
        step = max(1, _CHUNK_ELEMS // max(n, 1))
        ar = torch.arange(n)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            p = pos[r0:r1, None]
            keys = torch.rand(r1 - r0, n, generator=g)
            keys = torch.where(ar[None, :] <= p, keys, torch.full_like(keys, -1.0))
            kk = min(k, n)
            top = keys.topk(kk, dim=1).indices
            cnt = torch.clamp(p + 1, max=k)                        # valid slots per row
            slot = torch.arange(kk)[None, :]
            top = torch.where(slot < cnt, top, torch.full_like(top, -1))
            if kk < k:
                top = torch.cat([top, torch.full((r1 - r0, k - kk), -1, dtype=top.dtype)], 1)
            idx[r0:r1] = top
    elif cfg.pattern in ("long", "mtp"):
        if cfg.pattern == "long":
            win, n_win = 4096, k // 2
            # window end p ~ U[4096, n]: the window [p - 4096, p) lies inside [0, n)
            p = torch.randint(win, n + 1, (rows, 1), generator=g)
            start = p - win
        else:
            win, n_win = 8192, (3 * k) // 4
            start = torch.full((rows, 1), n - win, dtype=torch.int64)
        local = _distinct_uniform(rows, win, n_win, g) + start
        far = _distinct_uniform(rows, n, k - n_win, g, exclude=local)
        idx = _shuffle_rows(torch.cat([local, far], dim=1), g)
    else:
        raise ValueError(f"unknown index pattern {cfg.pattern!r}")
    return idx.to(torch.int32).reshape(cfg.b, cfg.m, k)


def make_inputs(cfg: Config | str, seed: int = 0, *, b: int | None = None,
                m: int | None = None):
    """``(q, kv, attn_sink, topk_idxs, scale)`` on the CPU for ``cfg``.

    ``b``/``m`` override the batch and query-row counts (used for bounded
    samples of a configuration); the distributions are unchanged.
    """
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    if b is not None or m is not None:
        cfg = dataclasses.replace(cfg, b=b if b is not None else cfg.b,
                                  m=m if m is not None else cfg.m)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(cfg.b, cfg.m, H, D, generator=g).to(torch.bfloat16)
    kv = torch.empty(cfg.b, cfg.kv_len, D, dtype=torch.bfloat16)
    step = max(1, _CHUNK_ELEMS // D)
    flat = kv.view(-1, D)
    for r0 in range(0, flat.shape[0], step):      # chunked: mtp kv is 16 GiB
        r1 = min(flat.shape[0], r0 + step)
        flat[r0:r1] = torch.randn(r1 - r0, D, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, generator=g, dtype=torch.float32)
    idx = make_indices(cfg, g)
    return q, kv, sink, idx, SCALE


def gathered_bytes(topk_idxs: torch.Tensor, kv_len: int, d: int = D) -> int:
    """Algorithmic gathered-KV bytes: valid slots x d x 2 B (bf16)."""
    valid = ((topk_idxs >= 0) & (topk_idxs < kv_len)).sum().item()
    return int(valid) * d * 2
