"""Row sharding of ``sparse_attn`` across the GPUs of one node.

Every query row (b, m) is independent: the reference runs one program per
row with no communication between programs (track-01/submission.py:290-291,
grid ``(m, b)`` at :1005).  So a job is split into contiguous ranges of the
flattened row index ``r = b * m_total + m``, one range per rank, balanced to
within one row; each rank runs the op on its own rows with its batch's KV
cache, and the output is assembled by one all-gather at the end (the only
collective, outside the op's hot path).

``sparse_attn_sharded`` is the SPMD entry: call it on every rank of a
``torch.distributed`` group (NCCL on GPUs) with the same full-size inputs (or
at least the rows and KV caches the rank needs) on the rank's device.
"""
from __future__ import annotations

import dataclasses

import torch

__all__ = ["RowPiece", "RowBlock", "partition_rows", "partition_blocks", "sparse_attn_sharded"]


@dataclasses.dataclass(frozen=True)
class RowPiece:
    """Rows ``m0:m1`` of batch item ``b`` (flattened rows ``r0:r1``)."""
    b: int
    m0: int
    m1: int
    r0: int
    r1: int


def row_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced range of ``n_rows`` for ``rank`` of ``world``."""
    return (rank * n_rows) // world, ((rank + 1) * n_rows) // world


def partition_rows(b: int, m: int, world: int, rank: int) -> list[RowPiece]:
    """The rows of ``rank``, cut at batch boundaries (one op call per piece)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    r0, r1 = row_range(b * m, world, rank)
    pieces = []
    r = r0
    while r < r1:
        bi, mi = divmod(r, m)
        end = min(r1, (bi + 1) * m)
        pieces.append(RowPiece(bi, mi, mi + (end - r), r, end))
        r = end
    return pieces


@dataclasses.dataclass(frozen=True)
class RowBlock:
    """Rows ``m0:m1`` of batch items ``b0:b1``: one op call over a contiguous
    slab (``q[b0:b1, m0:m1]``).  Either whole batch items (``m0 = 0``,
    ``m1 = m``) or a part of one batch item (``b1 = b0 + 1``)."""
    b0: int
    b1: int
    m0: int
    m1: int

    @property
    def rows(self) -> int:
        return (self.b1 - self.b0) * (self.m1 - self.m0)


def partition_blocks(b: int, m: int, world: int, rank: int) -> list[RowBlock]:
    """The rows of ``rank`` (as :func:`partition_rows`) as at most three
    slabs: a leading partial batch item, the whole batch items, a trailing
    partial one.  At one rank that is one block covering the whole job."""
    pieces = partition_rows(b, m, world, rank)
    blocks: list[RowBlock] = []
    for p in pieces:
        full = p.m0 == 0 and p.m1 == m
        last = blocks[-1] if blocks else None
        if full and last is not None and last.m0 == 0 and last.m1 == m and last.b1 == p.b:
            blocks[-1] = RowBlock(last.b0, p.b + 1, 0, m)
        else:
            blocks.append(RowBlock(p.b, p.b + 1, p.m0, p.m1))
    return blocks


def sparse_attn_sharded(q, kv, attn_sink, topk_idxs, scale, group=None, compute=None):
    """Run the rows of this rank and all-gather the full output on every rank.

    ``compute(q, kv, sink, idx, scale) -> o`` defaults to the B200 op
    (``sparse_attn.sparse_attn``); tests pass a CPU stand-in to exercise the
    partition and the gather on ``gloo`` without a GPU.
    """
    import torch.distributed as dist
    if compute is None:
        from .op import sparse_attn as compute
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, m, h, d = q.shape
    n_rows = b * m
    blocks = partition_blocks(b, m, world, rank)
    mine = [compute(q[k.b0:k.b1, k.m0:k.m1], kv[k.b0:k.b1], attn_sink,
                    topk_idxs[k.b0:k.b1, k.m0:k.m1], scale).reshape(-1, h, d)
            for k in blocks]
    local = torch.cat(mine) if mine else q.new_empty(0, h, d)
    # all_gather wants equal sizes: pad every rank's rows to the largest range
    chunk = max(row_range(n_rows, world, r)[1] - row_range(n_rows, world, r)[0]
                for r in range(world))
    padded = q.new_zeros(chunk, h, d)
    padded[:local.shape[0]] = local
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded, group=group)
    out = q.new_empty(n_rows, h, d)
    for r in range(world):
        a, e = row_range(n_rows, world, r)
        out[a:e] = gathered[r][:e - a]
    return out.reshape(b, m, h, d)
