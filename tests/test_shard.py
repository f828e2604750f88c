"""Row sharding across ranks: partition properties, and a world-size-2 gloo
run of the sharded entry point on CPU with the oracle as the per-rank compute.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sparse_attn.shard import partition_rows, row_range


@pytest.mark.parametrize("b,m,world", [(1, 64, 2), (64, 1, 8), (2, 8192, 8), (128, 2, 8),
                                       (3, 5, 4), (1, 3, 8)])
def test_partition_covers_every_row_once(b, m, world):
    seen = []
    sizes = []
    for rank in range(world):
        pieces = partition_rows(b, m, world, rank)
        n = 0
        for p in pieces:
            assert 0 <= p.b < b and 0 <= p.m0 < p.m1 <= m
            assert p.r1 - p.r0 == p.m1 - p.m0 and p.r0 == p.b * m + p.m0
            seen.extend(range(p.r0, p.r1))
            n += p.r1 - p.r0
        sizes.append(n)
    assert seen == list(range(b * m))
    assert max(sizes) - min(sizes) <= 1


def test_partition_matches_benchmark_shards():
    # long-context config: b=2, m=8192 over 8 GPUs -> 2048 rows per GPU
    assert [partition_rows(2, 8192, 8, r)[0].m1 - partition_rows(2, 8192, 8, r)[0].m0
            for r in range(8)] == [2048] * 8
    # MTP decode: b=128, m=2 over 8 GPUs -> 16 batch items per GPU
    assert all(len(partition_rows(128, 2, 8, r)) == 16 for r in range(8))
    assert row_range(10, 3, 2) == (6, 10)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import make_golden
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    from sparse_attn.shard import sparse_attn_sharded
    q, kv, sink, idx, scale = make_golden.make_case("masked")
    o = sparse_attn_sharded(q, kv, sink, idx, scale, compute=sparse_attn_oracle)
    if rank == 0:
        torch.save(o, result_path)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_gloo_world2_matches_unsharded(tmp_path):
    import make_golden
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    path = str(tmp_path / "o.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    o = torch.load(path)
    q, kv, sink, idx, scale = make_golden.make_case("masked")
    assert torch.equal(o, sparse_attn_oracle(q, kv, sink, idx, scale))
