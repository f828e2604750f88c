"""Row-sharded run over NCCL on 2 GPUs against the CPU oracle (GPU).

Skipped unless at least two GPUs are visible.  Each rank computes its row
range of a reduced long-context problem with the B200 op and the ranks
all-gather the output; the CPU oracle on the same inputs checks every row,
within the parity tolerance (atol = rtol = 2e-2).  NVLS is off
(NCCL_NVLS_ENABLE=0): the test needs only a plain all-gather.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    import dataclasses
    from sparse_attn.workloads import CONFIGS, make_inputs
    cfg = dataclasses.replace(CONFIGS["long"], b=2, m=96)
    return make_inputs(cfg, seed=5)


def _worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from sparse_attn.shard import sparse_attn_sharded
    q, kv, sink, idx, scale = _inputs()
    o = sparse_attn_sharded(q.to(dev), kv.to(dev), sink.to(dev), idx.to(dev), scale)
    torch.cuda.synchronize()
    if rank == 0:
        torch.save(o.cpu(), path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_nccl_two_gpus_matches_oracle(tmp_path):
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    path = str(tmp_path / "o.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    q, kv, sink, idx, scale = _inputs()
    ref = sparse_attn_oracle(q, kv, sink, idx, scale)
    from helpers import assert_close
    assert_close(torch.load(path), ref, what="2-GPU sharded vs oracle")
