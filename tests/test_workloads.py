"""Input generators: distinctness, ranges and the configs' index patterns (CPU)."""
import dataclasses

import torch

from sparse_attn.workloads import CONFIGS, gathered_bytes, make_indices, make_inputs


def _distinct(idx):
    s = idx.reshape(-1, idx.shape[-1]).sort(1).values
    return not bool(((s[:, 1:] == s[:, :-1]) & (s[:, 1:] >= 0)).any())


def test_plumbing_inputs_deterministic():
    a = make_inputs("plumbing", seed=0)
    b = make_inputs("plumbing", seed=0)
    for x, y in zip(a[:4], b[:4]):
        assert torch.equal(x, y)
    q, kv, sink, idx, scale = a
    assert q.shape == (1, 64, 16, 512) and q.dtype == torch.bfloat16
    assert kv.shape == (1, 1024, 512) and sink.shape == (16,) and idx.dtype == torch.int32
    assert _distinct(idx) and int(idx.min()) >= 0 and int(idx.max()) < 1024
    assert abs(scale - 512 ** -0.5) < 1e-12


def test_decode_indices():
    idx = make_indices(CONFIGS["decode"], torch.Generator().manual_seed(0))
    assert idx.shape == (64, 1, 2048) and _distinct(idx)
    assert int(idx.min()) >= 0 and int(idx.max()) < 32768
    assert gathered_bytes(idx, 32768) == 134217728


def test_causal_indices():
    idx = make_indices(CONFIGS["causal"], torch.Generator().manual_seed(0))[0]
    valid = idx >= 0
    assert int(valid.sum()) == 6292480
    cnt = valid.sum(1)
    assert torch.equal(cnt, torch.clamp(torch.arange(4096) + 1, max=2048))
    # padding sits at the row end and every valid index is causal
    assert bool((valid[:, :-1] | ~valid[:, 1:]).all())
    assert bool((idx.max(1).values <= torch.arange(4096)).all())
    assert _distinct(idx)


def test_mtp_and_long_patterns_small():
    cfg = dataclasses.replace(CONFIGS["mtp"], b=4)
    idx = make_indices(cfg, torch.Generator().manual_seed(0))
    assert _distinct(idx) and int(idx.min()) >= 0 and int(idx.max()) < 131072
    local = (idx >= 131072 - 8192).sum(-1)
    assert bool((local >= 1536).all())
    cfg = dataclasses.replace(CONFIGS["long"], b=1, m=16)
    idx = make_indices(cfg, torch.Generator().manual_seed(1))
    assert _distinct(idx) and int(idx.min()) >= 0 and int(idx.max()) < 65536
