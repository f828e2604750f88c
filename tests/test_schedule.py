"""The row schedule of the prefill kernels, restated on the CPU.

``snake_row`` mirrors ``snake_row`` in kernelgen-challenge_b200/csrc/sa_common.cuh,
and ``row_units`` mirrors ``sa_row_units_kernel`` in csrc/sa_ws.cu.  The GPU
parity tests check the kernels' outputs.  These check the schedule's own
properties: every row runs exactly once, and the causal configuration's CTA
loads are balanced.
"""
import pytest
import torch

from sparse_attn.workloads import CONFIGS, make_indices

UK = 64  # keys per unit (ws and fp8 kernels)


def snake_row(k, g, G, R):
    pos = k * G + ((G - 1 - g) if k & 1 else g)
    return R - 1 - pos if pos < R else -1


def rows_of_cta(g, G, R):
    out, k = [], 0
    while (r := snake_row(k, g, G, R)) >= 0:
        out.append(r)
        k += 1
    return out


def row_units(idx_row, kv_len):
    valid = (idx_row >= 0) & (idx_row < kv_len)
    nz = valid.nonzero()
    last = int(nz[-1]) if nz.numel() else -1
    return 1 if last < 0 else (last + UK) // UK


@pytest.mark.parametrize("G,R", [(1, 2), (3, 40), (37, 1200), (148, 4096), (148, 16384),
                                 (296, 4097)])
def test_every_row_exactly_once(G, R):
    seen = sorted(r for g in range(G) for r in rows_of_cta(g, G, R))
    assert seen == list(range(R))
    counts = [len(rows_of_cta(g, G, R)) for g in range(G)]
    assert max(counts) - min(counts) <= 1


def test_row_units_follow_the_last_valid_slot():
    kv_len = 1000
    row = torch.full((300,), -1, dtype=torch.int32)
    assert row_units(row, kv_len) == 1          # no valid slot: one unit, o = 0
    row[0] = 5
    assert row_units(row, kv_len) == 1
    row[64] = 7
    assert row_units(row, kv_len) == 2
    row[299] = kv_len                            # out of range: not valid
    assert row_units(row, kv_len) == 2
    row[130] = -3
    assert row_units(row, kv_len) == 2


def test_causal_loads_balanced():
    """Causal prefill (row i: min(i+1, 2048) valid slots, then -1): with the
    snake order every CTA's load (units + one per row) is within one row of
    the mean, against 913 unit-equivalents per CTA for contiguous ranges."""
    cfg = CONFIGS["causal"]
    idx = make_indices(cfg, torch.Generator().manual_seed(0))[0]
    R, G = idx.shape[0], 148
    units = [row_units(idx[r], cfg.kv_len) for r in range(R)]
    assert units[0] == 1 and units[-1] == 32 and units[2047] == 32 and units[63] == 1
    loads = [sum(units[r] + 1 for r in rows_of_cta(g, G, R)) for g in range(G)]
    mean = sum(loads) / G
    assert max(loads) <= mean + 33
    assert max(loads) < 0.8 * (R * (cfg.topk // UK + 1) / G)
