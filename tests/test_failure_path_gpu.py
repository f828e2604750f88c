"""The bounded-wait failure path of the pipelined kernels (GPU).

Every mbarrier wait in the sa_fwd (warp-specialized) and sa_fwd_fp8 kernels
gives up after a bounded number of polls, records an error code that
``sa_device_status`` reports, stops issuing copies, waits for those already in
flight and returns.  These tests make a wait run out without faulting
anything: ``SA_OPT_TEST_STALL`` withholds one arrival on the first ring slot
(a flag that nothing else sets) and ``SA_OPT_SPIN_LIMIT`` shortens the wait.
They then check that the call returned, that the status word carries the
consumer's code, that ``sa_device_status_reset`` clears it, and that the next
call is correct against the CPU oracle.  The calls are decode-shaped: a few
units per CTA, split rows merged by the combine kernel.
"""
import dataclasses

import pytest
import torch

from helpers import assert_close
from oracle.sparse_attn_oracle import sparse_attn_fp8_oracle, sparse_attn_oracle
from sparse_attn import _lib, quantize_kv_fp8, sparse_attn_fp8_out, sparse_attn_out
from sparse_attn.workloads import CONFIGS, make_inputs  # noqa: F401

pytestmark = pytest.mark.gpu

# a wait on a ring slot's full barrier (8) or on a free slot (1) runs out; ws
# reports 100 + code, fp8 200 + code
WS_CODES = (101, 108)
FP8_CODES = (201, 208)


def _cuda(*ts):
    return [t.cuda() if torch.is_tensor(t) else t for t in ts]


@pytest.fixture
def stalled():
    """Short waits plus the withheld arrival, always undone afterwards."""
    _lib.device_status_reset()
    old_spin = _lib.set_option(_lib.SA_OPT_SPIN_LIMIT, 2048)
    old_stall = _lib.set_option(_lib.SA_OPT_TEST_STALL, 1)
    try:
        yield
    finally:
        _lib.set_option(_lib.SA_OPT_TEST_STALL, old_stall)
        _lib.set_option(_lib.SA_OPT_SPIN_LIMIT, old_spin)
        torch.cuda.synchronize()
        _lib.device_status_reset()


def _sample(cfg_name, seed, **over):
    cfg = dataclasses.replace(CONFIGS[cfg_name], **over) if over else cfg_name
    return make_inputs(cfg, seed=seed)


def test_ws_wait_runs_out_then_recovers(stalled):
    q, kv, sink, idx, scale = _sample("decode", 3, b=8)
    qd, kvd, sd, idd = _cuda(q, kv, sink, idx)
    o = torch.empty_like(qd)
    sparse_attn_out(o, qd, kvd, sd, idd, scale)  # returns: nothing waits forever
    torch.cuda.synchronize()
    assert _lib.device_status() in WS_CODES
    _lib.device_status_reset()
    assert _lib.device_status() == 0
    # healthy again: defaults restored, same call, right answer
    _lib.set_option(_lib.SA_OPT_TEST_STALL, 0)
    _lib.set_option(_lib.SA_OPT_SPIN_LIMIT, 0)
    sparse_attn_out(o, qd, kvd, sd, idd, scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert_close(o, sparse_attn_oracle(q, kv, sink, idx, scale), what="after recovery")


def test_fp8_wait_runs_out_then_recovers(stalled):
    q, kv, sink, idx, scale = _sample("decode", 5, b=4)
    qd, kvd, sd, idd = _cuda(q, kv, sink, idx)
    kv8, ks = quantize_kv_fp8(kvd)
    o = torch.empty_like(qd)
    sparse_attn_fp8_out(o, qd, kv8, ks, sd, idd, scale)
    torch.cuda.synchronize()
    assert _lib.device_status() in FP8_CODES
    _lib.device_status_reset()
    _lib.set_option(_lib.SA_OPT_TEST_STALL, 0)
    _lib.set_option(_lib.SA_OPT_SPIN_LIMIT, 0)
    sparse_attn_fp8_out(o, qd, kv8, ks, sd, idd, scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = sparse_attn_fp8_oracle(q, kv8.cpu(), ks.cpu(), sink, idx, scale)
    assert_close(o, ref, what="fp8 after recovery")


def test_options_validate():
    assert _lib.lib().sa_set_option(99, 0) == _lib.SA_ERR_INVALID_ARG
    assert _lib.lib().sa_set_option(_lib.SA_OPT_TEST_STALL, 2) == _lib.SA_ERR_INVALID_ARG
    assert _lib.lib().sa_get_option(_lib.SA_OPT_TEST_STALL) == 0
