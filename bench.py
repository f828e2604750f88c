"""Benchmark of the B200 ``sparse_attn`` hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config long] [--kv bf16|fp8] [--variant auto|mma|tcgen05|ws]
    python bench.py --op gather          random-row gather ceiling (no math)
    python bench.py --suite reftable     the reference's own 10-workload table

A "step" is one pass of the op over the configuration's whole batch (default:
BASELINE config "long", b=2 m=8192 kv_len=65536 topk=2048, h=16 d=512, the
largest configuration that fits one GPU).  With N ranks (torchrun, one
process per GPU) the job is strong-scaled: rank r runs the query rows
``shard.partition_blocks(b, m, N, r)`` gives it (contiguous row ranges, no
collective on the data path) with its batch items' KV caches resident; the
step time is the max over ranks and ``value`` = the job's query-tokens / that
time.  The one collective of the sharded op, the all-gather of o, is timed
separately (``allgather``), outside the op's timed region.

``value`` is timed with CUDA events on the launching stream, inputs resident
in HBM, L2 flushed (256 MiB write) before every timed step and the flush kept
outside the events.  ``e2e`` is the same metric through the public op with the
step's q and topk_idxs copied from pinned host memory and o copied back inside
the timed region (the KV cache and sink stay resident, as a serving KV cache
does).  ``per_config`` repeats the measurement for the other BASELINE configs
(decode, causal, MTP at one GPU; MTP batch-sharded at N > 1), each with its
roofline, CPU baseline and e2e.  ``triton_reference`` times the reference's
own GPU kernel (its Triton "universal" kernel, track-01/submission.py:276-347,
called through its unmodified ``sparse_attn``) on the same inputs when the
reference is installed under ``baseline/_ref``.

``--impl reference`` times the reference's CPU algorithm (the oracle port of
track-01/reference/reference.py) on all host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kernelgen-challenge_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from sparse_attn.workloads import CONFIGS, D, H, SCALE, make_indices  # noqa: E402

METRIC = "sparse_attn query-tokens/s at topk=2048"
UNIT = "query-tokens/s"
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20
REF_DIR = ROOT / "baseline" / "_ref" / "track-01"
# steps of each per-config measurement: enough timed work (>= ~0.1 s of op
# time) for the clock sampler to see the load
PER_CONFIG_STEPS = {"decode": 3000, "mtp": 1000, "causal": 200, "long": 50}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="long")
    ap.add_argument("--variant", choices=["auto", "mma", "tcgen05", "ws", "wt"], default="auto")
    ap.add_argument("--grid", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline legs (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="measure the --config line only")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip the reference Triton kernel timing")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16",
                    help="KV cache format: bf16 (the reference's) or e4m3 + fp32 per-token "
                         "scale (sparse_attn_fp8)")
    ap.add_argument("--op", choices=["sparse_attn", "sparse_attn_bwd", "hc_sinkhorn", "indexer",
                                     "gather"],
                    default="sparse_attn",
                    help="sparse_attn_bwd: the backward pass on --config; indexer: the top-k "
                         "index producer on --config's b, m, kv_len, topk; "
                         "hc_sinkhorn: the track-02 op on its 1k-1-64 prefill shape; "
                         "gather: the random-row gather ceiling (copies only, no math)")
    ap.add_argument("--suite", choices=["none", "reftable"], default="none",
                    help="reftable: the reference's 10-workload table "
                         "(track-01/workloads.py:15-26) through the reference's torch "
                         "oracle, its Triton kernel and this library")
    ap.add_argument("--kv-policy", type=int, default=-1, choices=[-1, 0, 1, 2],
                    help="L2 policy of the KV gathers (library option SA_OPT_KV_POLICY): -1 "
                         "by the call's reuse, 0 evict_first, 1 evict_normal, 2 evict_last")
    ap.add_argument("--gather-only", action="store_true",
                    help="diagnostic: the forward kernel gathers and discards its rows "
                         "(library option SA_OPT_GATHER_ONLY); no valid output")
    ap.add_argument("--graph", action="store_true",
                    help="capture one op call in a CUDA graph and time its replays")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip the one profiled call that counts our kernel launches")
    return ap.parse_args()


class L2Flush:
    """Untimed L2 flush between timed steps: a 256 MiB write (the whole 126 MB
    L2 is replaced), then a read of another 256 MiB buffer, so the lines the
    write left dirty are written back here, outside the timed region, and the
    next step starts from a cold, clean L2.  ``read=False`` keeps the write
    alone (the step then also pays for writing those dirty lines back)."""

    def __init__(self, dev, read=True):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(L2_FLUSH_BYTES // 8, dtype=torch.int64, device=dev) if read else None

    def zero_(self):
        self.w.zero_()
        if self.r is not None:
            self._acc = self.r.sum()

    describe = ("flushed before every timed step (256 MiB write, then a 256 MiB read so the "
                "dirty lines are written back), flush untimed")


def emit(args, d):
    """Print one op's JSON line, or hand it back when the default run
    collects the other ops' lines into its own."""
    if getattr(args, "collect", False):
        return d
    print(json.dumps(d), flush=True)
    return d


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), ws


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            j = json.loads(p.read_text())
            return float(j["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------------------
# clock sampling (NVML, polled during the timed region)
# ----------------------------------------------------------------------------
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int):
        self.samples, self.reasons = [], set()
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = device_index
            if vis:
                ids = [v.strip() for v in vis.split(",") if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    phys = int(ids[device_index])
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False
        self._stop = threading.Event()

    def _sample(self):
        nv = self.nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for b, name in _REASONS.items():
            if bits & b:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if not self.ok:
            return None
        self._stop.set()
        self.t.join()
        try:
            self._sample()
        except Exception:
            pass
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(self.reasons - {"gpu_idle"})}


# ----------------------------------------------------------------------------
# inputs
# ----------------------------------------------------------------------------
def block_inputs(cfg, blk, seed, device):
    """Seeded inputs of the row block ``blk`` of ``cfg``, made on the device
    (indices on the CPU, then copied).  The KV cache of batch item j is seeded
    by j alone, so ranks that hold rows of the same batch item see the same
    cache; q and the indices are seeded by the block's first row."""
    nb, mm = blk.b1 - blk.b0, blk.m1 - blk.m0
    g = torch.Generator(device=device).manual_seed(seed * 7919 + blk.b0 * 65537 + blk.m0)
    q = torch.randn(nb, mm, H, D, generator=g, device=device, dtype=torch.bfloat16)
    kv = torch.empty(nb, cfg.kv_len, D, device=device, dtype=torch.bfloat16)
    for i in range(nb):
        kv[i].normal_(generator=torch.Generator(device=device).manual_seed(
            seed * 1000003 + blk.b0 + i))
    sink = torch.randn(H, generator=torch.Generator(device=device).manual_seed(seed),
                       device=device, dtype=torch.float32)
    icfg = dataclasses.replace(cfg, b=nb, m=mm)
    idx = make_indices(icfg, torch.Generator().manual_seed(seed + 104729 * blk.b0 + blk.m0),
                       m0=blk.m0).to(device)
    return q, kv, sink, idx


def profile_our_kernels(fn, flush, reps=5):
    """Our kernels launched per call of ``fn``, their mean device duration, and
    the mean device timeline of a call (gap after the preceding kernel, span
    from our first kernel's start to our last kernel's end), from a CUPTI trace
    of ``reps`` L2-flushed calls made outside every timed region.
    Returns (launches per call, {name: mean us}) or (None, {error})."""
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(reps):
                flush.zero_()
                fn()
            torch.cuda.synchronize()
        kern = sorted((e for e in prof.events() if e.device_type.name == "CUDA"),
                      key=lambda e: e.time_range.start)
        per, gaps, spans, n = {}, [], [], 0
        prev_end, first_start, last_end = None, None, None
        for e in kern:
            ours = "sa_" in e.name and "_kernel" in e.name
            if ours:
                short = e.name.split("(")[0].split("::")[-1]
                per.setdefault(short, []).append(e.time_range.end - e.time_range.start)
                n += 1
                if first_start is None:
                    first_start = e.time_range.start
                    if prev_end is not None:
                        gaps.append(first_start - prev_end)
                last_end = e.time_range.end
            else:
                if first_start is not None:
                    spans.append(last_end - first_start)
                    first_start = None
                prev_end = e.time_range.end
        if first_start is not None:
            spans.append(last_end - first_start)
        out = {k: statistics.mean(v) for k, v in per.items()}
        if gaps:
            out["gap_after_previous_kernel"] = statistics.mean(gaps)
        if spans:
            out["span_first_start_to_last_end"] = statistics.mean(spans)
        return n // reps, out
    except Exception as e:  # profiler unavailable: report unknown
        return None, {"profiler failed": str(e)}


# ----------------------------------------------------------------------------
# CPU legs (oracle port of the reference algorithm)
# ----------------------------------------------------------------------------
def cpu_sample_inputs(cfg, rows, seed=0):
    from sparse_attn.workloads import make_inputs
    if cfg.m >= rows:
        q, kv, sink, idx, scale = make_inputs(cfg, seed, b=1)
        return q[:, :rows].contiguous(), kv, sink, idx[:, :rows].contiguous(), scale, rows
    b = max(1, rows // cfg.m)
    q, kv, sink, idx, scale = make_inputs(cfg, seed, b=b)
    return q, kv, sink, idx, scale, b * cfg.m


CPU_IMPL = "fp32 torch CPU restatement of reference.py (oracle/sparse_attn_oracle.py)"
REF_IMPL = ("the unmodified track-01/reference/reference.py (its torch CPU path), from the "
            "copy baseline/install_reference.sh puts in baseline/_ref")


def cpu_impl(cfg=None):
    """(fn, cores, kind, description): the reference's algorithm on the host
    cores.  Where the reference's own reference.py is installed
    (baseline/_ref) and the configuration has no -1 slots (reference.py
    raises on them: the causal rows' padding), that function itself
    ("reference"); otherwise its restatement with the masking rule, written
    with the same torch ops ("port")."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ref = REF_DIR / "reference" / "reference.py"
    if cfg is not None and cfg.pattern != "causal" and ref.exists():
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        import importlib
        return importlib.import_module("reference.reference").sparse_attn, cores, "reference", REF_IMPL
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    return sparse_attn_oracle, cores, "port", CPU_IMPL


def cpu_throughput(cfg, rows, min_seconds, max_reps):
    fn, cores, _, _ = cpu_impl(cfg)
    q, kv, sink, idx, scale, n = cpu_sample_inputs(cfg, rows)
    fn(q, kv, sink, idx, scale)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        fn(q, kv, sink, idx, scale)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            break
    return n * reps / el, n, reps, el, cores


def run_reference(args):
    rank, _, _ = dist_env()
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    fn, cores, kind, desc = cpu_impl(cfg)
    rows = 16
    q, kv, sink, idx, scale, n = cpu_sample_inputs(cfg, rows)
    for _ in range(max(args.warmup, 0)):
        fn(q, kv, sink, idx, scale)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(q, kv, sink, idx, scale)
    el = time.perf_counter() - t0
    val = n * args.steps / el
    sample = (f"{n} query rows of config '{cfg.name}' per step (b=1 slice, kv_len={cfg.kv_len}, "
              f"topk={cfg.topk}), {desc}")
    line = {
        "metric": METRIC, "value": val, "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded CPU generator)",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "h": H, "d": D,
                   "kv_len": cfg.kv_len, "topk": cfg.topk, "sample_rows_per_step": n},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU leg
# ----------------------------------------------------------------------------
def measure_e2e(idx_maker, q, kv, kscale, sink, idx, dev, stream, flush, K, barrier, world,
                job_tokens, fp8):
    """The metric through the public op with host-resident q and indices.

    Every step copies its q and indices from pinned host memory to the GPU,
    runs ``sparse_attn_out`` (or ``sparse_attn_fp8_out``: the public op with a
    caller-owned output, as a serving loop calls it) and copies o back to
    pinned host memory.  Pipelined, as a serving loop runs it (captured in CUDA
    graphs, see below): the copies of later steps overlap the op of earlier
    ones, on two copy streams.  L2 is not flushed here; instead the steps rotate over four
    distinct index sets, whose gathered rows (4 x the valid slots x row bytes)
    exceed the 126 MB L2.  ``serial`` repeats the measurement without any overlap
    and with the 256 MiB flush before every step (the device-timed value's
    conditions)."""
    import sparse_attn
    ke = min(K, 100)
    nset = 4
    q_h = q.cpu().pin_memory()
    idx_cpu = [idx.cpu()] + [idx_maker(r) for r in range(1, nset)]
    idx_hs = [t.pin_memory() for t in idx_cpu]
    # A serving loop stages each step's q and indices in one pinned slab, so
    # one host-to-device copy per step carries both (two copies cost ~15 %).
    qb, ib = q.numel() * q.element_size(), idx.numel() * idx.element_size()
    slab_h = []
    for r in range(nset):
        h = torch.empty(qb + ib, dtype=torch.uint8).pin_memory()
        h[:qb].copy_(q_h.reshape(-1).view(torch.uint8))
        h[qb:].copy_(idx_hs[r].reshape(-1).view(torch.uint8))
        slab_h.append(h)

    def op_out(o, qd, idd):
        if fp8:
            sparse_attn.sparse_attn_fp8_out(o, qd, kv, kscale, sink, idd, SCALE)
        else:
            sparse_attn.sparse_attn_out(o, qd, kv, sink, idd, SCALE)
        return o

    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    step_bytes = qb + ib + qb
    S = int(max(2, min(32, (256 << 20) // step_bytes)))
    if S >= 8:
        # Short steps (decode, MTP): one CUDA graph holds S steps, each with its
        # own device buffers: the host-to-device copies run in order on one
        # copy stream, step j's op waits only for its own inputs (so it
        # overlaps the copies of later steps), and its device-to-host copy runs
        # on a second copy stream.  Replaying the graph keeps the host out of
        # the loop, as a decode server does.  S is as large as 256 MiB of step
        # buffers allows (32 at decode): every graph boundary drains the
        # pipeline once.
        slab_d = [torch.empty(qb + ib, dtype=torch.uint8, device=dev) for _ in range(S)]
        qd = [x[:qb].view(q.dtype).view(q.shape) for x in slab_d]
        idd = [x[qb:].view(idx.dtype).view(idx.shape) for x in slab_d]
        od = [torch.empty_like(q) for _ in range(S)]
        o_hs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(S)]
        op_out(od[0], qd[0].copy_(q), idd[0].copy_(idx))  # workspace of the capture stream
        torch.cuda.synchronize()
        graphs = []
        for gi in range(nset):  # one graph per rotation of the index sets
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                cs = torch.cuda.current_stream()
                cin.wait_stream(cs)
                cout.wait_stream(cs)
                ins = []
                with torch.cuda.stream(cin):
                    for j in range(S):
                        slab_d[j].copy_(slab_h[(gi * S + j) % nset], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(cin)
                        ins.append(ev)
                for j in range(S):
                    cs.wait_event(ins[j])
                    out = op_out(od[j], qd[j], idd[j])
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    with torch.cuda.stream(cout):
                        cout.wait_event(ev)
                        o_hs[j].copy_(out, non_blocking=True)
                cs.wait_stream(cin)
                cs.wait_stream(cout)
            graphs.append(gr)
        reps = max(1, ke // S)
        for gr in graphs:
            gr.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        t0.record(stream)
        for r in range(reps):
            graphs[r % nset].replay()
        t1.record(stream)
        barrier()
        p_ms = t0.elapsed_time(t1)
        ke_p = reps * S
        how = (f"CUDA graphs of {S} steps replayed: each step's H2D copy of q and the indices "
               "(one pinned slab), op into a preallocated o, D2H copy of o; copies of later "
               "steps overlap the op of earlier ones (two copy streams); 4 rotating index "
               "sets instead of an L2 flush")
    else:
        # Long steps (prefill): the same pipeline driven from the host without
        # graphs (the host's enqueue time is small against a step), over NB
        # rotating buffer sets, so it never drains: step k's H2D copy waits only
        # until op k - NB has read its slab, its op for its inputs and for the
        # D2H copy of step k - NB to have read its output buffer.  The copies
        # of steps k + 1 and k - 1 run during op k on the two copy streams.
        NB = 3
        slab_d = [torch.empty(qb + ib, dtype=torch.uint8, device=dev) for _ in range(NB)]
        qd = [x[:qb].view(q.dtype).view(q.shape) for x in slab_d]
        idd = [x[qb:].view(idx.dtype).view(idx.shape) for x in slab_d]
        od = [torch.empty_like(q) for _ in range(NB)]
        o_hs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(NB)]
        cs = stream
        op_done = [torch.cuda.Event() for _ in range(NB)]
        in_done = [torch.cuda.Event() for _ in range(NB)]
        out_done = [torch.cuda.Event() for _ in range(NB)]

        def run(first, n):
            for k in range(first, first + n):
                j = k % NB
                with torch.cuda.stream(cin):
                    if k >= NB:
                        cin.wait_event(op_done[j])
                    slab_d[j].copy_(slab_h[k % nset], non_blocking=True)
                    in_done[j].record(cin)
                cs.wait_event(in_done[j])
                if k >= NB:
                    cs.wait_event(out_done[j])
                with torch.cuda.stream(cs):
                    op_out(od[j], qd[j], idd[j])
                op_done[j].record(cs)
                with torch.cuda.stream(cout):
                    cout.wait_event(op_done[j])
                    o_hs[j].copy_(od[j], non_blocking=True)
                    out_done[j].record(cout)

        ke_p = max(ke, 3 * NB)
        run(0, NB)  # warm-up: workspace, module loads
        cs.wait_stream(cin)
        cs.wait_stream(cout)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        t0.record(cs)
        run(NB, ke_p)
        cs.wait_stream(cin)
        cs.wait_stream(cout)
        t1.record(cs)
        barrier()
        torch.cuda.synchronize()
        p_ms = t0.elapsed_time(t1)
        how = (f"{NB} rotating buffer sets driven from the host (no graph, no drain): each "
               "step's H2D copy of q and the indices (one pinned slab), op into a "
               "preallocated o, D2H copy of o; the copies of the next and previous steps "
               "overlap each op (two copy streams); 4 rotating index sets instead of an "
               "L2 flush")

    # serial: copy in, op, copy out on one stream, L2 flushed before each step
    def serial_step(k):  # the drop-in call, as a caller with no staging would make it
        qs = q_h.to(dev, non_blocking=True)
        ids = idx_hs[k % nset].to(dev, non_blocking=True)
        o = (sparse_attn.sparse_attn_fp8(qs, kv, kscale, sink, ids, SCALE) if fp8
             else sparse_attn.sparse_attn(qs, kv, sink, ids, SCALE))
        o_hs[0].copy_(o, non_blocking=True)

    es = [torch.cuda.Event(enable_timing=True) for _ in range(ke)]
    ee = [torch.cuda.Event(enable_timing=True) for _ in range(ke)]
    barrier()
    for k in range(ke):
        flush.zero_()
        es[k].record(stream)
        serial_step(k)
        ee[k].record(stream)
    barrier()
    s_ms = sum(a.elapsed_time(b) for a, b in zip(es, ee))
    te = torch.tensor([p_ms, s_ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    p_ms, s_ms = float(te[0]), float(te[1])
    return {"value": job_tokens * ke_p / (p_ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": q_h.numel() * q_h.element_size()
            + idx_hs[0].numel() * idx_hs[0].element_size(),
            "d2h_bytes_per_step": q.numel() * q.element_size(),
            "steps": ke_p, "kv_cache_resident": True,
            "api": "sparse_attn.sparse_attn_fp8_out" if fp8 else "sparse_attn.sparse_attn_out",
            "pipelined": how,
            "serial": {"value": job_tokens * ke / (s_ms / 1e3),
                       "api": "sparse_attn.sparse_attn_fp8" if fp8 else "sparse_attn.sparse_attn",
                       "note": "no overlap, two H2D copies, 256 MiB L2 flush before every "
                               "step"}}


def run_hc_sinkhorn(args):
    """hc_split_sinkhorn (track-02) on the 1k-1-64 prefill shape [64, 1024, 24]
    (track-02/workloads.py:25), tokens/s; 192 algorithmic bytes per token
    (24 fp32 in, 24 out).  The CPU leg times the torch restatement of
    track-02/reference/reference.py."""
    b, s_ = 64, 1024
    if args.impl == "reference":
        from oracle.hc_sinkhorn_oracle import hc_split_sinkhorn_oracle
        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(0)
        mixes, sc, base = torch.randn(b, s_, 24, generator=g), torch.randn(3, generator=g), \
            torch.randn(24, generator=g)
        for _ in range(max(args.warmup, 0)):
            hc_split_sinkhorn_oracle(mixes, sc, base)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            hc_split_sinkhorn_oracle(mixes, sc, base)
        el = time.perf_counter() - t0
        val = b * s_ * args.steps / el
        print(json.dumps({"metric": "hc_split_sinkhorn tokens/s", "value": val, "unit": "tokens/s",
                          "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
                          "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
                          "cpu_baseline": {"value": val, "unit": "tokens/s",
                                           "cores": os.cpu_count(), "kind": "port",
                                           "sample": "full [64,1024,24] per step"},
                          "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    import sparse_attn
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    mixes = torch.randn(b, s_, 24, generator=g, device=dev)
    sc, base = torch.randn(3, generator=g, device=dev), torch.randn(24, generator=g, device=dev)
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        sparse_attn.hc_split_sinkhorn(mixes, sc, base)
    K = args.steps
    st = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    en = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize()
    for k in range(K):
        flush.zero_()
        st[k].record(stream)
        sparse_attn.hc_split_sinkhorn(mixes, sc, base)
        en[k].record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(e) for a, e in zip(st, en)) / K
    tokens = b * s_
    peak, kind = measured_peaks()
    achieved = tokens * 192 / (ms / 1e3) / 1e9
    return emit(args, {
        "metric": "hc_split_sinkhorn tokens/s", "value": tokens / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": K, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic (seeded randn)",
        "config": {"workload": "track-02 1k-1-64 prefill", "shape": [b, s_, 24],
                   "l2": "flushed before every timed step, flush untimed"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "note": "192 algorithmic bytes per token"}})


def run_backward(args):
    """The backward pass (sa_bwd) on one configuration: query-tokens/s of
    gradient computation, L2 flushed before every step.  The CPU leg
    (--impl reference) times autograd of the fp32 oracle on 8 rows."""
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        from oracle.sparse_attn_oracle import sparse_attn_oracle_grads
        torch.set_num_threads(os.cpu_count() or 1)
        q, kv, sink, idx, scale, n = cpu_sample_inputs(cfg, 8)
        do = torch.randn(q.shape).to(torch.bfloat16)
        t0 = time.perf_counter()
        for _ in range(max(1, args.steps)):
            sparse_attn_oracle_grads(q, kv, sink, idx, scale, do)
        el = time.perf_counter() - t0
        val = n * max(1, args.steps) / el
        print(json.dumps({"metric": "sparse_attn backward query-tokens/s", "value": val,
                          "unit": "query-tokens/s", "impl": "reference",
                          "config": {"workload": cfg.name, "sample_rows": n},
                          "cpu_baseline": {"value": val, "unit": "query-tokens/s",
                                           "cores": os.cpu_count(), "kind": "port",
                                           "sample": f"{n} rows, autograd of the fp32 oracle"}}),
              flush=True)
        return
    import sparse_attn
    from sparse_attn.op import _forward_train
    dev = torch.device("cuda", 0)
    from sparse_attn.shard import RowBlock
    q, kv, sink, idx = block_inputs(cfg, RowBlock(0, cfg.b, 0, cfg.m), 1000, dev)
    o, lse = _forward_train(q, kv, sink, idx, SCALE)  # the training forward keeps the lse
    do = torch.randn(q.shape, device=dev, dtype=torch.bfloat16)
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        sparse_attn.sparse_attn_backward(q, kv, sink, idx, SCALE, o, do, lse)
    K = args.steps
    st = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    en = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize()
    for k in range(K):
        flush.zero_()
        st[k].record(stream)
        sparse_attn.sparse_attn_backward(q, kv, sink, idx, SCALE, o, do, lse)
        en[k].record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(e) for a, e in zip(st, en)) / K
    valid = int(((idx >= 0) & (idx < cfg.kv_len)).sum().item())
    return emit(args, {
        "metric": "sparse_attn backward query-tokens/s", "value": cfg.b * cfg.m / (ms / 1e3),
        "unit": "query-tokens/s", "n_gpus": 1, "steps": K, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "kv_len": cfg.kv_len,
                   "topk": cfg.topk, "includes": "zeroing of the fp32 dkv buffer, sa_bwd "
                   "(one pass, given the training forward's lse), dkv cast to bf16"},
        "gathered_kv_gbs": valid * D * 2 / (ms / 1e3) / 1e9})


def run_indexer(args):
    """The top-k index producer on --config's (b, m, kv_len, topk): 64 index
    heads x 128 dims, bf16, all keys valid; query-tokens/s, L2 flushed before
    every step.  The CPU leg times the torch oracle on 4 rows."""
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        from oracle.indexer_oracle import indexer_topk_oracle
        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(0)
        rows = 4
        q = torch.randn(1, rows, 64, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(1, cfg.kv_len, 128, generator=g).to(torch.bfloat16)
        w = torch.rand(1, rows, 64, generator=g)
        ln = torch.full((1, rows), cfg.kv_len, dtype=torch.int32)
        t0 = time.perf_counter()
        for _ in range(max(1, args.steps)):
            indexer_topk_oracle(q, k, w, ln, cfg.topk)
        el = time.perf_counter() - t0
        print(json.dumps({"metric": "indexer query-tokens/s", "impl": "reference",
                          "value": rows * max(1, args.steps) / el, "unit": "query-tokens/s",
                          "config": {"workload": cfg.name, "sample_rows": rows}}), flush=True)
        return
    import sparse_attn
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(cfg.b, cfg.m, 64, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(cfg.b, cfg.kv_len, 128, generator=g, device=dev, dtype=torch.bfloat16)
    w = torch.rand(cfg.b, cfg.m, 64, generator=g, device=dev)
    ln = torch.full((cfg.b, cfg.m), cfg.kv_len, dtype=torch.int32, device=dev)
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        sparse_attn.indexer_topk(q, k, w, ln, cfg.topk)
    K = args.steps
    st = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    en = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize()
    for i in range(K):
        flush.zero_()
        st[i].record(stream)
        sparse_attn.indexer_topk(q, k, w, ln, cfg.topk)
        en[i].record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(e) for a, e in zip(st, en)) / K
    rows = cfg.b * cfg.m
    flops = 2.0 * rows * cfg.kv_len * 64 * 128
    return emit(args, {
        "metric": "indexer query-tokens/s", "value": rows / (ms / 1e3), "unit": "query-tokens/s",
        "n_gpus": 1, "steps": K, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "kv_len": cfg.kv_len,
                   "topk": cfg.topk, "index_heads": 64, "index_dim": 128},
        "score_tflops": flops / (ms / 1e3) / 1e12})


# ----------------------------------------------------------------------------
# GPU leg: one configuration, this rank's rows
# ----------------------------------------------------------------------------
class Case:
    """This rank's share of one configuration, resident on the device: one op
    call per row block (``shard.partition_blocks``; one block at one GPU)."""

    def __init__(self, cfg, rank, world, dev, seed, fp8=False, variant=0, grid=0):
        import sparse_attn
        from sparse_attn.shard import partition_blocks
        self.cfg, self.dev, self.fp8, self.variant, self.grid = cfg, dev, fp8, variant, grid
        self.seed = seed
        self.blocks = partition_blocks(cfg.b, cfg.m, world, rank)
        self.parts = []
        valid = 0
        for blk in self.blocks:
            q, kv, sink, idx = block_inputs(cfg, blk, seed, dev)
            valid += int(((idx >= 0) & (idx < cfg.kv_len)).sum().item())
            ks = None
            if fp8:  # quantised once, outside every timed region, by the library's kernel
                kv, ks = sparse_attn.quantize_kv_fp8(kv)
            self.parts.append((q, kv, ks, sink, idx, torch.empty_like(q)))
        torch.cuda.synchronize(dev)
        self.valid = valid
        self.gathered = valid * (D + 4 if fp8 else 2 * D)
        self.rows = sum(b.rows for b in self.blocks)
        nbytes = max([sparse_attn.workspace_bytes(b.b1 - b.b0, b.m1 - b.m0, cfg.topk, dev)
                      for b in self.blocks] + [256])
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)

    def step(self):
        import sparse_attn
        st = torch.cuda.current_stream(self.dev)
        for q, kv, ks, sink, idx, o in self.parts:
            if self.fp8:
                sparse_attn.sparse_attn_fp8_out(o, q, kv, ks, sink, idx, SCALE, self.ws,
                                                grid=self.grid, stream=st)
            else:
                sparse_attn.sparse_attn_out(o, q, kv, sink, idx, SCALE, self.ws,
                                            variant=self.variant, grid=self.grid, stream=st)

    def idx_maker(self, r):
        """A fresh index set for the single block (e2e's rotating sets)."""
        blk = self.blocks[0]
        icfg = dataclasses.replace(self.cfg, b=blk.b1 - blk.b0, m=blk.m1 - blk.m0)
        return make_indices(icfg, torch.Generator().manual_seed(self.seed + 7919 * r), m0=blk.m0)

def timed_steps(step, K, flush, stream, barrier, clocks_dev=None):
    """K L2-flushed steps timed by CUDA events (flush outside the events).
    Returns (per-step ms list, clock summary)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    sampler = ClockSampler(clocks_dev) if clocks_dev is not None else None
    barrier()
    if sampler:
        sampler.start()
    for k in range(K):
        flush.zero_()
        starts[k].record(stream)
        step()
        ends[k].record(stream)
    barrier()
    clocks = sampler.stop() if sampler else None
    return [s.elapsed_time(e) for s, e in zip(starts, ends)], clocks


def max_over_ranks(vals, dev, world):
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def l2_copy_gbs(dev, reps=20):
    """Measured L2 bandwidth denominator: a plain device copy of a 24 MiB
    buffer into another (48 MiB in all, L2-resident after the first pass),
    20 copies back to back in one CUDA graph (no launch gaps), read + write
    bytes over the best CUDA-event time of ``reps`` graph replays."""
    n = 24 << 20
    a = torch.empty(n, dtype=torch.uint8, device=dev).fill_(1)
    b = torch.empty_like(a)
    inner = 20
    for _ in range(3):
        b.copy_(a)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(inner):
            b.copy_(a)
    st = torch.cuda.current_stream(dev)
    graph.replay()
    best = None
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / inner
        best = ms if best is None else min(best, ms)
    return 2 * n / (best / 1e3) / 1e9


def traffic_for(key):
    tpath = ROOT / "profiles" / "traffic.json"
    if not tpath.exists():
        return None
    try:
        return json.loads(tpath.read_text()).get(key)
    except Exception:
        return None


def measure_config(cfg, args, rank, world, dev, flush, barrier, K, *, headline, fp8,
                   variant, l2_gbs, with_e2e, with_cpu):
    """Time this rank's share of ``cfg``; returns the result dict (rank 0's
    view: times are max over ranks, bytes and launches are this rank's)."""
    case = Case(cfg, rank, world, dev, seed=1000, fp8=fp8, variant=variant, grid=args.grid)
    stream = torch.cuda.current_stream(dev)
    step = case.step
    if args.graph:
        case.step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            case.step()
        step = graph.replay
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    per_call, kernel_us = (None, {}) if args.no_launch_count else profile_our_kernels(step, flush)
    step_ms, clocks = timed_steps(step, K, flush, stream, barrier, dev.index)
    total_ms = sum(step_ms)
    max_total_ms, = max_over_ranks([total_ms], dev, world)
    job_tokens = cfg.b * cfg.m
    value = job_tokens * K / (max_total_ms / 1e3)
    mean_ms = total_ms / K
    peak, peak_kind = measured_peaks()
    achieved = case.gathered / (mean_ms / 1e3) / 1e9
    key = f"{cfg.name}:fp8" if fp8 else f"{cfg.name}:{args.variant}"
    traffic = traffic_for(key)
    if traffic is None and not fp8:
        traffic = traffic_for(f"{cfg.name}:auto")
    res = {
        "value": value, "unit": UNIT, "ms_per_step": max_total_ms / K, "steps": K,
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "h": H, "d": D,
                   "kv_len": cfg.kv_len, "topk": cfg.topk,
                   "rows_this_rank": case.rows, "blocks_this_rank": len(case.blocks)},
        "gathered_kv_gbs": case.gathered / (mean_ms / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)"
                     if peak_kind == "measured" else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_step": case.gathered,
                     "note": "achieved = valid gathered KV bytes of this GPU's rows ("
                             + ("516" if fp8 else "1024") + " per slot) / mean event time of "
                             "one step (every kernel of the op call)"},
        "gpu_launches": None if per_call is None else per_call * K,
        "kernel_us": kernel_us,
        "step_ms": {"mean": mean_ms, "min": min(step_ms), "median": statistics.median(step_ms)},
        "clocks": clocks,
    }
    # KV caches that fit in L2 are served from it: report the L2 fraction too
    kv_bytes = cfg.kv_len * (D + 4 if fp8 else 2 * D) * sum(b.b1 - b.b0 for b in case.blocks)
    if l2_gbs and kv_bytes <= (128 << 20):
        res["roofline_l2"] = {"bound": "l2", "achieved": achieved, "peak": l2_gbs,
                              "unit": "GB/s", "frac": achieved / l2_gbs,
                              "peak_source": "measured in this run: plain 24 MiB device "
                                             "copy, L2-resident, 20 per CUDA graph "
                                             "(read + write bytes)",
                              "kv_cache_bytes": kv_bytes}
    if with_e2e and len(case.blocks) == 1:
        q, kv, ks, sink, idx, _ = case.parts[0]
        res["e2e"] = measure_e2e(case.idx_maker, q, kv, ks, sink, idx, dev, stream, flush, K,
                                 barrier, world, job_tokens, fp8)
    else:
        res["e2e"] = None
    if with_cpu and world == 1:
        val, n, reps, el, cores = cpu_throughput(cfg, rows=16, min_seconds=8.0, max_reps=200)
        _, _, kind, desc = cpu_impl(cfg)
        res["cpu_baseline"] = {
            "value": val, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} query rows of '{cfg.name}' x {reps} reps ({el:.1f} s), {desc}"}
    else:
        res["cpu_baseline"] = None
    res["_case"] = case
    return res


def time_allgather(case, dev, world, reps=20):
    """The sharded op's one collective, timed alone: every rank's o rows
    (padded to the largest share) all-gathered over NCCL."""
    import torch.distributed as dist
    from sparse_attn.shard import row_range
    cfg = case.cfg
    n_rows = cfg.b * cfg.m
    chunk = max(row_range(n_rows, world, r)[1] - row_range(n_rows, world, r)[0]
                for r in range(world))
    local = torch.zeros(chunk, H, D, dtype=torch.bfloat16, device=dev)
    out = torch.empty(world * chunk, H, D, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev)
    for _ in range(3):
        dist.all_gather_into_tensor(out, local)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        dist.all_gather_into_tensor(out, local)
    e1.record(st)
    torch.cuda.synchronize()
    ms, = max_over_ranks([e0.elapsed_time(e1) / reps], dev, world)
    return {"ms": ms, "bytes_per_rank": local.numel() * 2,
            "note": "all_gather_into_tensor of each rank's o rows (padded to the largest "
                    "share), NCCL, outside the op's timed region"}


# The reference's Triton kernel (track-01/submission.py:276-347, launched by its
# sparse_attn at :1003-1021) is not run: on this pool's B200 it raised a CUDA
# fault ("an illegal memory access was encountered") on the decode
# configuration (b=64, m=1, kv_len=32768, topk=2048, every index inside
# [0, kv_len)), so it stays off the GPU.
TRITON_UNAVAILABLE = ("not run: the reference's Triton universal kernel "
                      "(track-01/submission.py:276-347) raised an illegal-memory-access fault "
                      "on this pool's B200 on the decode configuration, so it stays off the GPU")


def triton_reference(case):
    return {"unavailable": TRITON_UNAVAILABLE}


def run_gather_probe(args):
    """--op gather: random-row gather rates with no math (sa_probe_gather).
    128 MiB of rows per call from a 2 GiB cache (the decode config's size),
    L2 flushed before each call (write only, or write then read), CUDA events;
    the same kernel on sequential rows shows what the copy machinery reaches
    without scatter."""
    from sparse_attn import _lib
    import ctypes
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    cache = torch.empty(2 << 30, dtype=torch.uint8, device=dev)
    sink = torch.zeros(4096, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    flushes = {"write": L2Flush(dev, read=False), "write+read": L2Flush(dev, read=True)}
    st = torch.cuda.current_stream(dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak, kind = measured_peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    total = 128 << 20
    results = []

    def run(row_bytes, method, ctas, depth, pattern, fl, reps=20, total=total):
        n_rows = total // row_bytes
        # "random-l2": rows of a 4 MiB region (the causal config's KV cache), so
        # after the first touches every row comes from L2
        pool = ((4 << 20) if pattern == "random-l2" else (2 << 30)) // row_bytes
        rows = (torch.randint(0, pool, (n_rows,), generator=g, device=dev, dtype=torch.int32)
                if pattern.startswith("random")
                else torch.arange(n_rows, device=dev, dtype=torch.int32))
        flush = flushes[fl]

        def call():
            _lib.check(L.sa_probe_gather(cache.data_ptr(), row_bytes, rows.data_ptr(), n_rows,
                                         row_bytes, method, ctas, depth, sink.data_ptr(),
                                         err.data_ptr(), ctypes.c_void_p(st.cuda_stream)))
        for _ in range(3):
            flush.zero_()
            call()
        ms = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            call()
            e1.record(st)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        med = statistics.mean(ms)  # (CUDA events tick in ~2 us steps here: the mean)
        gbs = total / (med / 1e3) / 1e9
        results.append({"bytes": total, "row_bytes": row_bytes, "method": ["cp.async16", "bulk_tma_1d",
                                                           "ldg_nc16_regs"][method],
                        "ctas": ctas, "depth": depth, "pattern": pattern, "flush": fl,
                        "us": med * 1e3, "gbs": gbs, "frac_of_hbm": gbs / peak})

    for fl in ("write", "write+read"):
        for pattern in ("random", "sequential"):
            for method in (0, 1, 2):
                for ctas, depth in ((sms, 3), (sms, 6), (2 * sms, 3)):
                    if method == 2 and depth != 3:
                        continue
                    run(1024, method, ctas, depth, pattern, fl)
    for rb in (512, 2048, 4096):
        for method in (0, 1):
            run(rb, method, sms, 6, "random", "write+read")
            run(rb, method, 2 * sms, 3, "random", "write+read")
    for method in (0, 1, 2):
        run(1024, method, sms, 3, "random-l2", "write+read")
        run(1024, method, 2 * sms, 3, "random-l2", "write+read")
    # the read ceiling on a long kernel: 1 GiB per call (ramp-up and tail are
    # then a small share), sequential and random rows, all three forms
    for pattern in ("sequential", "random"):
        for method, ctas, depth in ((2, 2 * sms, 3), (2, 4 * sms, 3), (0, 2 * sms, 3),
                                    (1, 2 * sms, 3)):
            run(1024, method, ctas, depth, pattern, "write+read", reps=5, total=1 << 30)
    torch.cuda.synchronize()
    ok = int(err.item()) == 0
    best = max((r for r in results if r["pattern"] == "random" and r["row_bytes"] == 1024),
               key=lambda r: r["gbs"])
    print(json.dumps({
        "metric": "random 1 KiB row gather GB/s (copies only)", "value": best["gbs"],
        "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "waits_ok": ok,
        "config": {"workload": "gather probe", "bytes_per_call": total, "cache_bytes": 2 << 30,
                   "l2": "flushed before every call (see each result's 'flush'), untimed"},
        "peak": {"hbm_gbs": peak, "source": kind}, "best": best, "results": results}),
        flush=True)


def run_reftable(args):
    """--suite reftable: the reference's benchmark (track-01/bench.py:27-53)
    over its own 10-workload table (track-01/workloads.py:15-26, indices drawn
    with replacement as at :36): its torch reference (reference.py, on the GPU)
    and this library, each CUDA-event timed with L2 flushed before every call;
    the speedup over the torch reference per workload and its geometric mean,
    as the reference reports its own.  (Its Triton kernel is not run; see
    TRITON_UNAVAILABLE.)"""
    import sparse_attn
    from sparse_attn.workloads import REFERENCE_TABLE as WORKLOADS
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = L2Flush(dev)
    st = torch.cuda.current_stream(dev)
    have_ref = (REF_DIR / "reference" / "reference.py").exists()
    ref_fn = None
    if have_ref:
        sys.path.insert(0, str(REF_DIR))
        import importlib
        ref_fn = importlib.import_module("reference.reference").sparse_attn

    def bench_fn(fn, a, reps=30):
        for _ in range(3):
            fn(*a)
        torch.cuda.synchronize()
        ms = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn(*a)
            e1.record(st)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        return statistics.median(ms)

    rows = []
    for label, b, m, kv_len, topk in WORKLOADS:
        g = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(b, m, H, D, generator=g, device=dev, dtype=torch.bfloat16)
        kv = torch.randn(b, kv_len, D, generator=g, device=dev, dtype=torch.bfloat16)
        sink = torch.randn(H, generator=g, device=dev, dtype=torch.float32)
        idx = torch.randint(0, kv_len, (b, m, topk), generator=g, device=dev, dtype=torch.int32)
        a = (q, kv, sink, idx, SCALE)
        r = {"workload": label, "b": b, "m": m, "kv_len": kv_len, "topk": topk,
             "ours_ms": bench_fn(sparse_attn.sparse_attn, a)}
        if have_ref:
            try:
                r["torch_ref_ms"] = bench_fn(ref_fn, a, reps=10)
            except torch.cuda.OutOfMemoryError:
                r["torch_ref_ms"] = None
                torch.cuda.empty_cache()
        rows.append(r)
        del q, kv, idx
        torch.cuda.empty_cache()

    def geo(xs):
        xs = [x for x in xs if x]
        return math.exp(sum(math.log(x) for x in xs) / len(xs)) if xs else None
    for r in rows:
        if r.get("torch_ref_ms"):
            r["speedup_over_torch_ref"] = r["torch_ref_ms"] / r["ours_ms"]
    summary = {"geomean_speedup_over_torch_ref": geo([r["torch_ref_ms"] / r["ours_ms"]
                                                      for r in rows if r.get("torch_ref_ms")]),
               "triton_reference": TRITON_UNAVAILABLE}
    print(json.dumps({"suite": "reftable", "reference_available": have_ref, "rows": rows,
                      **summary}), flush=True)


def main():
    args = parse()
    if args.op == "indexer":
        return run_indexer(args)
    if args.op == "hc_sinkhorn":
        return run_hc_sinkhorn(args)
    if args.op == "sparse_attn_bwd":
        return run_backward(args)
    if args.op == "gather":
        return run_gather_probe(args)
    if args.suite == "reftable":
        return run_reftable(args)
    if args.impl == "reference":
        return run_reference(args)

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    if args.kv_policy != -1 or args.gather_only:
        from sparse_attn import _lib
        _lib.set_option(_lib.SA_OPT_KV_POLICY, args.kv_policy)
        _lib.set_option(_lib.SA_OPT_GATHER_ONLY, int(args.gather_only))
    variant = {"auto": 0, "mma": 1, "tcgen05": 2, "ws": 3, "wt": 4}[args.variant]
    fp8 = args.kv == "fp8"
    flush = L2Flush(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    l2_gbs = l2_copy_gbs(dev)
    cfg = CONFIGS[args.config]
    head = measure_config(cfg, args, rank, world, dev, flush, barrier, args.steps,
                          headline=True, fp8=fp8, variant=variant, l2_gbs=l2_gbs,
                          with_e2e=not args.no_e2e, with_cpu=not args.no_cpu_baseline)
    head_case = head.pop("_case")
    allgather = time_allgather(head_case, dev, world) if world > 1 else None
    triton = None
    if rank == 0 and world == 1 and not args.no_triton and not fp8:
        triton = triton_reference(head_case)
        if "ms_per_step" in triton:
            triton["ours_over_triton"] = triton["ms_per_step"] / head["ms_per_step"]
    del head_case
    torch.cuda.empty_cache()

    per_config = {}
    if not args.no_per_config:
        others = ["long", "decode", "causal", "mtp"] if world == 1 else ["mtp"]
        for name in others:
            if name == args.config:
                continue
            c = CONFIGS[name]
            r = measure_config(c, args, rank, world, dev, flush, barrier,
                               PER_CONFIG_STEPS.get(name, args.steps), headline=False, fp8=fp8,
                               variant=variant, l2_gbs=l2_gbs, with_e2e=not args.no_e2e,
                               with_cpu=not args.no_cpu_baseline)
            case = r.pop("_case")
            if rank == 0 and world == 1 and not args.no_triton and not fp8:
                r["triton_reference"] = triton_reference(case)
                if "ms_per_step" in r["triton_reference"]:
                    r["triton_reference"]["ours_over_triton"] = (
                        r["triton_reference"]["ms_per_step"] / r["ms_per_step"])
            if world > 1:
                r["allgather"] = time_allgather(case, dev, world)
            del case
            torch.cuda.empty_cache()
            per_config[name] = r

    # the other rows of the scope table, measured in the same run at one GPU:
    # the fp8 KV cache at decode, the backward pass, the top-k index producer,
    # track-02's hc_split_sinkhorn
    other_ops = {}
    if world == 1 and not args.no_per_config and not fp8:
        r = measure_config(CONFIGS["decode"], args, rank, world, dev, flush, barrier,
                           PER_CONFIG_STEPS["decode"], headline=False, fp8=True, variant=0,
                           l2_gbs=l2_gbs, with_e2e=False, with_cpu=False)
        r.pop("_case")
        per_config["decode:fp8"] = r
        torch.cuda.empty_cache()
        import copy
        for name, fn, over in (("sparse_attn_bwd:causal", run_backward,
                                {"config": "causal", "steps": 20}),
                               ("indexer:decode", run_indexer, {"config": "decode", "steps": 50}),
                               ("hc_split_sinkhorn", run_hc_sinkhorn, {"steps": 200})):
            a = copy.copy(args)
            a.collect, a.impl = True, "ours"
            for k, v in over.items():
                setattr(a, k, v)
            try:
                other_ops[name] = fn(a)
            except Exception as e:  # noqa: BLE001 - reported in the line, never fatal
                other_ops[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.empty_cache()

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    launches = head["gpu_launches"]
    line = {
        "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 KV (fp32 per-token scale), bf16 q/o" if fp8 else "bf16",
        "data": "synthetic (seeded; q/kv/sink randn on device, distinct indices per row "
                "drawn on the CPU with the config's pattern)",
        "config": {**head["config"], "global_batch": cfg.b, "seq_len": cfg.m,
                   "parallelism": f"query rows sharded over {world} GPU(s) "
                                  "(shard.partition_blocks), KV cache of each rank's batch "
                                  "items resident, no collective in the timed region",
                   "allgather": "of o, outside the timed region, timed separately"
                                if world > 1 else "none (one GPU)",
                   "l2": L2Flush.describe,
                   "variant": "fp8" if fp8 else args.variant, "grid": args.grid,
                   "kv_cache": "e4m3 + fp32 per-token scale" if fp8 else "bf16",
                   "launch": "CUDA graph replay" if args.graph else "stream launch",
                   "gather_only": bool(args.gather_only),
                   "kv_l2_policy": "by reuse (evict_first if m*topk < kv_len, else evict_last)"
                                   if args.kv_policy == -1 else
                                   ["evict_first", "evict_normal", "evict_last"][args.kv_policy]},
        "gathered_kv_gbs": head["gathered_kv_gbs"],
        "roofline": head["roofline"],
        "cpu_baseline": head["cpu_baseline"],
        "e2e": head["e2e"],
        "gpu_launches": launches,
        "kernel_us": head["kernel_us"],
        "step_ms": head["step_ms"],
        "clocks": head["clocks"],
        "l2_copy_gbs": l2_gbs,
    }
    if "roofline_l2" in head:
        line["roofline_l2"] = head["roofline_l2"]
    if allgather is not None:
        allgather["value_with_allgather"] = (cfg.b * cfg.m) / (
            (head["ms_per_step"] + allgather["ms"]) / 1e3)
        line["allgather"] = allgather
    if triton is not None:
        line["triton_reference"] = triton
    if per_config:
        line["per_config"] = per_config
    if other_ops:
        line["other_ops"] = other_ops
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
