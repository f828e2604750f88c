"""Benchmark of the B200 ``sparse_attn`` hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config decode] [--variant auto|mma|tcgen05]

A "step" is one call of the op over one batch of the configuration (default:
BASELINE config "decode", b=64 m=1 kv_len=32768 topk=2048, h=16 d=512).
``value`` is query-tokens/s of the whole job with inputs resident in HBM,
timed with CUDA events on the launching stream, L2 flushed (256 MiB write)
before every timed step and the flush kept outside the events.  ``e2e`` is the
same metric through the public op ``sparse_attn`` with the step's q and
topk_idxs copied from pinned host memory and o copied back inside the timed
region (the KV cache and sink stay resident, as a serving KV cache does).

Multi-GPU (torchrun, one process per GPU): every rank runs its own batch of
the configuration (weak scaling, query rows sharded by batch, no collective on
the data path); the time is the max over ranks.

``--impl reference`` times the reference's CPU algorithm (the oracle port of
track-01/reference/reference.py) on all host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="decode")
    ap.add_argument("--variant", choices=["auto", "mma", "tcgen05", "ws"], default="auto")
    ap.add_argument("--grid", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline leg (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16",
                    help="KV cache format: bf16 (the reference's) or e4m3 + fp32 per-token "
                         "scale (sparse_attn_fp8)")
    ap.add_argument("--op", choices=["sparse_attn", "sparse_attn_bwd", "hc_sinkhorn", "indexer"],
                    default="sparse_attn",
                    help="sparse_attn_bwd: the backward pass on --config; indexer: the top-k "
                         "index producer on --config's b, m, kv_len, topk; "
                         "hc_sinkhorn: the track-02 op on its 1k-1-64 prefill shape")
    ap.add_argument("--graph", action="store_true",
                    help="capture one op call in a CUDA graph and time its replays")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip the one profiled call that counts our kernel launches")
    return ap.parse_args()


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
def device_inputs(cfg, seed, device):
    """Seeded inputs made directly on the GPU (indices on the CPU, then copied)."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(cfg.b, cfg.m, H, D, generator=g, device=device, dtype=torch.bfloat16)
    kv = torch.randn(cfg.b, cfg.kv_len, D, generator=g, device=device, dtype=torch.bfloat16)
    sink = torch.randn(H, generator=g, device=device, dtype=torch.float32)
    idx = make_indices(cfg, torch.Generator().manual_seed(seed)).to(device)
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
            ours = "sa_" in e.name and ("fwd_kernel" in e.name or "combine" in e.name)
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


def cpu_impl():
    """The reference's algorithm on the host cores, written with the same torch
    ops as reference.py (the faster CPU form on the GPU hosts: torch's
    vectorised einsum beats the scalar C restatement in oracle/sa_host.c)."""
    from oracle.sparse_attn_oracle import sparse_attn_oracle
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    return sparse_attn_oracle, cores


def cpu_throughput(cfg, rows, min_seconds, max_reps):
    fn, cores = cpu_impl()
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
    fn, cores = cpu_impl()
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
              f"topk={cfg.topk}), {CPU_IMPL}")
    line = {
        "metric": METRIC, "value": val, "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded CPU generator)",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "h": H, "d": D,
                   "kv_len": cfg.kv_len, "topk": cfg.topk, "sample_rows_per_step": n},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU leg
# ----------------------------------------------------------------------------
def measure_e2e(cfg, q, kv, kscale, sink, idx, dev, stream, flush, K, barrier, world, tokens,
                fp8, seed):
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
    idx_cpu = [idx.cpu()] + [make_indices(cfg, torch.Generator().manual_seed(seed + 7919 * r))
                             for r in range(1, nset)]
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

    # One CUDA graph holds S steps, each with its own device buffers: the
    # host-to-device copies run in order on one copy stream, step j's op waits
    # only for its own inputs (so it overlaps the copies of later steps), and
    # its device-to-host copy runs on a second copy stream.  Replaying the
    # graph keeps the host out of the loop, as a decode server does.  S is as
    # large as 256 MiB of step buffers allows (32 at decode): every graph
    # boundary drains the pipeline once.
    step_bytes = qb + ib + qb
    S = int(max(2, min(32, (256 << 20) // step_bytes)))
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slab_d = [torch.empty(qb + ib, dtype=torch.uint8, device=dev) for _ in range(S)]
    qd = [x[:qb].view(q.dtype).view(q.shape) for x in slab_d]
    idd = [x[qb:].view(idx.dtype).view(idx.shape) for x in slab_d]
    od = [torch.empty_like(q) for _ in range(S)]
    o_hs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(S)]
    op_out(od[0], qd[0].copy_(q), idd[0].copy_(idx))  # workspace of the capture stream, module loads
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
    return {"value": world * tokens * ke_p / (p_ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": q_h.numel() * q_h.element_size()
            + idx_hs[0].numel() * idx_hs[0].element_size(),
            "d2h_bytes_per_step": q.numel() * q.element_size(),
            "steps": ke_p, "kv_cache_resident": True,
            "api": "sparse_attn.sparse_attn_fp8_out" if fp8 else "sparse_attn.sparse_attn_out",
            "pipelined": f"CUDA graphs of {S} steps replayed: each step's H2D copy of q and "
                         "the indices (one pinned slab), op into a preallocated o, D2H copy "
                         "of o; copies of later steps overlap the op of earlier ones (two "
                         "copy streams); 4 rotating index sets instead of an L2 flush",
            "serial": {"value": world * tokens * ke / (s_ms / 1e3),
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
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
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
    print(json.dumps({
        "metric": "hc_split_sinkhorn tokens/s", "value": tokens / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": K, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic (seeded randn)",
        "config": {"workload": "track-02 1k-1-64 prefill", "shape": [b, s_, 24],
                   "l2": "flushed before every timed step, flush untimed"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "note": "192 algorithmic bytes per token"}}),
        flush=True)


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
    q, kv, sink, idx = device_inputs(cfg, seed=1000, device=dev)
    o, lse = _forward_train(q, kv, sink, idx, SCALE)  # the training forward keeps the lse
    do = torch.randn(q.shape, device=dev, dtype=torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
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
    print(json.dumps({
        "metric": "sparse_attn backward query-tokens/s", "value": cfg.b * cfg.m / (ms / 1e3),
        "unit": "query-tokens/s", "n_gpus": 1, "steps": K, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "kv_len": cfg.kv_len,
                   "topk": cfg.topk, "includes": "zeroing of the fp32 dkv buffer, sa_bwd "
                   "(one pass, given the training forward's lse), dkv cast to bf16"},
        "gathered_kv_gbs": valid * D * 2 / (ms / 1e3) / 1e9}), flush=True)


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
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
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
    print(json.dumps({
        "metric": "indexer query-tokens/s", "value": rows / (ms / 1e3), "unit": "query-tokens/s",
        "n_gpus": 1, "steps": K, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "kv_len": cfg.kv_len,
                   "topk": cfg.topk, "index_heads": 64, "index_dim": 128},
        "score_tflops": flops / (ms / 1e3) / 1e12}), flush=True)


def main():
    args = parse()
    if args.op == "indexer":
        return run_indexer(args)
    if args.op == "hc_sinkhorn":
        return run_hc_sinkhorn(args)
    if args.op == "sparse_attn_bwd":
        return run_backward(args)
    if args.impl == "reference":
        return run_reference(args)

    import sparse_attn
    from sparse_attn import sparse_attn_out

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    variant = {"auto": 0, "mma": 1, "tcgen05": 2, "ws": 3}[args.variant]
    cfg = CONFIGS[args.config]
    q, kv, sink, idx = device_inputs(cfg, seed=1000 + rank, device=dev)
    o = torch.empty_like(q)
    ws = torch.zeros(sparse_attn.workspace_bytes(cfg.b, cfg.m, cfg.topk, local_rank),
                     dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    tokens = cfg.b * cfg.m
    valid = int(((idx >= 0) & (idx < cfg.kv_len)).sum().item())
    gathered = valid * D * 2

    fp8 = args.kv == "fp8"
    if fp8:
        # quantised once, outside every timed region, by the library's own kernel
        kv8, kscale = sparse_attn.quantize_kv_fp8(kv)
        del kv
        torch.cuda.synchronize()
        gathered = valid * (D + 4)  # e4m3 row + its fp32 scale

    def op_call():
        if fp8:
            sparse_attn.sparse_attn_fp8_out(o, q, kv8, kscale, sink, idx, SCALE, ws,
                                            grid=args.grid, stream=torch.cuda.current_stream(dev))
        else:
            sparse_attn_out(o, q, kv, sink, idx, SCALE, ws, variant=variant, grid=args.grid,
                            stream=torch.cuda.current_stream(dev))

    step = op_call
    if args.graph:
        # one op call (forward + combine launches, programmatic dependency kept)
        # captured once; every step replays it on the timed stream
        op_call()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            op_call()
        step = graph.replay

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    per_call, kernel_us = (None, {}) if args.no_launch_count else profile_our_kernels(step, flush)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    sampler = ClockSampler(local_rank)
    barrier()
    sampler.start()
    for k in range(K):
        flush.zero_()  # untimed: outside the events
        starts[k].record(stream)
        step()
        ends[k].record(stream)
    barrier()
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    max_total_ms = float(t.item())
    value = world * tokens * K / (max_total_ms / 1e3)

    # ---- end to end through the public op, host buffers ----
    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(cfg, q, kv8 if fp8 else kv, kscale if fp8 else None, sink, idx, dev,
                          stream, flush, K, barrier, world, tokens, fp8, seed=1000 + rank)

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    peak, peak_kind = measured_peaks()
    mean_ms = total_ms / K
    achieved = gathered / (mean_ms / 1e3) / 1e9
    traffic = None
    tpath = ROOT / "profiles" / "traffic.json"
    if tpath.exists():
        try:
            tj = json.loads(tpath.read_text())
            key = f"{args.config}:fp8" if fp8 else f"{args.config}:{args.variant}"
            traffic = tj.get(key, None if fp8 else tj.get(args.config))
        except Exception:
            traffic = None

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        val, n, reps, el, cores = cpu_throughput(cfg, rows=16, min_seconds=10.0, max_reps=200)
        cpu = {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{n} query rows of '{cfg.name}' x {reps} reps ({el:.1f} s), "
                         f"{CPU_IMPL}"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": max_total_ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 KV (fp32 per-token scale), bf16 q/o" if fp8 else "bf16",
        "data": "synthetic (seeded; q/kv/sink randn on device, distinct indices per row)",
        "config": {"workload": cfg.name, "b": cfg.b, "m": cfg.m, "h": H, "d": D,
                   "kv_len": cfg.kv_len, "topk": cfg.topk, "global_batch": cfg.b * world,
                   "parallelism": f"rows sharded by batch over {world} GPU(s), no collective",
                   "l2": "flushed (256 MiB write) before every timed step, flush untimed",
                   "variant": "fp8" if fp8 else args.variant, "grid": args.grid,
                   "kv_cache": "e4m3 + fp32 per-token scale" if fp8 else "bf16",
                   "launch": "CUDA graph replay" if args.graph else "stream launch"},
        "gathered_kv_gbs": gathered * world * K / (max_total_ms / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)"
                     if peak_kind == "measured" else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_step": gathered,
                     "note": "achieved = valid gathered KV bytes (" + ("516" if fp8 else "1024")
                             + " per slot) / mean event time of one op call (main + combine "
                             "kernels)"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": None if per_call is None else per_call * K,
        "kernel_us": kernel_us,
        "step_ms": {"mean": mean_ms, "min": min(step_ms), "median": statistics.median(step_ms)},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
