"""Benchmark: exact top-k search QPS on B200, with roofline, parity and CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one search of a query batch against the corpus, with queries and
corpus already resident in HBM (`value`); `e2e` repeats it through the public
API from pinned host queries (fp32) to host results. Default workload (config
c2): 1M x 768 fp16 unit-norm corpus PER GPU, batch 256, k=10, cosine. With N>1
ranks (torchrun) the corpus is row-sharded: rank r holds its own rows (global
chunks r*shard .. of the same generator), each step is a full sharded search
(local fused top-k + NCCL all-gather + merge), and `value` counts query x
shard units per second over all ranks (N*b/t); `qps_global` is b/t over the
whole N-shard corpus and `phases_us` splits a step into local search,
all-gather and merge. After the timed loops, `parity` checks a subset of query
rows of the search result against the CPU oracle on the stored corpus.

--impl reference times the reference's CPU search paths (oracle/cpu_paths.py:
Index(device="cpu") torch fp32, exact_topk_fp32, numpy_search) on the host
cores, on a bounded sample of the same workload, scaled to the same unit.

--sweep [--sweep-batches 1,8,256 --sweep-chunks 0,74 --report table.md] times the
search over batch sizes and plan hints on one GPU instead (JSON rows + a
markdown table with roofline fractions).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "cuda-vector-search_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "QPS and % roofline (TC TFLOP/s or HBM GB/s), 1M×768 b256 k10, 1–8 B200"
CHUNK = 1 << 18

L2_BYTES = 126 << 20  # B200 L2 size, rounded up

CONFIGS = {
    # name: rows per GPU, dim, batch, k, metric
    "c1": dict(n=100_000, d=384, b=32, k=10, metric="cosine"),
    "c2": dict(n=1_000_000, d=768, b=256, k=10, metric="cosine"),
    "c3": dict(n=4_000_000, d=768, b=1, k=10, metric="ip"),
    "c4k100": dict(n=1_000_000, d=384, b=256, k=100, metric="cosine"),
    "c4k256": dict(n=1_000_000, d=384, b=256, k=256, metric="cosine"),
    "c5": dict(n=16_000_000, d=768, b=1024, k=100, metric="cosine"),
}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic(config: str):
    """Per-launch DRAM bytes of the search kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    j = json.loads(p.read_text())
    return j.get(config)


def workload_name(cfg) -> str:
    return (f"{cfg['n'] // 1000}k x {cfg['d']} fp16 unit-norm corpus per GPU, batch {cfg['b']}, "
            f"k={cfg['k']}, {cfg['metric']}")


# ---------------------------------------------------------------------------
# Shared by both arms
# ---------------------------------------------------------------------------
def bench_config(args, cfg, world: int) -> dict:
    """The `config` object of the JSON line; identical in both arms."""
    d_pad = -(-cfg["d"] // 64) * 64
    corpus_bytes = 2 * cfg["n"] * d_pad
    flushed = corpus_bytes < 2 * L2_BYTES
    return {
        "workload": workload_name(cfg),
        "config": args.config,
        "rows_per_gpu": cfg["n"], "total_rows": cfg["n"] * world, "dim": cfg["d"], "batch": cfg["b"],
        "k": cfg["k"], "metric": cfg["metric"],
        "l2": (f"corpus ({corpus_bytes / 1e9:.3f} GB per GPU) fits in the 126 MB L2: a {2 * L2_BYTES >> 20} MiB "
               "buffer is written before every timed step, outside the step's CUDA-event interval; "
               "the end-to-end steps then run one at a time") if flushed else
              f"inputs larger than L2 ({corpus_bytes / 1e9:.2f} GB corpus per GPU vs 126 MB L2)",
        "value_unit": (f"queries x {cfg['n'] // 1000}k-row shards per second over all ranks (N*b/t)" if world > 1
                       else "queries per second"),
    }


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# CPU baseline: the reference's CPU search paths (oracle/cpu_paths.py)
# ---------------------------------------------------------------------------
CPU_SAMPLE_ROWS = 1 << 18  # one chunk of the reference's exact_topk_fp32


def cpu_sample(cfg, rows: int, seed: int):
    """Unit-norm fp16 corpus rows and queries with the benchmark's distribution."""
    import numpy as np

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cfg["d"]), dtype=np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    q = rng.standard_normal((cfg["b"], cfg["d"]), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    return x.astype(np.float16), q.astype(np.float16)


def cpu_paths(cfg, rows: int):
    """{name: (callable running one search of all queries over the sample, what it is)}.

    Each callable includes the per-call query preparation of its path (cosine
    normalisation), as the reference's search does."""
    import numpy as np
    import torch

    from oracle import index_cpu_search, normalize_rows_fp16, numpy_search, torch_exact_topk_fp32

    torch.set_num_threads(os.cpu_count() or 1)
    x16, q16 = cpu_sample(cfg, rows, seed=7)
    cos = cfg["metric"] == "cosine"
    k = cfg["k"]
    x32_t = torch.from_numpy(x16.astype(np.float32))  # Index(device="cpu") stores fp32 rows
    x16_t = torch.from_numpy(x16)
    x32_np = x16.astype(np.float32)
    q_t = torch.from_numpy(q16).float()

    def prep_t():
        return q_t / q_t.norm(dim=1, keepdim=True).clamp_min(1e-12) if cos else q_t

    def prep_np():
        return normalize_rows_fp16(q16).astype(np.float32) if cos else q16.astype(np.float32)

    return {
        "torch_index_cpu": (lambda: index_cpu_search(prep_t(), x32_t, k),
                            "reference Index(device='cpu').search: fp32 torch.matmul + torch.topk "
                            "(index.py:131, reference.py:8-15)"),
        "torch_exact_topk_fp32": (lambda: torch_exact_topk_fp32(prep_t(), x16_t, k),
                                  "reference exact_topk_fp32 on the fp16 rows (reference.py:18-34)"),
        "numpy_search": (lambda: numpy_search(prep_np(), x32_np, k),
                         "reference numpy_search (bench/bench_baselines.py:45-50)"),
    }


def cpu_baseline(cfg):
    """The three reference CPU paths timed with the reference's median method
    (bench/timing.py) on a 2^18-row sample; the fastest is the baseline."""
    rows = min(cfg["n"], CPU_SAMPLE_ROWS)
    scale = cfg["n"] / rows
    from oracle import time_call

    paths = {}
    for name, (fn, what) in cpu_paths(cfg, rows).items():
        ms, reps = time_call(fn, target_s=1.0, max_reps=20)
        paths[name] = {"ms_per_sample": round(ms, 3), "reps": reps,
                       "qps": round(cfg["b"] / (ms / 1e3 * scale), 2), "what": what}
    best = min(paths, key=lambda nm: paths[nm]["ms_per_sample"])
    return {
        "value": paths[best]["qps"],
        "unit": "QPS",
        "cores": os.cpu_count(),
        "cpu_model": cpu_model(),
        "kind": "port",
        "path": best,
        "sample": (f"all {cfg['b']} queries x {rows} of {cfg['n']} corpus rows per call (median of reps, "
                   f"reference bench/timing.py method), scaled x{scale:.3g} to the full corpus; fastest of "
                   f"the reference's three CPU paths, restated in oracle/cpu_paths.py"),
        "paths": paths,
    }


def run_reference(args, cfg):
    """The reference's CPU implementation of the search on the host cores.

    Each step is one call of the fastest of the reference's CPU paths (chosen by
    a short median timing first) over a bounded sample: all queries against up
    to 2^18 corpus rows, fewer if K steps would take more than ~90 s. The line's
    ms_per_step is the measured time of such a step; `value` scales it to the
    full corpus (config rows / sample rows, given as `row_scale`)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import time_call

    W = max(args.warmup, 0)
    rows = min(cfg["n"], CPU_SAMPLE_ROWS)
    paths = cpu_paths(cfg, rows)
    probe = {nm: time_call(fn, target_s=0.3, max_reps=5)[0] for nm, (fn, _) in paths.items()}
    best = min(probe, key=probe.get)
    budget_ms = 90e3 / max(args.steps, 1)
    if probe[best] > budget_ms and rows > 8192:
        rows = max(8192, int(rows * budget_ms / probe[best]) // 1024 * 1024)
        paths = cpu_paths(cfg, rows)
    fn, what = paths[best]
    for _ in range(min(W, 3)):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    scale = cfg["n"] / rows
    qps = cfg["b"] / (t * scale)
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(qps, 2),
        "unit": "QPS",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": W,
        "ms_per_step": round(t * 1e3, 3),
        "ms_per_step_median": round(statistics.median(times) * 1e3, 3),
        "row_scale": round(scale, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": bench_config(args, cfg, args.gpus),
        "cpu_baseline": {
            "value": round(qps, 2), "unit": "QPS", "cores": os.cpu_count(), "cpu_model": cpu_model(),
            "kind": "port", "path": best,
            "sample": (f"each step: all {cfg['b']} queries x {rows} of {cfg['n']} corpus rows through {what}; "
                       f"ms_per_step is that measured step, value scales it x{scale:.4g} to the full corpus; "
                       f"path chosen as the fastest of {sorted(probe)} by a median timing "
                       f"({', '.join(f'{k}={v:.1f} ms' for k, v in sorted(probe.items()))})"),
        },
        "e2e": {"value": round(qps, 2), "unit": "QPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def make_shard(torch, n, d, seed, first_chunk, device):
    """Unit-norm fp16 rows generated per 2^18-row chunk with a per-GLOBAL-chunk
    seed (reference bench/bench_gpu.py:36-43), so any sharding yields the same
    global corpus."""
    x = torch.empty((n, d), dtype=torch.float16, device=device)
    for c, start in enumerate(range(0, n, CHUNK)):
        g = torch.Generator(device=device).manual_seed(seed * 100003 + first_chunk + c)
        blk = torch.randn(min(CHUNK, n - start), d, device=device, generator=g)
        x[start : start + blk.shape[0]] = (blk / blk.norm(dim=1, keepdim=True)).half()
    return x


def make_queries(torch, b, d, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(b, d, device=device, generator=g)
    return (q / q.norm(dim=1, keepdim=True)).half()


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # nvidia-smi missing: report no clocks
            self.proc = None

    def stop(self, windows=None):
        """Summary of the samples taken inside `windows` = [(start, end), ...] host
        times (time.time()) of the timed loops; all samples if fewer than 3 fall in them."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                try:
                    parts[0] = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    parts[0] = None
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = rows
        if windows:
            sel = [r for r in rows if r[0] is not None and any(w0 <= r[0] <= w1 for w0, w1 in windows)]
            inside = sel if len(sel) >= 3 else rows
        sm = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in inside if r[3].replace(".", "").isdigit()]
        pw = [float(r[4]) for r in inside if r[4].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in inside for j in range(4) if r[6 + j].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside), "power_w_median": statistics.median(pw) if pw else None,
                "window": "timed region" if inside is not rows else "whole run (too few samples inside)"}


def parity_check(torch, local_index, q_dev, result, k, row_offset, world, rows=8):
    """Checks `rows` query rows of a finished search against the CPU oracle.

    Every rank streams its own stored shard to the host in 2^19-row blocks and
    computes the oracle's top-(k+1) for the selected queries with global row
    ids; rank 0 merges the ranks' lists (oracle.merge_topk) and compares them
    with the search result. Runs after the timed loops, never inside them.
    Returns the comparison on rank 0 (None elsewhere)."""
    import numpy as np
    import torch.distributed as dist

    from oracle import compare_topk, exact_topk_blocks, merge_topk

    d = local_index.dim
    b = q_dev.shape[0]
    sel = np.unique(np.linspace(0, b - 1, min(b, rows)).astype(np.int64))
    dev = q_dev.device
    q32 = local_index._prep_queries(q_dev)[torch.as_tensor(sel, device=dev), :d].float().cpu().numpy()
    x = local_index._x

    def blocks(step=1 << 19):
        for s in range(0, x.shape[0], step):
            yield row_offset + s, x[s : s + step].cpu()[:, :d].float().numpy()

    kk = k + 1
    lv, li = exact_topk_blocks(q32, blocks(), kk)
    if lv.shape[1] < kk:  # a shard with fewer rows than k + 1
        pad = kk - lv.shape[1]
        lv = np.concatenate([lv, np.full((lv.shape[0], pad), -np.inf, np.float32)], 1)
        li = np.concatenate([li, np.full((li.shape[0], pad), np.iinfo(np.int64).max, np.int64)], 1)
    if world > 1:
        tv = torch.from_numpy(np.ascontiguousarray(lv)).to(dev)
        ti = torch.from_numpy(np.ascontiguousarray(li)).to(dev)
        gv = torch.empty((world,) + tuple(tv.shape), dtype=tv.dtype, device=dev)
        gi = torch.empty((world,) + tuple(ti.shape), dtype=ti.dtype, device=dev)
        dist.all_gather_into_tensor(gv, tv)
        dist.all_gather_into_tensor(gi, ti)
        gv, gi = gv.cpu().numpy(), gi.cpu().numpy()
        lv, li = merge_topk(list(gv), list(gi), kk)
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    got_v = result[0].cpu().numpy()[sel]
    got_i = result[1].cpu().numpy()[sel]
    res = compare_topk(got_v, got_i, lv, li, k)
    res["what"] = (f"{len(sel)} of {b} query rows (evenly spaced) of one search after the timed loops, vs the CPU "
                   f"oracle (numpy fp32 exact top-k, oracle/exact.py) on the stored corpus of all {world} rank(s)")
    return res


def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import cuda_vector_search as cvs
    from cuda_vector_search import _ext

    mod = _ext.load()
    n, d, b, k = cfg["n"], cfg["d"], cfg["b"], cfg["k"]
    chunks_per_shard = (n + CHUNK - 1) // CHUNK
    x = make_shard(torch, n, d, seed=1, first_chunk=rank * chunks_per_shard, device=dev)
    if world > 1:
        index = cvs.ShardedIndex(x, metric=cfg["metric"], device=dev, copy=False)
        local_index = index.local
    else:
        index = cvs.Index(x, metric=cfg["metric"], device=dev, copy=False)
        local_index = index
    q_dev = make_queries(torch, b, d, seed=2, device=dev)
    q_host = q_dev.float().cpu().pin_memory()
    del x

    def step(q):
        return index.search(q, k)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step(q_dev)
    barrier()

    # A corpus that fits in L2 would stay there from one step to the next; such
    # configs write a buffer twice the L2 size before every timed step, outside
    # the step's CUDA-event interval, and time the steps one by one.
    corpus_bytes = 2 * n * local_index._x.shape[1]
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if corpus_bytes < 2 * L2_BYTES else None
    step_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)] if flush_buf is not None else []

    def flush(s):
        flush_buf.fill_(s & 255)

    # Timed region: device-resident queries, CUDA events on the launching stream.
    stream = torch.cuda.current_stream()
    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, bb in ev_pairs:  # torch creates the CUDA event on first record
        a.record(stream)
        bb.record(stream)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    host_t0 = time.time()
    t0.record(stream)
    for s in range(args.steps):
        if flush_buf is not None:
            flush(s)
            step_evs[s][0].record(stream)
        mod.set_profile_events(ev_pairs[s][0].cuda_event, ev_pairs[s][1].cuda_event)
        step(q_dev)
        if flush_buf is not None:
            step_evs[s][1].record(stream)
    t1.record(stream)
    barrier()
    host_t1 = time.time()
    mod.set_profile_events(0, 0)
    ms_total = sum(a.elapsed_time(bb) for a, bb in step_evs) if flush_buf is not None else t0.elapsed_time(t1)
    kern_ms = [a.elapsed_time(bb) for a, bb in ev_pairs]

    # End to end through the public API: pinned host fp32 queries in, host results out.
    # It starts from the same rested state as the loop above: after ~200 ms of
    # back-to-back searches the 1 kW power cap lowers the SM clock, and without
    # the pause this loop would run in that window while the first did not.
    # Each step's results land in pinned host buffers; the barrier after the loop
    # waits for the last of them. As a serving loop would run it, step s's results
    # are read back on a read-back stream after step s+1 has been issued, so the
    # copy overlaps step s+1's search and step s+1's query upload is not queued
    # behind it. The compute stream waits for that copy before step s+2, so the
    # result tensors' memory is reused in stream order (no record_stream, which
    # would make the allocator grow its pool with cudaMalloc calls that stall the
    # host). The pinned result buffers are allocated, and the path warmed up
    # (upload ring, allocator blocks), before the timed loop: a pinned allocation
    # (cudaHostAlloc) takes milliseconds and leaves the GPU idle meanwhile.
    v_host = torch.empty((b, k), dtype=torch.float32, pin_memory=True)
    i_host = torch.empty((b, k), dtype=torch.int64, pin_memory=True)
    rb_stream = torch.cuda.Stream(device=dev)
    searched = [torch.cuda.Event() for _ in range(2)]
    read_back = torch.cuda.Event()

    def read(res, ev):
        rb_stream.wait_event(ev)
        with torch.cuda.stream(rb_stream):
            v_host.copy_(res[0], non_blocking=True)
            i_host.copy_(res[1], non_blocking=True)
        read_back.record(rb_stream)
        stream.wait_event(read_back)

    def e2e_loop_flushed(steps):
        # One step at a time (no pipelining across the flushes), each timed alone.
        for s in range(steps):
            flush(s)
            step_evs[s][0].record(stream)
            cur = index.search(q_host, k)
            v_host.copy_(cur[0], non_blocking=True)
            i_host.copy_(cur[1], non_blocking=True)
            step_evs[s][1].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(bb) for a, bb in step_evs[:steps])

    def e2e_loop(steps):
        prev = None
        for s in range(steps):
            cur = index.search(q_host, k)
            searched[s & 1].record(stream)
            if prev is not None:
                read(prev, searched[(s - 1) & 1])
            prev = cur
        read(prev, searched[(steps - 1) & 1])

    e2e_loop(max(args.warmup, 3))
    e2e_t0, e2e_t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    time.sleep(0.3)
    barrier()
    host_e0 = time.time()
    e2e_t0.record(stream)
    e2e_flushed_ms = e2e_loop_flushed(args.steps) if flush_buf is not None else None
    if flush_buf is None:
        e2e_loop(args.steps)
    e2e_t1.record(stream)
    barrier()
    host_t2 = time.time()
    # The samples taken while either loop kept the GPU busy (not the pause between).
    clk = clocks.stop(windows=[(host_t0, host_t1), (host_e0, host_t2)])
    e2e_ms_total = e2e_flushed_ms if flush_buf is not None else e2e_t0.elapsed_time(e2e_t1)

    # Untimed afterwards: the same K steps without the profiling events. The
    # events sit between the kernels of a search and break their programmatic-
    # launch chain (measured: +10 us per C1 call, +1% at C2), so the timed loop
    # above, which carries them for the roofline, slightly overstates the step.
    barrier()
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    u0.record(stream)
    for s in range(args.steps):
        if flush_buf is not None:
            flush(s)
            step_evs[s][0].record(stream)
        step(q_dev)
        if flush_buf is not None:
            step_evs[s][1].record(stream)
    u1.record(stream)
    barrier()
    plain_ms_total = sum(a.elapsed_time(bb) for a, bb in step_evs) if flush_buf is not None else u0.elapsed_time(u1)

    # Untimed afterwards: where a sharded step's time goes (CUDA events on the
    # current stream around the local search, the all-gather and the merge).
    # Steps run back to back as in the timed loop (no host synchronisation
    # between them, which would turn host-side skew between the ranks into
    # all-gather time); each step records its own four events.
    phases = [0.0, 0.0, 0.0]
    if world > 1:
        reps = min(args.steps, 20)
        pevs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(reps)]
        barrier()
        for pev in pevs:
            index.phase_events = pev
            step(q_dev)
        index.phase_events = None
        torch.cuda.synchronize()
        for pev in pevs:
            for j in range(3):
                phases[j] += pev[j].elapsed_time(pev[j + 1]) * 1e3 / reps
    tt = torch.tensor([ms_total, e2e_ms_total, sum(kern_ms), plain_ms_total] + phases, dtype=torch.float64,
                      device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms_total, kern_total, plain_ms_total = tt.tolist()[:4]
    phases = tt.tolist()[4:]
    parity = None if args.no_parity else parity_check(torch, local_index, q_dev, step(q_dev), k,
                                                       index.row_offset if world > 1 else 0, world)
    ms = ms_total / args.steps
    kern_avg = kern_total / args.steps
    value = world * b / (ms / 1e3)
    e2e_value = world * b / (e2e_ms_total / args.steps / 1e3)

    if rank == 0:
        hbm_peak, tc_peak, peak_src = load_peaks()
        d_pad = local_index._x.shape[1]
        flops = 2.0 * b * n * d
        alg_bytes = 2.0 * n * d_pad + 2.0 * b * d_pad + 12.0 * b * k
        tflops = flops / (kern_avg / 1e3) / 1e12
        gbs = alg_bytes / (kern_avg / 1e3) / 1e9
        tc_time = flops / (tc_peak * 1e12)
        hbm_time = alg_bytes / (hbm_peak * 1e9)
        bound = "tensor" if tc_time >= hbm_time else "hbm"
        traffic = load_traffic(args.config)
        roof_tc = {"bound": "tensor", "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                   "frac": round(tflops / tc_peak, 4), "traffic": traffic,
                   "note": f"bf16 dense burst peak, {peak_src}"}
        roof_hbm = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(gbs / hbm_peak, 4), "traffic": traffic,
                    "note": f"copy bandwidth, {peak_src}; algorithmic bytes = corpus + queries + results"}
        roofline = roof_tc if bound == "tensor" else roof_hbm
        # Our kernels per step: query preparation fused with the workspace clear,
        # search, merge of the segment lists (+ the merge of the gathered shard lists).
        launches_per_step = 3 if world == 1 else 4
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "QPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic",
            "config": bench_config(args, cfg, world),
            "qps_global": round(b / (ms / 1e3), 1),
            "roofline": roofline,
            "roofline_other": roof_hbm if bound == "tensor" else roof_tc,
            "kernel_ms": round(kern_avg, 4),
            "e2e": {"value": round(e2e_value, 1), "unit": "QPS",
                    "h2d_bytes_per_step": int(q_host.numel() * q_host.element_size()),
                    "d2h_bytes_per_step": int(v_host.numel() * 4 + i_host.numel() * 8)},
            "clocks": clk,
            "gpu_launches": launches_per_step * args.steps,
            "parity": parity,
            "without_kernel_events": {
                "ms_per_step": round(plain_ms_total / args.steps, 4),
                "value": round(world * b / (plain_ms_total / args.steps / 1e3), 1),
                "note": ("the same K steps after the timed loop without the per-step profiling events that time "
                         "the search kernel (they break the launch chain between its kernels); untimed, max over ranks"),
            },
        }
        if world > 1:
            out["phases_us"] = {"local_search": round(phases[0], 1), "all_gather": round(phases[1], 1),
                                "merge": round(phases[2], 1),
                                "note": "max over ranks of the mean of up to 20 untimed back-to-back steps after the timed loops; all_gather includes waiting for the slowest rank's local search"}
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(cfg)
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_sweep(args, cfg):
    """Plan sweep on one GPU (the reference's bench/sweep.py + report.py role):
    for the config's corpus, every batch size in --sweep-batches and every plan
    hint (bq 0 = automatic, 128 = one-CTA tiles, 256 = CTA pairs; chunks 0 =
    one CTA (pair) per SM, or the given counts), the live CUDA-event time of the
    search kernel and of the whole call. Prints one JSON row per point and a
    markdown table; --report PATH also writes the table there."""
    import torch

    import cuda_vector_search as cvs
    from cuda_vector_search import _ext

    mod = _ext.load()
    dev = torch.device("cuda", 0)
    n, d, k = cfg["n"], cfg["d"], cfg["k"]
    x = make_shard(torch, n, d, seed=1, first_chunk=0, device=dev)
    index = cvs.Index(x, metric=cfg["metric"], device=dev, copy=False)
    hbm_peak, tc_peak, _ = load_peaks()
    d_pad = index._x.shape[1]
    batches = [int(v) for v in args.sweep_batches.split(",")]
    chunk_list = [int(v) for v in args.sweep_chunks.split(",")]
    rows = []
    for b in batches:
        q = index._prep_queries(make_queries(torch, b, d, seed=2, device=dev))
        for bq in (0, 128, 256):
            if bq == 256 and b <= 128:
                continue
            for chunks in chunk_list:
                for _ in range(3):
                    mod.fused_topk(q, index._x, k, bq, chunks)
                torch.cuda.synchronize()
                reps = max(3, args.steps)
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
                for a_, b_ in evs:
                    a_.record()
                    b_.record()
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                t0.record()
                for a_, b_ in evs:
                    mod.set_profile_events(a_.cuda_event, b_.cuda_event)
                    _, _, plan = mod.fused_topk(q, index._x, k, bq, chunks)
                t1.record()
                torch.cuda.synchronize()
                mod.set_profile_events(0, 0)
                kern = sum(a_.elapsed_time(b_) for a_, b_ in evs) / reps
                call = t0.elapsed_time(t1) / reps
                tflops = 2.0 * b * n * d / (kern / 1e3) / 1e12
                gbs = (2.0 * n * d_pad + 2.0 * b * d_pad + 12.0 * b * k) / (kern / 1e3) / 1e9
                row = {"config": args.config, "n": n, "d": d, "b": b, "k": k, "bq": bq, "chunks": chunks,
                       "plan": plan.tolist(), "kernel_ms": round(kern, 4), "call_ms": round(call, 4),
                       "qps": round(b / (call / 1e3), 1), "tflops": round(tflops, 1), "gbs": round(gbs, 1),
                       "tc_frac": round(tflops / tc_peak, 4), "hbm_frac": round(gbs / hbm_peak, 4)}
                rows.append(row)
                print(json.dumps(row), flush=True)
    lines = [f"Plan sweep, {args.config}: {n} x {d} fp16, k={k}, {cfg['metric']} (one B200; kernel = CUDA events "
             f"around the search kernel, call = whole fused_topk)", "",
             "| b | bq hint | chunks | plan | kernel ms | call ms | QPS | TF/s | GB/s | TC frac | HBM frac |",
             "|---|---|---|---|---|---|---|---|---|---|---|"]
    for r in rows:
        lines.append(f"| {r['b']} | {r['bq']} | {r['chunks']} | {r['plan']} | {r['kernel_ms']} | {r['call_ms']} | "
                     f"{r['qps']:.0f} | {r['tflops']} | {r['gbs']} | {r['tc_frac']} | {r['hbm_frac']} |")
    table = "\n".join(lines)
    print(table)
    if args.report:
        Path(args.report).write_text(table + "\n")


def run_merge_case(args):
    """Profiling case for the multi-GPU merge kernel on one GPU: merge_lists over
    gathered [ranks, b, k] lists of the C5 8-GPU shape (8 x 1024 x 100), five
    calls (no timing, no JSON line)."""
    import torch

    from cuda_vector_search import _ext

    mod = _ext.load()
    ranks, b, k = 8, 1024, 100
    g = torch.Generator(device="cuda").manual_seed(3)
    v = torch.rand(ranks, b, k, device="cuda", generator=g).sort(dim=2, descending=True).values.contiguous()
    i = torch.randint(0, 1 << 30, (ranks, b, k), device="cuda", generator=g)
    for _ in range(5):
        mod.merge_lists(v, i, k)
    torch.cuda.synchronize()
    print("merge_lists case done", flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    # 200 steps: ~80 ms at C2, long enough for several clock samples inside the
    # timed loop (nvidia-smi samples every 20 ms), short enough to stay below
    # the power cap's reaction time.
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the post-timing oracle check (profiling runs)")
    ap.add_argument("--rows", type=int, default=0, help="override rows per GPU (profiling runs)")
    ap.add_argument("--batch", type=int, default=0, help="override the batch size (profiling runs)")
    ap.add_argument("--sweep", action="store_true", help="plan sweep instead of the benchmark line")
    ap.add_argument("--sweep-batches", default="1,2,8,32,128,256,512,1024")
    ap.add_argument("--sweep-chunks", default="0")
    ap.add_argument("--report", default="", help="with --sweep: write the markdown table to this path")
    ap.add_argument("--merge-case", action="store_true",
                    help="profiling case: merge_lists over [8, 1024, 100] gathered lists (one GPU)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.rows:
        cfg["n"] = args.rows
    if args.batch:
        cfg["b"] = args.batch
    if args.merge_case:
        run_merge_case(args)
    elif args.sweep:
        run_sweep(args, cfg)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
