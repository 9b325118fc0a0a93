"""Benchmark of the MLA decode step (the one hot path of lechebs/ada-mla).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One step = one weight-absorbed decode O* = softmax(Q* C^T) C[:, :512] of the
configured batch with inputs already resident in HBM.  Default workload is
BASELINE config 1 (B=1, n_h=128, N=4096, fp16) on every rank: with N GPUs each
rank decodes its own sequence (sequence sharding, no data-path collective), so
per-GPU work is fixed ("scaling": "weak").  Every run (any N) also measures the
two multi-GPU layouts of the north star and reports them under "multi_gpu":
config 3 with its KV length split over the N ranks (local decode + one NCCL
all-gather of the (O, LSE) partials + LSE merge, strong scaling) and config 2
with its 128 sequences sharded over the ranks (strong scaling, no collective).

Metric: latent-KV HBM GB/s = algorithmic cache bytes of all ranks / step time
(max over ranks), plus us/step.  L2: every step reads a different copy of the
inputs from a ring whose total size is >= 3x the L2, so each step streams its
cache from HBM.  The timed region is one replay of a CUDA graph of exactly K
steps launched through the C ABI (mla_b200_decode_batched_f16) with
preallocated buffers; NVML clock readings are taken back to back from just
before that replay until it has finished.

roofline.launch_us is the average duration of the main decode kernel: CUDA
events recorded by the library immediately around that launch on its stream,
in an eager run whose launches were queued behind a device-side sleep (so no
host latency and no graph event nodes sit inside the interval).

`--page-size P` (P a multiple of 32) runs the same step on a paged copy of
the cache: shuffled pages of P tokens in a pool, addressed through a block
table (mla_b200_decode_paged_f16); the metric still counts each sequence's own
cache bytes.

`--kv-dtype fp8` runs it on an e4m3 copy of the cache (kv scale 1;
mla_b200_decode_batched_fp8); the metric then counts the e4m3 bytes (576 per
token), so compare us/step with the fp16 line.

`--mtp K` decodes K draft tokens per sequence (mla_b200_decode_mtp_f16): one
pass over the cache when K x n_h <= 128, else one 128-row pass per draft with
the repeated reads served by L2; the metric counts each sequence's cache bytes
once (config keys `draft_tokens`, `tokens_per_step`).

`--dtype bf16` runs the step on bf16 copies of Q* and the cache
(mla_b200_decode_batched_bf16, bf16 output); same bytes per token.

`--impl reference` times the reference's own FP32 CPU kernel
(run_mla_decode_cpu, compiled from the reference sources into oracle/_ref, or
our C restatement when that build is absent) on all host cores, rank 0 only,
on the same workload and `config`.  That arm never loads this repository's
CUDA libraries (the workload generators are loaded by file path, not through
the ada_mla package).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_PARENT = os.path.join(ROOT, "ada-mla_b200")
sys.path.insert(0, PKG_PARENT)
sys.path.insert(0, ROOT)

HEAD_DIM_K = 576
METRIC = "MLA decode latent-KV HBM GB/s (us/step alongside)"
UNIT = "GB/s"
PROFILES = os.path.join(ROOT, "profiles")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def load_workloads():
    """The synthetic workload generators (ada_mla/workloads.py), loaded by path
    so that the package's __init__ -- which loads the CUDA libraries -- does not
    run.  The module itself imports only torch."""
    name = "_mla_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_PARENT, "ada_mla", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def ncu_traffic(cfg: int):
    """DRAM bytes (read + write) of one launch of the main decode kernel on this
    config, as recorded in its committed ncu summary (profiles/), with the
    summary's file name and the commit the capture ran on."""
    path = os.path.join(PROFILES, f"tc_decode_cfg{cfg}_ncu.md")
    try:
        with open(path) as f:
            text = f.read()
    except OSError:
        return None, None
    m = re.search(r"^traffic_bytes_per_launch:\s*([0-9.eE+]+)", text, re.M)
    c = re.search(r"^captured_at_commit:\s*(\S+)", text, re.M)
    if not m:
        return None, None
    return float(m.group(1)), f"profiles/{os.path.basename(path)} (commit {c.group(1) if c else '?'})"


def workload_config(args, wl, world: int) -> dict:
    """The `config` object of the JSON line: the workload only, identical for
    both arms at the same arguments and world size."""
    variant = ("dense" if wl.cu_seqlens is None else "packed varlen")
    if args.page_size > 0:
        variant = f"paged cache: shuffled {args.page_size}-token pages"
    if args.kv_dtype == "fp8":
        variant += ", e4m3 cache"
    if args.dtype == "bf16":
        variant += ", bf16"
    return {
        "workload": f"cfg{args.config}: B={wl.batch} n_h={wl.num_heads} N={wl.max_seq_len} per rank "
                    f"({variant}), softmax scale folded into Q*",
        "cfg": args.config, "batch_per_rank": wl.batch, "num_heads": wl.num_heads,
        "seq_len": wl.max_seq_len, "total_tokens_per_rank": wl.total_tokens,
        "page_size": args.page_size if args.page_size > 0 else None,
        "draft_tokens": args.mtp if args.mtp > 1 else 1,
        "tokens_per_step": wl.batch * max(args.mtp, 1) * world,
        "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
        "l2": "GPU arm: every timed step reads its own copy of the inputs from a rotating ring "
              ">= 3x L2 (inputs larger than L2)",
    }


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML reads only; no setting is changed)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, interval_s: float = 0.002):
        self.interval_s = interval_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _sample(self):
        n = self._nvml
        mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
        try:
            reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            reasons = n.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.samples.append((mhz, reasons))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            if self.interval_s > 0:
                time.sleep(self.interval_s)

    def __enter__(self):
        if self._nvml is not None:
            try:
                self._sample()  # one reading just before the timed region starts
            except Exception:
                pass
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_init():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_replay(graph, steps: int, world: int, local: int, align=None):
    """Times ONE replay of `graph` (exactly `steps` steps) with CUDA events,
    bracketed by a barrier and a synchronize; returns (ms per step, max over
    ranks, clocks sampled by NVML while that replay runs).  `align`: one
    untimed step of a cross-rank exchange, enqueued before the start event so
    that every rank's events start when that exchange completes on all ranks
    (otherwise the first timed exchange waits out the ranks' host skew after
    the barrier, charged to the earliest rank)."""
    import torch

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local, interval_s=0.0)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        if align is not None:
            align()
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ev0.elapsed_time(ev1), world) / steps
    return ms, sampler.summary()


def native_libs_loaded() -> list[str]:
    """Shared objects of this repository mapped into this process."""
    try:
        with open("/proc/self/maps") as f:
            paths = {line.split()[-1] for line in f if line.rstrip().endswith(".so")}
    except OSError:
        return []
    return sorted(p for p in paths if p.startswith(ROOT) or "ada_mla" in p or "mla_b200" in p)


# ---------------------------------------------------------------------------
# CPU baseline / reference arm
# ---------------------------------------------------------------------------
def _cpu_decode(wl_cpu, seqs, impl: str, threads: int):
    import numpy as np

    import oracle

    q = wl_cpu.query.float().numpy()
    nbytes = 0
    for b in seqs:
        c = wl_cpu.cache_rows(b).float().numpy()
        qs = (q[b].astype(np.float64) * np.sqrt(HEAD_DIM_K)).astype(np.float32)
        oracle.run_mla_decode_cpu(qs, c, impl=impl, threads=threads)
        nbytes += c.shape[0] * HEAD_DIM_K * 2
    return nbytes


def cpu_decode_sample(wl_cpu, impl: str, threads: int, min_seconds: float):
    """Runs the reference CPU kernel on the whole (small) workload until
    min_seconds of wall time have passed.  Returns (GB/s, seconds, repetitions)."""
    bytes_done = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        bytes_done += _cpu_decode(wl_cpu, range(wl_cpu.batch), impl, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return bytes_done / el / 1e9, el, reps


def cpu_kind():
    import oracle

    return "reference" if oracle.have_ref() else "port"


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_arm(args):
    """--impl reference: the reference's FP32 CPU kernel on all host cores,
    rank 0 only, on the whole job's workload (world x the per-rank sequences of
    the GPU arm); each step is that decode, or a bounded sample of its
    sequences for the large configs."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    W = load_workloads()
    wl = W.make_workload(args.config, seed=0, device="cpu")
    kind = cpu_kind()
    impl = "reference" if kind == "reference" else "oracle"
    threads = cpu_cores()
    # whole-job work = world copies of the per-rank workload; a step decodes a
    # bounded sample of it (every sequence of cfg1, the first sequences of the
    # others) so that the run ends within minutes
    limit = 1 if args.config == 3 else (2 if args.config == 2 else 8)
    seqs = list(range(min(wl.batch, limit)))
    for _ in range(args.warmup):
        _cpu_decode(wl, seqs, impl, threads)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += _cpu_decode(wl, seqs, impl, threads)
    el = time.perf_counter() - t0
    gbs = nbytes / el / 1e9
    # us per step of the whole job's decode at this throughput
    job_bytes = wl.cache_bytes * world
    ms = job_bytes / (gbs * 1e9) * 1e3
    loaded = native_libs_loaded()
    if any("mla_b200" in p or "_ada_mla_ext" in p for p in loaded):
        raise SystemExit(f"reference arm loaded this repository's CUDA libraries: {loaded}")
    sample = (f"{len(seqs)} of {wl.batch} sequence(s) of cfg{args.config} per step "
              f"({sum(wl.seqlens[b] for b in seqs)} tokens), {args.steps} steps, {el:.2f} s; "
              f"ms_per_step scaled to the whole job ({world} x {wl.batch} sequences)")
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "us_per_step": ms * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, wl, world),
        "cpu_baseline": {"value": gbs, "unit": UNIT, "cores": threads, "kind": kind,
                         "cpu": cpu_model(), "sample": sample},
        "e2e": {"value": gbs, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "native_libs_loaded": loaded,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def kernel_launch_us(step, n_launch: int) -> float:
    """Average duration of the main decode kernel over n_launch eager steps.

    The library records the events immediately around that launch on its
    stream (mla_b200_set_kernel_timing).  A device-side sleep queued first
    keeps the GPU busy while the host enqueues every step, so the steps then
    run back to back and no host latency falls between the two events."""
    import torch

    from ada_mla import capi

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_launch)]
    for a, e in evs:  # torch creates the CUDA event at its first record
        a.record()
        e.record()
    s = torch.cuda.current_stream()
    # one pass to learn the host enqueue time, then a sleep that covers it
    t0 = time.perf_counter()
    for i in range(n_launch):
        step(i, s.cuda_stream)
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    torch.cuda._sleep(int(max(host_s * 2.0, 1e-3) * 2.0e9))  # ~2 GHz cycles
    for i in range(n_launch):
        capi.set_kernel_timing(*evs[i])
        step(i, s.cuda_stream)
    capi.set_kernel_timing(None, None)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(e) for a, e in evs) * 1e3


def kernel_span_us(step, steps: int, cap) -> float:
    """Mean device-side span of the main decode kernel over a graph of `steps`
    steps (mla_b200_set_kernel_span: %globaltimer at its first CTA's start
    and its last CTA's end, one slot per captured launch)."""
    import torch

    from ada_mla import capi

    span = torch.empty((steps, 2), dtype=torch.int64, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        capi.set_kernel_span(span)
        try:
            with torch.cuda.graph(g, stream=cap):
                for i in range(steps):
                    step(i, cap.cuda_stream)
        finally:
            capi.set_kernel_span(None)
    vals = []
    for _ in range(3):
        span[:, 0].fill_(-1)  # UINT64_MAX
        span[:, 1].fill_(0)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        d = (span[:, 1] - span[:, 0]).double()
        vals.append(float(d.mean()) / 1e3)
    del g
    return min(vals)


def run_ours(args):
    import torch

    rank, world, local = dist_init()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import ada_mla
    from ada_mla import capi
    from ada_mla.workloads import make_workload, paged_layout

    hbm_peak, _, peak_kind = _peaks()
    L2 = torch.cuda.get_device_properties(dev).L2_cache_size or (126 << 20)

    wl = make_workload(args.config, seed=1000 * rank, device=dev)
    step_bytes = wl.cache_bytes // (2 if args.kv_dtype == "fp8" else 1) + wl.query.numel() * wl.query.element_size()
    ring = max(2, -(-3 * L2 // step_bytes)) if not args.no_rotate else 1
    ring = min(ring, max(1, int(40e9 // step_bytes)))
    qs = [wl.query] + [wl.query.clone() for _ in range(ring - 1)]
    cs = [wl.cache] + [wl.cache.clone() for _ in range(ring - 1)]
    cu = wl.cu_seqlens
    total = wl.total_tokens
    b, nh, maxlen = wl.batch, wl.num_heads, wl.max_seq_len
    ws_bytes = capi.workspace_size(b, nh, total, maxlen, args.splits)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty((b, nh, 512), dtype=torch.float16, device=dev)
    lib = capi.lib()
    cache_2d = [c.view(-1, HEAD_DIM_K) for c in cs]
    paged = args.page_size > 0
    fp8 = args.kv_dtype == "fp8"
    mtp = args.mtp > 1
    if mtp and (paged or fp8):
        raise SystemExit("--mtp combines with neither --page-size nor --kv-dtype fp8")
    if mtp:
        g = torch.Generator(device=dev).manual_seed(77 + rank)
        qm = (torch.randn((b, args.mtp, nh, HEAD_DIM_K), generator=g, device=dev) / 192 ** 0.5).half()
        qs = [qm] + [qm.clone() for _ in range(ring - 1)]
        ws_bytes = lib.mla_b200_workspace_size_mtp(b, args.mtp, nh, total, maxlen, args.splits)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        out = torch.empty((b, args.mtp, nh, 512), dtype=torch.float16, device=dev)
    if fp8 and paged:
        raise SystemExit("--kv-dtype fp8 and --page-size do not combine")
    bf16 = args.dtype == "bf16"
    if bf16 and (paged or fp8 or mtp):
        raise SystemExit("--dtype bf16 combines with none of --page-size, --kv-dtype fp8, --mtp")
    if bf16:
        qs = [x.bfloat16() for x in qs]
        cs = [x.bfloat16() for x in cs]
        cache_2d = [c.view(-1, HEAD_DIM_K) for c in cs]
        out = torch.empty((b, nh, 512), dtype=torch.bfloat16, device=dev)
    cache_bytes = wl.cache_bytes // (2 if fp8 else 1)  # algorithmic bytes one step reads
    if fp8:
        cs8 = []
        while cs:  # convert copy by copy (the fp16 ring need not exist at once in both forms)
            cs8.append(cs.pop(0).view(-1, HEAD_DIM_K).to(torch.float8_e4m3fn))
        del cache_2d
        ws_bytes = lib.mla_b200_workspace_size_fp8(b, nh, total, maxlen, args.splits)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    if paged:
        pl = paged_layout(wl, args.page_size, seed=rank)
        pools = [pl.scatter(c) for c in cs]  # the ring's copies, each in its own pool
        del cs, cache_2d
        ws_bytes = capi.workspace_size(b, nh, b * maxlen, maxlen, args.splits)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        step_bytes = pools[0].numel() * pools[0].element_size() + wl.query.numel() * wl.query.element_size()

    def step(i, stream):
        if mtp:
            st = lib.mla_b200_decode_mtp_f16(
                qs[i % ring].data_ptr(), cache_2d[i % ring].data_ptr(),
                None if cu is None else cu.data_ptr(), b, args.mtp, nh, total, maxlen, 1.0,
                args.splits, out.data_ptr(), capi.OUT_F16, None, ws.data_ptr(), ws_bytes, stream)
        elif fp8:
            st = lib.mla_b200_decode_batched_fp8(
                qs[i % ring].data_ptr(), cs8[i % ring].data_ptr(), 1.0,
                None if cu is None else cu.data_ptr(), b, nh, total, maxlen, 1.0, args.splits,
                out.data_ptr(), capi.OUT_F16, None, ws.data_ptr(), ws_bytes, stream)
        elif bf16:
            st = lib.mla_b200_decode_batched_bf16(
                qs[i % ring].data_ptr(), cache_2d[i % ring].data_ptr(),
                None if cu is None else cu.data_ptr(), b, nh, total, maxlen, 1.0, args.splits,
                out.data_ptr(), capi.OUT_BF16, None, ws.data_ptr(), ws_bytes, stream)
        elif paged:
            st = lib.mla_b200_decode_paged_f16(
                qs[i % ring].data_ptr(), pools[i % ring].data_ptr(), pl.block_table.data_ptr(),
                pl.seq_lens.data_ptr(), b, nh, pl.num_pages, pl.page_size, pl.block_table.shape[1],
                maxlen, 1.0, args.splits, out.data_ptr(), capi.OUT_F16, None, ws.data_ptr(),
                ws_bytes, stream)
        else:
            st = lib.mla_b200_decode_batched_f16(
                qs[i % ring].data_ptr(), cache_2d[i % ring].data_ptr(),
                None if cu is None else cu.data_ptr(), b, nh, total, maxlen, 1.0, args.splits,
                out.data_ptr(), capi.OUT_F16, None, ws.data_ptr(), ws_bytes, stream)
        if st != 0:
            raise RuntimeError(f"decode failed: {capi.status_string(st)}")

    # warm-up (eager), then capture exactly K steps into one graph
    s = torch.cuda.current_stream().cuda_stream
    for i in range(args.warmup):
        step(i, s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        step(0, cap.cuda_stream)  # one eager call on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                step(i, cap.cuda_stream)
    graph.replay()  # warm the graph itself
    torch.cuda.synchronize()
    ms_step, clocks = timed_replay(graph, args.steps, world, local)
    value = world * cache_bytes / (ms_step * 1e-3) / 1e9
    del graph

    # per-launch duration of the dominant (main decode) kernel: its device-side
    # span (first CTA start to last CTA end) in a second capture of the same K
    # steps, and CUDA events around each launch (which add its launch latency)
    kernel_us = kernel_span_us(step, args.steps, cap)
    launch_us = kernel_launch_us(step, max(args.steps, 50))
    achieved = cache_bytes / (kernel_us * 1e-6) / 1e9
    traffic, traffic_src = (None, None) if (paged or fp8 or mtp or bf16) else ncu_traffic(args.config)

    # end-to-end through the public API: pinned host inputs -> device, decode,
    # result -> host, every step
    # (paged: the pool, block table and lengths all cross from the host)
    src = pools[0] if paged else (cs8[0].view(wl.cache.shape) if fp8 else
                                  (cs[0] if bf16 else wl.cache))
    qh = [(qs[0] if mtp or bf16 else wl.query).cpu().pin_memory() for _ in range(2)]
    ch = [src.cpu().pin_memory() for _ in range(2)]
    qd, cd = torch.empty_like(qh[0], device=dev), torch.empty_like(src)
    oh = torch.empty(tuple(out.shape), dtype=out.dtype).pin_memory()
    if paged:
        bth, slh = pl.block_table.cpu().pin_memory(), pl.seq_lens.cpu().pin_memory()
        btd, sld = torch.empty_like(pl.block_table), torch.empty_like(pl.seq_lens)

    def e2e_step(i):
        qd.copy_(qh[i % 2], non_blocking=True)
        cd.copy_(ch[i % 2], non_blocking=True)
        if mtp:
            o = ada_mla.mla_decode_mtp(qd, cd, cu, max_seq_len=maxlen, softmax_scale=1.0,
                                       num_splits=args.splits)
        elif paged:
            btd.copy_(bth, non_blocking=True)
            sld.copy_(slh, non_blocking=True)
            o = ada_mla.mla_decode_paged(qd, cd, btd, sld, max_seq_len=maxlen, softmax_scale=1.0,
                                         num_splits=args.splits)
        else:
            o = ada_mla.mla_decode_batched(qd, cd, cu, max_seq_len=maxlen, softmax_scale=1.0,
                                           num_splits=args.splits, kv_scale=1.0)
        oh.copy_(o, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 200))
    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / e2e_steps
    e2e_value = world * cache_bytes / (e2e_ms * 1e-3) / 1e9
    h2d = qh[0].numel() * qh[0].element_size() + ch[0].numel() * ch[0].element_size()
    if paged:
        h2d += bth.numel() * 4 + slh.numel() * 4
    d2h = oh.numel() * oh.element_size()
    del qh, ch, qd, cd

    err = ada_mla.mla_get_device_error()
    if err != 0:
        raise RuntimeError(f"device error word set: {err}")

    chunk, splits = capi.plan(b, nh, total, maxlen, torch.cuda.get_device_properties(dev).multi_processor_count)
    kernels_per_step = 2 + (1 if cu is not None or paged else 0) + (1 if fp8 else 0)
    config = workload_config(args, wl, world)
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "us_per_step": ms_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if bf16 else "f16" + (" (e4m3 cache)" if fp8 else ""),
            "data": "synthetic",
            "config": config,
            "run": {"num_splits": splits if args.splits <= 0 else args.splits, "chunk_tokens": chunk,
                    "ring_copies": ring, "ring_mib": round(ring * step_bytes / 2**20)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_source": peak_kind,
                         "traffic": traffic, "traffic_source": traffic_src,
                         "kernel": "mla::tc::tc_decode_kernel",
                         "kernel_us": kernel_us,
                         "timing": "achieved = algorithmic bytes / kernel_us; kernel_us = mean device-side "
                                   "span of the kernel (first CTA start to last CTA end, %globaltimer) over "
                                   "a graph of the K steps; launch_us = mean CUDA-event interval around each "
                                   "launch on its stream (adds the launch latency)",
                         "launch_us": launch_us,
                         "algorithmic_bytes_per_launch": cache_bytes},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": e2e_ms * 1e3,
                    "api": ("ada_mla.mla_decode_mtp" if mtp else "ada_mla.mla_decode_paged" if paged
                            else "ada_mla.mla_decode_batched")},
            "gpu_launches": args.steps * kernels_per_step,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            wl_cpu = load_workloads().make_workload(args.config, seed=0, device="cpu") \
                if args.config in (0, 1) else None
            if wl_cpu is not None:
                threads = cpu_cores()
                kind = cpu_kind()
                gbs, el, reps = cpu_decode_sample(wl_cpu, "reference" if kind == "reference" else "oracle",
                                                  threads, args.cpu_seconds)
                line["cpu_baseline"] = {"value": gbs, "unit": UNIT, "cores": threads, "kind": kind,
                                        "cpu": cpu_model(),
                                        "sample": f"{reps} full cfg{args.config} decodes "
                                                  f"({el:.1f} s wall)"}
    del qs, wl
    if not args.no_multi:
        mg = multi_gpu_lines(args, rank, world, local)
        if line is not None:
            line["multi_gpu"] = mg
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# the multi-GPU layouts (strong scaling over the ranks of this run)
# ---------------------------------------------------------------------------
def _ring_len(step_bytes: int, dev) -> int:
    """Copies of a step's inputs so that consecutive steps read >= 3x L2 of
    distinct data (capped at 40 GB)."""
    import torch

    l2 = torch.cuda.get_device_properties(dev).L2_cache_size or (126 << 20)
    return max(1, min(-(-3 * l2 // max(step_bytes, 1)), int(40e9 // max(step_bytes, 1))))


def _graph_of(fn, steps):
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=cap):
            for _ in range(steps):
                fn()
    graph.replay()
    torch.cuda.synchronize()
    return graph


def kv_split_line(cfg: int, steps: int, rank: int, world: int, local: int, exchange: str = "p2p") -> dict:
    """One sequence's KV length split over the ranks: local decode of the rank's
    slice, then the exchange: "p2p" = this library's exchange kernel over NVLink
    peer memory (the slice's split merge fused in), "nccl" = the slice's merge
    into a packed (O, LSE) buffer, one NCCL all-gather and the LSE merge."""
    import torch

    from ada_mla import multigpu
    from ada_mla.workloads import make_workload

    dev = torch.device("cuda", local)
    wl = make_workload(cfg, seed=0, device=dev)
    n = wl.max_seq_len
    dec = multigpu.KvSplitDecoder(exchange=exchange)
    lo, hi = dec.bounds(n)
    slice_bytes = max(1, (hi - lo) * wl.batch * HEAD_DIM_K * 2)
    ring = _ring_len(slice_bytes, dev)
    slices = [wl.cache[:, lo:hi].clone() for _ in range(ring)]
    it = [0]

    def fn():
        dec(wl.query, slices[it[0] % ring], 1.0)
        it[0] += 1

    graph = _graph_of(fn, steps)
    ms, clocks = timed_replay(graph, steps, world, local, align=fn)
    del graph
    stages = dec.stage_times_us(wl.query, slices[0], 1.0, reps=20)
    dec.close()
    how = ("one exchange kernel: the slice's split merge, (O, LSE) stored into every rank's buffer over "
           "NVLink peer memory, then merged" if exchange == "p2p"
           else "NCCL all-gather of (O, LSE) + LSE merge")
    return {"workload": f"cfg{cfg}: B={wl.batch} n_h={wl.num_heads} N={n}, KV length split over "
                        f"{world} GPU(s): local decode + {how}", "exchange": exchange,
            "scaling": "strong", "us_per_step": ms * 1e3,
            "value": wl.cache_bytes / (ms * 1e-3) / 1e9, "unit": UNIT,
            "stages_us_rank0": stages, "clocks_sm_mhz": clocks.get("sm_mhz")}


def sharded_line(cfg: int, steps: int, rank: int, world: int, local: int) -> dict:
    """A batch's sequences sharded over the ranks (LPT on length), each rank
    decoding its own with no collective on the data path."""
    import torch

    import ada_mla
    from ada_mla import multigpu
    from ada_mla.workloads import make_workload, seqlens_for

    dev = torch.device("cuda", local)
    lens = seqlens_for(cfg, seed=0)
    mine = multigpu.shard_sequences(lens, world)[rank]
    wl = make_workload(cfg, seed=0, device=dev, seqlens=[lens[i] for i in mine])
    ring = _ring_len(wl.cache_bytes, dev)
    caches = [wl.cache] + [wl.cache.clone() for _ in range(ring - 1)]
    it = [0]

    def fn():
        ada_mla.mla_decode_batched(wl.query, caches[it[0] % ring], wl.cu_seqlens,
                                   max_seq_len=wl.max_seq_len, softmax_scale=1.0)
        it[0] += 1

    graph = _graph_of(fn, steps)
    ms, clocks = timed_replay(graph, steps, world, local)
    del graph
    total_bytes = sum(lens) * HEAD_DIM_K * 2
    return {"workload": f"cfg{cfg}: {len(lens)} sequences sharded over {world} GPU(s) by LPT on "
                        f"length (rank 0: {len(mine)} sequences, {wl.total_tokens} tokens), no collective",
            "scaling": "strong", "us_per_step": ms * 1e3,
            "value": total_bytes / (ms * 1e-3) / 1e9, "unit": UNIT,
            "clocks_sm_mhz": clocks.get("sm_mhz")}


def multi_gpu_lines(args, rank, world, local) -> dict:
    import torch

    out = {}
    steps = max(10, min(args.steps, 50))
    lines = {
        "cfg3_kv_split": lambda: kv_split_line(3, steps, rank, world, local, "p2p"),
        "cfg3_kv_split_nccl": lambda: kv_split_line(3, steps, rank, world, local, "nccl"),
        "cfg2_sharded": lambda: sharded_line(2, steps, rank, world, local),
    }
    for name, fn in lines.items():
        # every rank runs the same steps, so an error raised by the library's
        # argument checks or allocations is raised on every rank alike; it is
        # reported in the line instead of costing the headline
        try:
            out[name] = fn()
        except Exception as e:  # noqa: BLE001
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def run_kv(args):
    """--mode kv: only the KV-split line of the configured (dense) config."""
    rank, world, local = dist_init()
    import torch

    torch.cuda.set_device(local)
    line = kv_split_line(args.config, args.steps, rank, world, local, "p2p")
    torch.cuda.empty_cache()
    line["nccl_exchange"] = kv_split_line(args.config, args.steps, rank, world, local, "nccl")
    if rank == 0:
        line.update({"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                     "ms_per_step": line["us_per_step"] / 1e3, "higher_is_better": True,
                     "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                     "config": {"workload": line["workload"], "cfg": args.config,
                                "parallelism": f"kv-split x{world}"}})
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_absorbed(args):
    """--mode absorbed: the projections on either side of the decode, on the
    tcgen05 projection kernel, for config --config's batch at 128 heads (d = d_v
    = 128): Q absorption alone, O projection alone (weight-read GB/s: each layer
    has its own weights, so a ring of weight copies >= 3x L2 is cycled), and the
    whole step absorb -> decode -> project.  The same products through torch.bmm
    (cuBLAS) are timed alongside."""
    import torch

    rank, world, local = dist_init()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from ada_mla import absorbed, capi
    from ada_mla.workloads import make_workload

    wl = make_workload(args.config, seed=0, device=dev)
    b, nh, d, dv = wl.batch, wl.num_heads, 128, 128
    g = torch.Generator(device=dev).manual_seed(5)
    q_nope = (torch.randn((b, nh, d), generator=g, device=dev)).half()
    q_rope = (torch.randn((b, nh, 64), generator=g, device=dev) / 192 ** 0.5).half()
    w_bytes = nh * d * 512 * 2
    ring = _ring_len(2 * w_bytes, dev)
    w_uk = [(torch.randn((nh, d, 512), generator=g, device=dev) / 512 ** 0.5).half() for _ in range(ring)]
    w_uv = [(torch.randn((nh, 512, dv), generator=g, device=dev) / 512 ** 0.5).half() for _ in range(ring)]
    o_star = torch.randn((b, nh, 512), generator=g, device=dev).half()
    q_star = torch.empty((b, nh, 576), dtype=torch.float16, device=dev)
    out = torch.empty((b, nh, dv), dtype=torch.float16, device=dev)
    it = [0]
    steps = max(10, min(args.steps, 100))

    def timed(fn):
        it[0] = 0

        def step():
            fn(it[0] % ring)
            it[0] += 1

        graph = _graph_of(step, steps)
        ms, clocks = timed_replay(graph, steps, world, local)
        del graph
        return ms * 1e3, clocks.get("sm_mhz")

    res = {}
    us, mhz = timed(lambda i: capi.absorb_q(q_nope, q_rope, w_uk[i], q_star))
    res["absorb_q"] = {"us": us, "weight_GBps": w_bytes / (us * 1e-6) / 1e9, "sm_mhz": mhz}
    us, mhz = timed(lambda i: capi.project_o(o_star, w_uv[i], out))
    res["project_o"] = {"us": us, "weight_GBps": w_bytes / (us * 1e-6) / 1e9, "sm_mhz": mhz}
    us, _ = timed(lambda i: torch.bmm(q_nope.transpose(0, 1), w_uk[i], out=q_star.new_empty((nh, b, 512))))
    res["absorb_q_torch_bmm"] = {"us": us, "weight_GBps": w_bytes / (us * 1e-6) / 1e9}
    us, _ = timed(lambda i: torch.bmm(o_star.transpose(0, 1), w_uv[i]))
    res["project_o_torch_bmm"] = {"us": us, "weight_GBps": w_bytes / (us * 1e-6) / 1e9}
    cache = wl.cache
    us_dec, _ = timed(lambda i: absorbed.mla_decode_batched(q_star, cache, wl.cu_seqlens,
                                                            max_seq_len=wl.max_seq_len, softmax_scale=1.0))
    us, mhz = timed(lambda i: absorbed.mla_decode_absorbed(
        q_nope, q_rope, w_uk[i], cache, w_uv[i], wl.cu_seqlens, max_seq_len=wl.max_seq_len, softmax_scale=1.0))
    res["pipeline"] = {"us": us, "decode_only_us": us_dec, "sm_mhz": mhz}
    if rank == 0:
        print(json.dumps({"mode": "absorbed", "config": {"workload": f"cfg{args.config}: B={b} n_h={nh} d={d} "
                                                                     f"d_v={dv} fp16, weights ring x{ring}"},
                          "hbm_peak_GBps": _peaks()[0], "results": res}), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=[1, 2, 3, 4])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--splits", type=int, default=-1)
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"],
                    help="bf16: decode bf16 copies of Q* and the cache")
    ap.add_argument("--mtp", type=int, default=1,
                    help="draft tokens per sequence decoded in one pass (multi-token decode)")
    ap.add_argument("--kv-dtype", default="fp16", choices=["fp16", "fp8"],
                    help="fp8: decode an e4m3 copy of the cache")
    ap.add_argument("--page-size", type=int, default=0,
                    help="decode a paged copy of the cache (pages of this many tokens)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-multi", action="store_true",
                    help="skip the multi_gpu lines (cfg3 KV split, cfg2 sharded)")
    ap.add_argument("--no-rotate", action="store_true")
    ap.add_argument("--mode", default="shard", choices=["shard", "kv", "absorbed"],
                    help="shard: every rank decodes its own sequence(s), no collective (default); "
                         "kv: only the KV-split line of --config; absorbed: the projections around "
                         "the decode and the whole absorbed step")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.mode == "kv":
        run_kv(args)
    elif args.mode == "absorbed":
        run_absorbed(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
