"""Benchmark of the MLA decode step (the one hot path of lechebs/ada-mla).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One step = one weight-absorbed decode O* = softmax(Q* C^T) C[:, :512] of the
configured batch with inputs already resident in HBM.  Default workload is
BASELINE config 1 (B=1, n_h=128, N=4096, fp16) on every rank: with N GPUs each
rank decodes its own sequence (sequence sharding, no data-path collective), so
per-GPU work is fixed ("scaling": "weak").

Metric: latent-KV HBM GB/s = algorithmic cache bytes of all ranks / step time
(max over ranks), plus us/step.  L2: every step reads a different copy of the
inputs from a ring whose total size is >= 3x the L2, so each step streams its
cache from HBM.  The timed region is a CUDA graph of exactly K steps launched
through the C ABI (mla_b200_decode_batched_f16) with preallocated buffers.

`--page-size P` (P a multiple of 32) runs the same step on a paged copy of
the cache: shuffled pages of P tokens in a pool, addressed through a block
table (mla_b200_decode_paged_f16); the metric still counts each sequence's own
cache bytes.

`--kv-dtype fp8` runs it on an e4m3 copy of the cache (kv scale 1;
mla_b200_decode_batched_fp8); the metric then counts the e4m3 bytes (576 per
token), so compare us/step with the fp16 line.

`--mtp K` decodes K draft tokens per sequence in one pass over the cache
(mla_b200_decode_mtp_f16, K x n_h <= 128): the same bytes per step for K times
the tokens (config keys `draft_tokens`, `tokens_per_step`).

`--dtype bf16` runs the step on bf16 copies of Q* and the cache
(mla_b200_decode_batched_bf16, bf16 output); same bytes per token.

`--impl reference` times the reference's own FP32 CPU kernel
(run_mla_decode_cpu, compiled from the reference sources into oracle/_ref, or
our C restatement when that build is absent) on all host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ada-mla_b200"))
sys.path.insert(0, ROOT)

HEAD_DIM_K = 576
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# main decode kernel per config, from an `ncu --set full` capture of this kernel
# on this workload (cfg 1: 4.95 MB read, 0 written; cfg 3: 152.0 + 4.0 MB).
NCU_TRAFFIC = {1: 4.949e6, 3: 156.02e6}
METRIC = "MLA decode latent-KV HBM GB/s (us/step alongside)"
UNIT = "GB/s"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML reads only; no setting is changed)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
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
            time.sleep(0.002)

    def __enter__(self):
        if self._nvml is not None:
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
def dist_init(n_gpus: int):
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


# ---------------------------------------------------------------------------
# CPU baseline / reference arm
# ---------------------------------------------------------------------------
def cpu_decode_sample(wl_cpu, impl: str, threads: int, min_seconds: float):
    """Runs the reference CPU kernel on the whole (small) workload until
    min_seconds of wall time have passed.  Returns (GB/s, sample description)."""
    import numpy as np

    import oracle

    q = wl_cpu.query.float().numpy()
    bytes_done = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        for b in range(wl_cpu.batch):
            c = wl_cpu.cache_rows(b).float().numpy()
            qs = (q[b].astype(np.float64) * np.sqrt(HEAD_DIM_K)).astype(np.float32)
            oracle.run_mla_decode_cpu(qs, c, impl=impl, threads=threads)
            bytes_done += c.shape[0] * HEAD_DIM_K * 2
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return bytes_done / el / 1e9, el, reps


def cpu_kind():
    import oracle

    return "reference" if oracle.have_ref() else "port"


def run_reference_arm(args):
    """--impl reference: the reference's FP32 CPU kernel on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from ada_mla.workloads import make_workload

    wl = make_workload(args.config, seed=0, device="cpu")
    kind = cpu_kind()
    impl = "reference" if kind == "reference" else "oracle"
    threads = os.cpu_count() or 1
    import numpy as np

    import oracle

    q = wl.query.float().numpy()
    cbytes = wl.cache_bytes

    def one_step():
        for b in range(wl.batch):
            c = wl.cache_rows(b).float().numpy()
            qs = (q[b].astype(np.float64) * np.sqrt(HEAD_DIM_K)).astype(np.float32)
            oracle.run_mla_decode_cpu(qs, c, impl=impl, threads=threads)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    el = time.perf_counter() - t0
    ms = el / args.steps * 1e3
    gbs = cbytes * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "us_per_step": ms * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cfg{args.config}: B={wl.batch} n_h={wl.num_heads} "
                               f"N={wl.max_seq_len} (full decode per step)", "cfg": args.config},
        "cpu_baseline": {"value": gbs, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"whole cfg{args.config} decode per step, {args.steps} steps"},
        "e2e": {"value": gbs, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch

    rank, world, local = dist_init(args.gpus)
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
        if args.mtp * nh > 128:
            raise SystemExit(f"--mtp {args.mtp} x {nh} heads exceeds 128 rows")
        g = torch.Generator(device=dev).manual_seed(77 + rank)
        qm = (torch.randn((b, args.mtp, nh, HEAD_DIM_K), generator=g, device=dev) / 192 ** 0.5).half()
        qs = [qm] + [qm.clone() for _ in range(ring - 1)]
        ws_bytes = capi.workspace_size(b, args.mtp * nh, total, maxlen, args.splits)
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

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms_total = max_over_ranks(ev0.elapsed_time(ev1), world)
    ms_step = ms_total / args.steps
    value = world * cache_bytes / (ms_step * 1e-3) / 1e9

    # per-launch duration of the dominant (main decode) kernel: the library
    # records these events immediately around that launch on its stream; in
    # stream capture they become event-record nodes, so a second graph of the
    # same steps times every launch at replay (no host launch latency inside)
    n_launch = max(args.steps, 50)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_launch)]
    for a, e in evs:  # torch creates its CUDA event on first record
        a.record()
        e.record()
    torch.cuda.synchronize()
    tgraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(tgraph, stream=cap):
            for i in range(n_launch):
                capi.set_kernel_timing(*evs[i])
                step(i, cap.cuda_stream)
            capi.set_kernel_timing(None, None)
    tgraph.replay()
    torch.cuda.synchronize()
    launch_ms = statistics.mean(a.elapsed_time(e) for a, e in evs)
    del tgraph
    achieved = cache_bytes / (launch_ms * 1e-3) / 1e9

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

    err = ada_mla.mla_get_device_error()
    if err != 0:
        raise RuntimeError(f"device error word set: {err}")

    chunk, splits = capi.plan(b, nh, total, maxlen, torch.cuda.get_device_properties(dev).multi_processor_count)
    kernels_per_step = 2 + (1 if cu is not None or paged else 0) + (1 if fp8 else 0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "us_per_step": ms_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if bf16 else "f16" + (" (e4m3 cache)" if fp8 else ""),
            "data": "synthetic",
            "config": {"workload": f"cfg{args.config}: B={b} n_h={nh} N={maxlen} per rank "
                                   + (f"(paged cache: shuffled {args.page_size}-token pages, "
                                      f"{pl.num_pages} pages), " if paged else
                                      f"({'packed varlen' if cu is not None else 'dense'}"
                                      f"{', e4m3 cache' if fp8 else ''}), ")
                                   + "softmax scale folded into Q*",
                       "page_size": args.page_size if paged else None,
                       "draft_tokens": args.mtp if mtp else 1,
                       "tokens_per_step": b * (args.mtp if mtp else 1) * world,
                       "cfg": args.config, "batch_per_rank": b, "num_heads": nh,
                       "seq_len": maxlen, "total_tokens_per_rank": total,
                       "num_splits": splits if args.splits <= 0 else args.splits,
                       "chunk_tokens": chunk,
                       "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                       "l2": f"rotating ring of {ring} input copies ({ring * step_bytes / 2**20:.0f} MiB "
                             f">= 3x L2)" if ring > 1 else "no rotation"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_source": peak_kind,
                         "traffic": None if paged or fp8 else NCU_TRAFFIC.get(args.config),
                         "kernel": "mla::tc::tc_decode_kernel",
                         "launch_us": launch_ms * 1e3,
                         "algorithmic_bytes_per_launch": cache_bytes},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": e2e_ms * 1e3,
                    "api": ("ada_mla.mla_decode_mtp" if mtp else "ada_mla.mla_decode_paged" if paged
                            else "ada_mla.mla_decode_batched")},
            "gpu_launches": args.steps * kernels_per_step,
            "clocks": sampler.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            from ada_mla.workloads import make_workload as mk

            wl_cpu = mk(args.config, seed=0, device="cpu") if args.config in (0, 1) else None
            if wl_cpu is not None:
                threads = os.cpu_count() or 1
                kind = cpu_kind()
                gbs, el, reps = cpu_decode_sample(wl_cpu, "reference" if kind == "reference" else "oracle",
                                                  threads, args.cpu_seconds)
                line["cpu_baseline"] = {"value": gbs, "unit": UNIT, "cores": threads, "kind": kind,
                                        "sample": f"{reps} full cfg{args.config} decodes "
                                                  f"({el:.1f} s wall)"}
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_kv(args):
    """--mode kv: ONE workload (identical on every rank) whose KV length is split
    across the ranks; each step = local decode of the rank's slice + NCCL
    all-gather of the (O, LSE) partials + LSE merge, captured in one CUDA graph.
    Total work is fixed as N grows ("scaling": "strong")."""
    import torch

    rank, world, local = dist_init(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import torch.distributed as dist

    from ada_mla import multigpu
    from ada_mla.workloads import make_workload

    wl = make_workload(args.config, seed=0, device=dev)
    assert wl.cu_seqlens is None, "kv mode takes a dense config (1 or 3)"
    n = wl.max_seq_len
    dec = multigpu.KvSplitDecoder() if world > 1 else None
    lo, hi = dec.bounds(n) if dec else (0, n)
    cache_slice = wl.cache[:, lo:hi].contiguous()

    def step():
        if dec is None:
            import ada_mla

            return ada_mla.mla_decode_batched(wl.query, cache_slice, softmax_scale=1.0)
        return dec(wl.query, cache_slice, 1.0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        step()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=cap):
            for _ in range(args.steps):
                step()
    graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms_step = max_over_ranks(ev0.elapsed_time(ev1), world) / args.steps
    value = wl.cache_bytes / (ms_step * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "us_per_step": ms_step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": f"cfg{args.config}: B={wl.batch} n_h={wl.num_heads} N={n}, KV length "
                                   f"split over {world} GPU(s), (O, LSE) all-gather + LSE merge",
                       "cfg": args.config, "parallelism": f"kv-split x{world}",
                       "l2": "single copy (no rotation)"},
            "clocks": sampler.summary()}), flush=True)
    del graph
    if world > 1:
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
    ap.add_argument("--no-rotate", action="store_true")
    ap.add_argument("--mode", default="shard", choices=["shard", "kv"],
                    help="shard: every rank decodes its own sequence(s), no collective (default); "
                         "kv: one sequence's KV length split across the ranks")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.mode == "kv":
        run_kv(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
