"""Benchmark: fp8 sparse-MLA decode on B200, B=64, H=128, top-k=2048 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5|idx|writer]

One step = one decode call over one batch (64 requests x 128 heads x 2048
selected 656-byte rows).  Multi-GPU: one process per GPU (torchrun), requests
and their KV pages sharded across GPUs (weak scaling, per-GPU batch fixed), no
collective on the hot path; the timed window is bracketed by barriers and the
step time is the max over ranks.  Rank 0 prints one JSON line.

value      = KV GB/s of the whole job = (N * B * topk * 656 bytes) / step time
e2e        = same metric through the public Python API with the step's q and
             indices copied from pinned host memory and out copied back, each
             direction on its own stream (double-buffered) so step i's copies
             overlap the decode of its neighbours, as a serving loop runs
roofline   = the decode call's achieved TFLOP/s (or GB/s for the HBM-bound
             shapes) over the same back-to-back window as ms_per_step (CUDA
             events on the launching stream; a split call's time includes its
             merge launch), against MEASURED_PEAKS.json; launch_us (events
             around each call, a second pass) is reported beside it
cpu_baseline = the oracle's numpy restatement of the reference's fp32 torch
             golden path, on a bounded sample of the same workload, rank 0, N=1
--impl reference = that CPU implementation alone, as the reference arm
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "vllm-fp8kv_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

METRIC = "fp8 sparse-MLA decode µs/call + KV GB/s, B=64,H=128,topk=2048, 1/2/4/8 GPU"
N_SETS = 4  # rotating (q, indices) sets: consecutive steps read disjoint KV rows


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) in a thread during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.samples, self.reasons = [], 0
        self.period = period_s
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception as e:  # NVML missing: report it instead of guessing
            self.err = repr(e)
            self.max_mhz = None

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit]
        med = float(np.median(self.samples)) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _traffic_per_launch(kernel: str, workload: str):
    """dram read+write bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", f"{kernel}_{workload}.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------- CPU arm
def cpu_reference_step_fn(shape_name: str, sample_requests: int, seed: int = 0):
    """Build a bounded CPU sample of the workload and return (fn, kv_bytes, desc).

    The sample keeps the per-request shape (heads, top-k, context length, page
    size, value distributions) and builds only `sample_requests` requests
    with their own KV pages, quantized by the oracle writer on the host."""
    from oracle import oracle as O
    from vllm_fp8kv import synthetic

    s = synthetic.SHAPES[shape_name]
    B = min(sample_requests, s.B)
    pool_slots = B * s.ctx if not s.shared_pool else max(B * 2048 * 64, 1 << 20)
    w = synthetic.make_host(s, seed=seed, B=B, pool_slots=min(pool_slots, s.pool_slots))
    pool = O.quantize_rows(w.kv_src_bits)
    q = synthetic.bf16_to_f32(w.q_bits)
    slots = w.slots

    def fn():
        return O.sparse_decode(q, pool, slots, w.sm_scale)

    desc = (f"{B} of {s.B} requests of {shape_name} (H={s.H}, topk={s.topk}, ctx={s.ctx}); "
            f"numpy fp32 restatement of ref_sparse_mla_decode + logsumexp, BLAS threads")
    return fn, B * s.topk * 656, desc


def shard_seeds(rank: int) -> tuple[int, int]:
    """Seeds of rank's shard: its own pool and requests, and its rotating
    q / top-k sets (weak scaling: every rank holds different data)."""
    return 1000 + rank, 2000 + rank


def gather_ranks(value, dist, device) -> list[float]:
    """Every rank's `value`, in rank order (after the timed regions)."""
    import torch

    if dist is None:
        return [float(value)]
    world = dist.get_world_size()
    out = [torch.zeros(1, dtype=torch.float64, device=device) for _ in range(world)]
    dist.all_gather(out, torch.tensor([float(value)], dtype=torch.float64, device=device))
    return [float(t.item()) for t in out]


def max_over_ranks(values, dist, device) -> list[float]:
    """Element-wise max of per-rank timings, on every rank (the slowest rank
    sets the job's step time).  `dist` is torch.distributed or None for one
    process.  Runs after the timed regions, never inside them."""
    import torch

    v = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        dist.barrier()
    return v.tolist()


def job_kv_gbs(world: int, kv_bytes_per_rank: int, ms: float) -> float:
    """KV GB/s of the whole job: every rank moves its own rows in `ms`."""
    return world * kv_bytes_per_rank / (ms * 1e-3) / 1e9


def run_reference_arm(args, rank):
    if rank != 0:
        return None
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(os.cpu_count())
    except Exception:
        pass
    fn, kv_bytes, desc = cpu_reference_step_fn(args.workload, args.cpu_sample)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    gbs = kv_bytes / dt / 1e9
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "sample": desc},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ---------------------------------------------------------------- GPU arm
def run_ours(args, rank, world, local_rank):
    import torch

    from vllm_fp8kv import synthetic
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import (
        decode_workspace_bytes,
        fp8_ds_mla_sparse_decode,
    )

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    s = synthetic.SHAPES[args.workload]
    if args.requests:
        # a smaller case of the same workload (profiling captures): fewer
        # requests; pools of disjoint contexts shrink with them
        import dataclasses

        pool = s.pool_slots if s.shared_pool else args.requests * s.ctx
        s = dataclasses.replace(s, B=args.requests, pool_slots=pool,
                                lead_masked_reqs=min(s.lead_masked_reqs, args.requests))
    pool_seed, set_seed = shard_seeds(rank)
    w = synthetic.make_device(s, seed=pool_seed, device=dev)
    splits = s.num_splits or None
    # rotating input sets over the same pool: fresh top-k rows every step
    g = torch.Generator(device=dev).manual_seed(set_seed)
    sets = [(w.q, w.slots)]
    for _ in range(N_SETS - 1):
        tok = torch.rand((s.B, s.ctx), generator=g, device=dev).argsort(dim=1)[:, : s.topk]
        tok = tok.to(torch.int32)
        if s.lead_masked_reqs:
            tok[: s.lead_masked_reqs, : s.lead_masked] = -1
        valid = tok >= 0
        t0 = torch.where(valid, tok, torch.zeros_like(tok)).long()
        page = torch.gather(w.block_table.long(), 1, t0 // 64)
        slots = torch.where(valid, page * 64 + t0 % 64, torch.full_like(page, -1)).to(torch.int32)
        q = torch.randn((s.B, s.H, 576), generator=g, device=dev).to(torch.bfloat16)
        sets.append((q, slots.contiguous()))
    ws_bytes = decode_workspace_bytes(s.B, s.H, 1, s.topk, splits or 0)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    kv = w.kv

    def step(i):
        q, sl = sets[i % N_SETS]
        return fp8_ds_mla_sparse_decode(q, kv, sl, w.sm_scale, return_lse=True,
                                        num_kv_splits=splits, workspace=ws)

    stream = torch.cuda.current_stream(dev)
    # clocks are sampled over the whole GPU phase (warm-up, the timed window,
    # the per-launch pass and the end-to-end pass): the timed window alone is
    # a few milliseconds
    clk = ClockSampler(dev.index if dev.index is not None else 0)
    clk.__enter__()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)

    # ---- device-timed window: K back-to-back steps between two events (the
    # reported step time; no event between steps, so consecutive launches
    # overlap their prologue/epilogue as a serving loop's do)
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    w0.record(stream)
    h0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # enqueue cost per call
    w1.record(stream)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    window_ms = w0.elapsed_time(w1)
    step_ms = window_ms / args.steps

    # ---- per-launch duration for the roofline: a second pass of K steps with
    # start/end events around each call on the launching stream
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        starts[i].record(stream)
        step(i)
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    launch_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(starts, ends)]))

    # ---- end to end through the public API: pinned host q/indices in, out back.
    # Copies run on their own streams (one per PCIe direction), double-buffered:
    # the H2D of step i+1 and the D2H of step i-1 overlap the decode of step i.
    hq = [sq.cpu().pin_memory() for sq, _ in sets]
    hi = [sl.cpu().pin_memory() for _, sl in sets]
    hout = [torch.empty((s.B, s.H, 512), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    hlse = [torch.empty((s.B, s.H), dtype=torch.float32).pin_memory() for _ in range(2)]
    dq = [torch.empty_like(sets[0][0]) for _ in range(2)]
    di = [torch.empty_like(sets[0][1]) for _ in range(2)]
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]   # D2H of buffer b finished
    inputs_free = [torch.cuda.Event() for _ in range(2)]  # decode of buffer b consumed dq/di

    def h2d(i):
        b, k = i & 1, i % N_SETS
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(inputs_free[b])
            dq[b].copy_(hq[k], non_blocking=True)
            di[b].copy_(hi[k], non_blocking=True)
            in_ready[b].record(copy_in)

    def e2e_run(n):
        for ev in inputs_free + out_done:
            ev.record(stream)
        h2d(0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                h2d(i + 1)
            stream.wait_event(in_ready[b])
            stream.wait_event(out_done[b])  # hout[b] / the previous out of buffer b are free
            out, lse = fp8_ds_mla_sparse_decode(dq[b], kv, di[b], w.sm_scale, return_lse=True,
                                                num_kv_splits=splits, workspace=ws)
            inputs_free[b].record(stream)
            done = torch.cuda.Event()
            done.record(stream)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done)
                out.record_stream(copy_out)
                lse.record_stream(copy_out)
                hout[b].copy_(out, non_blocking=True)
                hlse[b].copy_(lse, non_blocking=True)
                out_done[b].record(copy_out)
        stream.wait_stream(copy_in)
        stream.wait_stream(copy_out)

    e2e_run(args.warmup)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    clk.__exit__(None, None, None)
    h2d_b = sets[0][0].numel() * 2 + sets[0][1].numel() * 4
    d2h_b = hout[0].numel() * 2 + hlse[0].numel() * 4

    # ---- max over ranks (no collective on the hot path; this is after timing)
    per_rank_ms = gather_ranks(step_ms, dist, dev)
    step_ms, e2e_ms, launch_ms = max_over_ranks([step_ms, e2e_ms, launch_ms], dist, dev)

    from vllm_fp8kv.fp8_ds_mla_sparse_decode import decode_kernel_name

    kerns = decode_kernel_name(s.B, s.H, 1, s.topk, torch.bfloat16, splits or 0)
    kern = kerns.split("+")[0]
    launches_per_step = len(kerns.split("+"))
    line = None
    if rank == 0:
        kvb = synthetic.kv_bytes(s.B, s.topk)
        flops = synthetic.algorithmic_flops(s.B, s.H, s.topk)
        alg = synthetic.algorithmic_bytes(s.B, s.H, s.topk)
        peaks = _peaks()
        tensor_bound = s.H >= 64
        # the call's time in the reported back-to-back window (all of its
        # launches: a split call's merge is inside it)
        if tensor_bound:
            achieved = flops / (step_ms * 1e-3) / 1e12
            peak = peaks["bf16_tflops"]
            roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak}
        else:
            achieved = alg / (step_ms * 1e-3) / 1e9
            peak = peaks["hbm_gbs"]
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak}
        roof["peak_source"] = peaks["source"] + " (burst)"
        roof["kernel"] = kern
        roof["time_source"] = ("back-to-back window = ms_per_step"
                               + (" (decode + merge launches)" if launches_per_step > 1 else ""))
        roof["kernel_us"] = step_ms * 1e3
        roof["launch_us"] = launch_ms * 1e3
        roof["host_enqueue_us"] = host_ms * 1e3
        roof["traffic"] = _traffic_per_launch(kern, args.workload)
        roof["algorithmic_bytes_per_launch"] = alg
        roof["algorithmic_flops_per_launch"] = flops
        value = job_kv_gbs(world, kvb, step_ms)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "us_per_call": step_ms * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": f"{args.workload}: B={s.B} H={s.H} topk={s.topk} ctx={s.ctx} "
                            f"pool={s.pool_slots} slots page=64 per GPU",
                "per_gpu_batch": s.B, "global_batch": s.B * world, "heads": s.H,
                "topk": s.topk, "num_kv_splits": splits or "auto",
                "parallelism": f"request-sharded x{world}, no collective",
                "l2": f"{N_SETS} rotating q/top-k sets over a {s.pool_slots * 656 / 1e9:.2f} GB "
                      f"pool: {N_SETS * kvb / 1e6:.0f} MB of distinct rows per cycle > 126 MB L2",
            },
            "tflops": world * flops / (step_ms * 1e-3) / 1e12,
            "roofline": roof,
            "e2e": {"value": job_kv_gbs(world, kvb, e2e_ms), "unit": "GB/s",
                    "us_per_call": e2e_ms * 1e3, "h2d_bytes_per_step": h2d_b,
                    "d2h_bytes_per_step": d2h_b},
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clk.summary(),
        }
        if world > 1:
            line["per_rank_us"] = [round(v * 1e3, 2) for v in per_rank_ms]
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


# ---------------------------------------------------------------- indexer
def run_indexer(args):
    """The DSA indexer read path at the headline's request shape: 64 decode
    tokens (next_n 1), 64 index heads of dim 128, 32768-token contexts over
    their own fp8 key pages (random page permutations), top-2048 selection.
    One step = fp8_paged_mqa_logits + top_k_per_row_decode over one batch;
    four rotating query sets, keys 277 MB > L2."""
    import torch

    from vllm_fp8kv.indexer import PAGE_BYTES, fp8_paged_mqa_logits, indexer_topk

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, ctx, topk, nb_per = 64, 32768, 2048, 32768 // 64
    g = torch.Generator(device=dev).manual_seed(7)
    nb = B * nb_per
    k = torch.randn((nb * 64, 128), generator=g, device=dev)
    scale = (k.abs().amax(1) / 448.0).clamp_min(1e-30)
    kq = (k / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).view(nb, 64 * 128)
    pages = torch.empty((nb, PAGE_BYTES), dtype=torch.uint8, device=dev)
    pages[:, : 64 * 128] = kq
    pages[:, 64 * 128:] = scale.view(nb, 64).contiguous().view(torch.uint8)
    del k, kq
    bt = torch.randperm(nb, generator=g, device=dev).view(B, nb_per).to(torch.int32)
    ctxs = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    sets = []
    for _ in range(N_SETS):
        q = torch.randn((B, 1, 64, 128), generator=g, device=dev).to(torch.float8_e4m3fn)
        w = torch.randn((B, 64), generator=g, device=dev) / 8
        sets.append((q, w))
    logits = torch.empty((B, ctx), dtype=torch.float32, device=dev)
    out = torch.empty((B, topk), dtype=torch.int32, device=dev)

    def step(i, what="both"):
        q, w = sets[i % N_SETS]
        if what in ("both", "logits"):
            fp8_paged_mqa_logits(q, pages, w, ctxs, bt, None, ctx, logits=logits)
        if what in ("both", "topk"):
            from vllm_fp8kv.indexer import top_k_per_row_decode

            top_k_per_row_decode(logits, 1, ctxs, out, B, logits.stride(0), 1, topk)

    stream = torch.cuda.current_stream(dev)
    clk = ClockSampler(0)
    clk.__enter__()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    times = {}
    for what in ("both", "logits", "topk"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for i in range(args.steps):
            step(i, what)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        times[what] = e0.elapsed_time(e1) / args.steps
    clk.__exit__(None, None, None)
    key_bytes = B * ctx * 132
    logit_bytes = B * ctx * 4
    alg_logits = key_bytes + logit_bytes + B * 64 * 128 + B * 64 * 4 + B * nb_per * 4
    alg_topk = logit_bytes + B * topk * 4
    peaks = _peaks()
    achieved = alg_logits / (times["logits"] * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"] + " (burst)",
            "kernel": "indexer_logits_kernel", "time_source": "back-to-back window of logits calls",
            "kernel_us": times["logits"] * 1e3,
            "traffic": _traffic_per_launch("indexer_logits_kernel", "idx"),
            "algorithmic_bytes_per_launch": alg_logits}
    return {
        "metric": "DSA indexer fp8 paged MQA logits + top-k, B=64, 64 heads x 128, ctx 32768, top-2048",
        "value": key_bytes / (times["both"] * 1e-3) / 1e9, "unit": "GB/s (index keys)",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": times["both"],
        "us_per_call": times["both"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 MMA, f32 accumulate", "data": "synthetic",
        "config": {"workload": "idx: B=64 next_n=1 H=64 D=128 ctx=32768 topk=2048 page=64",
                   "l2": f"{N_SETS} rotating query sets over {key_bytes / 1e6:.0f} MB of keys > 126 MB L2"},
        "logits_us": times["logits"] * 1e3, "topk_us": times["topk"] * 1e3,
        "roofline": roof, "gpu_launches": 2 * args.steps, "clocks": clk.summary(),
    }


def run_writer(args):
    """The fp8_ds_mla cache writer (concat_and_cache_mla(..., "fp8_ds_mla")) on a
    65,536-token prefill chunk: bf16 latent + rope -> 656-byte rows at random
    distinct slots of the c2-sized pool (2,097,152 slots).  One step = one
    writer call; four rotating input sets (302 MB > L2).  Algorithmic bytes
    per token: 1152 read + 656 written + 8 of slot mapping."""
    import numpy as np
    import torch

    from oracle import oracle as O
    from vllm_fp8kv.cache_writer import concat_and_cache_mla

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N, slots = 65536, 2_097_152
    g = torch.Generator(device=dev).manual_seed(11)
    cache = torch.zeros((slots // 64, 64, 656), dtype=torch.uint8, device=dev)
    sets = []
    for _ in range(N_SETS):
        kv_c = torch.randn((N, 512), generator=g, device=dev).bfloat16()
        k_pe = torch.randn((N, 64), generator=g, device=dev).bfloat16()
        sm = torch.randperm(slots, generator=g, device=dev)[:N].to(torch.int64)
        sets.append((kv_c, k_pe, sm))
    one = torch.ones((), dtype=torch.float32, device=dev)

    def step(i):
        kv_c, k_pe, sm = sets[i % N_SETS]
        concat_and_cache_mla(kv_c, k_pe, cache, sm, "fp8_ds_mla", one)

    stream = torch.cuda.current_stream(dev)
    clk = ClockSampler(0)
    clk.__enter__()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps

    # end to end: each step's inputs from pinned host memory, one written row back
    host = [(kv_c.cpu().pin_memory(), k_pe.cpu().pin_memory(), sm.cpu().pin_memory())
            for kv_c, k_pe, sm in sets]
    dkv = torch.empty_like(sets[0][0]); dpe = torch.empty_like(sets[0][1]); dsm = torch.empty_like(sets[0][2])
    row_back = torch.empty((656,), dtype=torch.uint8).pin_memory()

    def e2e_step(i):
        hkv, hpe, hsm = host[i % N_SETS]
        dkv.copy_(hkv, non_blocking=True)
        dpe.copy_(hpe, non_blocking=True)
        dsm.copy_(hsm, non_blocking=True)
        concat_and_cache_mla(dkv, dpe, cache, dsm, "fp8_ds_mla", one)
        row_back.copy_(cache.view(-1, 656)[hsm[0].item()], non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    e_steps = max(3, args.steps // 20)
    e0.record(stream)
    for i in range(e_steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clk.__exit__(None, None, None)
    e2e_ms = e0.elapsed_time(e1) / e_steps

    bytes_step = N * (1152 + 656 + 8)
    peaks = _peaks()
    achieved = bytes_step / (ms * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"] + " (burst)",
            "kernel": "ds_mla_write_kernel", "time_source": "back-to-back window = ms_per_step",
            "kernel_us": ms * 1e3, "traffic": _traffic_per_launch("ds_mla_write_kernel", "writer"),
            "algorithmic_bytes_per_launch": bytes_step}
    line = {
        "metric": "fp8_ds_mla cache write GB/s (bf16 latent + rope -> 656-B rows)",
        "value": achieved, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "us_per_call": ms * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 -> e4m3", "data": "synthetic",
        "config": {"workload": f"writer: N={N} tokens, pool={slots} slots, random distinct slots",
                   "l2": f"{N_SETS} rotating input sets, {N_SETS * N * 1152 / 1e6:.0f} MB > 126 MB L2"},
        "roofline": roof,
        "e2e": {"value": bytes_step / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "us_per_call": e2e_ms * 1e3,
                "h2d_bytes_per_step": N * (1152 + 8), "d2h_bytes_per_step": 656},
        "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline:
        # the oracle writer (C restatement of the reference's writer) on a sample
        n = 8192
        src = (np.random.default_rng(0).standard_normal((n, 576)).astype(np.float32)
               .view(np.uint32) >> 16).astype(np.uint16)
        O.quantize_rows(src)
        t0 = time.perf_counter()
        reps = 0
        while True:
            O.quantize_rows(src)
            reps += 1
            if time.perf_counter() - t0 > 3.0:
                break
        dt = (time.perf_counter() - t0) / reps
        line["cpu_baseline"] = {"value": n * (1152 + 656 + 8) / dt / 1e9, "unit": "GB/s", "cores": 1,
                                "kind": "port",
                                "sample": f"{n} tokens through the oracle's C writer, {reps} timed calls"}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c2", choices=["c2", "c3", "c4", "c5", "idx", "writer"],
                    help="c2-c5: the decode shapes; idx: the DSA indexer read path; writer: the "
                         "fp8_ds_mla cache writer (one GPU)")
    ap.add_argument("--requests", type=int, default=0,
                    help="per-GPU batch override for profiling a smaller case (0 = the workload's)")
    ap.add_argument("--cpu-sample", type=int, default=8,
                    help="requests in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local_rank = _env_int("LOCAL_RANK", 0)

    if args.impl == "reference":
        line = run_reference_arm(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if args.workload in ("idx", "writer"):
        if rank == 0:
            print(json.dumps(run_indexer(args) if args.workload == "idx" else run_writer(args)), flush=True)
        return
    line = run_ours(args, rank, world, local_rank)
    if rank == 0 and line is not None:
        if world == 1 and not args.no_cpu_baseline:
            fn, kv_bytes, desc = cpu_reference_step_fn(args.workload, args.cpu_sample)
            fn()
            t0 = time.perf_counter()
            n = 0
            while True:
                fn()
                n += 1
                if time.perf_counter() - t0 > 5.0 or n >= 20:
                    break
            dt = (time.perf_counter() - t0) / n
            line["cpu_baseline"] = {"value": kv_bytes / dt / 1e9, "unit": "GB/s",
                                    "cores": os.cpu_count(), "kind": "port",
                                    "sample": desc + f"; {n} timed calls"}
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
