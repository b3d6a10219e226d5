"""Throughput of the B200 token-sampling path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload batch1024] [--impl ours|reference]

A step samples one batch of rows of the workload (default ``batch1024``:
1024 rows x vocab 152,064 fp32 logits N(0, 2^2) with 8 ids +8.0 per row,
history 64, repetition penalty 1.1, T 0.8, top-k 40, top-p 0.95) with the
inputs resident in HBM.  N > 1 runs as one process per GPU under torchrun;
every rank samples its own batch (batch sharding: no data-path collective),
so ``value`` is the rows all ranks sampled per second and ``scaling`` is weak.

Timing: W untimed steps, then K steps bracketed by a barrier and
cudaDeviceSynchronize, measured with CUDA events on the launching stream,
max over ranks.  The logits (623 MB per step) exceed the 126 MB L2, so no
flush is needed between steps.  The single-pass kernel is also timed on its
own (events around its launch) for the roofline; ``e2e`` is the same metric
through the host-buffer C entry point (H2D of each step's rows from pinned
memory, D2H of ids and states), and ``cpu_baseline`` is the reference's own
sampler (oracle/_ref, compiled from its sources) on the box's host cores.

``--impl reference`` times the reference CPU sampler alone on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/s at batch 1024×vocab 152064 fp32; % of B200 HBM peak"


def workload_of(args):
    """The named workload, at --batch rows per GPU when given (a smaller case
    of the same rows for profiler captures; bench lines keep the full size)."""
    from noel_b200.workloads import WORKLOADS

    w = WORKLOADS[args.workload]
    return w.resized(batch=args.batch) if args.batch else w


def metric_for(w) -> str:
    """The headline metric for the batch1024 workload; other workloads name
    their own shape (they are the other configurations, not the headline)."""
    if w.name == "batch1024" and w.batch == 1024:
        return METRIC
    return f"sampled rows/s, workload {w.name}: batch {w.batch}×vocab {w.vocab} {w.dtype}"


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def main_kernel(w) -> str:
    """The kernel that samples the workload's rows: the streaming kernel for
    full lists (top-k off), the block kernel for top-k above 120, else the
    one-CTA-per-row kernel (greedy and top-k up to 120)."""
    if w.temperature > 1e-4 and w.top_k <= 0:
        return "stream_rows_kernel"
    if w.temperature > 1e-4 and w.top_k > 120:
        return "sample_rows_block_kernel"
    return "sample_rows_kernel"


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of the workload's main kernel from the committed
    ncu summary (line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def reduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def cpu_reference_rows_per_s(w, logits_host: np.ndarray, hist_host, rng_host, threads: int):
    """The reference sampler (oracle/_ref) over the given rows; returns rows/s."""
    from oracle.oracle import RefSampler, make_config

    ref = RefSampler()
    cfg = make_config(**w.config_kwargs())
    ref.sample_batch(cfg, logits_host[: min(16, len(logits_host))], history=None if hist_host is None else
                     hist_host[: min(16, len(logits_host))], rng=rng_host[: min(16, len(logits_host))],
                     nthreads=threads)  # warm (page-in)
    t0 = time.perf_counter()
    ref.sample_batch(cfg, logits_host, history=hist_host, rng=rng_host, nthreads=threads)
    dt = time.perf_counter() - t0
    return len(logits_host) / dt, dt


def uniform_of(state) -> np.float32:
    """The reference's next uniform for an xorshift128+ state (sampler.c:8-21)."""
    a, b = int(state[0]), int(state[1])
    M = (1 << 64) - 1
    a ^= (a << 23) & M
    s1 = a ^ b ^ (a >> 18) ^ (b >> 5)
    return np.float32((((s1 + b) & M) >> 40)) * np.float32(1.0 / 16777216.0)


def boundary_draws(w, cand_vals, num_cands, rng0, rel=1e-5) -> int:
    """Rows whose draw r lands within rel x mass of a boundary of the running
    weight sums (sampler.c:155-191, replayed in fp32 on the reference's sorted
    weights): the draws a tolerance-based comparison would have to excuse."""
    hits = 0
    for b in range(len(rng0)):
        n = int(num_cands[b])
        if w.top_k > 0 and w.top_k < n:
            n = w.top_k
        n = min(n, cand_vals.shape[1])
        vals = cand_vals[b, :n].astype(np.float32)
        acc = np.cumsum(vals, dtype=np.float32)  # sequential fp32 sums
        mass = acc[-1] if n else np.float32(0)
        if 0.0 < w.top_p < 1.0 and n:
            keep = int(np.argmax(acc >= np.float32(w.top_p) * mass)) + 1
            acc, mass = acc[:keep], acc[keep - 1]
        if not n or mass <= 0:
            continue
        r = uniform_of(rng0[b]) * mass
        if np.min(np.abs(acc - r)) <= rel * mass:
            hits += 1
    return hits


def run_reference(args):
    """--impl reference: the reference's CPU sampler on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from noel_b200.workloads import WORKLOADS, generate_numpy
    from oracle.oracle import RefSampler

    w = workload_of(args)
    sample_rows = args.cpu_rows
    d = generate_numpy(w, seed=1, rows=sample_rows)
    threads = RefSampler().max_threads() if RefSampler.available() else os.cpu_count()
    for _ in range(args.warmup):
        cpu_reference_rows_per_s(w, d["logits"][:16], None if d["history"] is None else d["history"][:16],
                                 d["rng"][:16], threads)
    times = []
    for _ in range(args.steps):
        _, dt = cpu_reference_rows_per_s(w, d["logits"], d["history"], d["rng"], threads)
        times.append(dt)
    tot = sum(times)
    value = sample_rows * len(times) / tot
    line = {
        "impl": "reference", "metric": metric_for(w), "value": value, "unit": "rows/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_label(w),
        "data": "synthetic", "config": workload_config(w, args.gpus),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "reference",
                         "sample": f"{sample_rows} rows of {w.name} per step (one noel_sampler_t per "
                                   f"OpenMP thread, rows split across {threads} threads)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    del torch
    print(json.dumps(line), flush=True)


def dtype_label(w) -> str:
    """The logits' type; the arithmetic is fp32 either way (bf16 widens exactly)."""
    return "bf16" if w.dtype == "bf16" else "f32"


def workload_config(w, n_gpus):
    return {"workload": w.name, "batch_per_gpu": w.batch, "global_batch": w.batch * n_gpus, "vocab": w.vocab,
            "logits_dtype": w.dtype, "history": w.history, "temperature": w.temperature, "top_k": w.top_k,
            "top_p": w.top_p, "repetition_penalty": w.repetition_penalty,
            "parallelism": f"batch-sharded x{n_gpus}",
            "l2": f"no flush: {w.batch * w.vocab * (4 if w.dtype == 'f32' else 2) / 1e6:.0f} MB of logits "
                  f"per step > 126 MB L2"}


def run_ours(args):
    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import WORKLOADS, generate_torch

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    w = workload_of(args)
    d = generate_torch(w, dev, seed=1, row0=rank * w.batch)
    logits, hist, rng = d["logits"], d["history"], d["rng"]
    cfg = S.make_config(**w.config_kwargs())
    B, V = logits.shape
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    dtype = S.F32 if logits.dtype == torch.float32 else S.BF16
    hp, H, hld = (hist.data_ptr(), hist.shape[1], hist.stride(0)) if hist is not None else (None, 0, 0)

    def step(st=None):
        S.sample_batch_raw(cfg, logits.data_ptr(), dtype, B, V, logits.stride(0), hp, H, hld,
                           rng.data_ptr(), ids.data_ptr(), probs.data_ptr(), (st or stream).cuda_stream)

    rng0 = rng.clone()  # the states before any step, for the parity check
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if args.profile:  # a short, allocation-light run for ncu captures
        del d
        torch.cuda.empty_cache()
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return

    # One step captured as a CUDA graph (both kernels, the same arguments),
    # replayed once per timed step: the host launches one graph per step, so
    # ranks sharing the host's cores do not leave their GPUs waiting.
    graph = None
    try:
        cap = torch.cuda.Stream(dev)  # its scratch is made by a call before the capture
        with torch.cuda.stream(cap):
            step(cap)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            step(cap)
        graph = g
        graph.replay()
        torch.cuda.synchronize()
    except Exception as e:  # direct launches instead
        graph = None
        print(f"# CUDA graph capture unavailable ({e}); timing direct launches", file=sys.stderr)

    # ---- timed region: whole steps ----
    clocks = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t_ms = e0.elapsed_time(e1)
    t_ms = reduce_max(t_ms, world)
    rows = B * world * args.steps
    value = rows / (t_ms / 1e3)

    # ---- the single-pass kernel alone (events around its launch) ----
    kb = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ka = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        S.profile_events(kb[i], ka[i])
        step()
    S.profile_events(None, None)
    torch.cuda.synchronize()
    k_ms = float(np.mean([b.elapsed_time(a) for b, a in zip(kb, ka)]))
    k_ms = reduce_max(k_ms, world)
    peak, peak_kind = measured_peak()
    bytes_per_launch = w.bytes_per_row() * B
    achieved = bytes_per_launch / (k_ms / 1e3) / 1e9
    traffic = profile_traffic(main_kernel(w), w.name)

    # ---- end to end through the host-buffer C entry point ----
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    h_logits = logits.cpu().pin_memory()
    h_hist = hist.cpu().pin_memory() if hist is not None else None
    h_rng = rng.cpu().pin_memory()
    lg_np = h_logits.view(torch.int16).numpy().view(np.uint16) if dtype == S.BF16 else h_logits.numpy()
    hist_np = h_hist.numpy() if h_hist is not None else None
    rng_np = h_rng.numpy().view(np.uint64)
    S.sample_batch_host(cfg, lg_np, rng_np, history=hist_np)  # warm
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        S.sample_batch_host(cfg, lg_np, rng_np, history=hist_np)
    e2e_s = reduce_max(time.perf_counter() - t0, world)
    e2e_value = B * world * e2e_steps / e2e_s
    h2d = lg_np.nbytes + (hist_np.nbytes if hist_np is not None else 0) + rng_np.nbytes
    d2h = B * 4 + rng_np.nbytes

    # ---- CPU baseline and parity: the reference sampler on a bounded sample
    # of the same rows from the same initial states, rank 0.  The GPU's ids
    # and RNG states for those rows (one step from the initial states) must
    # equal the reference's bit for bit, or the run fails. ----
    cpu, parity = None, None
    if rank == 0 and not args.no_cpu:
        from oracle.oracle import RefSampler

        if RefSampler.available():
            n = min(args.cpu_rows, B)
            rng_p = rng0.clone()
            ids_p = torch.empty(B, dtype=torch.int32, device=dev)
            S.sample_batch_raw(cfg, logits.data_ptr(), dtype, B, V, logits.stride(0), hp, H, hld,
                               rng_p.data_ptr(), ids_p.data_ptr(), None, stream.cuda_stream)
            torch.cuda.synchronize()
            rng0_np = rng0[:n].cpu().numpy().view(np.uint64).copy()
            lg_ref = lg_np[:n].copy() if dtype == S.F32 else (lg_np[:n].astype(np.uint32) << 16).view(np.float32)
            threads = RefSampler().max_threads()
            ref_cfg = __import__("oracle.oracle", fromlist=["make_config"]).make_config(**w.config_kwargs())
            t0 = time.perf_counter()
            ref = RefSampler().sample_batch(ref_cfg, lg_ref, history=hist_np[:n].copy() if hist_np is not None
                                            else None, rng=rng0_np, n_list=64, nthreads=threads)
            rps = n / (time.perf_counter() - t0)
            g_ids = ids_p[:n].cpu().numpy()
            g_rng = rng_p[:n].cpu().numpy().view(np.uint64)
            mism = (g_ids != ref.ids) | (g_rng != ref.rng).any(axis=1)
            parity = {"rows": n, "mismatches": int(mism.sum()),
                      "boundary_draws": boundary_draws(w, ref.cand_vals, ref.num_cands, rng0_np),
                      "against": "the reference's src/sampler.c built into oracle/_ref, same rows and states"}
            if mism.any():
                print(json.dumps({"error": "parity", "parity": parity,
                                  "first_rows": np.where(mism)[0][:8].tolist()}), flush=True)
                sys.exit(1)
            cpu = {"value": rps, "unit": "rows/s", "cores": threads, "kind": "reference",
                   "sample": f"{n} rows of {w.name} (one noel_sampler_t per OpenMP thread)"}
        else:
            cpu = {"value": None, "unit": "rows/s", "cores": 0, "kind": "reference",
                   "sample": "oracle/_ref not built"}

    if rank == 0:
        line = {
            "metric": metric_for(w), "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": t_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype_label(w), "data": "synthetic",
            "config": workload_config(w, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": main_kernel(w), "kernel_ms": k_ms,
                         "bytes_per_launch": bytes_per_launch, "peak_source": f"{peak_kind} hbm_gbs"},
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "api": "noel_sampler_sample_batch_host (pinned host buffers)"},
            "clocks": clk,
            "gpu_launches": 2 * args.steps,
            "launch": "cuda_graph replay per step" if graph is not None else "direct",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_vocab_sharded(args):
    """The vocab-sharded workload: every rank holds columns [v_begin, v_begin +
    width) of all B rows; a step is select on every rank, one NCCL all-gather
    of the lists, and the merge (plus any full-row fallback).  All ranks
    sample the same B rows together, so ``value`` is B rows per step time and
    ``scaling`` is strong."""
    import torch

    from noel_b200 import sampler as S
    from noel_b200.sharded import NcclGather, sample_vocab_sharded, sample_vocab_sharded_local, shard_bounds
    from noel_b200.workloads import WORKLOADS, generate_torch

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    w = workload_of(args)
    d = generate_torch(w, dev, seed=1)  # the same full rows on every rank
    b0, width = shard_bounds(w.vocab, world)[rank]
    shard = d["logits"][:, b0:b0 + width].contiguous()
    hist, rng = d["history"], d["rng"]
    del d
    torch.cuda.empty_cache()
    cfg = S.make_config(**w.config_kwargs())
    gather = NcclGather() if world > 1 else None
    B = shard.shape[0]
    stream = torch.cuda.current_stream(dev)
    n_full = [0]

    def step(lg):
        if world > 1:
            ids, _, nf = sample_vocab_sharded(cfg, lg, b0, w.vocab, rng, history=hist, gather=gather)
        else:
            ids, _, nf = sample_vocab_sharded_local(cfg, lg, [(0, width)], rng, history=hist)
        n_full[0] += nf
        return ids

    for _ in range(max(args.warmup, 3)):
        step(shard)
    torch.cuda.synchronize()
    if args.profile:
        for _ in range(args.steps):
            step(shard)
        torch.cuda.synchronize()
        return
    n_full[0] = 0
    clocks = ClockSampler(local if world > 1 else torch.cuda.current_device())
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step(shard)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t_ms = reduce_max(e0.elapsed_time(e1), world)
    value = B * args.steps / (t_ms / 1e3)

    kb = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ka = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        S.profile_events(kb[i], ka[i])
        step(shard)
    S.profile_events(None, None)
    torch.cuda.synchronize()
    k_ms = reduce_max(float(np.mean([b.elapsed_time(a) for b, a in zip(kb, ka)])), world)
    peak, peak_kind = measured_peak()
    bytes_per_launch = B * (width * 4 + (hist.shape[1] * 4 if hist is not None else 0))
    achieved = bytes_per_launch / (k_ms / 1e3) / 1e9

    # end to end: the shard's rows from pinned host memory every step, ids back
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    h_shard = shard.cpu().pin_memory()
    h_ids = torch.empty(B, dtype=torch.int32).pin_memory()
    d_shard = torch.empty_like(shard)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        d_shard.copy_(h_shard, non_blocking=True)
        h_ids.copy_(step(d_shard), non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = reduce_max(time.perf_counter() - t0, world)

    if rank == 0:
        line = {
            "metric": f"sampled rows/s at batch {B}×vocab {w.vocab} {w.dtype}, vocab-sharded over {world} GPU(s)",
            "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": t_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(workload_config(w, 1), global_batch=B, batch_per_gpu=B,
                           parallelism=f"vocab-sharded x{world} ({width} columns per GPU)",
                           l2=f"no flush: {B * width * 4 / 1e6:.0f} MB of logits per GPU per step"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "kernel": "sample_rows_kernel (shard select)",
                         "kernel_ms": k_ms, "bytes_per_launch": bytes_per_launch,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "cpu_baseline": None,
            "e2e": {"value": B * e2e_steps / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": B * width * 4,
                    "d2h_bytes_per_step": B * 4, "steps": e2e_steps,
                    "api": "noel_b200.sharded (select, NCCL all-to-all of row blocks, merge, NCCL all-gather of results) from pinned host shards"},
            "rows_from_full_rows": n_full[0],
            "clocks": clk,
            "gpu_launches": 3 * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_engine_call(args):
    """The engine's call shape (src/engine.c:378-387): one row of host logits
    per generated token through noel_sampler_sample, history NULL, with the
    vocabulary truncated to 8192 (the engine's default) and in full
    (NOEL_FULL_VOCAB).  Both arms make the same calls on the same row from the
    same seed, so their id sequences must agree; the reference is its own
    sampler.c (oracle/_ref) on one host thread, as the engine runs it."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import ctypes as C

    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import WORKLOADS, generate_numpy
    from oracle.oracle import RefSampler

    torch.cuda.set_device(0)
    w = WORKLOADS["single_row"]
    for V in (8192, w.vocab):
        row = np.ascontiguousarray(generate_numpy(w.resized(vocab=V), seed=3)["logits"][0])  # pageable, like engine.c:59
        cfg = S.make_config(**dict(w.config_kwargs(), seed=1234))
        n = max(args.steps, 20) * 4
        smp = S.Sampler(cfg, max_vocab=V)
        for _ in range(max(args.warmup, 3) * 4):
            smp.sample(row)
        smp.set_config(cfg)  # reseeds (seed != 0, sampler.c:63-70)
        t0 = time.perf_counter()
        ids = [smp.sample(row) for _ in range(n)]
        us = (time.perf_counter() - t0) / n * 1e6
        line = {"metric": f"us per noel_sampler_sample call, engine call shape (host logits, history NULL), vocab {V}",
                "value": us, "unit": "us/call", "higher_is_better": False, "calls": n, "dtype": "f32",
                "data": "synthetic", "config": {"workload": "engine_call", "vocab": V, "temperature": w.temperature,
                                                "top_k": w.top_k, "top_p": w.top_p, "history": None}}
        if RefSampler.available():
            ref = RefSampler()
            L = ref.lib
            L.noel_sampler_init.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
            L.noel_sampler_sample.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
            L.noel_sampler_free.argtypes = [C.c_void_p]
            st = S.SamplerStruct()
            L.noel_sampler_init(C.byref(st), C.byref(cfg), V)
            nr = n if V <= 8192 else max(10, n // 8)
            rrow = row.copy()
            t0 = time.perf_counter()
            rids = [L.noel_sampler_sample(C.byref(st), rrow.ctypes.data, V, None, 0) for _ in range(nr)]
            rus = (time.perf_counter() - t0) / nr * 1e6
            L.noel_sampler_free(C.byref(st))
            line["reference"] = {"value": rus, "unit": "us/call", "calls": nr, "cores": 1,
                                 "kind": "reference", "sample": "src/sampler.c built into oracle/_ref, one thread"}
            line["parity"] = {"calls": nr, "mismatches": int(sum(a != b for a, b in zip(ids[:nr], rids)))}
        smp.free()
        print(json.dumps(line), flush=True)


def run_router(args):
    """The MoE router (src/sparsity.c:46-79) over a batch of tokens: 1,048,576
    tokens x 64 experts fp32 gate logits N(0, 3^2) (268 MB, larger than L2),
    top-8, per GPU.  value = routed tokens/s; the roofline is HBM (the logits
    read once, 8 B per routing entry written).  The reference's
    aether_route_top_k is timed on a bounded sample on the host cores and its
    ids are compared with the GPU's."""
    import torch

    from noel_b200 import sampler as S

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    T, E, K = (args.batch or 1048576), 64, 8
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn(T, E, device=dev, generator=g) * 3.0
    stream = torch.cuda.current_stream(dev)
    out = torch.empty(T, K, 2, dtype=torch.int32, device=dev)

    def step():
        S._check(S.lib().noel_moe_route_top_k(x.data_ptr(), T, E, E, K, out.data_ptr(),
                                              S.C.c_void_p(stream.cuda_stream)))

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if args.profile:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return
    clocks = ClockSampler(local if world > 1 else torch.cuda.current_device())
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t_ms = reduce_max(e0.elapsed_time(e1), world)
    value = T * world * args.steps / (t_ms / 1e3)
    k_ms = t_ms / args.steps
    peak, peak_kind = measured_peak()
    bytes_per_launch = T * E * 4 + T * K * 8
    achieved = bytes_per_launch / (k_ms / 1e3) / 1e9
    # end to end through the public Python API from pinned host memory
    h_x = x.cpu().pin_memory()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        ids, w = S.route_top_k(h_x.to(dev, non_blocking=True), K)
        ids.cpu(), w.cpu()
    e2e_s = reduce_max(time.perf_counter() - t0, world)
    cpu, parity = None, None
    if rank == 0 and not args.no_cpu:
        from oracle.oracle import RefAux

        if RefAux.available():
            n = min(T, 65536)
            xs = h_x[:n].numpy()
            ref = RefAux()
            ref.route_batch(xs[:1024], K)  # warm
            t0 = time.perf_counter()
            rid, _ = ref.route_batch(xs, K)
            rps = n / (time.perf_counter() - t0)
            step()
            torch.cuda.synchronize()
            gid = out[:n, :, 0].cpu().numpy()
            parity = {"tokens": n, "mismatches": int((gid != rid).any(axis=1).sum()),
                      "against": "the reference's src/sparsity.c built into oracle/_ref"}
            if parity["mismatches"]:
                print(json.dumps({"error": "parity", "parity": parity}), flush=True)
                sys.exit(1)
            cpu = {"value": rps, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"{n} tokens through aether_route_top_k, OpenMP over tokens"}
    if rank == 0:
        print(json.dumps({
            "metric": f"routed tokens/s, MoE router {E} experts top-{K} fp32", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "moe_router", "tokens_per_gpu": T, "experts": E, "top_k": K,
                       "parallelism": f"token-sharded x{world}",
                       "l2": f"no flush: {T * E * 4 / 1e6:.0f} MB of gate logits per step > 126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "kernel": "moe_route_kernel", "kernel_ms": k_ms,
                         "bytes_per_launch": bytes_per_launch, "peak_source": f"{peak_kind} hbm_gbs"},
            "cpu_baseline": cpu, "parity": parity,
            "e2e": {"value": T * world * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * E * 4,
                    "d2h_bytes_per_step": T * K * 8, "steps": e2e_steps,
                    "api": "noel_b200.sampler.route_top_k from pinned host logits"},
            "clocks": clk, "gpu_launches": args.steps,
        }), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_postreq(args):
    """The pipeline's sibling sampler (src/pipeline_stages.c:103-189).
    (1) The reference tool's own loop (tools/benchmark_cpu_offload.c:75-90:
    vocab 32,000, top-k 50, top-p 0.9, T 0.7; one host row, logits[0] = 12
    before each call, the row otherwise left as the previous call left it)
    through the drop-in noel_postreq_sample and through the reference's
    aether_postreq_sample on one host thread, from the same srand seed, id
    sequences compared; the tool's published figure is 98.81 us per token.
    (2) Batched: 1024 such rows resident on the GPU through
    noel_postreq_sample_batch (rows/s; each row read three times and written
    once by the kernel, 2 x 128 KB algorithmic)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch

    from noel_b200 import sampler as S
    from oracle.oracle import LIBC, PostreqParams, RefAux

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    V, K, P, T = 32000, 50, 0.9, 0.7
    g = np.random.Generator(np.random.PCG64(7))
    base = (g.random(V, dtype=np.float32) * 10.0).astype(np.float32)  # the tool's rand() / RAND_MAX * 10 row
    prm = S.postreq_params(T, P, K, 1.15, 2048, False)
    n = max(args.steps, 20) * 10
    row = base.copy()
    for _ in range(max(args.warmup, 3)):
        row[0] = 12.0
        S.postreq_sample(row, prm)
    row = base.copy()
    LIBC.srand(42)
    t0 = time.perf_counter()
    ids = []
    for _ in range(n):
        row[0] = 12.0
        ids.append(S.postreq_sample(row, prm))
    us = (time.perf_counter() - t0) / n * 1e6
    line = {"metric": "us per aether_postreq_sample call, vocab 32000, top-k 50, top-p 0.9, T 0.7 (the reference "
                      "tool's loop)", "value": us, "unit": "us/call", "higher_is_better": False, "calls": n,
            "dtype": "f32", "data": "synthetic", "published_reference_us": 98.81,
            "config": {"workload": "postreq_call", "vocab": V, "top_k": K, "top_p": P, "temperature": T}}
    if RefAux.available():
        ref = RefAux()
        rrow = base.copy()
        rp = PostreqParams(T, P, K, 1.15, 2048, False)
        LIBC.srand(42)
        t0 = time.perf_counter()
        rids = []
        for _ in range(n):
            rrow[0] = 12.0
            rids.append(ref.lib.aether_postreq_sample(rrow.ctypes.data_as(S.C.POINTER(S.C.c_float)), V,
                                                      S.C.byref(rp)))
        rus = (time.perf_counter() - t0) / n * 1e6
        line["reference"] = {"value": rus, "unit": "us/call", "cores": 1, "kind": "reference",
                             "sample": "src/pipeline_stages.c built into oracle/_ref, one thread, same loop"}
        line["parity"] = {"calls": n, "mismatches": int(sum(a != b for a, b in zip(ids, rids)))}
    print(json.dumps(line), flush=True)

    # batched, rows resident in HBM
    B = args.batch or 1024
    x0 = torch.from_numpy(np.tile(base, (B, 1))).to(dev)
    x0 += torch.randn(B, V, device=dev)  # distinct rows
    x = torch.empty_like(x0)
    u = torch.rand(B, device=dev)
    stream = torch.cuda.current_stream(dev)
    ids_d = torch.empty(B, dtype=torch.int32, device=dev)

    def step():
        S._check(S.lib().noel_postreq_sample_batch(S.C.byref(prm), x.data_ptr(), B, V, V, u.data_ptr(),
                                                   ids_d.data_ptr(), S.C.c_void_p(stream.cuda_stream)))

    for _ in range(max(args.warmup, 3)):
        x.copy_(x0)
        step()
    torch.cuda.synchronize()
    kt = []
    for _ in range(args.steps):
        x.copy_(x0)  # the kernel rewrites its rows: each step starts from the logits (outside the timed launch)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        torch.cuda.synchronize()
        kt.append(e0.elapsed_time(e1))
    k_ms = float(np.mean(kt))
    peak, peak_kind = measured_peak()
    bpl = B * V * 8
    print(json.dumps({
        "metric": f"sampled rows/s, aether_postreq_sample batch {B} x vocab {V}", "value": B / (k_ms / 1e3),
        "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "ms_per_step": k_ms, "higher_is_better": True,
        "dtype": "f32", "data": "synthetic", "config": {"workload": "postreq_batch", "batch": B, "vocab": V,
                                                        "top_k": K, "top_p": P, "temperature": T},
        "roofline": {"bound": "hbm", "achieved": bpl / (k_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": bpl / (k_ms / 1e3) / 1e9 / peak, "kernel": "postreq_sample_kernel",
                     "bytes_per_launch": bpl, "peak_source": f"{peak_kind} hbm_gbs"},
        "gpu_launches": args.steps}), flush=True)


def run_lmhead(args):
    """The LM head feeding the sampler (src/engine.c:377-387): bf16 output
    weights 152,064 x 4096 (1.25 GB, read from HBM every call), hidden states
    N(0, 1), the batch1024 sampling parameters, history NULL as the engine
    passes it; one token (the engine's decode step) and eight.  value =
    tokens/s through noel_lmhead_sample with inputs resident on the GPU; the
    roofline is the weights read once per call.  The reference (its own
    noel_gemv_quantized on the host cores, then noel_sampler_sample) is timed
    on one token and its logits and token compared with the GPU's."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import WORKLOADS, row_states

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    V, D = 152064, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    w = (torch.randn(V, D, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    cfgkw = WORKLOADS["batch1024"].config_kwargs()
    cfg = S.make_config(**cfgkw)
    peak, peak_kind = measured_peak()
    stream = torch.cuda.current_stream(dev)
    for B in (1, 8):
        x = torch.randn(B, D, device=dev, generator=g)
        rng = torch.from_numpy(row_states(3, np.arange(B)).view(np.int64).copy()).to(dev)
        logits = torch.empty(B, V, device=dev)
        ids = torch.empty(B, dtype=torch.int32, device=dev)

        def step():
            S._check(S.lib().noel_lmhead_sample(S.C.byref(cfg), w.data_ptr(), S.HEAD_BF16, D, x.data_ptr(), D, B, D,
                                                V, None, 0, 0, rng.data_ptr(), ids.data_ptr(), None,
                                                logits.data_ptr(), S.C.c_void_p(stream.cuda_stream)))

        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        wbytes = V * D * 2
        line = {"metric": f"tokens/s, LM head {V} x {D} bf16 + sampler, {B} token(s) per call",
                "value": B / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": args.steps,
                "higher_is_better": True, "dtype": "bf16 weights, f32 accumulate", "data": "synthetic",
                "config": {"workload": "lmhead", "batch": B, "hidden": D, "vocab": V, **cfgkw},
                "roofline": {"bound": "hbm", "achieved": wbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": wbytes / (ms / 1e3) / 1e9 / peak, "bytes_per_launch": wbytes,
                             "kernel": "lmhead_gemv_kernel + the sampler", "peak_source": f"{peak_kind} hbm_gbs"},
                "gpu_launches": 3 * args.steps}
        if B == 1 and not args.no_cpu:
            from oracle.oracle import RefAux, RefSampler, make_config

            if RefAux.available() and RefSampler.available():
                wh = w.view(torch.int16).cpu().numpy().view(np.uint16)
                xh = x.cpu().numpy()
                aux = RefAux()
                t0 = time.perf_counter()
                ref_logits = aux.gemv(wh, 30, xh)
                gemv_s = time.perf_counter() - t0
                rng0 = row_states(3, np.arange(1))
                t0 = time.perf_counter()
                rid = RefSampler().sample_batch(make_config(**cfgkw), ref_logits, rng=rng0, nthreads=1).ids
                samp_s = time.perf_counter() - t0
                # the GPU on the same token from the same state
                rng.copy_(torch.from_numpy(rng0.view(np.int64).copy()).to(dev))
                step()
                torch.cuda.synchronize()
                same = np.array_equal(logits.cpu().numpy().view(np.uint32), ref_logits.view(np.uint32))
                line["cpu_baseline"] = {"value": 1.0 / (gemv_s + samp_s), "unit": "tokens/s", "cores": os.cpu_count(),
                                        "kind": "reference",
                                        "sample": "one token: noel_gemv_quantized (BF16, all host threads) then "
                                                  "noel_sampler_sample (one thread)",
                                        "gemv_ms": gemv_s * 1e3, "sample_ms": samp_s * 1e3}
                line["parity"] = {"logits_bit_exact": bool(same), "ids_equal": bool(ids.cpu().numpy()[0] == rid[0])}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="batch1024")
    ap.add_argument("--cpu-rows", type=int, default=512)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile", action="store_true", help="only W + K steps, for ncu")
    ap.add_argument("--batch", type=int, default=0, help="rows per GPU instead of the workload's (profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "vocab_sharded":
        run_vocab_sharded(args)
    elif args.workload == "engine_call":
        run_engine_call(args)
    elif args.workload == "moe_router":
        run_router(args)
    elif args.workload == "postreq":
        run_postreq(args)
    elif args.workload == "lmhead":
        run_lmhead(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
