#!/usr/bin/env python
"""Flash-Born attention benchmark on B200: fwd+bwd TFLOP/s (BASELINE config C2 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|c1|c3|c4]

One step = one forward + backward of Born attention over one batch of synthetic inputs resident
in HBM (C2: B=8, H=16, N=2048, d=64, bf16, causal, per-head scale 8, eps 1e-12; Q, K, V from
torch seed 0, dO from seed 1, drawn in fp32 then cast).  The timed steps replay one captured
step (public-API forward + autograd backward) as a CUDA graph, so a small shard's device time is
not hidden behind the host's per-step Python work; ``eager_ms_per_step`` gives the eager figure
(``--eager`` times eagerly throughout).  With N GPUs (one process per GPU,
launched by torch.distributed.run) the one problem is split over the ranks (strong scaling):
every rank takes a rectangle of its (batch, head) units from sharding.plan_shards -- C2's 128
units become 64 / 32 / 16 per GPU at N = 2 / 4 / 8 (heads split), C3's 32 heads 4 per GPU at
N = 8 -- and runs it with no collective on the data path (the units are independent); value =
the problem's FLOPs / the slowest rank's device time.  ``--weak`` gives every rank a whole
problem of its own instead (weak scaling); the strong run also reports that figure under
``"weak_scaling"``.

FLOPs are algorithmic: 14 d per valid (query, key) pair (forward QK^T and PV, backward S
recompute, dP, dV, dK, dQ), elementwise work not counted.

With the default C2 workload the run also times C3 and C4 the same way (split over the ranks,
``--extra-steps`` steps each) and reports them under ``"workloads"``.

The same run then times the end-to-end data-parallel training step of the C5 GPT (d_model 1024,
6 layers, flash-Born attention, per-GPU batch 16 x 1024 tokens; NCCL gradient all-reduce across
the N ranks) and reports it under ``"gpt"`` in tokens/s (``--no-gpt`` skips it).

Rank 0 prints one JSON line.  ``--impl reference`` times the reference algorithm's CPU path
(the torch eager restatement in oracle/eager_torch.py, all host threads) on a bounded sample of
the same workload and prints the same line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

# A device-side delay (in SM clock cycles, ~0.5 ms) placed before a timed region so that the host
# has queued the timed launches when the region starts: the events then time device work, not
# the host's launch latency.
HEAD_START_CYCLES = 1_000_000

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    # name: (B, H, N, D, causal, description)
    "c1": (2, 4, 256, 64, True, "C1 B=2 H=4 N=256 d=64 causal (bf16 on GPU)"),
    "c2": (8, 16, 2048, 64, True, "C2 B=8 H=16 N=2048 d=64 causal bf16"),
    "c3": (1, 32, 16384, 128, True, "C3 B=1 H=32 N=16384 d=128 causal bf16, unit-norm*sqrt(d) Q/K"),
    "c4": (4, 16, 8192, 64, True, "C4 B=4 H=16 N=8192 d=64 doc-masked bf16 (geometric doc lengths, mean 512)"),
}


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant kernel,
# from an ncu capture of a named build: (bytes, source).  A static figure: a rebuilt kernel keeps
# reporting it until it is profiled again, which is why its source names the profiled build.
PROFILED_TRAFFIC = {
    ("c2", "bwd"): (294.6e6, "static: ncu capture of tc_bwd_kernel at C2, build b5a6055"),
    ("c2", "fwd"): (130.6e6, "static: ncu capture of tc_fwd_kernel at C2, build b5a6055"),
}


def profiled_traffic(workload: str, kernel: str):
    """(bytes per launch, source) of the dominant kernel from PROFILED_TRAFFIC, or (None, reason)."""
    return PROFILED_TRAFFIC.get((workload, kernel), (None, "not profiled for this workload"))


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def doc_ids_geometric(B: int, N: int, mean: float, seed: int) -> np.ndarray:
    """Per row: geometric document lengths (mean ``mean``, support >= 1) until N is covered."""
    rng = np.random.default_rng(seed)
    doc = np.zeros((B, N), dtype=np.int32)
    for b in range(B):
        t, d = 0, 0
        while t < N:
            L = int(rng.geometric(1.0 / mean))
            doc[b, t:t + L] = d
            t += L
            d += 1
    return doc


def valid_pairs(workload: str, B: int, H: int, N: int, doc: np.ndarray | None) -> int:
    if doc is None:
        return B * H * N * (N + 1) // 2
    total = 0
    for b in range(B):
        _, counts = np.unique(doc[b], return_counts=True)
        total += int(np.sum(counts.astype(np.int64) * (counts + 1) // 2))
    return total * H


def make_inputs(workload: str, rank: int):
    """CPU fp32 inputs of one rank's slice (rank 0 = the exact BASELINE recipe)."""
    B, H, N, D, causal, _ = WORKLOADS[workload]
    seed_qkv = {"c1": 0, "c2": 0, "c3": 2, "c4": 3}[workload] + 1000 * rank
    torch.manual_seed(seed_qkv)
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, H, N, D)
    v = torch.randn(B, H, N, D)
    if workload == "c3":
        q = q / q.norm(dim=-1, keepdim=True) * math.sqrt(D)
        k = k / k.norm(dim=-1, keepdim=True) * math.sqrt(D)
    torch.manual_seed(1 + 1000 * rank)
    do = torch.randn(B, H, N, D)
    doc = doc_ids_geometric(B, N, 512.0, 3 + 1000 * rank) if workload == "c4" else None
    scale = math.sqrt(D)  # the caller's head_scale init, sqrt(head_dim) (layers/attention.py:390,429)
    return q, k, v, do, doc, scale


class ClockSampler:
    """nvidia-smi samples (every 200 ms) of one GPU while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.rows.append([x.strip() for x in line.split(",")])

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for n, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [p for p in vis.split(",") if p.strip()]
    if parts and all(p.strip().isdigit() for p in parts) and local_rank < len(parts):
        return int(parts[local_rank])
    return local_rank


def gpu_local_cpus(gpu_index: int) -> set[int] | None:
    """The host CPUs NVML reports as local to a GPU (its NUMA node), or None when unknown."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:  # noqa: BLE001 -- no NVML, no GPU, no affinity support
        return None


def pinned_near_gpu(gpu_index: int, tensors):
    """Pinned host copies of ``tensors``, allocated by this thread while it runs on the GPU's
    local CPUs, so the pages sit on the GPU's NUMA node (a remote node halves the copy rate on
    multi-socket hosts); the thread's CPU set is restored afterwards."""
    cpus = gpu_local_cpus(gpu_index)
    old = os.sched_getaffinity(0) if cpus else None
    try:
        if cpus:
            os.sched_setaffinity(0, cpus)
        return [t.pin_memory() for t in tensors]
    finally:
        if old is not None:
            os.sched_setaffinity(0, old)


def cpu_eager_sample(workload: str, target_s: float, max_units: int | None = None):
    """Time the reference's CPU eager algorithm on whole (batch, head) units of the workload.

    Returns (flops_per_s, units, seconds, threads)."""
    from oracle.eager_torch import eager_unit_fwd_bwd

    B, H, N, D, causal, _ = WORKLOADS[workload]
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    gen = torch.Generator().manual_seed(0)
    doc = doc_ids_geometric(1, N, 512.0, 3)[0] if workload == "c4" else None
    doc_t = None if doc is None else torch.from_numpy(doc)
    pairs = valid_pairs(workload, 1, 1, N, None if doc is None else doc[None])
    flops_unit = 14 * D * pairs
    units, t0 = 0, time.perf_counter()
    while True:
        q, k, v, do = (torch.randn(N, D, generator=gen) for _ in range(4))
        eager_unit_fwd_bwd(q, k, v, do, math.sqrt(D), causal, 1e-12, 0, doc_t)
        units += 1
        el = time.perf_counter() - t0
        if el >= target_s or (max_units is not None and units >= max_units):
            break
    return flops_unit * units / el, units, el, threads, flops_unit


def run_reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return  # under torchrun rank 0 alone runs the CPU reference
    B, H, N, D, causal, desc = WORKLOADS[args.workload]
    # warm-up units, then K timed steps, each a bounded sample (whole (b,h) units)
    per_step_s = float(os.environ.get("FB_REF_STEP_SECONDS", "3.0"))
    for _ in range(max(1, min(args.warmup, 2))):
        cpu_eager_sample(args.workload, 0.0, max_units=1)
    rates, secs, units_total, flops_total = [], 0.0, 0, 0.0
    threads = 1
    flops_unit = 0
    for _ in range(args.steps):
        rate, units, el, threads, flops_unit = cpu_eager_sample(args.workload, per_step_s)
        rates.append(rate)
        secs += el
        units_total += units
        flops_total += rate * el
    value = flops_total / secs / 1e12
    line = {
        "impl": "reference",
        "metric": "born_attn_fwd_bwd_tflops",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True,
        "scaling": "weak" if args.weak else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": desc, "global_batch": B * world if args.weak else B, "seq_len": N, "heads": H,
                   "head_dim": D},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{units_total} whole (batch, head) units of {args.workload} (N={N}, d={D}), "
                                   f"{flops_unit / 1e9:.2f} GFLOP each, fp32, torch eager restatement of "
                                   "flash_born.py:681-690 + autograd, one unit at a time"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist

    from quantumdlblocks_b200 import flash_born_attention
    from quantumdlblocks_b200.kernels import flash_born as fbm
    from quantumdlblocks_b200.sharding import max_over_ranks

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    B, H, N, D, causal, desc = WORKLOADS[args.workload]
    split = world > 1 and not args.weak
    # strong scaling (default with N > 1 ranks): every rank takes its shard of the one BASELINE
    # problem (rank 0's inputs), a rectangle of (batch, head) units from sharding.plan_shards,
    # held contiguously on its GPU; weak scaling: every rank runs a whole problem of its own
    q_cpu, k_cpu, v_cpu, do_cpu, doc_np, scale_val = make_inputs(args.workload, 0 if split else rank)
    pairs_full = valid_pairs(args.workload, B, H, N, doc_np)
    shard = None
    if split:
        from quantumdlblocks_b200.sharding import plan_shards

        shard = plan_shards(B, H, N, world, is_causal=causal, doc_ids=doc_np)[rank]
        bs, hs = slice(shard.b0, shard.b1), slice(shard.h0, shard.h1)
        q_cpu, k_cpu, v_cpu, do_cpu = (x[bs, hs].contiguous() for x in (q_cpu, k_cpu, v_cpu, do_cpu))
        doc_np = None if doc_np is None else np.ascontiguousarray(doc_np[bs])
    Bl, Hl = q_cpu.shape[0], q_cpu.shape[1]
    bf = torch.bfloat16
    q = q_cpu.to(bf).to(dev).requires_grad_(True)
    k = k_cpu.to(bf).to(dev).requires_grad_(True)
    v = v_cpu.to(bf).to(dev).requires_grad_(True)
    do = do_cpu.to(bf).to(dev)
    doc = None if doc_np is None else torch.from_numpy(doc_np).to(dev)
    scale = torch.full((1, Hl, 1, 1), scale_val, device=dev, requires_grad=True)
    pairs = valid_pairs(args.workload, Bl, Hl, N, doc_np)  # this rank's valid pairs
    flops_step = 14.0 * D * pairs
    # FLOPs of the whole job per step: the one problem (split) or one problem per rank (weak)
    flops_job = 14.0 * D * pairs_full * (1 if split else world)

    launches = {"fwd": 0, "bwd": 0}

    def step(qq, kk, vv, dd):
        out = flash_born_attention(qq, kk, vv, scale, is_causal=causal, eps=1e-12, doc_ids=doc)
        launches["fwd"] = fbm.last_launch_count()
        grads = torch.autograd.grad(out, (qq, kk, vv, scale), dd)
        launches["bwd"] = fbm.last_launch_count()
        return out, grads

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    if args.mode == "prologue":
        run_prologue_mode(args, rank, flush, dev)
        return
    if args.mode == "families":
        run_families_mode(args, rank, flush, dev, flops_step)
        return
    if args.mode == "triton-reference":
        run_triton_reference_mode(args, rank, flush, dev, q, k, v, do, scale, doc, causal, flops_step)
        return
    if args.mode == "gpt":
        gpt = run_gpt(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(gpt), flush=True)
        return
    if args.mode != "step":
        run_kernel_mode(args, q, k, v, do, scale, doc, causal, flops_step, D, pairs, flush, rank, world, dev)
        return
    for _ in range(args.warmup):
        step(q, k, v, do)
    torch.cuda.synchronize()
    rc, site = fbm.device_status()
    if rc != 0:
        raise RuntimeError(f"device status {rc} (site {site}) after warm-up")

    # The timed steps replay one captured step (the public API's forward + autograd backward, the
    # same kernels and allocations as an eager step) as a CUDA graph: a small shard's step (C2 at
    # N = 8: ~75 us of device work) is shorter than the host's ~0.2 ms of Python, ctypes and
    # autograd work per step, which eager timing would measure instead.  The eager per-step time
    # is reported beside it.
    graph, graph_err = (None, "disabled by --eager") if args.eager else capture_step(lambda: step(q, k, v, do), dev)

    def timed_steps(n: int, use_graph: bool) -> float:
        ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        barrier()
        torch.cuda.synchronize()
        # A device-side delay ahead of the timed steps lets the host queue them up, so that short
        # runs (a few steps) time the device work rather than the host's first launches; it lies
        # outside every per-step event pair.
        torch.cuda._sleep(min(n, 200) * HEAD_START_CYCLES)
        for i in range(n):
            flush.zero_()  # L2 flush (256 MiB > 126 MB L2), outside the per-step events
            ev_s[i].record()
            if use_graph:
                graph.replay()
            else:
                step(q, k, v, do)
            ev_e[i].record()
        torch.cuda.synchronize()
        barrier()
        return float(sum(ev_s[i].elapsed_time(ev_e[i]) for i in range(n)))

    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    t_ms = timed_steps(args.steps, graph is not None)
    clocks = sampler.stop()
    eager_steps = max(3, min(args.steps, 50))
    if graph is not None:
        for _ in range(2):  # untimed: eager allocations after the graph's private pool was taken
            step(q, k, v, do)
        t_eager = timed_steps(eager_steps, False)
    else:
        t_eager = t_ms * eager_steps / args.steps
    gpu_launches = args.steps * (launches["fwd"] + launches["bwd"])

    # per-kernel timing of the forward and backward launches (C-ABI through the custom ops)
    sc_flat = scale.detach().reshape(-1).float().contiguous()
    qd, kd, vd = q.detach(), k.detach(), v.detach()
    reps = max(5, min(50, args.steps))
    t_fwd, t_bwd = 0.0, 0.0
    out_d, z_d = torch.ops.flashborn_b200.born_fwd(qd, kd, vd, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
    n_fwd_launch = fbm.last_launch_count()
    for _ in range(reps):
        flush.zero_()
        torch.cuda._sleep(HEAD_START_CYCLES)  # the host queues both launches before their events
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        out_d, z_d = torch.ops.flashborn_b200.born_fwd(qd, kd, vd, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
        a1.record()
        flush.zero_()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        torch.ops.flashborn_b200.born_bwd(do, qd, kd, vd, out_d, z_d, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
        b1.record()
        torch.cuda.synchronize()
        t_fwd += a0.elapsed_time(a1)
        t_bwd += b0.elapsed_time(b1)
    n_bwd_launch = fbm.last_launch_count()
    t_fwd /= reps
    t_bwd /= reps
    path_fwd = "tcgen05" if _path_is_tc(qd, False) else "general"
    path_bwd = "tcgen05" if _path_is_tc(qd, True) else "general"

    # End-to-end through the public API: every step copies its inputs from pinned host memory and
    # its output and gradients back to pinned host memory.  The copies run on their own streams
    # (the GPU's copy engines), pipelined across steps: step i+1's inputs stream in and step i-1's
    # results stream out while step i computes; every byte still crosses PCIe inside the timed
    # region, which ends when the last step's results are on the host.
    e2e_steps = max(3, min(args.steps, args.e2e_steps))
    gpu_index = physical_gpu_index(local_rank)
    hq, hk, hv, hdo = pinned_near_gpu(gpu_index, [x.to(bf) for x in (q_cpu, k_cpu, v_cpu, do_cpu)])
    h_out = [pinned_near_gpu(gpu_index, [torch.empty_like(hq) for _ in range(4)]) for _ in range(2)]
    slots = [[torch.empty(hq.shape, dtype=bf, device=dev) for _ in range(4)] for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def e2e_run(n_steps: int) -> None:
        slot_free = [None, None]    # compute finished reading a device slot's inputs
        in_ready = [None] * n_steps
        e0.record(comp)
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)

        def load(i):
            with torch.cuda.stream(s_in):
                if slot_free[i % 2] is not None:
                    s_in.wait_event(slot_free[i % 2])
                for dst, src in zip(slots[i % 2], (hq, hk, hv, hdo)):
                    dst.copy_(src, non_blocking=True)
                in_ready[i] = torch.cuda.Event()
                in_ready[i].record(s_in)

        load(0)
        for i in range(n_steps):
            if i + 1 < n_steps:
                load(i + 1)
            comp.wait_event(in_ready[i])
            xq, xk, xv, xd = slots[i % 2]
            out, (gq, gk, gv, _) = step(xq.detach().requires_grad_(True), xk.detach().requires_grad_(True),
                                        xv.detach().requires_grad_(True), xd)
            done = torch.cuda.Event()
            done.record(comp)
            slot_free[i % 2] = done
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for dst, src in zip(h_out[i % 2], (out, gq, gk, gv)):
                    src.record_stream(s_out)  # the allocator keeps it until this copy ends
                    dst.copy_(src, non_blocking=True)
        comp.wait_stream(s_out)
        e1.record(comp)

    e2e_run(2)  # untimed: first use of these buffer sizes in the caching allocator
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_run(e2e_steps)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    # whole-job bytes: each rank copies its own inputs in and its results out
    h2d = world * 4 * hq.numel() * hq.element_size()
    d2h = world * 4 * hq.numel() * hq.element_size()

    # a job takes as long as its slowest rank
    t_ms, e2e_ms, t_fwd, t_bwd, t_eager = max_over_ranks([t_ms, e2e_ms, t_fwd, t_bwd, t_eager], device=dev)

    peaks, peak_src = load_peaks()
    value = flops_job * args.steps / (t_ms / 1e3) / 1e12
    e2e_value = flops_job * e2e_steps / (e2e_ms / 1e3) / 1e12

    # with the strong split, weak scaling as an extra figure: every rank runs a whole problem of
    # its own (seeds offset by rank), same step, same timing rule
    weak = None
    if split:
        wq, wk, wv, wdo, wdoc_np, _ = make_inputs(args.workload, rank)
        wq, wk, wv = (x.to(bf).to(dev).requires_grad_(True) for x in (wq, wk, wv))
        wdo = wdo.to(bf).to(dev)
        wdoc = None if wdoc_np is None else torch.from_numpy(wdoc_np).to(dev)
        wscale = torch.full((1, H, 1, 1), scale_val, device=dev, requires_grad=True)

        def wstep():
            o = flash_born_attention(wq, wk, wv, wscale, is_causal=causal, eps=1e-12, doc_ids=wdoc)
            torch.autograd.grad(o, (wq, wk, wv, wscale), wdo)

        for _ in range(args.warmup):
            wstep()
        wev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(min(args.steps, 200) * HEAD_START_CYCLES)
        for i in range(args.steps):
            flush.zero_()
            wev[i][0].record()
            wstep()
            wev[i][1].record()
        torch.cuda.synchronize()
        (w_ms,) = max_over_ranks([sum(a.elapsed_time(b) for a, b in wev)], device=dev)
        w_flops = torch.tensor([14.0 * D * valid_pairs(args.workload, B, H, N, wdoc_np)], dtype=torch.float64,
                               device=dev)
        dist.all_reduce(w_flops)  # every rank's problem counts (document masks differ per rank)
        weak = {"value": float(w_flops.item()) * args.steps / (w_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": w_ms / args.steps, "scaling": "weak",
                "what": f"every rank runs a whole {args.workload} problem of its own (global batch {B * world})"}
        del wq, wk, wv, wdo
    flops_fwd = 4.0 * D * pairs
    flops_bwd = 10.0 * D * pairs
    dominant = "bwd" if t_bwd >= t_fwd else "fwd"
    dom_flops, dom_ms = (flops_bwd, t_bwd) if dominant == "bwd" else (flops_fwd, t_fwd)
    achieved = dom_flops / (dom_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic, traffic_src = profiled_traffic(args.workload, dominant)

    others = None
    if args.workload == "c2" and not args.weak and args.extra_steps > 0:
        others = {w: run_other_workload(args, w, rank, world, dev, flush, peaks) for w in ("c3", "c4")}

    gpt = None if args.no_gpt else run_gpt(args, rank, world, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, units, el, threads, flops_unit = cpu_eager_sample(args.workload, args.cpu_seconds)
        cpu = {"value": rate / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{units} whole (batch, head) units of {args.workload} (N={N}, d={D}) in {el:.1f} s, "
                         "fp32, torch eager restatement of flash_born.py:681-690 + autograd"}

    if rank == 0:
        line = {
            "metric": "born_attn_fwd_bwd_tflops",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": t_ms / args.steps,
            "eager_ms_per_step": t_eager / eager_steps,
            "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": desc, "global_batch": B if split else B * world, "seq_len": N, "heads": H,
                       "head_dim": D,
                       "parallelism": (f"(batch, head) units split over {world} ranks, rank 0 holds batch "
                                       f"[{shard.b0},{shard.b1}) x heads [{shard.h0},{shard.h1}) = {shard.units} "
                                       "units; no collective" if split else
                                       f"{world} rank(s), one whole problem each, no collective"),
                       "flops_per_step_per_rank": flops_step,
                       "flops_per_step_job": flops_job,
                       "l2": "flushed before every step (256 MiB write); per-step CUDA events exclude the flush",
                       "timing": ("CUDA-graph replays of one captured step (public-API forward + autograd backward); "
                                  "eager_ms_per_step: the same step launched eagerly" if graph is not None else
                                  f"eager steps (graph capture unavailable: {graph_err or 'disabled by --eager'})")},
            "weak_scaling": weak,
            "per_gpu_tflops": value / world,
            "pct_of_bf16_peak_sustained": 100.0 * value / world / float(
                peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])),
            "roofline": {"bound": "tensor", "kernel": f"{dominant} ({path_bwd if dominant == 'bwd' else path_fwd})",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"bf16_tflops (burst) of {peak_src}",
                         "traffic": traffic if world == 1 else None,
                         "traffic_source": ("dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant "
                                            "kernel, " + traffic_src) if world == 1 else "not profiled for a shard",
                         "fwd_ms": t_fwd, "bwd_ms": t_bwd, "fwd_launches": n_fwd_launch,
                         "bwd_launches": n_bwd_launch,
                         "fwd_tflops": flops_fwd / (t_fwd / 1e3) / 1e12,
                         "bwd_tflops": flops_bwd / (t_bwd / 1e3) / 1e12},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "api": "quantumdlblocks_b200.flash_born_attention + autograd",
                    "copies": "pinned host buffers; H2D and D2H on two copy streams, pipelined across steps"},
            "gpu_launches": gpu_launches,
            "cpu_baseline": cpu,
            "workloads": others,
            "gpt": gpt,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def capture_step(fn, dev: torch.device):
    """(graph, None) with ``fn`` captured as a CUDA graph after two warm-up calls on a side stream
    and one checked replay, or (None, reason) when capture fails."""
    from quantumdlblocks_b200.kernels import flash_born as fbm

    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        rc, site = fbm.device_status()
        if rc != 0:
            raise RuntimeError(f"device status {rc} (site {site}) after the graph's first replay")
        return graph, None
    except Exception as exc:  # noqa: BLE001 -- report it and time eagerly
        return None, f"{type(exc).__name__}: {str(exc)[:160]}"


def run_other_workload(args, workload: str, rank: int, world: int, dev: torch.device, flush: torch.Tensor,
                       peaks: dict) -> dict:
    """C3 or C4 timed inside the default run, split over the ranks like the headline problem
    (C3: 32 heads, 4 per GPU at N = 8; C4: heads split): ``--extra-steps`` fwd+bwd steps after two
    warm-up steps, L2 flushed before each, CUDA events on this rank's stream, max over ranks;
    then the forward and backward launches timed separately (C-ABI through the custom ops)."""
    import torch.distributed as dist

    from quantumdlblocks_b200 import flash_born_attention
    from quantumdlblocks_b200.kernels import flash_born as fbm
    from quantumdlblocks_b200.sharding import max_over_ranks, plan_shards

    B, H, N, D, causal, desc = WORKLOADS[workload]
    q_cpu, k_cpu, v_cpu, do_cpu, doc_np, scale_val = make_inputs(workload, 0)
    pairs_full = valid_pairs(workload, B, H, N, doc_np)
    shard = plan_shards(B, H, N, world, is_causal=causal, doc_ids=doc_np)[rank]
    bs, hs = slice(shard.b0, shard.b1), slice(shard.h0, shard.h1)
    bf = torch.bfloat16
    q, k, v = (x[bs, hs].to(bf).to(dev).requires_grad_(True) for x in (q_cpu, k_cpu, v_cpu))
    do = do_cpu[bs, hs].to(bf).to(dev)
    del q_cpu, k_cpu, v_cpu, do_cpu
    doc = None if doc_np is None else torch.from_numpy(np.ascontiguousarray(doc_np[bs])).to(dev)
    Hl = q.shape[1]
    scale = torch.full((1, Hl, 1, 1), scale_val, device=dev, requires_grad=True)
    pairs = valid_pairs(workload, q.shape[0], Hl, N, None if doc_np is None else doc_np[bs])

    def step():
        out = flash_born_attention(q, k, v, scale, is_causal=causal, eps=1e-12, doc_ids=doc)
        torch.autograd.grad(out, (q, k, v, scale), do)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    graph, graph_err = (None, "disabled by --eager") if args.eager else capture_step(step, dev)
    if world > 1:
        dist.barrier()
    steps = args.extra_steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda._sleep(steps * HEAD_START_CYCLES)
    for i in range(steps):
        flush.zero_()
        ev[i][0].record()
        if graph is not None:
            graph.replay()
        else:
            step()
        ev[i][1].record()
    torch.cuda.synchronize()
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    sc_flat = scale.detach().reshape(-1).float().contiguous()
    qd, kd, vd = q.detach(), k.detach(), v.detach()
    t_fwd = t_bwd = 0.0
    for _ in range(3):
        flush.zero_()
        torch.cuda._sleep(HEAD_START_CYCLES)
        a0, a1, b0, b1 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
        a0.record()
        out_d, z_d = torch.ops.flashborn_b200.born_fwd(qd, kd, vd, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
        a1.record()
        flush.zero_()
        b0.record()
        torch.ops.flashborn_b200.born_bwd(do, qd, kd, vd, out_d, z_d, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
        b1.record()
        torch.cuda.synchronize()
        t_fwd += a0.elapsed_time(a1) / 3
        t_bwd += b0.elapsed_time(b1) / 3
    rc, site = fbm.device_status()
    if rc != 0:
        raise RuntimeError(f"device status {rc} (site {site}) in {workload}")
    t_ms, t_fwd, t_bwd = max_over_ranks([t_ms, t_fwd, t_bwd], device=dev)
    value = 14.0 * D * pairs_full * steps / (t_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    bwd_tf = 10.0 * D * pairs / (t_bwd / 1e3) / 1e12  # this rank's shard (the slowest rank's time)
    res = {"metric": "born_attn_fwd_bwd_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
           "per_gpu_tflops": value / world, "ms_per_step": t_ms / steps, "steps": steps, "warmup": 2,
           "scaling": "strong",
           "config": {"workload": desc, "seq_len": N, "heads": H, "head_dim": D,
                      "parallelism": f"(batch, head) units split over {world} ranks, rank 0 holds batch "
                                     f"[{shard.b0},{shard.b1}) x heads [{shard.h0},{shard.h1}); no collective",
                      "flops_per_step_job": 14.0 * D * pairs_full,
                      "l2": "flushed before every step (256 MiB write); per-step CUDA events exclude the flush",
                      "timing": "CUDA-graph replays of one captured step" if graph is not None else
                                f"eager steps ({graph_err})"},
           "fwd_ms": t_fwd, "bwd_ms": t_bwd, "bwd_tflops_per_gpu": bwd_tf, "bwd_frac": bwd_tf / peak,
           "peak_source": "bf16_tflops (burst), measured"}
    del q, k, v, do, doc, scale, qd, kd, vd, out_d, z_d, graph
    torch.cuda.empty_cache()
    return res


def run_gpt(args, rank: int, world: int, dev: torch.device) -> dict:
    """C5: data-parallel training step of the d_model 1024, 6-layer, 16 x 64-head flash-Born GPT
    (vocab 50,257, 127 M parameters, random init from seed 0, bf16 autocast, AdamW), per-GPU batch
    16 x 1024 tokens of Zipf(1.1) ids.  Every step copies its tokens from pinned host memory, runs
    forward + backward + optimiser step; with N > 1 ranks DistributedDataParallel all-reduces the
    gradients over NCCL in buckets during the backward.  Timed with CUDA events, max over ranks."""
    from quantumdlblocks_b200.gpt import BornGPT, GPTConfig, make_ddp, param_count, train_step, zipf_tokens
    from quantumdlblocks_b200.kernels import flash_born as fbm
    from quantumdlblocks_b200.sharding import max_over_ranks

    cfg = GPTConfig()
    batch = args.gpt_batch
    torch.manual_seed(0)
    model = BornGPT(cfg).to(dev)
    n_params = param_count(model)
    net = make_ddp(model, dev) if world > 1 else model
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    n_batches = 4
    host = [torch.from_numpy(zipf_tokens(batch, cfg.seq_len, cfg.vocab_size, seed=1000 * rank + i)).pin_memory()
            for i in range(n_batches)]
    launches = {"n": 0}

    def step(i):
        tok = host[i % n_batches].to(dev, non_blocking=True)
        loss = train_step(net, opt, tok)
        return loss

    for i in range(args.gpt_warmup):
        step(i)
    torch.cuda.synchronize()
    losses = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.gpt_steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for i in range(args.gpt_steps):
        ev[i][0].record()
        losses.append(step(i))
        ev[i][1].record()
    torch.cuda.synchronize()
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    (t_ms,) = max_over_ranks([t_ms], device=dev)
    rc, site = fbm.device_status()
    if rc != 0:
        raise RuntimeError(f"device status {rc} (site {site}) in the GPT step")
    tokens = world * batch * cfg.seq_len * args.gpt_steps
    attn_flops = 14.0 * (cfg.d_model // cfg.n_heads) * cfg.seq_len * (cfg.seq_len + 1) / 2 * cfg.n_heads * cfg.n_layers
    dense_flops = 6.0 * n_params  # per token: every weight (the tied head included) in 3 GEMMs
    res = {
        "metric": "gpt_train_tokens_per_s", "value": tokens / (t_ms / 1e3), "unit": "tokens/s",
        "per_gpu": tokens / world / (t_ms / 1e3), "ms_per_step": t_ms / args.gpt_steps, "steps": args.gpt_steps,
        "warmup": args.gpt_warmup, "n_gpus": world,
        "config": {"workload": "C5 d_model=1024 L=6 H=16x64 seq=1024 vocab=50257 tied, flash-Born attention, "
                               "bf16 autocast, AdamW", "per_gpu_batch": batch, "params": n_params,
                   "data": "synthetic Zipf(1.1) token ids, host-pinned, copied every step",
                   "allreduce": (f"NCCL via DistributedDataParallel, 25 MB buckets overlapped with the backward, "
                                 f"{world} ranks") if world > 1 else "none (1 rank)"},
        "model_tflops_per_gpu": (dense_flops * batch * cfg.seq_len + attn_flops * batch) * args.gpt_steps
                                 / (t_ms / 1e3) / 1e12,
        "loss_first_last": [float(losses[0]), float(losses[-1])],
        "h2d_bytes_per_step": batch * (cfg.seq_len + 1) * 8,
    }
    del net, model, opt
    torch.cuda.empty_cache()
    return res


def run_prologue_mode(args, rank: int, flush: torch.Tensor, dev: torch.device) -> None:
    """--mode prologue: the attention layer's fused operand prologue at the C5 layer shape
    (B=16, T=1024, 16 heads x 64, bf16 projection, fp32 residual stream): qkv_prologue forward and
    backward and the row L2 normalisation forward and backward, and the GPT loss (fused
    cross-entropy over 16,384 x 50,304 bf16 logits) forward and backward, the head epilogue (gated
    XSA, output gate, head merge) forward and forward + backward, each timed with CUDA
    events after an L2 flush, against the HBM roofline (algorithmic bytes: every input element read
    once, every output element written once)."""
    from quantumdlblocks_b200.kernels import flash_born as fbm
    from quantumdlblocks_b200.kernels.prologue import (_l2norm_rows, _l2norm_rows_bwd, _qkv_prologue,
                                                       _qkv_prologue_bwd, rope_tables)

    B, T, H, hd = 16, 1024, 16, 64
    D = H * hd
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(B, T, 3 * D, generator=g, device=dev).to(torch.bfloat16)
    cos, sin = rope_tables(T, hd, device=dev)
    dq, dk, dv = (torch.randn(B, H, T, hd, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    x = torch.randn(B, T, D, generator=g, device=dev)
    dy = torch.randn(B, T, D, generator=g, device=dev)
    n = qkv.numel()
    cases = {
        "qkv_prologue_fwd": (lambda: _qkv_prologue(qkv, cos, sin, H, 1e-12), 2 * n * 2),
        "qkv_prologue_bwd": (lambda: _qkv_prologue_bwd(qkv, cos, sin, dq, dk, dv, H, 1e-12), (n * 2 // 3 + 2 * n) * 2),
        "l2norm_rows_fwd": (lambda: _l2norm_rows(x, 1e-12), 2 * x.numel() * 4),
        "l2norm_rows_bwd": (lambda: _l2norm_rows_bwd(x, dy, 1e-12), 3 * x.numel() * 4),
    }
    # the GPT loss at the C5 shape: 16,384 rows of 50,304 bf16 logits (fwd reads them once; bwd
    # reads them and writes the gradient), through the C ABI with preallocated buffers
    import ctypes

    from quantumdlblocks_b200 import _lib

    rows, vocab = B * T, 50304
    logits = torch.randn(rows, vocab, generator=g, device=dev).to(torch.bfloat16)
    tgt = torch.randint(0, 50257, (rows,), generator=g, device=dev)
    lse, loss = (torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(2))
    dlog = torch.empty_like(logits)
    gs = torch.ones(1, dtype=torch.float32, device=dev)
    xa = _lib.FbXentArgs()
    xa.rows, xa.vocab, xa.ld = rows, vocab, vocab
    xa.logits, xa.targets, xa.lse, xa.loss = logits.data_ptr(), tgt.data_ptr(), lse.data_ptr(), loss.data_ptr()
    xa.grad, xa.gscale = dlog.data_ptr(), gs.data_ptr()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    cases["xent_fwd"] = (lambda: _lib.check(lib.fb_xent_fwd(ctypes.byref(xa), stream), "xent"), rows * vocab * 2)
    cases["xent_bwd"] = (lambda: _lib.check(lib.fb_xent_bwd(ctypes.byref(xa), stream), "xent"), rows * vocab * 4)
    # the layer's head epilogue (gated XSA + output gate + head merge) at the C5 layer shape
    from quantumdlblocks_b200.kernels.epilogue import finalize_heads

    eo = dq.detach().clone().requires_grad_(True)
    ev = dk.detach().clone().requires_grad_(True)
    ea = torch.zeros(H, device=dev).requires_grad_(True)
    ex = x.detach().clone().requires_grad_(True)
    ew, eb = torch.zeros(H, 6, device=dev).requires_grad_(True), torch.zeros(H, device=dev).requires_grad_(True)
    edy = torch.randn(B, T, D, generator=g, device=dev).to(torch.bfloat16)
    hb = eo.numel() * 2

    def epi_fwd():
        with torch.no_grad():
            finalize_heads(eo, ev, ea, ex, ew, eb)

    def epi_step():
        torch.autograd.grad(finalize_heads(eo, ev, ea, ex, ew, eb), (eo, ev, ea, ex, ew, eb), edy)

    cases["heads_epilogue_fwd"] = (epi_fwd, 3 * hb)  # read O, V; write Y
    cases["heads_epilogue_fwd_bwd"] = (epi_step, 3 * hb + 5 * hb)  # + read dY, O, V; write dO, dV
    peaks, src = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    res = {}
    for name, (fn, nbytes) in cases.items():
        for _ in range(args.warmup):
            fn()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(HEAD_START_CYCLES)  # the host queues the launch before the timed region
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            fn()
            a1.record()
            torch.cuda.synchronize()
            total += a0.elapsed_time(a1)
        us = 1e3 * total / args.steps
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us": us, "bytes": nbytes, "gbs": gbs, "frac_hbm": gbs / hbm}
    rc, _ = fbm.device_status()
    if rank == 0:
        print(json.dumps({"mode": "prologue", "shape": {"B": B, "T": T, "heads": H, "head_dim": hd},
                          "hbm_peak_gbs": hbm, "peak_source": f"hbm_gbs of {src}", "kernels": res,
                          "device_status": rc}), flush=True)


def run_families_mode(args, rank: int, flush: torch.Tensor, dev: torch.device, flops_plain: float) -> None:
    """--mode families: complex-phase and paired-heads Born attention, forward + backward through
    the public API at the C2 shape (B=8, H=16, N=2048, d=64, causal, bf16, unit-norm Q and K as
    the layer passes them).  Each family is two plain terms' worth of work (complex: (q, k) and
    (q, rot k) over all heads; paired: four head-half terms over H/2 heads), so its algorithmic
    FLOPs are 2 x the plain C2 step's; timed with CUDA events after an L2 flush."""
    from quantumdlblocks_b200 import complex_phase_born_attention, paired_heads_born_attention
    from quantumdlblocks_b200.kernels import flash_born as fbm

    B, H, N, D = 8, 16, 2048, 64
    g = torch.Generator(device=dev).manual_seed(0)
    q, k = (torch.nn.functional.normalize(torch.randn(B, H, N, D, generator=g, device=dev), dim=-1) for _ in range(2))
    v = torch.randn(B, H, N, D, generator=g, device=dev)
    q, k, v = (x.to(torch.bfloat16).requires_grad_(True) for x in (q, k, v))
    do = torch.randn(B, H, N, D, generator=g, device=dev).to(torch.bfloat16)
    cases = {
        "complex_phase": (complex_phase_born_attention, torch.full((1, H, 1, 1), 8.0, device=dev)),
        "paired_heads": (paired_heads_born_attention, torch.full((1, H // 2, 1, 1), 8.0, device=dev)),
    }
    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    res = {}
    for name, (fn, sc) in cases.items():
        sc = sc.requires_grad_(True)

        def step():
            out = fn(q, k, v, sc, is_causal=True, eps=1e-12)
            return torch.autograd.grad(out, (q, k, v, sc), do)

        for _ in range(args.warmup):
            step()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(16 * HEAD_START_CYCLES)  # the host queues the step before the timed region
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            step()
            a1.record()
            torch.cuda.synchronize()
            total += a0.elapsed_time(a1)
        ms = total / args.steps
        tf = 2.0 * flops_plain / (ms / 1e3) / 1e12
        res[name] = {"ms": ms, "flops": 2.0 * flops_plain, "tflops": tf, "frac_bf16_peak": tf / peak}
    rc, _ = fbm.device_status()
    if rank == 0:
        print(json.dumps({"mode": "families", "shape": {"B": B, "H": H, "N": N, "D": D, "causal": True},
                          "peak_tflops": peak, "peak_source": f"bf16_tflops (burst) of {src}", "families": res,
                          "device_status": rc}), flush=True)


def run_triton_reference_mode(args, rank, flush, dev, q, k, v, do, scale, doc, causal, flops_step) -> None:
    """--mode triton-reference: the reference's own GPU path -- ``flash_born_attention`` of
    qdlblocks (``kernels/flash_born.py:655-690``, Triton kernels ``:80-430``), unmodified, imported
    from ``baseline/_ref`` -- forward + backward on this GPU at the workload's shape and inputs,
    timed like the benchmark step (L2 flushed, CUDA events).  The bar on a B200 is that code
    JIT-compiled for it.  The same inputs then run through this package's op and the two results
    are compared (max-rel), so the figure is known to be of the same computation."""
    from quantumdlblocks_b200 import flash_born_attention

    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "qdlblocks")):
        if rank == 0:
            print(json.dumps({"mode": "triton-reference", "unavailable": "baseline/_ref holds no qdlblocks package"}))
        return
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import warnings

    warnings.filterwarnings("ignore")
    from qdlblocks.kernels.flash_born import HAS_TRITON
    from qdlblocks.kernels.flash_born import flash_born_attention as ref_attention

    def grads(fn):
        out = fn(q, k, v, scale, is_causal=causal, eps=1e-12, doc_ids=doc)
        return (out, *torch.autograd.grad(out, (q, k, v, scale), do))

    t0 = time.perf_counter()
    grads(ref_attention)  # first call: Triton compiles its kernels for this GPU
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    for _ in range(args.warmup):
        grads(ref_attention)
    total = 0.0
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(16 * HEAD_START_CYCLES)  # the host queues the step before the timed region
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        grads(ref_attention)
        a1.record()
        torch.cuda.synchronize()
        total += a0.elapsed_time(a1)
    ms = total / args.steps
    ref = grads(ref_attention)
    ours = grads(flash_born_attention)
    names = ("out", "dq", "dk", "dv")
    diff = {n: float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30))
            for n, a, b in zip(names, ours[:4], ref[:4])}
    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    tf = flops_step / (ms / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({"mode": "triton-reference", "workload": args.workload, "has_triton": bool(HAS_TRITON),
                          "ms_per_step": ms, "tflops": tf, "frac_bf16_peak": tf / peak,
                          "peak_source": f"bf16_tflops (burst) of {src}", "first_call_s": compile_s,
                          "max_rel_ours_vs_reference": diff,
                          "what": "qdlblocks flash_born_attention (Triton) fwd + autograd bwd, unmodified, "
                                  "from baseline/_ref"}), flush=True)


def run_kernel_mode(args, q, k, v, do, scale, doc, causal, flops_step, D, pairs, flush, rank, world, dev) -> None:
    """--mode fwd|bwd: launch only the forward or only the backward kernels through the custom
    ops (one C-ABI call per step), W warm-up + K timed launches, for profilers and kernel timing."""
    from quantumdlblocks_b200.kernels import flash_born as fbm

    sc_flat = scale.detach().reshape(-1).float().contiguous()
    qd, kd, vd = q.detach(), k.detach(), v.detach()
    fwd = torch.ops.flashborn_b200.born_fwd
    bwd = torch.ops.flashborn_b200.born_bwd
    out_d, z_d = fwd(qd, kd, vd, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)

    def one():
        if args.mode == "fwd":
            fwd(qd, kd, vd, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)
        else:
            bwd(do, qd, kd, vd, out_d, z_d, sc_flat, None, doc, causal, 1e-12, 0, 0.0, False)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(HEAD_START_CYCLES)  # the host queues the launch before the timed region
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one()
        e1.record()
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    ms = total / args.steps
    flops = (4.0 if args.mode == "fwd" else 10.0) * D * pairs
    rc, site = fbm.device_status()
    if rank == 0:
        print(json.dumps({"mode": args.mode, "workload": args.workload, "ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
                          "launches": fbm.last_launch_count(), "device_status": rc}), flush=True)


def _path_is_tc(q: torch.Tensor, backward: bool) -> bool:
    import ctypes

    from quantumdlblocks_b200 import _lib

    a = _lib.FbAttnArgs()
    B, H, T, D = q.shape
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, T, D
    a.dtype = a.out_dtype = _lib.FB_BF16
    a.is_causal = 1
    a.scale, a.scale_numel = 1, 1
    for n in ("q", "k", "v", "out", "dout", "dq", "dk", "dv"):
        setattr(a, n + "_stride", _lib._I64x4(*q.stride()))
    return _lib.load().fb_select_path(ctypes.byref(a), int(backward)) == _lib.FB_PATH_TCGEN05


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--weak", action="store_true",
                    help="with N > 1: every rank runs a whole problem (weak scaling) instead of its shard of one")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpt", action="store_true", help="skip the C5 GPT training-step measurement")
    ap.add_argument("--eager", action="store_true", help="time the steps eagerly instead of as CUDA-graph replays")
    ap.add_argument("--extra-steps", type=int, default=5,
                    help="steps of C3 and C4 timed in the default C2 run (0 skips them)")
    ap.add_argument("--gpt-steps", type=int, default=10)
    ap.add_argument("--gpt-warmup", type=int, default=3)
    ap.add_argument("--gpt-batch", type=int, default=16)
    ap.add_argument("--mode", choices=["step", "fwd", "bwd", "prologue", "families", "gpt", "triton-reference"],
                    default="step",
                    help="step: the benchmark (fwd+bwd); fwd / bwd: one kernel family only (profiling); "
                         "prologue: the attention layer's fused operand kernels at the C5 shape; "
                         "families: complex-phase and paired-heads attention at the C2 shape; "
                         "gpt: only the C5 GPT training step; triton-reference: the reference's own Triton "
                         "kernels (baseline/_ref) on this GPU, same inputs")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
