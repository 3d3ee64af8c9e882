"""Benchmark: attention fwd and fwd+bwd TFLOP/s (fp16, head_dim 64) on 1..8 B200s.

One step = one forward + backward of ``tattn.attention`` over one batch (BASELINE config 2 per GPU:
fp16, B4 H16 N4096 D64, non-causal; ``--config cfg3`` / ``cfg5`` select the causal long-context and
the scaling configs). Multi-GPU runs shard (batch, head) pairs across ranks with no collective on the
hot path (weak scaling: every rank runs the config-2 batch); each rank times on the device with CUDA
events, rank 0 reports the max over ranks. FLOPs follow the reference (bench/bench.py:31-35):
4*B*H*N^2*D, halved when causal, x3.5 for fwd+bwd.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2|cfg3|cfg5] [--impl reference]

``--impl reference`` times the reference's CPU path (the oracle restatement of
src/tattn/reference.py's tiled_forward/tiled_backward) on the host cores, on a bounded sample of the
same workload, and prints the same JSON line with "impl": "reference".

``--compare`` (one GPU) prints one JSON line per implementation and config, in the spirit of the
reference's bench/bench.py comparison table (bench.py:62-76, 128-171): this library, torch's
scaled_dot_product_attention with each backend (flash, cuDNN, memory-efficient) and a naive
materialised softmax, each with fwd and fwd+bwd TFLOP/s, peak extra memory and the max-abs error of O
and the gradients against an fp32 definition on two (b, h) pairs. The other implementations are
library kernels shown for context only; they are not part of this library's path.
"""

from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "triton-attn_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "attention fwd and fwd+bwd TFLOP/s (fp16, hd64) at 1/2/4/8 B200 vs fp16 peak"
CONFIGS = {
    # name: (batch per GPU, heads, seq, head_dim, causal)
    "cfg2": (4, 16, 4096, 64, False),
    "cfg3": (1, 16, 16384, 64, True),
    "cfg5": (64, 16, 8192, 64, True),  # scaling config: (batch, head) pairs split over the ranks
}
T4_PUBLISHED = {"cfg2": 16.9, "cfg3": 15.9}  # the reference's published fwd+bwd TFLOP/s on a T4 (results/t4.json)
L2_BYTES = 126 * 2**20
# DRAM bytes (read + write) of one launch of the dominant kernel, from the committed ncu capture
# profiles/bwd_dkdv_cfg2.md (dram__bytes_read.sum + dram__bytes_write.sum); None for other configs.
NCU_TRAFFIC = {("cfg2", "dkdv"): 136_370_176 + 43_040_000, ("cfg2", "bwd_fused"): 203_631_872 + 92_393_472}


def flops(b: int, h: int, n: int, d: int, causal: bool, mode: str) -> float:
    f = 4.0 * b * h * n * n * d
    if causal:
        f /= 2
    return f * (3.5 if mode == "fwd+bwd" else 1.0)


def shard(pairs: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous (batch, head) pair range [lo, hi) of `rank`: pairs are independent in the forward
    and the backward, so ranks need no data exchange; sizes differ by at most one pair."""
    return pairs * rank // world, pairs * (rank + 1) // world


def max_over_ranks(ms: float, device=None) -> float:
    """Device time of the slowest rank (MAX all-reduce of one scalar, outside the timed region)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return ms
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"tflops": p["bf16_tflops"], "tflops_sustained": p.get("bf16_tflops_sustained"),
                "hbm_gbs": p["hbm_gbs"], "source": "measured"}  # fmt: skip
    return {"tflops": 1590.0, "tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


# ------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle samples every 50 ms while the timed region runs. Entering waits
    (at most 5 s, before the region starts) for the first sample, since nvidia-smi takes longer to
    start than a short timed region lasts; leaving waits (at most 0.3 s) for one more sample if none
    arrived during the region. Only samples from the region's start on are summarised."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")  # fmt: skip

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []
        self.first = 0
        self._t: threading.Thread | None = None

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )  # fmt: skip
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t0 = time.monotonic()
            while not self.lines and self.proc.poll() is None and time.monotonic() - t0 < 5.0:
                time.sleep(0.005)
            self.first = len(self.lines)
        except OSError:
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            t0 = time.monotonic()
            while len(self.lines) <= self.first and self.proc.poll() is None and time.monotonic() - t0 < 0.3:
                time.sleep(0.002)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._t is not None:
                self._t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons, power = [], None, set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines[self.first:]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}  # fmt: skip


# ------------------------------------------------------------------------------------------- CPU
def _cpu_worker(args: tuple) -> tuple:
    """Time the oracle's tiled forward+backward on (b, h) pairs [lo, hi), once with `blocks` and once
    with 2*`blocks` outer blocks: (fwd_1, bwd_1, fwd_2, bwd_2) seconds."""
    import numpy as np

    from oracle import tiled_backward, tiled_forward

    (b_h, n, d, causal, lo, hi, blocks, seed) = args
    rng = np.random.default_rng(seed + lo)
    shape = (hi - lo, n, d)
    q, k, v, do = (rng.standard_normal(shape).astype(np.float16) for _ in range(4))
    out = []
    for nb in (blocks, 2 * blocks):
        t0 = time.perf_counter()
        o, m = tiled_forward(q, k, v, causal, row_blocks=nb)
        t1 = time.perf_counter()
        tiled_backward(q, k, v, o, m, do, causal, col_blocks=nb)
        t2 = time.perf_counter()
        out += [t1 - t0, t2 - t1]
    return tuple(out)


def _pair_fraction(nb: int, taken: int, causal: bool, reverse: bool) -> float:
    """Fraction of the block-pair loop covered by the first `taken` outer blocks (16x16 blocks)."""
    if not causal:
        return taken / nb
    # forward: query block i does i+1 key blocks; backward: key block j does nb-j query blocks.
    w = [(nb - i) if reverse else (i + 1) for i in range(nb)]
    return sum(w[:taken]) / sum(w)


def cpu_pool(cfg: str, workers: int):
    """A pool of `workers` spawned processes for cpu_baseline (spawned, so it is safe after CUDA init)."""
    b, h = CONFIGS[cfg][:2]
    return mp.get_context("spawn").Pool(max(1, min(workers, b * h)))


def _extrapolate(t1: float, t2: float, f1: float, f2: float) -> float:
    """Full-loop time from samples t1, t2 covering loop fractions f1 < f2 of the block-pair loop:
    t = setup + W * f, so W = (t2 - t1) / (f2 - f1) and full = setup + W (setup >= 0)."""
    w = max(t2 - t1, 0.0) / max(f2 - f1, 1e-9)
    return max(t1 - w * f1, 0.0) + w


def cpu_baseline(cfg: str, budget_s: float, workers: int, pool=None, blocks: int | None = None) -> dict:
    """The reference's CPU path (oracle restatement of reference.py's 16x16-block tiled forward and
    backward, fp16 inputs upcast to fp32) on a bounded sample of the workload, in `workers` spawned
    processes that split the (batch, head) pairs. Each worker times the first `blocks` and the first
    2*`blocks` outer blocks; the difference gives the per-block cost without the fixed setup (fp32
    copies, delta, output buffers), and the full-workload time is setup + the whole block loop.
    Returns TFLOP/s for the full workload."""
    b, h, n, d, causal = CONFIGS[cfg]
    pairs = b * h
    nb = (n + 15) // 16
    workers = max(1, min(workers, pairs))
    bounds = [(pairs * i // workers, pairs * (i + 1) // workers) for i in range(workers)]
    own = pool is None
    if own:
        pool = cpu_pool(cfg, workers)
    try:
        if blocks is None:  # size the sample from a one-block probe so it takes about budget_s
            probe = pool.map(_cpu_worker, [(pairs, n, d, causal, lo, hi, 1, 0) for lo, hi in bounds])
            per_blk = max((r[2] + r[3]) / 2 for r in probe)  # upper bound: setup included
            blocks = max(1, min(nb // 2, int(budget_s / (3 * per_blk))))
        res = pool.map(_cpu_worker, [(pairs, n, d, causal, lo, hi, blocks, 0) for lo, hi in bounds])
    finally:
        if own:
            pool.close()
            pool.join()
    take = blocks
    ff = [_pair_fraction(nb, take, causal, False), _pair_fraction(nb, 2 * take, causal, False)]
    fb = [_pair_fraction(nb, take, causal, True), _pair_fraction(nb, 2 * take, causal, True)]
    t_fwd = max(_extrapolate(r[0], r[2], *ff) for r in res)
    t_bwd = max(_extrapolate(r[1], r[3], *fb) for r in res)
    total = flops(b, h, n, d, causal, "fwd+bwd")
    return {
        "value": total / (t_fwd + t_bwd) / 1e12,
        "unit": "TFLOP/s",
        "cores": workers,
        "kind": "port",
        "sample": (f"{cfg} all {pairs} (b,h) pairs, first {take} and first {2 * take} of {nb} 16-row "
                   f"query blocks (fwd) and key blocks (bwd); full time = setup + per-block cost x "
                   f"block-pair count"),  # fmt: skip
        "blocks": take,
        "fwd_s_extrapolated": t_fwd,
        "bwd_s_extrapolated": t_bwd,
    }


# ------------------------------------------------------------------------------------------- GPU
def _kernel_times(q, k, v, do, causal, scale, iters: int) -> dict:
    """Average device time (CUDA events on the launching stream) of each library kernel."""
    import torch

    from tattn import _lib, api

    lib = _lib.load()
    z, h, n, d = q.shape
    o, m = api._forward(q, k, v, causal, scale)
    delta = torch.empty((z, h, n), device=q.device, dtype=torch.float32)
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    st = _lib.strides_array(q.stride(), k.stride(), v.stride(), do.stride())
    stream = torch.cuda.current_stream().cuda_stream
    ci = int(causal)
    calls = {
        "fwd": lambda: lib.tattn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), m.data_ptr(),
                                     _lib.strides_array(q.stride(), k.stride(), v.stride(), o.stride()),
                                     z, h, n, d, 0, ci, scale, 0, stream),
        "preprocess": lambda: lib.tattn_bwd_preprocess(o.data_ptr(), do.data_ptr(), delta.data_ptr(),
                                                       _lib.strides_array(o.stride(), do.stride()),
                                                       z, h, n, d, 0, stream),
        "dkdv": lambda: lib.tattn_bwd_dkdv(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), dk.data_ptr(),
                                           dv.data_ptr(), m.data_ptr(), delta.data_ptr(), st, z, h, n, d, 0, ci,
                                           scale, 0, stream),
        "dq": lambda: lib.tattn_bwd_dq(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), dq.data_ptr(),
                                       m.data_ptr(), delta.data_ptr(), st, z, h, n, d, 0, ci, scale, 0, stream),
    }  # fmt: skip
    if d <= 64:  # the backward the API runs for these shapes: delta, fused kernel, dQ scaling
        ws = torch.empty((z, h, n, d), device=q.device, dtype=torch.float32)
        st5 = _lib.strides_array(q.stride(), k.stride(), v.stride(), o.stride(), do.stride())
        calls["bwd_fused"] = lambda: lib.tattn_bwd_fused(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), dq.data_ptr(), dk.data_ptr(),
            dv.data_ptr(), m.data_ptr(), delta.data_ptr(), ws.data_ptr(), st5, z, h, n, d, 0, ci, scale, stream)
    out = {}
    for name, fn in calls.items():
        for _ in range(3):
            _lib.check(name, fn())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / iters
    return out


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from tattn import _lib, attention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    b, h, n, d, causal = CONFIGS[args.config]
    if args.config == "cfg5":  # strong scaling of the fixed 1024 (b, h) pairs
        lo, hi = shard(b * h, rank, world)
        b_local, h_local = 1, hi - lo
    else:  # weak scaling: each rank runs the whole config on its own (batch, head) shard
        b_local, h_local = b, h
    scale = 1.0 / math.sqrt(d)
    shape = (b_local, h_local, n, d)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q, k, v, do = (torch.randn(shape, generator=g, device=dev).to(torch.float16) for _ in range(4))
    qg, kg, vg = (t.detach().requires_grad_() for t in (q, k, v))

    def step():
        out = attention(qg, kg, vg, causal=causal)
        return torch.autograd.grad(out, (qg, kg, vg), do)

    def fwd_only():
        with torch.no_grad():
            return attention(q, k, v, causal=causal)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError("device status word set during warm-up")

    def timed(fn, iters):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), dev)

    with ClockSampler(local) as clk:
        ms_total = timed(step, args.steps)
    ms_step = ms_total / args.steps
    if args.lean:  # profiling runs: warm-up + timed steps only
        if rank == 0:
            total = flops(b_local, h_local, n, d, causal, "fwd+bwd") * world
            print(json.dumps({"lean": True, "config": args.config, "ms_per_step": ms_step,
                              "tflops": total / (ms_step * 1e-3) / 1e12}), flush=True)  # fmt: skip
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    for _ in range(3):
        fwd_only()
    ms_fwd = timed(fwd_only, args.steps) / args.steps

    # e2e: every step copies its inputs q, k, v, dO from pinned host memory to the device, runs the
    # public API's forward and backward, and copies O, dq, dk, dv back to pinned host memory.
    # Serial: all on one stream. Pipelined (the reported value): copies on their own streams with two
    # device input sets, so step k's compute overlaps step k+1's host->device copy and step k-1's
    # device->host copy (PCIe is full duplex), as an input pipeline feeding a training loop would.
    host_in = [t.cpu().pin_memory() for t in (q, k, v, do)]
    host_out = [[torch.empty(shape, dtype=torch.float16).pin_memory() for _ in range(4)] for _ in range(2)]
    dev_in = [[torch.empty(shape, device=dev, dtype=torch.float16) for _ in range(4)] for _ in range(2)]
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def compute_from(bufs):
        qd, kd, vd = (t.detach().requires_grad_() for t in bufs[:3])
        out = attention(qd, kd, vd, causal=causal)
        grads = torch.autograd.grad(out, (qd, kd, vd), bufs[3])
        return (out.detach(), *grads)

    def e2e_serial_step():
        for dst, src in zip(dev_in[0], host_in):
            dst.copy_(src, non_blocking=True)
        for dst, src in zip(host_out[0], compute_from(dev_in[0])):
            dst.copy_(src, non_blocking=True)

    def e2e_pipelined(iters):
        main = torch.cuda.current_stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        start = torch.cuda.Event()
        start.record(main)

        def h2d(kk):
            slot = kk % 2
            s_h2d.wait_event(start)
            if kk >= 2:
                s_h2d.wait_event(in_free[slot])  # the compute of step kk - 2 has read this set
            with torch.cuda.stream(s_h2d):
                for dst, src in zip(dev_in[slot], host_in):
                    dst.copy_(src, non_blocking=True)
                in_ready[slot].record(s_h2d)

        h2d(0)
        for kk in range(iters):
            slot = kk % 2
            if kk + 1 < iters:
                h2d(kk + 1)
            main.wait_event(in_ready[slot])
            outs = compute_from(dev_in[slot])
            in_free[slot].record(main)
            done = torch.cuda.Event()
            done.record(main)
            s_d2h.wait_event(done)
            with torch.cuda.stream(s_d2h):
                for dst, src in zip(host_out[slot], outs):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(s_d2h)
        tail = torch.cuda.Event()
        tail.record(s_d2h)
        main.wait_event(tail)  # the timed region ends after the last device->host copy

    def timed_pipelined(iters):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_pipelined(iters)
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), dev)

    n_e2e = max(3, args.steps // 2)
    for _ in range(2):
        e2e_serial_step()
    e2e_pipelined(3)
    torch.cuda.synchronize()
    ms_e2e_serial = timed(e2e_serial_step, n_e2e) / n_e2e
    ms_e2e = timed_pipelined(n_e2e) / n_e2e
    if _lib.device_status() != 0:
        raise RuntimeError("device status word set during the timed region")

    kt = _kernel_times(q, k, v, do, causal, scale, max(5, args.steps))
    if world > 1:
        kt_t = torch.tensor([kt[k_] for k_ in sorted(kt)], device=dev, dtype=torch.float64)
        dist.all_reduce(kt_t, op=dist.ReduceOp.MAX)
        kt = dict(zip(sorted(kt), kt_t.tolist()))

    per_rank_fb = flops(b_local, h_local, n, d, causal, "fwd+bwd")
    per_rank_f = flops(b_local, h_local, n, d, causal, "fwd")
    total_fb = per_rank_fb * world
    total_f = per_rank_f * world
    value = total_fb / (ms_step * 1e-3) / 1e12
    fwd_tflops = total_f / (ms_fwd * 1e-3) / 1e12
    pk = peaks()
    # GEMM FLOPs each kernel actually performs per launch (2 flops per MAC; causal halves the pairs).
    pair_flops = 2.0 * b_local * h_local * n * n * d * (0.5 if causal else 1.0)
    # bwd_fused: 5 GEMMs (S, dP, dV, dK, dQ) per pair; its time includes the delta pass and the dQ scaling.
    kflops = {"fwd": 2 * pair_flops, "dkdv": 4 * pair_flops, "dq": 3 * pair_flops, "bwd_fused": 5 * pair_flops}
    step_kernels = ("fwd", "bwd_fused") if "bwd_fused" in kt else ("fwd", "dkdv", "dq")  # what a step runs
    dom = max(step_kernels, key=lambda kk: kt[kk])
    achieved = kflops[dom] / (kt[dom] * 1e-3) / 1e12
    bytes_in = 4 * b_local * h_local * n * d * 2
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "strong" if args.config == "cfg5" else "weak",
            "vs_baseline": round(value / T4_PUBLISHED[args.config], 2) if args.config in T4_PUBLISHED else None,
            "vs_baseline_ref": "the reference's published fwd+bwd on a Tesla T4 (its results/t4.json)",
            "dtype": "fp16",
            "data": "synthetic: q,k,v,dO ~ N(0,1) cast to fp16, seeded per rank",
            "config": {
                "workload": f"{args.config}: fp16 fwd+bwd B{b_local} H{h_local} N{n} D{d} "
                            f"{'causal' if causal else 'non-causal'} per GPU",
                "global_batch_heads": b_local * h_local * world,
                "seq_len": n,
                "head_dim": d,
                "causal": causal,
                "parallelism": f"(batch, head) sharding over {world} GPU(s), no collective on the hot path",
                "l2": f"working set {8 * bytes_in // 4 / 2**20:.0f} MiB per step > 126 MB L2 (inputs larger than L2)",
            },  # fmt: skip
            "fwd_tflops": round(fwd_tflops, 2),
            "fwd_ms": round(ms_fwd, 4),
            "fwd_frac_of_peak": round(fwd_tflops / world / pk["tflops"], 4),
            "fwd_bwd_frac_of_peak": round(value / world / pk["tflops"], 4),
            "peak_tflops_per_gpu": pk["tflops"],
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json bf16_tflops, burst; fp16 dense equals bf16)",
            "kernel_ms": {k_: round(v_, 4) for k_, v_ in kt.items()},
            "roofline": {
                "kernel": dom,
                "bound": "tensor",
                "achieved": round(achieved, 1),
                "peak": pk["tflops"],
                "unit": "TFLOP/s",
                "frac": round(achieved / pk["tflops"], 4),
                "traffic": NCU_TRAFFIC.get((args.config, dom)),
                "traffic_source": (f"ncu capture (profiles/{'bwd_fused' if dom == 'bwd_fused' else 'bwd_dkdv'}_cfg2.md)"
                                   if (args.config, dom) in NCU_TRAFFIC else None),
                "flops_per_launch": kflops[dom],
            },
            "e2e": {
                "value": round(total_fb / (ms_e2e * 1e-3) / 1e12, 2),
                "unit": "TFLOP/s",
                "ms_per_step": round(ms_e2e, 3),
                "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_in,
                "path": "tattn.attention with pinned host q,k,v,dO copied in and O,dq,dk,dv copied out every "
                        "step; copies on their own streams, double-buffered, overlapping the neighbouring "
                        "steps' compute",
                "serial": {"value": round(total_fb / (ms_e2e_serial * 1e-3) / 1e12, 2),
                           "ms_per_step": round(ms_e2e_serial, 3),
                           "path": "the same with copies and compute on one stream"},
            },
            "gpu_launches": 4 * args.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(args.config, args.cpu_budget, max(1, os.cpu_count() or 1))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_compare(args) -> None:
    """Comparison table (see the module docstring): one JSON line per (config, implementation)."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from tattn import attention

    dev = torch.device("cuda", 0)

    def naive(q, k, v, causal, scale):
        s_ = (q @ k.transpose(-1, -2)).float() * scale
        if causal:
            n_ = q.shape[-2]
            s_ = s_.masked_fill(torch.ones(n_, n_, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
        return (torch.softmax(s_, -1).to(q.dtype) @ v)

    def sdpa(backend):
        def f(q, k, v, causal, scale):
            with sdpa_kernel([backend]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)
        return f

    impls = {
        "tattn_b200": lambda q, k, v, causal, scale: attention(q, k, v, causal=causal, sm_scale=scale),
        "sdpa_flash": sdpa(SDPBackend.FLASH_ATTENTION),
        "sdpa_cudnn": sdpa(SDPBackend.CUDNN_ATTENTION),
        "sdpa_efficient": sdpa(SDPBackend.EFFICIENT_ATTENTION),
        "naive": naive,
    }
    for cfg in ("cfg2", "cfg3"):
        b, h, n, d, causal = CONFIGS[cfg]
        scale = 1.0 / math.sqrt(d)
        g = torch.Generator(device=dev).manual_seed(1234)
        q, k, v, do = (torch.randn((b, h, n, d), generator=g, device=dev).to(torch.float16) for _ in range(4))
        # fp32 definition on two (b, h) pairs for the error columns
        pairs = [(0, 0), (b - 1, h - 1)]
        refs = {}
        for bi, hi in pairs:
            qf, kf, vf = (t[bi, hi].float().requires_grad_() for t in (q, k, v))
            of = naive(qf, kf, vf, causal, scale)
            gq, gk, gv = torch.autograd.grad(of, (qf, kf, vf), do[bi, hi].float())
            refs[(bi, hi)] = (of.detach(), gq, gk, gv)
        for name, fn in impls.items():
            line = {"compare": name, "config": cfg, "shape": [b, h, n, d], "causal": causal}
            try:
                qg, kg, vg = (t.detach().requires_grad_() for t in (q, k, v))

                def step():
                    o_ = fn(qg, kg, vg, causal, scale)
                    return o_, torch.autograd.grad(o_, (qg, kg, vg), do)

                def fwd():
                    with torch.no_grad():
                        return fn(q, k, v, causal, scale)

                o_, grads = step()
                err = {"o": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
                for (bi, hi), (of, gq, gk, gv) in refs.items():
                    for key, a_, r_ in (("o", o_, of), ("dq", grads[0], gq), ("dk", grads[1], gk), ("dv", grads[2], gv)):
                        err[key] = max(err[key], (a_[bi, hi].float() - r_).abs().max().item())
                del o_, grads
                torch.cuda.synchronize()
                base = torch.cuda.memory_allocated(dev)
                torch.cuda.reset_peak_memory_stats(dev)
                step()
                torch.cuda.synchronize()
                peak = torch.cuda.max_memory_allocated(dev) - base
                for fn_, key in ((fwd, "fwd"), (step, "fwd+bwd")):
                    for _ in range(3):
                        fn_()
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    iters = max(3, args.steps // 4)
                    e0.record()
                    for _ in range(iters):
                        fn_()
                    e1.record()
                    torch.cuda.synchronize()
                    ms = e0.elapsed_time(e1) / iters
                    line[f"{key}_ms"] = round(ms, 4)
                    line[f"{key}_tflops"] = round(flops(b, h, n, d, causal, key) / (ms * 1e-3) / 1e12, 1)
                line["peak_extra_mib_fwd_bwd"] = round(peak / 2**20, 1)
                line["max_abs_err_vs_fp32"] = {k_: float(f"{v_:.3g}") for k_, v_ in err.items()}
            except Exception as e:  # a backend that does not support this GPU / shape
                line["unavailable"] = f"{type(e).__name__}: {str(e).splitlines()[0][:160] if str(e) else ''}"
            print(json.dumps(line), flush=True)
            torch.cuda.empty_cache()


def run_reference(args) -> None:
    """The reference's CPU implementation of the path (oracle port), rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = max(1, os.cpu_count() or 1)
    vals = []
    # Each step is one bounded sample of the same size (blocks sized once, from the first warm-up
    # step, so that all steps together cost about cpu_budget seconds).
    per_step = args.cpu_budget / max(1, args.steps)
    with cpu_pool(args.config, cores) as pool:
        first = cpu_baseline(args.config, per_step, cores, pool)
        for _ in range(args.warmup - 1):
            cpu_baseline(args.config, per_step, cores, pool, blocks=first["blocks"])
        t0 = time.perf_counter()
        for _ in range(args.steps):
            vals.append(cpu_baseline(args.config, per_step, cores, pool, blocks=first["blocks"]))
        wall = time.perf_counter() - t0
    b, h, n, d, causal = CONFIGS[args.config]
    value = statistics.median(v["value"] for v in vals)
    cb = dict(vals[-1])
    cb["value"] = round(value, 6)
    line = {
        "metric": METRIC,
        "value": round(value, 6),
        "unit": "TFLOP/s",
        "impl": "reference",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(flops(b, h, n, d, causal, "fwd+bwd") / (value * 1e12) * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong" if args.config == "cfg5" else "weak",
        "vs_baseline": None,
        "dtype": "fp16 inputs, fp32 arithmetic (reference CPU path)",
        "data": "synthetic: q,k,v,dO ~ N(0,1) cast to fp16",
        "config": {"workload": f"{args.config}: fp16 fwd+bwd B{b} H{h} N{n} D{d} {'causal' if causal else 'non-causal'}",
                   "seq_len": n, "head_dim": d, "causal": causal},  # fmt: skip
        "cpu_baseline": cb,
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 1),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU work for the CPU baseline")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--lean", action="store_true", help="warm-up + timed steps only (for profiler runs)")
    ap.add_argument("--compare", action="store_true",
                    help="comparison table against torch SDPA backends and a naive softmax (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.compare:
        run_compare(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
