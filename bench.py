"""Benchmark: attention fwd and fwd+bwd TFLOP/s (fp16, head_dim 64) on 1..8 B200s.

The headline line is BASELINE config 5, the scaling config: fp16 causal forward + backward over a fixed
B64 H16 N8192 D64 problem whose 1,024 (batch, head) pairs are split evenly over the ranks (strong
scaling; 1,024 / 512 / 256 / 128 pairs per GPU at 1 / 2 / 4 / 8 GPUs). One step = one forward and one
backward of ``tattn.attention`` over the rank's pairs. Pairs are independent in the forward and the
backward (the reference's grid axis 1 is Z*H, kernels.py:96-98), so ranks exchange no data; each rank
times on the device with CUDA events and rank 0 reports the max over ranks. FLOPs follow the
reference (bench/bench.py:31-35): 4*B*H*N^2*D, halved when causal, x3.5 for fwd+bwd.

Configs 2 (B4 H16 N4096 non-causal) and 3 (B1 H16 N16384 causal) run on every rank as well, whole
(they are single-GPU configs), and are reported per GPU under "configs": the north_star's forward
target (>= 60% of peak) is stated on config 2. ``--config cfg2|cfg3`` makes one of them the headline
instead (weak scaling: every rank runs the whole config).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg5|cfg2|cfg3] [--impl reference]

``--impl reference`` times the reference's CPU path (the numpy restatement of src/tattn/reference.py's
tiled_forward / tiled_backward in oracle/) on the host cores: each step runs complete (batch, head)
pairs of the same config, one per worker process, every key and query block of them, and the line
reports their FLOPs over the step's wall time.

``--variants`` (one GPU) times every tile variant of the library's tile table (forward, split backward)
and the fused backward at configs 2 and 3 and a config-5 slice, one JSON line each.

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
    # name: (batch, heads, seq, head_dim, causal)
    "cfg2": (4, 16, 4096, 64, False),
    "cfg3": (1, 16, 16384, 64, True),
    "cfg5": (64, 16, 8192, 64, True),
}
STRONG = {"cfg5"}  # configs whose fixed (batch, head) pairs are split over the ranks
# The reference's published fwd+bwd TFLOP/s on a Tesla T4 for the config-2 and config-3 shapes
# (its results/t4.json); it publishes nothing for config 5.
T4_PUBLISHED = {"cfg2": 16.9, "cfg3": 15.9}
L2_BYTES = 126 * 2**20
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each kernel per (batch,
# head) pair, from an ncu capture of the current build on a 64-pair slice of config 5 (inputs 5 x 64 MiB
# > L2; the command is NCU_TRAFFIC_SOURCE), divided by the captured pairs. Scaled by the pairs a launch
# processes, as the traffic grows with them.
NCU_TRAFFIC_PER_PAIR: dict[tuple[str, str], float] = {
    ("cfg5", "bwd_fused"): (540_986_368 + 303_763_712) / 64,
    ("cfg5", "fwd"): (210_691_072 + 50_971_648) / 64,
}
NCU_TRAFFIC_SOURCE = ("ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none "
                      "-k regex:'bwd_fused|fwd_f16' -s 6 -c 2 python bench.py --lean --pairs 64 --steps 2 --warmup 3")


def flops(b: int, h: int, n: int, d: int, causal: bool, mode: str) -> float:
    f = 4.0 * b * h * n * n * d
    if causal:
        f /= 2
    return f * (3.5 if mode == "fwd+bwd" else 1.0)


def shard(pairs: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous (batch, head) pair range [lo, hi) of `rank`: pairs are independent in the forward
    and the backward, so ranks need no data exchange; sizes differ by at most one pair."""
    return pairs * rank // world, pairs * (rank + 1) // world


def local_pairs(cfg: str, rank: int, world: int) -> int:
    """(batch, head) pairs one rank runs: its shard of a strong-scaling config, else the whole config."""
    b, h = CONFIGS[cfg][:2]
    if cfg in STRONG:
        lo, hi = shard(b * h, rank, world)
        return hi - lo
    return b * h


def config_dict(cfg: str, world: int) -> dict:
    """The `config` object of the JSON line (identical in both arms)."""
    b, h, n, d, causal = CONFIGS[cfg]
    strong = cfg in STRONG
    pairs = b * h
    return {
        "workload": (f"{cfg}: fp16 fwd+bwd B{b} H{h} N{n} D{d} {'causal' if causal else 'non-causal'}"
                     + (f", {pairs} (batch, head) pairs split over {world} GPU(s)" if strong
                        else f" on each of {world} GPU(s)")),  # fmt: skip
        "global_batch_heads": pairs if strong else pairs * world,
        "seq_len": n,
        "head_dim": d,
        "causal": causal,
        "parallelism": f"(batch, head) sharding over {world} GPU(s), no collective on the hot path",
        "l2": f"inputs {4 * (pairs // (world if strong else 1)) * n * d * 2 / 2**20:.0f} MiB per GPU per step > 126 MB L2",
    }


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
def _cpu_init() -> None:
    """Pool initializer: one BLAS thread per worker process (the workers already fill the cores)."""
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"


def _cpu_task(args: tuple) -> tuple[int, float, float]:
    """One worker's share of a CPU step: the reference's tiled forward and backward (oracle restatement,
    16x16 blocks, fp16 inputs upcast to fp32) over `npairs` complete (batch, head) pairs of length n.
    Returns (pid, forward seconds, backward seconds); input generation is not timed."""
    import numpy as np

    from oracle import tiled_backward, tiled_forward

    n, d, causal, npairs, seed = args
    rng = np.random.default_rng(seed)
    q, k, v, do = (rng.standard_normal((npairs, n, d)).astype(np.float16) for _ in range(4))
    t0 = time.perf_counter()
    o, m = tiled_forward(q, k, v, causal)
    t1 = time.perf_counter()
    tiled_backward(q, k, v, o, m, do, causal)
    t2 = time.perf_counter()
    return os.getpid(), t1 - t0, t2 - t1


def cpu_pool(workers: int):
    """Spawned worker processes (spawn, so a pool started after CUDA initialisation is safe)."""
    return mp.get_context("spawn").Pool(max(1, workers), initializer=_cpu_init)


def cpu_step(cfg: str, pool, workers: int, pairs_per_worker: int = 1, seed: int = 0) -> dict:
    """One CPU step: `workers` tasks of `pairs_per_worker` whole pairs each, run in parallel. The step's
    time is the busiest worker process's compute time (a process that ran two tasks counts both)."""
    _, _, n, d, causal = CONFIGS[cfg]
    tasks = [(n, d, causal, pairs_per_worker, seed * 1000 + i) for i in range(workers)]
    res = pool.map(_cpu_task, tasks, chunksize=1)
    per_pid: dict[int, list[float]] = {}
    for pid, tf, tb in res:
        acc = per_pid.setdefault(pid, [0.0, 0.0])
        acc[0] += tf
        acc[1] += tb
    busiest = max(per_pid.values(), key=sum)
    pairs = workers * pairs_per_worker
    secs = sum(busiest)
    return {"seconds": secs, "fwd_s": busiest[0], "bwd_s": busiest[1], "pairs": pairs,
            "tflops": flops(1, pairs, n, d, causal, "fwd+bwd") / secs / 1e12}  # fmt: skip


def cpu_sample_text(cfg: str, workers: int, pairs_per_worker: int) -> str:
    b, h, n, d, causal = CONFIGS[cfg]
    return (f"{workers * pairs_per_worker} of the {b * h} (batch, head) pairs of {cfg} per step, each a complete "
            f"N={n} D={d} {'causal' if causal else 'non-causal'} forward + backward (every 16x16 block of the "
            f"reference's tiled loops), {pairs_per_worker} pair(s) in each of {workers} worker processes; "
            f"TFLOP/s = the pairs' FLOPs / the busiest worker's compute time")  # fmt: skip


def cpu_baseline(cfg: str, workers: int) -> dict:
    """The `cpu_baseline` object of the GPU arm's line: one CPU step (after one warm-up step) on a pool of
    `workers` processes, i.e. `workers` complete pairs of the same config."""
    with cpu_pool(workers) as pool:
        cpu_step(cfg, pool, workers, 1, seed=99)
        r = cpu_step(cfg, pool, workers, 1, seed=1)
    return {"value": round(r["tflops"], 6), "unit": "TFLOP/s", "cores": workers, "kind": "port",
            "sample": cpu_sample_text(cfg, workers, 1), "seconds": round(r["seconds"], 2)}  # fmt: skip


# ------------------------------------------------------------------------------------------- GPU
def _isolated_kernel_times(q, k, v, do, causal, scale, iters: int) -> dict:
    """Average device time (CUDA events on the launching stream, back-to-back launches) of each entry
    point on the rank's inputs: the forward, the fused backward call the API takes, and the
    reference-style split backward (preprocess, dK/dV, dQ) for comparison."""
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
    ws = torch.empty(lib.tattn_bwd_fused_workspace_bytes(z, h, n, d), device=q.device, dtype=torch.uint8)
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


class _Timer:
    """Device time of `iters` calls of `fn`: barrier, synchronize, CUDA events on the current stream,
    synchronize; the max over ranks."""

    def __init__(self, world: int, dev) -> None:
        self.world, self.dev = world, dev

    def __call__(self, fn, iters: int) -> float:
        import torch
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), self.dev)


def _inputs(pairs: int, n: int, d: int, dev, seed: int):
    import torch

    g = torch.Generator(device=dev).manual_seed(seed)
    shape = (1, pairs, n, d)
    return [torch.randn(shape, generator=g, device=dev).to(torch.float16) for _ in range(4)]


def _side_config(cfg: str, steps: int, warmup: int, timer: _Timer, dev, rank: int, pk: dict) -> dict:
    """Whole config `cfg` on this rank (weak): fwd+bwd and fwd-only device times, per GPU, max over ranks."""
    import torch

    from tattn import attention

    b, h, n, d, causal = CONFIGS[cfg]
    q, k, v, do = _inputs(b * h, n, d, dev, 4321 + rank)
    q, k, v, do = (t.view(b, h, n, d) for t in (q, k, v, do))
    qg, kg, vg = (t.detach().requires_grad_() for t in (q, k, v))

    def step():
        out = attention(qg, kg, vg, causal=causal)
        return torch.autograd.grad(out, (qg, kg, vg), do)

    def fwd():
        with torch.no_grad():
            return attention(q, k, v, causal=causal)

    for _ in range(warmup):
        step()
        fwd()
    ms_fb = timer(step, steps) / steps
    ms_f = timer(fwd, steps) / steps
    fb = flops(b, h, n, d, causal, "fwd+bwd") / (ms_fb * 1e-3) / 1e12
    f = flops(b, h, n, d, causal, "fwd") / (ms_f * 1e-3) / 1e12
    out = {
        "workload": f"fp16 B{b} H{h} N{n} D{d} {'causal' if causal else 'non-causal'}, whole config on each GPU",
        "fwd_bwd_tflops_per_gpu": round(fb, 2),
        "fwd_bwd_ms": round(ms_fb, 4),
        "fwd_tflops_per_gpu": round(f, 2),
        "fwd_ms": round(ms_f, 4),
        "fwd_frac_of_peak": round(f / pk["tflops"], 4),
        "fwd_bwd_frac_of_peak": round(fb / pk["tflops"], 4),
    }
    if cfg in T4_PUBLISHED:
        out["fwd_bwd_vs_t4_published"] = round(fb / T4_PUBLISHED[cfg], 2)
    del q, k, v, do, qg, kg, vg
    torch.cuda.empty_cache()
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
    timer = _Timer(world, dev)
    pk = peaks()
    cfg = args.config
    _, _, n, d, causal = CONFIGS[cfg]
    pairs = args.pairs or local_pairs(cfg, rank, world)
    scale = 1.0 / math.sqrt(d)
    shape = (1, pairs, n, d)
    q, k, v, do = _inputs(pairs, n, d, dev, 1234 + rank)
    qg, kg, vg = (t.detach().requires_grad_() for t in (q, k, v))

    def step():
        out = attention(qg, kg, vg, causal=causal)
        return torch.autograd.grad(out, (qg, kg, vg), do)

    # In-step split of the device time: events around the forward call and the backward call of every
    # timed step (recorded on the launching stream; the host enqueues far ahead of these ms-long
    # kernels, so each interval is the device time of that call's kernels).
    marks: list[tuple] = []

    def step_marked():
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        out = attention(qg, kg, vg, causal=causal)
        e[1].record()
        grads = torch.autograd.grad(out, (qg, kg, vg), do)
        e[2].record()
        marks.append(e)
        return grads

    def fwd_only():
        with torch.no_grad():
            return attention(q, k, v, causal=causal)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError("device status word set during warm-up")

    with ClockSampler(local) as clk:
        ms_total = timer(step_marked, args.steps)
    ms_step = ms_total / args.steps
    fwd_in_step = statistics.fmean(m[0].elapsed_time(m[1]) for m in marks)
    bwd_in_step = statistics.fmean(m[1].elapsed_time(m[2]) for m in marks)
    split = torch.tensor([fwd_in_step, bwd_in_step], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(split, op=dist.ReduceOp.MAX)
    fwd_in_step, bwd_in_step = split.tolist()
    if args.lean:  # profiling runs: warm-up + timed steps only
        if rank == 0:
            total = flops(1, pairs, n, d, causal, "fwd+bwd") * world
            print(json.dumps({"lean": True, "config": cfg, "pairs_per_gpu": pairs, "ms_per_step": ms_step,
                              "tflops": total / (ms_step * 1e-3) / 1e12}), flush=True)  # fmt: skip
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    for _ in range(3):
        fwd_only()
    ms_fwd = timer(fwd_only, args.steps) / args.steps

    # ---- e2e: every step copies its inputs q, k, v, dO from pinned host memory to the device, runs the
    # public API's forward and backward, and copies O, dq, dk, dv back into pinned host memory.
    # Serial: all on one stream. Pipelined: copies on their own streams with two device input sets, so
    # step k's compute overlaps step k+1's host->device copy and step k-1's device->host copy (PCIe is
    # full duplex). Each step's outputs stay referenced until the compute stream has waited for their
    # device->host copy, so the caching allocator reuses their memory only in stream order.
    host_in = [t.cpu().pin_memory() for t in (q, k, v, do)]
    host_out = [torch.empty(shape, dtype=torch.float16).pin_memory() for _ in range(4)]
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
        for dst, src in zip(host_out, compute_from(dev_in[0])):
            dst.copy_(src, non_blocking=True)

    def e2e_pipelined(iters: int) -> None:
        main = torch.cuda.current_stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_copied = [torch.cuda.Event() for _ in range(2)]
        held: list = [None, None]
        start = torch.cuda.Event()
        start.record(main)

        def h2d(kk: int) -> None:
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
            if held[slot] is not None:  # step kk - 2's outputs have been copied out: release them
                main.wait_event(out_copied[slot])
                held[slot] = None
            outs = compute_from(dev_in[slot])
            in_free[slot].record(main)
            done = torch.cuda.Event()
            done.record(main)
            s_d2h.wait_event(done)
            with torch.cuda.stream(s_d2h):
                for dst, src in zip(host_out, outs):
                    dst.copy_(src, non_blocking=True)
            out_copied[slot].record(s_d2h)
            held[slot] = outs
        # The copy-out stream is in order: the timed region ends after its last copy.
        main.wait_event(out_copied[(iters - 1) % 2])

    n_e2e = max(3, args.steps)
    for _ in range(2):
        e2e_serial_step()
    e2e_pipelined(3)
    torch.cuda.synchronize()
    ms_e2e_serial = timer(e2e_serial_step, n_e2e) / n_e2e
    ms_e2e_pipe = timer(lambda: e2e_pipelined(n_e2e), 1) / n_e2e
    del dev_in
    torch.cuda.empty_cache()
    if _lib.device_status() != 0:
        raise RuntimeError("device status word set during the timed region")

    kt = _isolated_kernel_times(q.view(shape), k.view(shape), v.view(shape), do.view(shape), causal, scale,
                                max(5, args.steps))  # fmt: skip
    if world > 1:
        kt_t = torch.tensor([kt[k_] for k_ in sorted(kt)], device=dev, dtype=torch.float64)
        dist.all_reduce(kt_t, op=dist.ReduceOp.MAX)
        kt = dict(zip(sorted(kt), kt_t.tolist()))
    del q, k, v, do, qg, kg, vg
    torch.cuda.empty_cache()

    side = {}
    if not args.no_side:
        for other in ("cfg2", "cfg3"):
            if other != cfg:
                side[other] = _side_config(other, args.steps, args.warmup, timer, dev, rank, pk)

    # Pairs all ranks processed per step: the whole strong-scaling config (its shards), else every rank's own.
    all_pairs = CONFIGS[cfg][0] * CONFIGS[cfg][1] if (cfg in STRONG and not args.pairs) else pairs * world
    total_fb = flops(1, all_pairs, n, d, causal, "fwd+bwd")
    total_f = flops(1, all_pairs, n, d, causal, "fwd")
    value = total_fb / (ms_step * 1e-3) / 1e12
    fwd_tflops = total_f / (ms_fwd * 1e-3) / 1e12
    # GEMM FLOPs per launch on this rank (2 flops per MAC; causal halves the pairs): the forward's 2
    # GEMMs; the fused backward's 5 (S, dP, dV, dK, dQ), whose call also runs the delta pass and the dQ
    # scaling; the split path's 4 + 3.
    pair_flops = 2.0 * pairs * n * n * d * (0.5 if causal else 1.0)
    kflops = {"fwd": 2 * pair_flops, "bwd_fused": 5 * pair_flops, "dkdv": 4 * pair_flops, "dq": 3 * pair_flops}
    step_kernels = {"fwd": fwd_in_step, "bwd_fused": bwd_in_step}
    dom = max(step_kernels, key=lambda kk: step_kernels[kk])
    achieved = kflops[dom] / (step_kernels[dom] * 1e-3) / 1e12
    bytes_in = 4 * pairs * n * d * 2
    traffic = NCU_TRAFFIC_PER_PAIR.get((cfg, dom))
    if rank == 0:
        e2e_best = min(ms_e2e_serial, ms_e2e_pipe)
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "strong" if cfg in STRONG else "weak",
            "vs_baseline": round(value / T4_PUBLISHED[cfg], 2) if cfg in T4_PUBLISHED else None,
            "dtype": "fp16",
            "data": "synthetic: q,k,v,dO ~ N(0,1) cast to fp16, seeded per rank",
            "config": config_dict(cfg, world),
            "fwd_tflops": round(fwd_tflops, 2),
            "fwd_ms": round(ms_fwd, 4),
            "fwd_frac_of_peak": round(fwd_tflops / world / pk["tflops"], 4),
            "fwd_bwd_frac_of_peak": round(value / world / pk["tflops"], 4),
            "peak_tflops_per_gpu": pk["tflops"],
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json bf16_tflops, burst; fp16 dense equals bf16)",
            "in_step_ms": {"fwd": round(fwd_in_step, 4), "bwd": round(bwd_in_step, 4)},
            "kernel_ms_isolated": {k_: round(v_, 4) for k_, v_ in kt.items()},
            "roofline": {
                "kernel": "bwd_fused_kernel (tattn_bwd_fused call)" if dom == "bwd_fused" else "fwd_f16_kernel",
                "bound": "tensor",
                "achieved": round(achieved, 1),
                # the kernel is timed inside a seconds-long run of steps at the power cap, so its peak is
                # the sustained GEMM rate (MEASURED_PEAKS.json bf16_tflops_sustained); the burst fraction
                # is given beside it
                "peak": pk["tflops_sustained"] or pk["tflops"],
                "peak_kind": "sustained" if pk.get("tflops_sustained") else "burst",
                "unit": "TFLOP/s",
                "frac": round(achieved / (pk["tflops_sustained"] or pk["tflops"]), 4),
                "frac_of_burst": round(achieved / pk["tflops"], 4),
                "traffic": round(traffic * pairs) if traffic else None,
                "traffic_source": ("one launch on a 64-pair slice of the config, per pair x the pairs of this "
                                   "launch: " + NCU_TRAFFIC_SOURCE) if traffic else None,
                # the op's own tensors: backward reads q, k, v, O, dO, M and writes dq, dk, dv (the fp32 dQ
                # workspace is the implementation's); forward reads q, k, v and writes O, M
                "algorithmic_bytes": (8 if dom == "bwd_fused" else 4) * pairs * n * d * 2 + 4 * pairs * n,
                # the fused kernel's fp32 dQ sums, written (reduce-adds leaving L2) and read back once for
                # the fp16 dq: the part of `traffic` above the op's own tensors
                "workspace_bytes": 8 * pairs * n * d if dom == "bwd_fused" else 0,
                "flops_per_launch": kflops[dom],
                "timing": "CUDA events around each call inside the timed steps, mean over steps, max over ranks",
            },
            "e2e": {
                "value": round(total_fb / (e2e_best * 1e-3) / 1e12, 2),
                "unit": "TFLOP/s",
                "ms_per_step": round(e2e_best, 3),
                "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_in,
                "path": ("tattn.attention + autograd on each rank's pairs, with q, k, v, dO copied in from pinned "
                         "host memory and O, dq, dk, dv copied back to pinned host memory every step; the "
                         "faster of the two schedules below"),
                "pipelined": {"value": round(total_fb / (ms_e2e_pipe * 1e-3) / 1e12, 2),
                              "ms_per_step": round(ms_e2e_pipe, 3),
                              "path": "copies on their own streams, double-buffered, overlapping the neighbouring "
                                      "steps' compute"},
                "serial": {"value": round(total_fb / (ms_e2e_serial * 1e-3) / 1e12, 2),
                           "ms_per_step": round(ms_e2e_serial, 3),
                           "path": "copies and compute on one stream"},
                "iterations": n_e2e,
            },  # fmt: skip
            "configs": side,
            "gpu_launches": args.steps * LAUNCHES_PER_STEP,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(cfg, max(1, os.cpu_count() or 1))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# Library kernels one fwd+bwd step launches: the forward; the delta pass and the fused backward kernel
# (which also scales dQ).
LAUNCHES_PER_STEP = 3


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


def run_variants(args) -> None:
    """Every tile variant of the tile table (tattn.api.TILE_CONFIGS, i.e. the library's csrc/tiles.h) on
    one GPU, one JSON line each: the forward variants, the split backward (dK/dV + dQ) variants, and the
    fused backward, at configs 2 and 3 and a 128-pair slice of config 5. This is the evidence behind the
    default per (D, causal): the same launches under ncu give each variant's tensor-pipe activity."""
    import torch

    from tattn import _lib, api

    dev = torch.device("cuda", 0)
    cases = {"cfg2": CONFIGS["cfg2"], "cfg3": CONFIGS["cfg3"], "cfg5_slice128": (8,) + CONFIGS["cfg5"][1:],
             "cfg2_d128": (4, 16, 4096, 128, False), "cfg2_d128_causal": (4, 16, 4096, 128, True)}
    timer = _Timer(1, dev)
    for name, (b, h, n, d, causal) in cases.items():
        q, k, v, do = (t.view(b, h, n, d) for t in _inputs(b * h, n, d, dev, 77))
        sc = 1.0 / math.sqrt(d)
        f = flops(b, h, n, d, causal, "fwd")
        o, m = api._forward(q, k, v, causal, sc)
        runs = [("fwd", i + 1, cfg, lambda cfg=cfg: api._forward(q, k, v, causal, sc, config=cfg), f)
                for i, cfg in enumerate(api.TILE_CONFIGS["fwd"]) if api.tile_supported(cfg, "fwd", d)]
        runs += [("bwd_split", i + 1, cfg, lambda cfg=cfg: api._backward(q, k, v, o, m, do, causal, sc, config=cfg),
                  2.5 * f) for i, cfg in enumerate(api.TILE_CONFIGS["bwd"]) if api.tile_supported(cfg, "bwd", d)]
        # the API's own fp16 backward: the fused kernel
        runs.append(("bwd_fused", 0, {},
                     lambda: api._backward(q, k, v, o, m, do, causal, sc), 2.5 * f))
        for kind, idx, cfg, fn, fl in runs:
            for _ in range(args.warmup):
                fn()
            ms = timer(fn, args.steps) / args.steps
            # tile_cfg 0 of tattn_fwd / the split backward resolves to this variant; the API's fp16 backward
            # is the fused kernel
            default = _lib.load().tattn_tile_default(api._KIND["fwd" if kind == "fwd" else "bwd"], d, int(causal), 0)
            print(json.dumps({"variants": name, "kind": kind, "tile_cfg": idx, **cfg, "ms": round(ms, 4),
                              "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
                              "default": kind == "bwd_fused" or idx == default}),
                  flush=True)  # fmt: skip
        del q, k, v, do, o, m
        torch.cuda.empty_cache()
    if _lib.device_status() != 0:
        raise RuntimeError("device status word set during the variant sweep")


def run_reference(args) -> None:
    """The reference's CPU implementation of the path (oracle restatement), rank 0 only: W warm-up steps,
    then K timed steps, each `workers` complete (batch, head) pairs of the config in parallel."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cfg = args.config
    cores = max(1, os.cpu_count() or 1)
    steps = []
    t_start = time.perf_counter()
    with cpu_pool(cores) as pool:
        for i in range(args.warmup):
            cpu_step(cfg, pool, cores, 1, seed=10_000 + i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            steps.append(cpu_step(cfg, pool, cores, 1, seed=i))
        wall = time.perf_counter() - t0
    _, _, n, d, causal = CONFIGS[cfg]
    pairs = steps[0]["pairs"]
    secs = sum(s["seconds"] for s in steps)
    value = flops(1, pairs * len(steps), n, d, causal, "fwd+bwd") / secs / 1e12
    line = {
        "metric": METRIC,
        "value": round(value, 6),
        "unit": "TFLOP/s",
        "impl": "reference",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(secs / len(steps) * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong" if cfg in STRONG else "weak",
        "vs_baseline": None,
        "dtype": "fp32 (fp16 inputs upcast, as the reference's CPU path does)",
        "data": "synthetic: q,k,v,dO ~ N(0,1) cast to fp16",
        "config": config_dict(cfg, world),
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": cpu_sample_text(cfg, cores, 1)},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 1),
        "total_wall_s": round(time.perf_counter() - t_start, 1),
    }  # fmt: skip
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg5")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pairs", type=int, default=0,
                    help="override the (batch, head) pairs per GPU (profiling a slice of a config)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-side", action="store_true", help="skip the extra per-GPU configs 2 and 3")
    ap.add_argument("--lean", action="store_true", help="warm-up + timed steps only (for profiler runs)")
    ap.add_argument("--compare", action="store_true",
                    help="comparison table against torch SDPA backends and a naive softmax (one GPU)")
    ap.add_argument("--variants", action="store_true", help="time every tile variant of the tile table (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.compare:
        run_compare(args)
        return
    if args.variants:
        run_variants(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
