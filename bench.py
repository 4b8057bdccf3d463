"""Benchmark: batched small-matrix exponential, forward + Frechet backward, matrices/s.

Headline workload: config 5 of the benchmark set -- FP32 [1,048,576, 32, 32], entries
N(0,1)/sqrt(32) scaled by lognormal(0,1) per matrix -- with the batch split evenly over the N
GPUs (one process per GPU, no collective in the timed region; strong scaling).  A step is one
forward ``fh.matrix_exp(x)`` plus one ``torch.autograd.grad(y, x, g)`` through the public API
on the rank's shard, inputs resident in HBM (4.3 GB per tensor, larger than L2).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference package's CPU path (native torch.linalg.matrix_exp +
autograd, flash_hypercons/ops/matrix_exp/__init__.py:26-29,95-96) on the host cores, rank 0
only, on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HEADLINE = 5
METRIC = "fwd+bwd matrices/s"
SECONDARY = (2, 3, 4)
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "ncu_traffic.json")


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, default=HEADLINE, choices=[1, 2, 3, 4, 5])
    p.add_argument("--no-extras", action="store_true", help="skip the secondary configs, e2e and CPU baseline")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU work of the CPU baseline sample")
    p.add_argument("--batch", type=int, default=None,
                   help="use only the first BATCH matrices of the config (small cases for profiling)")
    p.add_argument("--stream-mix-only", action="store_true",
                   help="run only the fused stream-mixing leg (with --batch: that many tokens per rank)")
    return p.parse_args()


def workloads_module():
    """``flash_hyperconnections_b200/workloads.py`` loaded by file path.  It needs torch only;
    importing it through the package would run the package ``__init__``, which loads this
    repository's native libraries -- and the reference arm must not map them."""
    import importlib.util

    name = "_fhx_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "flash_hyperconnections_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses resolve their module through sys.modules
    spec.loader.exec_module(mod)
    return mod


# ----------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------
class Dist:
    """One process per GPU (torchrun env vars); NCCL for GPU runs, gloo for the CPU arm.
    Collectives are used only outside the timed region: barriers around it and a MAX
    all-reduce of the per-rank times."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        self.backend = None

    def init(self, backend: str):
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=300))
            self.pg = dist
            self.backend = backend

    def barrier(self):
        if self.pg is not None:
            if self.backend == "nccl":
                self.pg.barrier(device_ids=[self.local_rank])
            else:
                self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        device = f"cuda:{self.local_rank}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([value], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.pg is None:
            return value
        device = f"cuda:{self.local_rank}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([value], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def sum_ints(self, values: list[int]) -> list[int]:
        if self.pg is None:
            return list(values)
        device = f"cuda:{self.local_rank}" if self.backend == "nccl" else "cpu"
        t = torch.tensor(values, dtype=torch.int64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return [int(v) for v in t.tolist()]

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


# ----------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            pass

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        mhz, max_mhz, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            if self.uuid and not parts[0].endswith(self.uuid.replace("GPU-", "")):
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max_mhz, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ----------------------------------------------------------------------------------------
# the step
# ----------------------------------------------------------------------------------------
def fwd_bwd(fh, a, g):
    x = a.detach().requires_grad_()
    y = fh.matrix_exp(x)
    (grad,) = torch.autograd.grad(y, x, g)
    return y, grad


def count_our_launches(fh, a, g) -> int:
    """Kernels of libfhx launched by one step, from the library's own launch counter."""
    from flash_hyperconnections_b200 import _native

    lib = _native.load_cabi()
    torch.cuda.synchronize()
    before = lib.fhx_launch_count()
    fwd_bwd(fh, a, g)
    torch.cuda.synchronize()
    return int(lib.fhx_launch_count() - before)


def time_steps(fh, a, g, steps: int, warmup: int, dist: Dist, flush: torch.Tensor | None = None):
    """Device time of `steps` fwd+bwd steps: total ms, and per-phase kernel ms (fwd, bwd)."""
    for _ in range(warmup):
        fwd_bwd(fh, a, g)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if flush is None:
        start.record()
        for e0, e1, e2 in ev:
            e0.record()
            x = a.detach().requires_grad_()
            y = fh.matrix_exp(x)
            e1.record()
            torch.autograd.grad(y, x, g)
            e2.record()
        end.record()
        torch.cuda.synchronize()
        total = start.elapsed_time(end)
    else:
        total = 0.0
        for e0, e1, e2 in ev:
            flush.add_(1.0)  # write more than L2 between timed iterations
            e0.record()
            x = a.detach().requires_grad_()
            y = fh.matrix_exp(x)
            e1.record()
            torch.autograd.grad(y, x, g)
            e2.record()
        torch.cuda.synchronize()
        total = sum(e0.elapsed_time(e2) for e0, _, e2 in ev)
    dist.barrier()
    torch.cuda.synchronize()
    fwd = [e0.elapsed_time(e1) for e0, e1, _ in ev]
    bwd = [e1.elapsed_time(e2) for _, e1, e2 in ev]
    return total, statistics.mean(fwd), statistics.mean(bwd)


# Cycles of the spin kernel that precedes each device-only step (about 0.5 ms at 1.9 GHz).
HOST_LEAD_CYCLES = 1_000_000


def kernel_device_us(fh, a, g, flush: torch.Tensor, reps: int = 5) -> dict | None:
    """Mean device duration of each libfhx kernel of an eager step (L2 flushed before each step),
    from the CUDA profiler's kernel records: the kernels alone, without the launch and event
    overhead that event-timed phases of a few microseconds include."""
    from torch.profiler import ProfilerActivity, profile

    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(reps):
                flush.add_(1.0)
                fwd_bwd(fh, a, g)
            torch.cuda.synchronize()
        out = {}
        for ev in prof.key_averages():
            if "fhx::" not in ev.key:
                continue
            total = getattr(ev, "device_time_total", None)
            if total is None:
                total = getattr(ev, "cuda_time_total", 0.0)
            name = ev.key.split("(")[0].replace("void ", "").replace("fhx::", "")
            out[name] = round(float(total) / max(1, int(ev.count)), 2)
        return out or None
    except Exception:  # the CUDA profiler is unavailable (e.g. under ncu)
        return None


def device_phase_ms(fh, a, g, steps: int, flush: torch.Tensor):
    """Device time of the forward and backward kernels of one eager step, without host gaps: for
    small batches the host (Python, dispatcher, autograd engine) takes longer to issue a step than
    the GPU takes to run it, so events around the phases of `time_steps` also count the GPU waiting
    for the next launch.  Here a spin kernel after each L2 flush lets the host run ahead, and the
    events around each phase see only its kernels (plus the launch and event overhead of a few
    microseconds that separates them).  Medians over the steps."""
    fwd, bwd = [], []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1, e2 in ev:
        flush.add_(1.0)
        torch.cuda._sleep(HOST_LEAD_CYCLES)
        e0.record()
        x = a.detach().requires_grad_()
        y = fh.matrix_exp(x)
        e1.record()
        torch.autograd.grad(y, x, g)
        e2.record()
    torch.cuda.synchronize()
    for e0, e1, e2 in ev:
        fwd.append(e0.elapsed_time(e1))
        bwd.append(e1.elapsed_time(e2))
    return statistics.median(fwd), statistics.median(bwd)


def graph_step_ms(fh, a, g, steps: int, warmup: int, flush: torch.Tensor | None):
    """Device time per step of one fwd+bwd step captured in a CUDA graph and replayed (the launch-
    overhead answer for small batches), and whether the replayed results equal an eager step."""
    x = a.detach().clone().requires_grad_()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            y = fh.matrix_exp(x)
            torch.autograd.grad(y, x, g)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = fh.matrix_exp(x)
        (grad,) = torch.autograd.grad(y, x, g)
    for _ in range(warmup):
        graph.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        if flush is not None:
            flush.add_(1.0)
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)
    y_eager, grad_eager = fwd_bwd(fh, a, g)
    same = bool(torch.equal(y, y_eager) and torch.equal(grad, grad_eager))
    del graph
    return ms, same


def fused_step_ms(fh, a, g, steps: int, warmup: int, flush: torch.Tensor | None):
    """Device time per call of ``fh.matrix_exp_and_grad`` (forward and backward of exp in one
    Frechet launch, for a known upstream gradient), and whether its gradient equals the
    autograd step's bit for bit."""
    for _ in range(warmup):
        fh.matrix_exp_and_grad(a, g)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        if flush is not None:
            flush.add_(1.0)
        e0.record()
        fh.matrix_exp_and_grad(a, g)
        e1.record()
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)
    _, grad = fh.matrix_exp_and_grad(a, g)
    _, grad_ref = fwd_bwd(fh, a, g)
    return ms, bool(torch.equal(grad, grad_ref))


# End-to-end pipeline shape (matrices per chunk, streams), measured on B200 over PCIe with
# config 5: 8192 x 4 gave 5.25 M matrices/s, 32768 x 2 gave 4.45 M, 4096 x 8 gave 5.03 M.
E2E_CHUNK = 8192
E2E_STREAMS = 4


def result_digest(fh, a, g) -> list[int]:
    """Integer sums of the raw bits of Y and of the gradient of this rank's shard (one more step,
    after the timed region).  Summed over ranks they give a whole-batch digest that must be the same
    at every GPU count: the shards are generated identically and no matrix depends on another."""
    y, grad = fwd_bwd(fh, a, g)
    out = []
    for t in (y.detach(), grad):
        bits = t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)
        out.append(int(bits.to(torch.int64).sum().item()))
    del y, grad
    return out


def e2e_steps(fh, cfg, a_host, g_host, steps: int, warmup: int, dist: Dist, device,
              chunk: int = E2E_CHUNK, nstreams: int = E2E_STREAMS):
    """Same metric through the public API from pinned host buffers: every step copies its
    inputs host->device, runs fwd+bwd and copies Y and the gradient back, pipelined in chunks
    over several streams (round robin, so that one chunk's upload, another's compute and a
    third's download overlap).  Returns (seconds per step, h2d bytes, d2h bytes)."""
    batch = a_host.shape[0]
    chunk = min(batch, chunk)
    n = cfg.n
    streams = [torch.cuda.Stream(device=device) for _ in range(nstreams)]
    dev_a = [torch.empty((chunk, n, n), dtype=cfg.dtype, device=device) for _ in range(nstreams)]
    dev_g = [torch.empty((chunk, n, n), dtype=cfg.dtype, device=device) for _ in range(nstreams)]
    y_host = torch.empty_like(a_host).pin_memory()
    grad_host = torch.empty_like(a_host).pin_memory()

    def one_step():
        for i, lo in enumerate(range(0, batch, chunk)):
            k = i % nstreams
            s = streams[k]
            hi = min(lo + chunk, batch)
            with torch.cuda.stream(s):
                xa = dev_a[k][: hi - lo]
                xg = dev_g[k][: hi - lo]
                xa.copy_(a_host[lo:hi], non_blocking=True)
                xg.copy_(g_host[lo:hi], non_blocking=True)
                src = xa.mT if cfg.transposed else xa
                y, grad = fwd_bwd(fh, src, xg)
                y_host[lo:hi].copy_(y.detach(), non_blocking=True)
                grad_host[lo:hi].copy_(grad, non_blocking=True)
        for s in streams:
            s.synchronize()

    for _ in range(warmup):
        one_step()
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    torch.cuda.synchronize()
    elapsed = (time.perf_counter() - t0) / steps
    dist.barrier()
    nbytes = a_host.numel() * a_host.element_size()
    return elapsed, 2 * nbytes, 2 * nbytes


LINK_BYTES = 256 << 20
LINK_REPS = 8


def link_gbs_per_direction(device, dist: Dist, nbytes: int = LINK_BYTES, reps: int = LINK_REPS) -> float:
    """Pinned host<->device copy bandwidth of this rank's link with both directions running at once
    (the bound of the e2e leg, which uploads and downloads concurrently), GB/s per direction.  The
    ranks start together (barrier) so that the figure includes the host-memory and PCIe-switch
    sharing that the e2e leg itself sees at N > 1."""
    h_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nbytes, dtype=torch.uint8, device=device)
    d_out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    up, down = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)

    def both():
        cur = torch.cuda.current_stream(device)
        up.wait_stream(cur)
        down.wait_stream(cur)
        with torch.cuda.stream(up):
            d_in.copy_(h_in, non_blocking=True)
        with torch.cuda.stream(down):
            h_out.copy_(d_out, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)

    both()
    torch.cuda.synchronize(device)
    dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        both()
    end.record()
    torch.cuda.synchronize(device)
    dist.barrier()
    return reps * nbytes / (start.elapsed_time(end) * 1e6)


# ----------------------------------------------------------------------------------------
# roofline
# ----------------------------------------------------------------------------------------
def frechet_kernel_name(n: int) -> str:
    """The kernel that fhx_frechet launches for n x n matrices (the roofline's dominant kernel)."""
    if n <= 4:
        return f"fhx::expm_reg_kernel<{n}, Frechet> (fhx_frechet)"
    tile = {8: "8, 4, 4", 16: "16, 2, 4", 32: "32, 2, 4"}[8 if n <= 8 else 16 if n <= 16 else 32]
    return f"fhx::expm_team_kernel<{tile}, Frechet> (fhx_frechet)"


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "sm_max_mhz": 1965.0}, "fallback"


def fp32_fma_peak_tflops(sm_count: int, mhz: float) -> float:
    # 128 FP32 lanes per SM, one FMA (2 flops) per lane per clock.
    return sm_count * 128 * 2 * mhz * 1e6 / 1e12


def load_traffic(config_index: int):
    try:
        with open(TRAFFIC_PATH) as f:
            data = json.load(f)
        return data.get(str(config_index))
    except (OSError, ValueError):
        return None


def measure_config(fh, cfg, rank, world, dist, steps, warmup, device, with_e2e, batch=None, with_graph=False):
    from flash_hyperconnections_b200 import roofline as R

    W = workloads_module()

    start, count = W.shard(cfg, rank, world) if world > 1 else (0, cfg.batch)
    if batch is not None:
        count = min(count, batch)
    a, g = W.generate(cfg, start, count, device=device)
    torch.cuda.synchronize()
    steps_per_matrix = R.mandated_steps(a)
    fwd_flops = 2.0 * R.kernel_size(cfg.n) ** 3 * float(steps_per_matrix.sum().item())
    bwd_flops = 3.0 * fwd_flops
    in_bytes = a.numel() * a.element_size()
    flush = None
    if 3 * in_bytes < 256 * 2**20:  # inputs fit in L2: flush it between timed iterations
        flush = torch.empty(64 * 2**20, dtype=torch.float32, device=device)
    launches = count_our_launches(fh, a, g)
    total_ms, fwd_ms, bwd_ms = time_steps(fh, a, g, steps, warmup, dist, flush)
    eager_phase_ms = None
    if flush is not None:
        # the per-kernel figures without the host gaps that the eager step contains
        eager_phase_ms = {"fwd": fwd_ms, "bwd": bwd_ms}
        fwd_ms, bwd_ms = device_phase_ms(fh, a, g, max(steps, 5), flush)
    kernel_us = kernel_device_us(fh, a, g, flush) if flush is not None else None
    digest = result_digest(fh, a, g)
    graph = graph_step_ms(fh, a, g, steps, warmup, flush) if with_graph else None
    fused = fused_step_ms(fh, a, g, steps, warmup, flush)
    result = {
        "digest": digest,
        "count": count,
        "total_ms": total_ms,
        "fwd_ms": fwd_ms,
        "bwd_ms": bwd_ms,
        "eager_phase_ms": eager_phase_ms,
        "kernel_device_us": kernel_us,
        "fwd_flops": fwd_flops,
        "bwd_flops": bwd_flops,
        "launches_per_step": launches,
        "mean_steps": float(steps_per_matrix.double().mean().item()),
        "bytes": R.algorithmic_bytes(count, cfg.n, cfg.elem_bytes),
        "l2": "L2 flushed (256 MB write) between timed iterations" if flush is not None
        else f"inputs larger than L2 ({in_bytes / 1e9:.2f} GB per tensor per rank)",
    }
    if graph is not None:
        result["graph_ms"], result["graph_matches_eager"] = graph
    result["fused_ms"], result["fused_grad_matches"] = fused
    if with_e2e:
        e2e_count = min(count, 131072)
        a_host = (a[:e2e_count].mT.contiguous() if cfg.transposed else a[:e2e_count]).cpu().pin_memory()
        g_host = g[:e2e_count].cpu().pin_memory()
        del a, g
        torch.cuda.empty_cache()
        sec, h2d, d2h = e2e_steps(fh, cfg, a_host, g_host, max(2, min(steps, 5)), 1, dist, device)
        result["e2e"] = {"sec_per_step": sec, "count": e2e_count, "h2d": h2d, "d2h": d2h,
                         "link_gbs": link_gbs_per_direction(device, dist)}
    return result


# ----------------------------------------------------------------------------------------
# hyper-connection stream mixing (config 2's mixing matrices applied to residual streams)
# ----------------------------------------------------------------------------------------
MIX_TOKENS = 65536   # config 2: 16 sequences x 4096 tokens
MIX_STREAMS = 4
MIX_WIDTH = 4096     # residual stream width D (model dimension)


def measure_stream_mix(fh, dist, steps, warmup, device, tokens=None):
    """fwd+bwd of Y = exp(H) X per token: the fused kernels (fh.mix_streams) against the unfused
    composition (fh.matrix_exp, then a batched matmul, with autograd through both), bf16, on
    this rank's shard of the tokens.  Inputs are larger than L2."""
    W = workloads_module()
    cfg = W.CONFIGS[2]
    tokens = min(tokens or MIX_TOKENS, MIX_TOKENS) // dist.world
    start = dist.rank * tokens
    h, _ = W.generate(cfg, start, tokens, device=device)
    gen = torch.Generator(device="cpu")
    gen.manual_seed(90412 + dist.rank)
    x = torch.randn((tokens, MIX_STREAMS, MIX_WIDTH), generator=gen).to(torch.bfloat16).to(device)
    dy = torch.randn((tokens, MIX_STREAMS, MIX_WIDTH), generator=gen).to(torch.bfloat16).to(device)

    def fused():
        hh = h.detach().requires_grad_()
        xx = x.detach().requires_grad_()
        y = fh.mix_streams(hh, xx)
        torch.autograd.grad(y, (xx, hh), dy)

    def unfused():
        hh = h.detach().requires_grad_()
        xx = x.detach().requires_grad_()
        y = fh.matrix_exp(hh) @ xx
        torch.autograd.grad(y, (xx, hh), dy)

    out = {}
    for name, fn in (("fused", fused), ("unfused", unfused)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = dist.max(e0.elapsed_time(e1) / steps)
    elt = 2
    per_token = 5 * MIX_STREAMS * MIX_WIDTH * elt + 3 * MIX_STREAMS**2 * elt  # X, Y, X, dY, dX; H, H, dH
    hbm = per_token * tokens / (out["fused"] * 1e6)
    del h, x, dy
    torch.cuda.empty_cache()
    return {
        "workload": f"bf16 H [{tokens * dist.world}, {MIX_STREAMS}, {MIX_STREAMS}] (config 2 generators) applied to "
                    f"streams [{tokens * dist.world}, {MIX_STREAMS}, {MIX_WIDTH}]; fwd + bwd (d streams, d H)",
        "value": tokens * dist.world / (out["fused"] / 1e3), "unit": "tokens/s", "ms_per_step": out["fused"],
        "unfused_ms_per_step": out["unfused"], "speedup_vs_unfused": out["unfused"] / out["fused"],
        "hbm": {"algorithmic_bytes_per_token": per_token, "achieved_gbs_per_gpu": hbm},
        "unfused": "fh.matrix_exp(H) @ X with autograd (exp launch, batched matmul, Frechet launch, matmul backward)",
    }


# ----------------------------------------------------------------------------------------
# CPU path of the reference (native torch + autograd on the host cores)
# ----------------------------------------------------------------------------------------
def cpu_reference_sample(cfg, target_seconds: float):
    from oracle import cpu_path

    W = workloads_module()

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    probe = 256 if cfg.n >= 16 else 2048
    a, g = W.generate(cfg, 0, min(probe, cfg.batch), device="cpu")
    cpu_path.time_fwd_bwd(a, g, repeat=1)  # first call pays one-time thread-pool costs
    t = cpu_path.time_fwd_bwd(a, g, repeat=1)
    rate = a.shape[0] / t
    count = int(min(cfg.batch, max(probe, rate * target_seconds)))
    count = max(probe, (count // probe) * probe)
    a, g = W.generate(cfg, 0, count, device="cpu")
    t = cpu_path.time_fwd_bwd(a, g, repeat=1)
    return {"value": count / t, "unit": "matrices/s", "cores": threads, "kind": "reference",
            "sample": f"first {count} matrices of {cfg.name}: native torch.linalg.matrix_exp + autograd.grad on CPU "
                      f"(the reference package's CPU path), {threads} threads, {t:.1f} s",
            "seconds": t}


def run_reference(args, dist):
    from oracle import cpu_path

    W = workloads_module()

    cfg = W.CONFIGS[args.config]
    if dist.rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    per_step = max(1.0, args.cpu_seconds / max(1, args.steps))
    probe = 256 if cfg.n >= 16 else 2048
    a, g = W.generate(cfg, 0, min(probe, cfg.batch), device="cpu")
    cpu_path.time_fwd_bwd(a, g, repeat=1)  # first call pays one-time thread-pool costs
    rate = a.shape[0] / cpu_path.time_fwd_bwd(a, g, repeat=1)
    count = int(min(cfg.batch, max(probe, rate * per_step)))
    count = max(probe, (count // probe) * probe) if count >= probe else count
    a, g = W.generate(cfg, 0, count, device="cpu")
    for _ in range(args.warmup):
        cpu_path.time_fwd_bwd(a, g, repeat=1)
    times = [cpu_path.time_fwd_bwd(a, g, repeat=1) for _ in range(args.steps)]
    total = sum(times)
    value = count * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "matrices/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, config generator)",
        "config": {"workload": cfg.name, "step_sample": count, "full_batch": cfg.batch, "n": cfg.n},
        "cpu_baseline": {"value": value, "unit": "matrices/s", "cores": threads, "kind": "reference",
                         "sample": f"first {count} matrices of {cfg.name} per step: native torch.linalg.matrix_exp "
                                   f"+ autograd.grad on CPU, the reference package's CPU path"},
        "e2e": {"value": value, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
def main():
    args = parse_args()
    dist = Dist()
    if args.impl == "reference":
        dist.init("gloo")
        try:
            run_reference(args, dist)
        finally:
            dist.close()
        return

    import flash_hypercons as fh

    W = workloads_module()
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    dist.init("nccl")
    cfg = W.CONFIGS[args.config]
    if args.stream_mix_only:
        res = measure_stream_mix(fh, dist, max(5, args.steps), args.warmup, device, tokens=args.batch)
        if dist.rank == 0:
            print(json.dumps({"stream_mix": res}), flush=True)
        dist.close()
        return
    sampler = ClockSampler(dist.local_rank) if dist.rank == 0 else None

    if sampler:
        sampler.start()
    main_res = measure_config(fh, cfg, dist.rank, dist.world, dist, args.steps, args.warmup, device,
                              with_e2e=not args.no_extras, batch=args.batch)
    clocks = sampler.stop() if sampler else None

    digest = dist.sum_ints(main_res["digest"])
    total_ms = dist.max(main_res["total_ms"])
    fwd_ms = dist.max(main_res["fwd_ms"])
    bwd_ms = dist.max(main_res["bwd_ms"])
    # algorithmic work of the whole job (every rank's shard), for the per-GPU roofline
    fused_ms = dist.max(main_res["fused_ms"])
    fused_ok = dist.sum(0.0 if main_res["fused_grad_matches"] else 1.0) == 0.0
    fwd_flops = dist.sum(main_res["fwd_flops"])
    bwd_flops = dist.sum(main_res["bwd_flops"])
    sum_steps = dist.sum(main_res["mean_steps"] * main_res["count"])
    ms_per_step = total_ms / args.steps
    global_batch = main_res["count"] * dist.world
    value = global_batch / (ms_per_step / 1e3)
    e2e = None
    if "e2e" in main_res:
        sec = dist.max(main_res["e2e"]["sec_per_step"])
        e2e_total = main_res["e2e"]["count"] * dist.world
        e2e = {"value": e2e_total / sec, "unit": "matrices/s",
               "h2d_bytes_per_step": main_res["e2e"]["h2d"] * dist.world,
               "d2h_bytes_per_step": main_res["e2e"]["d2h"] * dist.world,
               "batch": e2e_total, "path": "pinned host -> fh.matrix_exp + autograd.grad -> pinned host, "
                                           f"{E2E_STREAMS} streams, {E2E_CHUNK}-matrix chunks"}
        # the e2e leg's own roofline: each rank's host link, both directions at once, measured
        # with every rank copying at the same time
        link = -dist.max(-main_res["e2e"]["link_gbs"])  # slowest rank's link
        per_dir = main_res["e2e"]["h2d"] / (sec * 1e9)    # bytes each way per rank per second
        e2e["link"] = {"bound": "pcie", "achieved_gbs_per_direction": per_dir,
                       "measured_gbs_per_direction": link, "frac": per_dir / link,
                       "aggregate_host_gbs": 2 * per_dir * dist.world,
                       "measured": f"pinned {LINK_BYTES >> 20} MB host->device and device->host copies on two streams "
                                   f"at once, x{LINK_REPS}, all ranks together"}

    extras = {}
    if not args.no_extras:
        # Secondary configs, sharded over the ranks like the headline one (same collective steps
        # on every rank).
        for idx in SECONDARY:
            if idx == args.config:
                continue
            sub = W.CONFIGS[idx]
            steps = max(5, args.steps)
            r = measure_config(fh, sub, dist.rank, dist.world, dist, steps, args.warmup, device, with_e2e=False,
                               with_graph=idx == 2 and dist.world == 1)
            sub_digest = dist.sum_ints(r["digest"])
            sub_total = dist.max(r["total_ms"])
            sub_fwd = dist.max(r["fwd_ms"])
            sub_bwd = dist.max(r["bwd_ms"])
            sub_fwd_flops = dist.sum(r["fwd_flops"]) / dist.world
            sub_bwd_flops = dist.sum(r["bwd_flops"]) / dist.world
            sub_steps = dist.sum(r["mean_steps"] * r["count"])
            sub_fused = dist.max(r["fused_ms"])
            sub_fused_ok = dist.sum(0.0 if r["fused_grad_matches"] else 1.0) == 0.0
            ms = sub_total / steps
            extras[sub.name] = {
                "value": sub.batch / (ms / 1e3), "unit": "matrices/s", "ms_per_step": ms, "n_gpus": dist.world,
                "result_digest": {"y_bits_sum": sub_digest[0], "grad_bits_sum": sub_digest[1]},
                "fwd_kernel_ms": sub_fwd, "bwd_kernel_ms": sub_bwd,
                "kernel_ms_note": ("device time of each phase's kernels, a spin kernel letting the host run "
                                   "ahead (the eager step's phases, host gaps included: eager_phase_ms)"
                                   if r["eager_phase_ms"] is not None else "device time of each phase of the step"),
                "eager_phase_ms": ({k: dist.max(v) for k, v in r["eager_phase_ms"].items()}
                                   if r["eager_phase_ms"] is not None else None),
                "kernel_device_us": r["kernel_device_us"],
                "fwd_tflops_per_gpu": sub_fwd_flops / (sub_fwd * 1e9),
                "bwd_tflops_per_gpu": sub_bwd_flops / (sub_bwd * 1e9),
                "hbm_gbs_per_gpu": r["bytes"] / (ms * 1e6), "mean_products_per_matrix": sub_steps / sub.batch,
                "l2": r["l2"],
                "fused_fwd_bwd": {"ms_per_step": sub_fused, "value": sub.batch / (sub_fused / 1e3),
                                  "grad_matches_autograd": sub_fused_ok,
                                  "path": "fh.matrix_exp_and_grad: forward and backward in one Frechet launch"},
            }
            if "graph_ms" in r:
                extras[sub.name]["cuda_graph"] = {
                    "ms_per_step": r["graph_ms"], "value": sub.batch / (r["graph_ms"] / 1e3),
                    "matches_eager": r["graph_matches_eager"],
                    "path": "one fwd+bwd step (fh.matrix_exp + autograd.grad) captured in torch.cuda.CUDAGraph, replayed",
                }
    stream_mix = None
    if not args.no_extras:
        stream_mix = measure_stream_mix(fh, dist, max(5, args.steps), args.warmup, device)
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_extras:
        cpu = cpu_reference_sample(cfg, args.cpu_seconds)

    if dist.rank == 0:
        peaks, peak_src = load_peaks()
        props = torch.cuda.get_device_properties(device)
        max_mhz = float(peaks.get("sm_max_mhz", 1965.0))
        fma_peak = fp32_fma_peak_tflops(props.multi_processor_count, max_mhz)
        # per GPU: the job's algorithmic flops / N over the max-over-ranks kernel time
        bwd_tflops = bwd_flops / dist.world / (bwd_ms * 1e9)
        fwd_tflops = fwd_flops / dist.world / (fwd_ms * 1e9)
        traffic = load_traffic(args.config)
        hbm_gbs = main_res["bytes"] / (ms_per_step * 1e6)
        roofline = {
            "bound": "fp32_fma",
            "kernel": frechet_kernel_name(cfg.n),
            "achieved": bwd_tflops,
            "peak": fma_peak,
            "unit": "TFLOP/s",
            "frac": bwd_tflops / fma_peak,
            "peak_source": f"nominal FP32 FMA: {props.multi_processor_count} SMs x 128 lanes x 2 flops x "
                           f"{max_mhz:.0f} MHz (clocks.max.sm, {peak_src} MEASURED_PEAKS.json has no FP32-FMA figure)",
            "traffic": traffic,
            "forward": {"achieved": fwd_tflops, "frac": fwd_tflops / fma_peak},
            "step": {"achieved": (fwd_flops + bwd_flops) / dist.world / (ms_per_step * 1e9),
                     "frac": (fwd_flops + bwd_flops) / dist.world / (ms_per_step * 1e9) / fma_peak},
            "hbm": {"achieved_gbs_per_gpu": hbm_gbs, "peak_gbs": peaks.get("hbm_gbs"),
                    "frac": hbm_gbs / float(peaks.get("hbm_gbs", 6650.0))},
            "flops_definition": "2 P^3 (pi(m)+s) fwd, 6 P^3 (pi(m)+s) bwd per matrix, (m, s) from the kernel's rule; "
                                "summed over every rank's shard, per GPU",
        }
        if clocks and clocks.get("sm_mhz"):
            roofline["frac_at_sampled_clock"] = bwd_tflops / fp32_fma_peak_tflops(props.multi_processor_count,
                                                                                  clocks["sm_mhz"])
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "matrices/s",
            "n_gpus": dist.world,
            "result_digest": {"y_bits_sum": digest[0], "grad_bits_sum": digest[1],
                              "note": "sum over ranks of the raw bits of Y and the gradient; the same at every GPU count"},
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded host-side generator, same matrices at every GPU count and in the CPU arm; "
                    "see flash_hyperconnections_b200/workloads.py)",
            "config": {"workload": f"config{cfg.index}:{cfg.name} fwd+bwd", "global_batch": global_batch, "n": cfg.n,
                       "io_dtype": str(cfg.dtype).replace("torch.", ""), "parallelism": f"batch shards x{dist.world}, "
                       "no collective", "l2": main_res["l2"],
                       "mean_products_per_matrix": sum_steps / global_batch},
            "gpu_launches": main_res["launches_per_step"] * args.steps,
            "kernel_ms": {"fwd": fwd_ms / 1.0, "bwd": bwd_ms / 1.0},
            "kernel_device_us": main_res.get("kernel_device_us"),
            "fused_fwd_bwd": {"ms_per_step": fused_ms, "value": global_batch / (fused_ms / 1e3),
                              "grad_matches_autograd": fused_ok,
                              "path": "fh.matrix_exp_and_grad(x, g): forward and backward of exp in one Frechet launch "
                                      "(for callers that hold the upstream gradient); not the headline step"},
            "roofline": roofline,
            "clocks": clocks,
        }
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = {k: v for k, v in cpu.items() if k != "seconds"}
        if extras:
            line["secondary_configs"] = extras
        if stream_mix:
            peak_hbm = float(peaks.get("hbm_gbs", 6650.0))
            stream_mix["hbm"]["peak_gbs"] = peak_hbm
            stream_mix["hbm"]["frac"] = stream_mix["hbm"]["achieved_gbs_per_gpu"] / peak_hbm
            line["stream_mix"] = stream_mix
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
