#!/usr/bin/env python
"""MoC forward+backward throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

One step = the MoC module's training step on one batch of synthetic input: router
(z @ router^T, softmax) -> convolution -> backward of both (dx, dz, dconv_bases,
drouter).  Config 2: B=4, T=4096, D=z_dim=2048, K=16, S=4, bf16, softmax router,
init_std 0.002, router weight N(0, 0.02); x, z, dy ~ N(0, 1) from a seeded generator.

* ``value``      tokens/s of the whole job: the step is captured once in a CUDA graph
                 and replayed K times with inputs resident in HBM (192 MiB of x, z, dy
                 per rank, larger than the 126 MB L2), timed with CUDA events.
* ``e2e``        the same metric through the public API (``MoC`` forward + backward,
                 eager), with x, z, dy copied from pinned host memory every step and the
                 step's result, the parameter gradients dconv_bases and drouter, copied
                 back, both inside the timed region (``h2d_bytes_per_step`` /
                 ``d2h_bytes_per_step`` count exactly those copies).
* ``roofline``   the dominant kernel timed alone (CUDA events on its stream):
                 algorithmic bytes per launch / average launch time vs measured HBM peak.
* ``cpu_baseline`` the CPU oracle (a port of the reference's PyTorch path) on the full
                 config-2 batch, rank 0 at N=1 only.
* ``workloads``  (default workload, N=1) short runs of the other BASELINE workloads on
                 the same GPU: config 3 (varlen), config 4 (decode) and config 5 (large,
                 one GPU's share), each with its own value and roofline; and the fused
                 q / k / v projection + convolution (proj): prefill, and its training step
                 fused against unfused.

With N > 1 (torchrun, one rank per GPU) every rank runs its own config-2 batch
(weak scaling) and the step adds one all-reduce of [dconv_bases | drouter]; after the
timed region every rank checks that no all-reduce gave up waiting for a peer.
``--impl reference`` times the reference's CPU path (the oracle port) instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mixture-of-convolutions_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

CONFIG = {"B": 4, "T": 4096, "D": 2048, "Dz": 2048, "K": 16, "S": 4, "router": "softmax", "activation": None,
          "init_std": 0.002, "router_std": 0.02}
# config 5, per rank: the large data-parallel case (B=32 over 8 GPUs, so 4 sequences per GPU),
# bases at the fan-in std sqrt(K / (3 S))
CONFIG_LARGE = {"B": 4, "T": 8192, "D": 4096, "Dz": 4096, "K": 32, "S": 8, "router": "softmax", "activation": None,
                "init_std": (32 / (3 * 8)) ** 0.5, "router_std": 0.02}
METRIC = "MoC fwd+bwd tokens/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def step_bytes_per_token(D: int, Dz: int, K: int) -> int:
    """Algorithmic HBM bytes per token of one module fwd+bwd (bf16): forward reads x, z
    and writes y; backward reads dy, x, z and writes dx, dz; alpha is written once and
    read once: 2*(5D + 3Dz) + 4K."""
    return 2 * (5 * D + 3 * Dz) + 4 * K


KERNEL_BYTES_PER_TOKEN = {
    # per-launch algorithmic bytes per token (bf16): reads + writes the kernel must do
    "conv_backward": lambda c: 2 * c["D"] * 3 + 2 * c["K"] * 2,   # x, dy in; dx out; alpha in, dalpha out
    "conv_forward": lambda c: 2 * c["D"] * 2 + 2 * c["K"],        # x in, y out, alpha in
    "router_forward": lambda c: 2 * c["Dz"] + 2 * c["K"],         # z in, alpha out
    "router_backward": lambda c: 2 * c["Dz"] * 2 + 4 * c["K"],    # z in, dz out, alpha + dalpha in
}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        out = {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
        if "bf16_tflops" in d:
            out["bf16_tflops"] = float(d["bf16_tflops"])
        return out
    return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback"}


# ----------------------------------------------------------------------------- clocks

_SAMPLER_SRC = r"""
import sys, time, pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByPciBusId(sys.argv[1].encode())
out = open(sys.argv[2], "w", buffering=1)
out.write("max %d\n" % pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
while True:
    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    try:
        reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    except Exception:
        reasons = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
    out.write("%.6f %d %d\n" % (time.time(), mhz, reasons))
    time.sleep(0.001)
"""


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons of one GPU through NVML
    every ~1 ms in a child process (free of this process's GIL), tagged with wall time."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device: torch.device, out_dir: str) -> None:
        import subprocess

        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        self.path = os.path.join(out_dir, f"clocks_{os.getpid()}.txt")
        self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, bus, self.path],
                                     stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        deadline = time.time() + 60
        while time.time() < deadline and self.proc.poll() is None:  # wait for the first sample
            if os.path.exists(self.path) and os.path.getsize(self.path) > 20:
                break
            time.sleep(0.05)

    def stop(self) -> None:
        if self.proc.poll() is None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self, t0: float, t1: float) -> dict:
        self.stop()
        max_mhz, samples = None, []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = line.split()
                    if parts and parts[0] == "max":
                        max_mhz = int(parts[1])
                    elif len(parts) == 3:
                        samples.append((float(parts[0]), int(parts[1]), int(parts[2])))
            os.remove(self.path)
        except OSError:
            pass
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": max_mhz, "reasons": ["no NVML samples"], "samples": 0}
        inside = [s for s in samples if t0 <= s[0] <= t1] or [min(samples, key=lambda s: abs(s[0] - t1))]
        mask = 0
        for s in inside:
            mask |= s[2]
        reasons = [name for name, bit in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max_mhz, "reasons": reasons,
                "samples": len(inside)}


# ----------------------------------------------------------------------------- workload

def make_module_and_inputs(cfg: dict, rank: int, device: torch.device):
    from moc import MoC

    torch.manual_seed(1234)  # the same parameters on every rank; data differs per rank
    m = MoC(dim=cfg["D"], z_dim=cfg["Dz"], kernel_size=cfg["S"], k=cfg["K"], activation=cfg["activation"],
            init_std=cfg["init_std"], router_activation=cfg["router"])
    with torch.no_grad():
        m.router.copy_(torch.randn(cfg["K"], cfg["Dz"], generator=torch.Generator().manual_seed(4321)) * cfg["router_std"])
    g = torch.Generator().manual_seed(4321 + 1 + rank)
    m = m.to(device=device, dtype=torch.bfloat16)
    shape = (cfg["B"], cfg["T"])
    host = {
        "x": torch.randn(*shape, cfg["D"], generator=g).bfloat16(),
        "z": torch.randn(*shape, cfg["Dz"], generator=g).bfloat16(),
        "dy": torch.randn(*shape, cfg["D"], generator=g).bfloat16(),
    }
    return m, host


def train_step(m, x, z, dy, reducer=None):
    """Forward + backward of the module; with `reducer` (N > 1) the parameter gradients
    come back summed over ranks by one all-reduce."""
    y, _ = m(x, z)
    grads = torch.autograd.grad(y, (x, z, m.conv_bases, m.router), dy)
    if reducer is not None:
        reducer(grads[2:])
    return y, grads


def time_region(fn, steps: int, stream: torch.cuda.Stream) -> float:
    """ms per call of fn over `steps` calls, CUDA events on `stream`."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def graph_time(fn, reps: int, device: torch.device) -> float:
    """Device time in ms of one fn() call: `reps` calls captured in one CUDA graph and
    replayed, so host launch overhead is excluded (CUDA events on the replay stream)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    stream = torch.cuda.current_stream(device)
    g.replay()
    ms = time_region(g.replay, 3, stream) / reps
    del g
    return ms


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------- CPU baseline

def cpu_baseline(cfg: dict, iters: int = 3, warmup: int = 1) -> dict:
    """The CPU oracle (a port of the reference's moc/reference.py + router, fp32) on the
    host's cores, all threads: config 2 on its full batch (B=4 x T=4096 tokens per step);
    config 5 on one of its 4 sequences per GPU (8192 tokens), tokens/s scaled from that
    sample.  Returns the mean over `iters` timed steps after `warmup` untimed ones."""
    from oracle import moc_oracle as O

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    large = cfg["D"] == CONFIG_LARGE["D"]
    B = 1 if large else cfg["B"]
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, cfg["T"], cfg["D"], generator=g)
    z = torch.randn(B, cfg["T"], cfg["Dz"], generator=g)
    dy = torch.randn(B, cfg["T"], cfg["D"], generator=g)
    w = torch.randn(cfg["K"], cfg["Dz"], generator=g) * cfg["router_std"]
    b = (torch.rand(cfg["K"], cfg["S"], cfg["D"], generator=g) * 2 - 1) * cfg["init_std"] * 3 ** 0.5
    for _ in range(warmup):
        O.module_grads(x, z, w, b, dy, cfg["router"], cfg["activation"], dtype=torch.float32)
    t0 = time.perf_counter()
    for _ in range(iters):
        O.module_grads(x, z, w, b, dy, cfg["router"], cfg["activation"], dtype=torch.float32)
    t = (time.perf_counter() - t0) / iters
    tokens = B * cfg["T"]
    if large:
        sample = (f"1 of the config's {cfg['B']} sequences per GPU ({tokens} tokens), fp32 fwd+bwd, mean of {iters} "
                  f"steps after {warmup} warm-up; tokens/s extrapolated from that sequence")
    else:
        sample = (f"the full config-2 batch ({B} x {cfg['T']} = {tokens} tokens per step), fp32 fwd+bwd, "
                  f"mean of {iters} steps after {warmup} warm-up")
    return {"value": tokens / t, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": sample, "sec_per_iter": t}


DECODE = {"B": 128, "Dz": 4096, "K": 16, "S": 4, "prompt": 512,
          "modules": (("q", 4096, "exp"), ("k", 1024, "exp"), ("v", 1024, "softmax"))}


def decode_bytes_per_step(c: dict) -> int:
    """Algorithmic HBM bytes of one decode step over all modules (bf16): per module x, z
    and y rows, the S-1 cached states read and the S states written, basis and router W."""
    total = 0
    for _, D, _ in c["modules"]:
        total += 2 * c["B"] * (D + c["Dz"] + D + (c["S"] - 1) * D + c["S"] * D)
        total += 2 * c["K"] * c["S"] * D + 2 * c["K"] * c["Dz"]
    return total


def run_decode(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Config 4: q / k / v MoC modules sharing z, caches prefilled from a 512-token prompt,
    then one token per step for every sequence (replicas only for N > 1: each rank decodes
    its own batch, no collective)."""
    from moc import MoC, _lib
    from moc.fused import decode_step

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:  # timing only: barrier and max over ranks
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    c = dict(DECODE)
    if args.batch is not None:
        c["B"] = args.batch
    torch.manual_seed(77)
    mods, caches = [], []
    g = torch.Generator().manual_seed(78 + rank)
    with torch.no_grad():
        z_p = torch.randn(c["B"], c["prompt"], c["Dz"], generator=g).bfloat16().to(device)
        for name, D, ract in c["modules"]:
            m = MoC(dim=D, z_dim=c["Dz"], kernel_size=c["S"], k=c["K"], init_std=0.002, router_activation=ract)
            m.router.copy_(torch.randn(c["K"], c["Dz"], generator=g) * 0.02)
            m = m.to(device=device, dtype=torch.bfloat16)
            x_p = torch.randn(c["B"], c["prompt"], D, generator=g).bfloat16().to(device)
            _, cache = m(x_p, z_p, output_final_state=True)
            mods.append(m)
            caches.append(cache.contiguous())
            del x_p
        del z_p
        host_x = [torch.randn(c["B"], 1, D, generator=g).bfloat16() for _, D, _ in c["modules"]]
        host_z = torch.randn(c["B"], 1, c["Dz"], generator=g).bfloat16()
        xs = [h.to(device) for h in host_x]
        z = host_z.to(device)

        def step():  # one fused decode step: one launch for all modules
            return decode_step(mods, xs, z, caches)

        def step_per_module():  # MoC.step per module: router + update, six launches
            return [m.step(x, z, cache)[0] for m, x, cache in zip(mods, xs, caches)]

        for _ in range(args.warmup):
            step_per_module()
        g_pm = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_pm):
            step_per_module()
        for _ in range(args.warmup):
            g_pm.replay()
        ms_per_module = max_over_ranks(time_region(g_pm.replay, args.steps, torch.cuda.current_stream(device)),
                                       world)
        del g_pm

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        l0 = _lib.launch_count()
        step()
        torch.cuda.synchronize()
        launches_per_step = _lib.launch_count() - l0
        stream = torch.cuda.current_stream(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(args.warmup):
            graph.replay()
        sampler = ClockSampler(device, os.environ.get("TMPDIR", "/tmp"))
        barrier(world)
        t0 = time.time()
        ms = time_region(graph.replay, args.steps, stream)
        t1 = time.time()
        barrier(world)
        ms = max_over_ranks(ms, world)
        clocks = sampler.summary(t0, t1)

        pin_x = [h.pin_memory() for h in host_x]
        pin_z = host_z.pin_memory()
        outs = [torch.empty(c["B"], 1, D, dtype=torch.bfloat16).pin_memory() for _, D, _ in c["modules"]]

        def e2e():
            for d, h in zip(xs, pin_x):
                d.copy_(h, non_blocking=True)
            z.copy_(pin_z, non_blocking=True)
            for o, y in zip(outs, step()):
                o.copy_(y, non_blocking=True)

        for _ in range(2):
            e2e()
        ms_e2e = max_over_ranks(time_region(e2e, max(3, min(args.steps, 50)), stream), world)
        # the same step as a serving loop runs it: copies in, fused step, copies out, all
        # captured in one CUDA graph (no host work per step)
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph):
            e2e()
        e2e_graph.replay()
        ms_e2e_graph = max_over_ranks(time_region(e2e_graph.replay, max(3, min(args.steps, 50)), stream), world)
        del e2e_graph
    nbytes = decode_bytes_per_step(c)
    peaks = measured_peaks()
    line = None
    if rank == 0:
        us = ms * 1e3
        line = {
            "metric": "MoC decode step latency (q, k, v modules)", "value": us, "unit": "us/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "config4: decode, q D=4096 / k D=1024 / v D=1024, z_dim=4096, K=16, S=4, "
                                   f"batch {c['B']}, caches prefilled from a {c['prompt']}-token prompt",
                       "parallelism": f"replicas{world}",
                       "timing": "CUDA graph of one fused decode step (all modules) replayed K times; CUDA events"},
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                         "algorithmic_bytes_per_step": nbytes,
                         "bound_us": nbytes / (peaks["hbm_gbs"] * 1e9) * 1e6},
            "e2e": {"value": ms_e2e * 1e3, "unit": "us/step",
                    "h2d_bytes_per_step": sum(h.numel() * 2 for h in host_x) + host_z.numel() * 2,
                    "d2h_bytes_per_step": sum(o.numel() * 2 for o in outs),
                    "what": "eager: pinned-host copies of x and z in, moc.fused.decode_step, copies of y out",
                    "graph_us": ms_e2e_graph * 1e3},
            "gpu_launches": launches_per_step * args.steps,
            "per_module_path_us": ms_per_module * 1e3,
            "clocks": clocks,
        }
    sampler.stop()
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


def varlen_lengths(total: int, seed: int) -> list[int]:
    """Config 3 sequence lengths: uniform in [64, 4096] from a seeded generator, the last
    one truncated so that they add up to `total`."""
    g = torch.Generator().manual_seed(seed)
    lens, acc = [], 0
    while acc < total:
        n = int(torch.randint(64, 4097, (1,), generator=g))
        n = min(n, total - acc)
        lens.append(n)
        acc += n
    return lens


def run_varlen(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Config 3: 16384 packed tokens of sequences with lengths uniform in [64, 4096], D=Dz=2048,
    K=16, S=4, exp router, fused SiLU; one MoC fwd+bwd per step, captured in a CUDA graph.
    Each rank runs its own packed batch (weak scaling, no collective: replicas)."""
    from moc import MoC, _lib
    import moc.ops as ops

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    total, D, K, S = 16384, 2048, 16, 4
    lens = varlen_lengths(total, 31 + rank)
    cu_cpu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
    cu = cu_cpu.to(device)
    chunks = ops.prepare_chunk_indices(cu, cu_seqlens_cpu=cu_cpu)
    torch.manual_seed(1234)
    m = MoC(dim=D, z_dim=D, kernel_size=S, k=K, activation="silu", init_std=0.002, router_activation="exp")
    with torch.no_grad():
        m.router.copy_(torch.randn(K, D, generator=torch.Generator().manual_seed(4321)) * 0.02)
    m = m.to(device=device, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(99 + rank)
    x = torch.randn(1, total, D, generator=g).bfloat16().to(device).requires_grad_()
    z = torch.randn(1, total, D, generator=g).bfloat16().to(device).requires_grad_()
    dy = torch.randn(1, total, D, generator=g).bfloat16().to(device)
    maxlen = max(lens)

    def step():
        y, _ = m(x, z, cu_seqlens=cu, max_seqlen=maxlen, chunk_indices=chunks)
        return torch.autograd.grad(y, (x, z, m.conv_bases, m.router), dy)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    l0 = _lib.launch_count()
    step()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - l0
    stream = torch.cuda.current_stream(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    sampler = ClockSampler(device, os.environ.get("TMPDIR", "/tmp"))
    barrier(world)
    t0 = time.time()
    ms = time_region(graph.replay, args.steps, stream)
    t1 = time.time()
    barrier(world)
    ms = max_over_ranks(ms, world)
    clocks = sampler.summary(t0, t1)
    nbytes = step_bytes_per_token(D, D, K) * total
    peaks = measured_peaks()
    line = None
    if rank == 0:
        line = {
            "metric": "MoC varlen fwd+bwd tokens/s", "value": total * world / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "config3: packed varlen MoC fwd+bwd, 16384 tokens, lengths U[64,4096], "
                                   "D=z_dim=2048, K=16, S=4, exp router, SiLU",
                       "n_seqs": len(lens), "parallelism": f"replicas{world}",
                       "timing": "CUDA graph of one step replayed K times; CUDA events"},
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                         "algorithmic_bytes_per_step": nbytes},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
    sampler.stop()
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


PROJ = {"B": 4, "T": 4096, "d_model": 4096, "K": 16, "S": 4,
        "modules": (("q", 4096, "exp"), ("k", 1024, "exp"), ("v", 1024, "softmax"))}


def run_proj(args, rank: int, world: int, local_rank: int) -> dict | None:
    """The fused projection + convolution forward: the q / k / v MoC modules of an attention
    block (README.md:115-129) at config 4's widths, prefill of B=4 x T=4096 tokens.  One step
    is the three routers and one moc_proj_forward_multi over qkv_proj.weight (h read once),
    captured in a CUDA graph; beside it the unfused path (one cuBLAS qkv GEMM, then each
    module's MoC forward on its slice).  Each rank runs its own batch (replicas)."""
    from moc import MoC, _lib, fused
    import moc.ops as ops

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    c = PROJ
    B, T, Dm = (c["B"] if args.batch is None else args.batch), c["T"], c["d_model"]
    torch.manual_seed(1234)
    mods = []
    for name, D, ract in c["modules"]:
        m = MoC(dim=D, z_dim=Dm, kernel_size=c["S"], k=c["K"], init_std=0.002, router_activation=ract)
        with torch.no_grad():
            m.router.normal_(0.0, 0.02)
        mods.append(m.to(device=device, dtype=torch.bfloat16))
    g = torch.Generator().manual_seed(77 + rank)
    d_total = sum(D for _, D, _ in c["modules"])
    w_qkv = (torch.randn(d_total, Dm, generator=g) / Dm ** 0.5).bfloat16().to(device)
    h = torch.randn(B, T, Dm, generator=g).bfloat16().to(device)  # x_norm: projected and routing input
    offs = [0]
    for _, D, _ in c["modules"]:
        offs.append(offs[-1] + D)
    w_rows = [w_qkv[offs[i]:offs[i + 1]] for i in range(len(mods))]

    def step_fused():  # inference: no autograd graph, so the launch writes y only
        with torch.no_grad():
            return fused.proj_forward_multi(h, w_qkv, mods, z=h)

    def q_only():
        with torch.no_grad():
            return fused.proj_forward(h, w_rows[0], mods[0], alpha=alpha_q)

    def step_unfused():
        with torch.no_grad():
            qkv = torch.matmul(h, w_qkv.T)
            return [m(qkv[..., offs[i]:offs[i + 1]], h)[0] for i, m in enumerate(mods)]

    # parity of the two paths on this workload (bf16 tolerance of the convolution tests)
    for a_, b_ in zip(step_fused(), step_unfused()):
        err = float((a_.float() - b_.float()).abs().max() / b_.float().abs().max().clamp_min(1e-30))
        assert err <= 2e-2, f"fused and unfused paths differ: {err:.3e}"
    for _ in range(args.warmup):
        step_fused()
    torch.cuda.synchronize()
    l0 = _lib.launch_count()
    step_fused()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - l0
    stream = torch.cuda.current_stream(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step_fused()
    for _ in range(args.warmup):
        graph.replay()
    sampler = ClockSampler(device, os.environ.get("TMPDIR", "/tmp"))
    barrier(world)
    t0 = time.time()
    ms = time_region(graph.replay, args.steps, stream)
    t1 = time.time()
    barrier(world)
    ms = max_over_ranks(ms, world)
    clocks = sampler.summary(t0, t1)
    ms_unfused = graph_time(step_unfused, max(3, min(args.steps, 10)), device)
    # the fused kernel alone on the widest module (router output precomputed)
    alpha_q = ops.launch_router_forward(h, mods[0].router.detach(), mods[0].router_activation)
    k_ms = graph_time(q_only, max(3, min(args.steps, 10)), device)
    k_flops = 2.0 * B * T * Dm * mods[0].dim
    # the training step of the same block: forward + backward of h, qkv_proj.weight and every
    # module's conv_bases and router, fused (the launch keeps each module's x for the backward)
    # against unfused (the projection GEMM writes qkv, each module reads its slice back)
    hq = h.detach().clone().requires_grad_()
    wq = w_qkv.detach().clone().requires_grad_()
    params = [p for m in mods for p in (m.conv_bases, m.router)]
    dys = [torch.randn(B, T, D, generator=g).bfloat16().to(device) for _, D, _ in c["modules"]]

    def train_fused():
        return torch.autograd.grad(fused.proj_forward_multi(hq, wq, mods, z=hq), [hq, wq] + params, grad_outputs=dys)

    def train_unfused():
        qkv = torch.matmul(hq, wq.T)
        ys = [m(qkv[..., offs[i]:offs[i + 1]], hq)[0] for i, m in enumerate(mods)]
        return torch.autograd.grad(ys, [hq, wq] + params, grad_outputs=dys)

    for a_, b_ in zip(train_fused(), train_unfused()):
        err = float((a_.float() - b_.float()).abs().max() / b_.float().abs().max().clamp_min(1e-30))
        assert err <= 2e-2, f"fused and unfused training gradients differ: {err:.3e}"
    reps = max(3, min(args.steps, 10))
    ms_train = max_over_ranks(graph_time(train_fused, reps, device), world)
    ms_train_unfused = max_over_ranks(graph_time(train_unfused, reps, device), world)
    peaks = measured_peaks()
    peak_tf = peaks.get("bf16_tflops", FALLBACK_BF16_TFLOPS)
    tokens = B * T
    line = None
    if rank == 0:
        line = {
            "metric": "MoC q/k/v projection + convolution prefill tokens/s", "value": tokens * world / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "fused projection (next-step item 2): q D=4096 / k D=1024 / v D=1024 MoC modules "
                                   "over d_model=4096, B=4, T=4096, K=16, S=4, routers exp/exp/softmax",
                       "parallelism": f"replicas{world}",
                       "timing": "CUDA graph of one step (3 routers + 1 fused launch for q, k, v) replayed K times; "
                                 "CUDA events"},
            "unfused_ms_per_step": ms_unfused,
            "unfused": "cuBLAS qkv GEMM (torch.matmul) + each module's router and MoC forward on its slice",
            "train_ms_per_step": ms_train, "train_unfused_ms_per_step": ms_train_unfused,
            "train": "forward + backward (gradients of h, qkv_proj.weight, each module's conv_bases and router): "
                     "fused = one moc_proj_forward_multi_save launch keeping each module's x, then per module "
                     "moc_backward and the router backward, then the dh / dweight GEMMs (cuBLAS) over the modules' "
                     "dx; unfused = the same through the qkv GEMM and each module's autograd; CUDA graph, CUDA events",
            "roofline": {"bound": "tensor", "kernel": "k_proj_conv (q module, D=4096)", "achieved": k_flops / (k_ms * 1e-3) / 1e12,
                         "peak": peak_tf, "peak_source": "measured" if "bf16_tflops" in peaks else "fallback",
                         "unit": "TFLOP/s", "frac": k_flops / (k_ms * 1e-3) / 1e12 / peak_tf,
                         "launch_ms": k_ms, "algorithmic_flops_per_launch": k_flops,
                         "note": "projection FLOPs only; the 8 recomputed halo rows per 120 output rows and the "
                                 "per-sequence tile padding are extra work not counted"},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
    sampler.stop()
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


def bench_config(cfg: dict, world: int) -> dict:
    """The workload description both arms print."""
    b = cfg["B"]
    if cfg["D"] == CONFIG_LARGE["D"]:
        name = (f"config5: large data-parallel MoC fwd+bwd, B={b} per GPU (B={b * world} over {world}), T=8192, "
                "D=z_dim=4096 K=32 S=8 bf16 softmax, fan-in init")
    else:
        name = f"config2: MoC module fwd+bwd, B={b} T=4096 D=z_dim=2048 K=16 S=4 bf16 softmax"
    if b != (CONFIG_LARGE if cfg["D"] == CONFIG_LARGE["D"] else CONFIG)["B"]:
        name += " (reduced batch, --batch)"
    in_mib = 3 * cfg["B"] * cfg["T"] * cfg["D"] * 2 // (1 << 20)
    return {"workload": name,
            "global_batch": cfg["B"] * world, "seq_len": cfg["T"], "D": cfg["D"], "z_dim": cfg["Dz"],
            "K": cfg["K"], "S": cfg["S"], "parallelism": f"dp{world}",
            "l2": f"inputs larger than L2 (x, z, dy = {in_mib} MiB per rank)",
            "timing": "CUDA graph of one step replayed K times; CUDA events; max over ranks"}


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's CPU path of the step (the oracle port of
    moc/reference.py + the router, fp32) on the host's cores, K timed steps after W warm-up
    steps, each the whole config-2 batch (config 5: one of its sequences).  Rank 0 only."""
    if rank != 0:
        return
    cfg = dict(CONFIG_LARGE if args.workload == "large" else CONFIG)
    base = cpu_baseline(cfg, iters=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": base["sec_per_iter"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(cfg, world),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference CPU path: oracle port of moc/reference.py + router (the reference is Python; "
                "its GPU path is Triton, timed separately in profiles/)",
    }
    print(json.dumps(line), flush=True)


def run_triton_reference(args) -> None:
    """The reference's own GPU path (its Triton kernels, the unmodified package installed in
    baseline/_ref) at config 2 on one GPU, beside this library's figures in profiles/: each
    operation and the module step as CUDA-graph replays timed with CUDA events.  Imports the
    reference's `moc` instead of this library's, so it runs alone in its process."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "moc")):
        print(json.dumps({"impl": "reference-triton", "unavailable": "the reference is not installed in baseline/_ref"}))
        return
    sys.path.insert(0, ref_dir)
    import moc as rmoc  # noqa: E402  (the reference package)
    from moc import ops as rops  # noqa: E402

    if not rmoc.__file__.startswith(ref_dir):
        raise RuntimeError(f"expected the reference package, imported {rmoc.__file__}")
    dev = torch.device("cuda", 0)
    side = torch.cuda.Stream(dev)
    torch.cuda.set_stream(side)  # every launch, warm-up included, on one non-default stream
    B, T, D, Dz, K, S = CONFIG["B"], CONFIG["T"], CONFIG["D"], CONFIG["Dz"], CONFIG["K"], CONFIG["S"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, T, D, generator=g).bfloat16().to(dev)
    z = torch.randn(B, T, Dz, generator=g).bfloat16().to(dev)
    dy = torch.randn(B, T, D, generator=g).bfloat16().to(dev)
    m = rmoc.MoC(dim=D, z_dim=Dz, kernel_size=S, k=K, init_std=0.002, router_activation="softmax")
    with torch.no_grad():
        m.router.normal_(0, 0.02)
    m = m.to(device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        alpha = torch.softmax(torch.nn.functional.linear(z, m.router), -1)
    basis = m.conv_bases.detach()

    def gtime(fn, reps=20):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            for _ in range(reps):
                fn()
        gr.replay()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(side)
        for _ in range(3):
            gr.replay()
        s1.record(side)
        torch.cuda.synchronize()
        return s0.elapsed_time(s1) / (3 * reps)

    xx, zz = x.clone().requires_grad_(), z.clone().requires_grad_()

    def step():
        y, _ = m(xx, zz)
        torch.autograd.grad(y, (xx, zz, m.conv_bases, m.router), dy)

    zr, wr = z.clone().requires_grad_(), m.router.detach().clone().requires_grad_()

    def router_fb():
        a = torch.softmax(torch.nn.functional.linear(zr, wr), -1)
        torch.autograd.grad(a, (zr, wr), alpha)

    t0 = time.time()
    for _ in range(2):  # the Triton autotuners run here
        step()
    torch.cuda.synchronize()
    res = {"impl": "reference-triton", "config": "config2: B=4 T=4096 D=z_dim=2048 K=16 S=4 bf16 softmax",
           "warmup_autotune_s": time.time() - t0, "triton": __import__("triton").__version__,
           "gpu": torch.cuda.get_device_name(0)}
    res["conv_forward_ms"] = gtime(lambda: rops.launch_forward(x, alpha, basis, activation_flag=0))
    res["conv_backward_ms"] = gtime(lambda: rops.launch_backward(x, alpha, basis, dy, dy, activation_flag=0,
                                                                  need_x=True))
    with torch.no_grad():
        res["router_forward_ms"] = gtime(lambda: torch.softmax(torch.nn.functional.linear(z, m.router), -1))
    res["router_fwd_bwd_ms"] = gtime(router_fb)
    res["module_step_ms"] = gtime(step, reps=10)
    res["tokens_per_s"] = B * T / (res["module_step_ms"] * 1e-3)
    print(json.dumps(res), flush=True)


# ----------------------------------------------------------------------------- main

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--triton-reference", action="store_true",
                    help="time the reference's own Triton GPU path (baseline/_ref) at config 2 and exit")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-workloads", action="store_true",
                    help="with the default workload on one GPU, skip the short varlen / decode / large runs "
                         "reported under the line's 'workloads' key")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per rank for train / large / proj / decode (a smaller case for ncu "
                         "captures, or a decode batch sweep; default: the config's)")
    ap.add_argument("--workload", choices=("train", "decode", "varlen", "large", "proj"), default="train",
                    help="train: config 2 (the headline); decode: config 4, three modules, batch 128; "
                         "varlen: config 3, packed sequences, exp router, SiLU; large: config 5, "
                         "4 sequences of 8192 tokens per GPU, D=4096, K=32, S=8; proj: the fused projection + "
                         "convolution forward of q/k/v modules (prefill)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.triton_reference:
        run_triton_reference(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    runners = {"train": run_train, "large": run_train, "decode": run_decode, "varlen": run_varlen, "proj": run_proj}
    line = runners[args.workload](args, rank, world, local_rank)
    if line is not None and args.workload == "train" and world == 1 and not args.no_extra_workloads:
        # the other BASELINE workloads, short runs on the same GPU, reported in the same line
        extra = {}
        for name in ("varlen", "decode", "large", "proj"):
            sub = argparse.Namespace(**vars(args))
            sub.workload, sub.steps, sub.warmup, sub.batch = name, min(args.steps, 20), 3, None
            sub.no_cpu_baseline = True
            torch.cuda.empty_cache()
            extra[name] = summarize(runners[name](sub, rank, world, local_rank))
        line["workloads"] = extra
    if line is not None:
        print(json.dumps(line), flush=True)


def summarize(line: dict) -> dict:
    """The keys of a workload's line that the headline line carries for it."""
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "higher_is_better", "config", "roofline",
            "kernel_ms", "e2e", "per_module_path_us", "gpu_launches", "clocks", "step_hbm_frac",
            "unfused_ms_per_step", "train_ms_per_step", "train_unfused_ms_per_step")
    return {k: line[k] for k in keep if k in line}


def run_train(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Config 2 (``--workload train``, the headline) or config 5 per GPU (``large``): the MoC
    module's training step, one batch per rank (weak scaling); for N > 1 the step adds the one
    all-reduce of [dconv_bases | drouter]."""
    from moc import _lib, dp

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    cfg = dict(CONFIG_LARGE if args.workload == "large" else CONFIG)
    if args.batch is not None:
        cfg["B"] = args.batch
    N_rank = cfg["B"] * cfg["T"]

    m, host = make_module_and_inputs(cfg, rank, device)
    x = host["x"].to(device).requires_grad_()
    z = host["z"].to(device).requires_grad_()
    dy = host["dy"].to(device)
    # the step's one collective: this library's NVLink all-reduce (MOC_ALLREDUCE=nccl: NCCL)
    reducer = None
    if world > 1:
        if os.environ.get("MOC_ALLREDUCE", "nvlink") != "nccl":
            try:  # every rank raises together if any rank cannot set up peer access
                reducer = dp.NVLinkGradAllReduce([m.conv_bases, m.router])
            except RuntimeError as e:
                print(f"rank {rank}: NVLink all-reduce unavailable ({e}); using NCCL", file=sys.stderr)
        if reducer is None:
            reducer = dp.GradAllReduce([m.conv_bases, m.router])

    # --- device-resident step, captured in a CUDA graph
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(args.warmup):  # (N > 1: NCCL communicator set up before the capture)
            train_step(m, x, z, dy, reducer)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    train_step(m, x, z, dy, reducer)
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - launches0

    # one graph per step: router + conv forward and backward, and for N > 1 the one
    # all-reduce of [dconv_bases | drouter]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _, g_grads = train_step(m, x, z, dy, reducer)
    stream = torch.cuda.current_stream(device)

    def graph_step():
        graph.replay()

    for _ in range(args.warmup):
        graph_step()
    sampler = ClockSampler(device, os.environ.get("TMPDIR", "/tmp"))
    barrier(world)
    t_wall0 = time.time()
    ms_step = time_region(graph_step, args.steps, stream)
    t_wall1 = time.time()
    barrier(world)
    ms_step = max_over_ranks(ms_step, world)
    clocks = sampler.summary(t_wall0, t_wall1)

    # --- end to end through the public API, host buffers.  Every step copies its inputs
    # x, z, dy from pinned host memory and reads the step's result (the parameter
    # gradients dconv_bases, drouter) back to pinned host memory.  Two device input slots
    # let the copy engine bring step n+1's inputs in while step n computes.
    pin = {k: v.pin_memory() for k, v in host.items()}
    out_host = {
        "dbasis": torch.empty(m.conv_bases.shape, dtype=torch.bfloat16).pin_memory(),
        "drouter": torch.empty(m.router.shape, dtype=torch.bfloat16).pin_memory(),
    }
    slots = [{k: torch.empty_like(v, device=device) for k, v in host.items()} for _ in range(2)]
    copy_stream = torch.cuda.Stream(device)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def h2d(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(used[slot])  # the step that last read this slot is done
            for k, v in pin.items():
                slots[slot][k].copy_(v, non_blocking=True)
            h2d_done[slot].record(copy_stream)

    def e2e_run(n_steps):
        copy_stream.wait_stream(stream)  # the copies start inside the timed region
        h2d(0)
        for n in range(n_steps):
            if n + 1 < n_steps:
                h2d((n + 1) % 2)
            sl = slots[n % 2]
            stream.wait_event(h2d_done[n % 2])
            xg = sl["x"].detach().requires_grad_()
            zg = sl["z"].detach().requires_grad_()
            _, grads = train_step(m, xg, zg, sl["dy"], reducer)
            used[n % 2].record(stream)
            out_host["dbasis"].copy_(grads[2], non_blocking=True)
            out_host["drouter"].copy_(grads[3], non_blocking=True)

    for ev in used:
        ev.record(stream)
    e2e_steps = max(3, min(args.steps, 10))
    e2e_run(2)
    barrier(world)
    ms_e2e = max_over_ranks(time_region(lambda: e2e_run(e2e_steps), 1, stream) / e2e_steps, world)
    h2d_bytes = sum(t.numel() * t.element_size() for t in pin.values())
    d2h_bytes = sum(t.numel() * t.element_size() for t in out_host.values())

    # --- per-kernel timing for the roofline (each C-ABI call timed alone)
    import moc.ops as ops

    xa = x.detach()
    with torch.no_grad():
        alpha = ops.launch_router_forward(z.detach(), m.router.detach(), cfg["router"])
    basis = m.conv_bases.detach()
    kernel_calls = {
        "router_forward": lambda: ops.launch_router_forward(z.detach(), m.router.detach(), cfg["router"]),
        "conv_forward": lambda: ops.launch_forward(xa, alpha, basis, activation_flag=0),
        "conv_backward": lambda: ops.launch_backward(xa, alpha, basis, dy, dy, activation_flag=0, need_x=True),
        "router_backward": lambda: ops.launch_router_backward(z.detach(), m.router.detach(), alpha, alpha,
                                                              cfg["router"]),
    }
    kernel_ms = {}
    reps = max(5, min(args.steps, 20))
    for name, fn in kernel_calls.items():
        kernel_ms[name] = graph_time(fn, reps, device)
    allreduce_ms = None
    if reducer is not None:  # every rank: the same collectives in the same order
        gcopy = [g.clone() for g in g_grads[2:]]
        barrier(world)
        allreduce_ms = max_over_ranks(time_region(lambda: reducer(gcopy), 10, stream), world)
    if hasattr(reducer, "check"):  # every rank: raises on all of them if any call gave up waiting
        reducer.check()
    dominant = max(kernel_ms, key=kernel_ms.get)
    peaks = measured_peaks()
    kbytes = KERNEL_BYTES_PER_TOKEN[dominant](cfg) * N_rank
    achieved = kbytes / (kernel_ms[dominant] * 1e-3) / 1e9
    traffic = profiled_traffic(dominant if args.workload == "train" else f"{args.workload}:{dominant}")

    step_bytes = step_bytes_per_token(cfg["D"], cfg["Dz"], cfg["K"]) * N_rank
    tokens_all = N_rank * world

    line = None
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": tokens_all / (ms_step * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": bench_config(cfg, world),
            "achieved_gbs": step_bytes / (ms_step * 1e-3) / 1e9,
            "step_hbm_frac": step_bytes / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "peak_source": peaks["source"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": traffic, "launch_ms": kernel_ms[dominant],
                         "algorithmic_bytes_per_launch": kbytes},
            "kernel_ms": kernel_ms,
            "grad_allreduce_ms": allreduce_ms,
            "grad_allreduce": type(reducer).__name__ if reducer is not None else None,
            "e2e": {"value": tokens_all / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": d2h_bytes, "ms_per_step": ms_e2e,
                    "what": "MoC module step through the public API (eager); x, z, dy copied in from pinned host "
                            "memory every step (double-buffered, overlapping the previous step) and the step's "
                            "parameter gradients read back"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            base = cpu_baseline(cfg)
            line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}

    sampler.stop()
    del graph
    if world > 1:
        dist.barrier()
        if hasattr(reducer, "close"):
            reducer.close()
        dist.barrier()
        dist.destroy_process_group()
    return line


def profiled_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` at this workload, from the committed ncu summary
    (profiles/*.md line 'traffic_bytes_per_launch <kernel> <bytes>'), else None."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if not name.endswith(".md"):
            continue
        with open(os.path.join(pdir, name)) as f:
            for line in f:
                parts = line.strip().strip("`").split()
                if len(parts) == 3 and parts[0] == "traffic_bytes_per_launch" and parts[1] == kernel:
                    return float(parts[2])
    return None


if __name__ == "__main__":
    main()
