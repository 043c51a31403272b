"""Benchmark: attention fwd+bwd TFLOP/s on B200 (1..8 GPUs), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload (default "c4"): causal fwd+bwd, B=8, S=8192, H=32, D=128, fp16,
q/k/v/dO ~ N(0,1) from seeded generators (synthetic data).  The 256
(batch, head) pairs are split by batch across the N ranks with no collective
(strong scaling: the total work is fixed).  One step = out = flash_attn(q, k, v,
causal=True); out.backward(dO) through the public autograd API.
FLOPs (benchmark convention): 4*B*H*S^2*D, halved for causal; fwd+bwd = 2.5x.

Extra keys beside the base contract:
  e2e          the same step with pinned-host inputs copied in and O, dQ, dK,
               dV copied back inside the timed region (copies of neighbouring
               steps overlap the compute: three streams, double-buffered inputs).
  roofline     the dominant kernel (the main backward kernel) timed alone with
               CUDA events; achieved = its algorithmic tensor FLOPs (5 GEMMs,
               2.5 x F_fwd) / its median duration; peak = MEASURED_PEAKS.json.
  cpu_baseline the reference's fp32 eager path (flash_attn_volta/ref.py from the
               unmodified package in baseline/_ref; the oracle restatement of it
               only where that copy is missing) on 8 (batch, head) pairs of the
               same workload, rank 0, N=1, extrapolated by FLOPs.
  headline_c3b the headline config (B=1, S=4096, H=8, D=128, causal) at N=1,
               with config 3's D=64 case (B=1, S=4096, H=16) under "c3a": fwd+bwd
               through the autograd API and the forward with LSE alone.
  clocks       nvidia-smi samples taken during the timed region.
--impl reference times the same CPU path on all host cores, each step = fwd+bwd
of 8 (batch, head) pairs of the workload; under torchrun only rank 0 runs it.
--impl reference-triton (informational) runs the reference's Triton kernels on
the GPU through its public API.
"""
from __future__ import annotations

import argparse
import contextlib
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

WORKLOADS = {
    # name: (B, S, H, D, causal, amp)
    "c4": (8, 8192, 32, 128, True, 1.0),
    "c3b": (1, 4096, 8, 128, True, 0.5),
    "c3a": (1, 4096, 16, 64, True, 0.5),
    "c1": (2, 1024, 8, 64, False, 1.0),
    # profiling case: the c4 shape with 1/16 of its (batch, head) pairs; q, k, v,
    # o, dO together (160 MiB) exceed L2, one launch is a few hundred us
    "p8k": (1, 8192, 16, 128, True, 1.0),
}
L2_BYTES = 126 * 1000 * 1000


# DRAM bytes (read + write) per launch of the main backward kernel over the
# workload's whole batch, from ncu (dram__bytes_read.sum + dram__bytes_write.sum)
# and where it came from; the summaries are under profiles/.
BWD_TRAFFIC_PER_LAUNCH = {
    "c4": (5.76e9, "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full c4 launch "
                   "(3.48 GB + 2.28 GB, 1 pass; profiles/traffic_c4_fwd_bwd_main.md)"),
}


def flops_fwd(B, S, H, D, causal):
    f = 4.0 * B * H * S * S * D
    return f * 0.5 if causal else f


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), "measured"
    return 1590.0, 1400.0, "fallback"


def load_hbm_peak():
    """Measured HBM copy bandwidth (GB/s) and its kind."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            v = json.load(f).get("hbm_gbs")
        if v:
            return float(v), "measured"
    return 6650.0, "fallback"


def merge_roofline(dev, rows, H, D, reps=20):
    """fa_sm100_merge (the ring's LSE merge) on one block of the ring's size:
    B=1, `rows` query rows, H heads, fp16 block output, not the first block.
    Algorithmic bytes per launch: read the fp32 running O and the block's O,
    write the running O (10 B per element), and per row read both LSEs and write
    one (12 B).  Median of `reps` CUDA-event timed launches; the tensors are
    larger than L2."""
    from flash_attn_volta_b200 import ops
    ops.load()
    acc_o = torch.zeros((1, rows, H, D), device=dev, dtype=torch.float32)
    acc_lse = torch.zeros((1, H, rows), device=dev, dtype=torch.float32)
    o = torch.randn((1, rows, H, D), device=dev, dtype=torch.float16)
    lse = torch.randn((1, H, rows), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        torch.ops.fav.merge_(acc_o, acc_lse, o, lse, False)
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        torch.ops.fav.merge_(acc_o, acc_lse, o, lse, False)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = float(statistics.median(times))
    nbytes = rows * H * D * (4 + 2 + 4) + rows * H * (4 + 4 + 4)
    achieved = nbytes / (ms * 1e-3) / 1e9
    peak, kind = load_hbm_peak()
    return {"kernel": "fa_merge_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "peak_kind": f"{kind} HBM copy",
            "bytes_per_launch": nbytes, "median_ms": ms,
            "shape": {"B": 1, "rows": rows, "H": H, "D": D}}


def gen_shard(B0, B1, S, H, D, amp, device, seed_base=1234):
    """q, k, v, dO for batches [B0, B1) — each batch index has its own seed so
    every GPU count sees the same global tensors."""
    outs = [torch.empty((B1 - B0, S, H, D), dtype=torch.float16, device=device) for _ in range(4)]
    for i, b in enumerate(range(B0, B1)):
        g = torch.Generator(device=device).manual_seed(seed_base + b)
        for t in outs:
            t[i].normal_(0.0, 1.0, generator=g)
            if amp != 1.0:
                t[i].mul_(amp)
    return outs


# ----------------------------------------------------------------------- clocks
_NVML_SAMPLER = r"""
import sys, time, pynvml
pynvml.nvmlInit()
uuid, idx, period = sys.argv[1], int(sys.argv[2]), float(sys.argv[3])
try:
    h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(idx)
mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
print("ready", flush=True)
while True:
    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    print(sm, mx, bits, flush=True)
    time.sleep(period)
"""


class ClockSampler:
    """SM clock and clock-event reasons sampled during a timed region.

    A child process reads NVML every 5 ms (the GPU matched to the CUDA device
    by UUID), else `nvidia-smi -lms 50`.  Only reads; changes nothing."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.kind = None

    def start(self):
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.gpu_index).uuid)
            self.proc = subprocess.Popen(
                [sys.executable, "-c", _NVML_SAMPLER, uuid, str(self.gpu_index), "0.005"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            if self.proc.stdout.readline().strip() == "ready":
                self.kind = "nvml"
                return
            self.proc.kill()
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.kind = "nvidia-smi"
        except Exception:
            self.proc = None

    def _collect(self):
        if self.kind == "nvml":
            time.sleep(0.01)  # a timed region shorter than the period still gets a sample
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return out

    def stop(self):
        if self.proc is None:
            return None
        out = self._collect()
        if self.kind == "nvml":
            rows = []
            for line in out.splitlines():
                f = line.split()
                if len(f) == 3 and all(x.isdigit() for x in f):
                    rows.append(tuple(int(x) for x in f))
            if not rows:
                return None
            reasons = sorted({n for _, _, bits in rows for n, m in self.REASONS if bits & m})
            return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                    "reasons": reasons, "samples": len(rows), "source": "nvml, 5 ms"}
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi, 50 ms"}


def gpu_local_cpus(index):
    """CPUs that NVML reports as closest to CUDA device `index` (those this
    process may run on), or an empty set when that is unknown."""
    try:
        import pynvml
        p = torch.cuda.get_device_properties(index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 1) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        return cpus & os.sched_getaffinity(0)
    except Exception:
        return set()


@contextlib.contextmanager
def near_gpu(index):
    """Run the body on the CPUs local to GPU `index`, so that host memory first
    touched there (pinned buffers: their pages are mapped when allocated) sits
    on the GPU's NUMA node; the previous affinity is restored on exit.  Yields
    whether the GPU's CPUs were known."""
    cpus = gpu_local_cpus(index)
    old = os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield bool(cpus)
    finally:
        if cpus:
            os.sched_setaffinity(0, old)


# ----------------------------------------------------------------------- CPU path
def cpu_reference():
    """The reference's own CPU attention (flash_attn_volta/ref.py:9-36,
    attention_ref) from the unmodified package installed in baseline/_ref, loaded
    as a single module (its package __init__ would import the Triton kernels);
    else this repo's oracle restatement of it.  Returns (fn, kind) with
    fn(q, k, v, causal) -> fp32 output."""
    path = os.path.join(ROOT, "baseline", "_ref", "flash_attn_volta", "ref.py")
    if os.path.exists(path):
        import importlib.util
        spec = importlib.util.spec_from_file_location("_fav_reference_ref", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return (lambda q, k, v, causal: mod.attention_ref(q, k, v, causal=causal,
                                                           dtype_out=torch.float32)), "reference"
    from oracle.attention_oracle import attention_fwd
    return (lambda q, k, v, causal: attention_fwd(q, k, v, causal=causal,
                                                  dtype=torch.float32)[0]), "port"


def cpu_pair_step(fn, S, D, causal, amp, seed=0):
    """One fwd+bwd of one (batch, head) pair through the CPU reference (fp32
    leaves made from seeded fp16 inputs, as the reference's tests do)."""
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = [(torch.randn((1, S, 1, D), generator=g) * amp).half() for _ in range(4)]
    leaves = [t.float().requires_grad_() for t in (q, k, v)]
    t0 = time.perf_counter()
    o = fn(*leaves, causal)
    o.backward(do.float())
    return time.perf_counter() - t0


def cpu_model():
    """Host CPU model name (from /proc/cpuinfo), or None."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


CPU_PAIRS = 8  # (batch, head) pairs per CPU sample, extrapolated by FLOPs


def cpu_baseline(S, D, causal, amp, budget_s=20.0):
    """Median over up to 3 samples of CPU_PAIRS (b, h) pairs each (about 10-30 s
    of CPU work at S=8192), after one warm-up pair."""
    torch.set_num_threads(os.cpu_count() or 1)
    fn, kind = cpu_reference()
    cpu_pair_step(fn, min(S, 1024), D, causal, amp)  # warm-up
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start < budget_s and len(times) < 3):
        times.append(sum(cpu_pair_step(fn, S, D, causal, amp, seed=100 * len(times) + p)
                         for p in range(CPU_PAIRS)))
    t = statistics.median(times)
    f = CPU_PAIRS * 2.5 * flops_fwd(1, S, 1, D, causal)
    return {"value": f / t / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": kind, "cpu_model": cpu_model(),
            "sample": f"median of {len(times)} samples, each fwd+bwd of {CPU_PAIRS} (batch, head) "
                      f"pairs, S={S}, D={D}, causal={causal}, fp32 "
                      f"({'flash_attn_volta/ref.py attention_ref + autograd' if kind == 'reference' else 'oracle restatement of ref.py'}), "
                      f"{t:.2f} s per sample; extrapolated to the workload by FLOPs"}


def run_reference(args, wl):
    """The driver's reference arm: the reference's CPU path on this host's cores,
    each step fwd+bwd of CPU_PAIRS (batch, head) pairs of the workload."""
    world, rank, _ = dist_env()
    B, S, H, D, causal, amp = WORKLOADS[wl]
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    fn, kind = cpu_reference()
    step = lambda i: sum(cpu_pair_step(fn, S, D, causal, amp, seed=CPU_PAIRS * i + p)  # noqa: E731
                         for p in range(CPU_PAIRS))
    for i in range(args.warmup):
        step(1000 + i)
    times = [step(i) for i in range(args.steps)]
    t = sum(times)
    f = CPU_PAIRS * 2.5 * flops_fwd(1, S, 1, D, causal) * len(times)
    val = f / t / 1e12
    line = {
        "impl": "reference", "metric": "attention fwd+bwd TFLOP/s", "value": val,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / len(times), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl, "B": B, "S": S, "H": H, "D": D, "causal": causal,
                   "step": f"fwd+bwd of {CPU_PAIRS} (batch, head) pairs on the host CPU",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": kind, "cpu_model": cpu_model(),
                         "sample": f"{len(times)} steps x {CPU_PAIRS} (b,h) pairs, S={S}, D={D}"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------- GPU path
def time_steps(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def run_ours(args, wl):
    import torch.distributed as dist
    from flash_attn_volta_b200 import _lib, check_status, flash_attn, flash_attn_forward
    from flash_attn_volta_b200.forward import _stream_ptr

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, S, H, D, causal, amp = WORKLOADS[wl]
    assert B % world == 0, f"batch {B} not divisible by {world} GPUs"
    # The headline config is timed first: right after the large workload the
    # SM clock stays in the power-capped state (1672 vs 1965 MHz, measured with
    # NVML) for a few seconds and the same small step takes ~20 % longer.  Its
    # own clock samples are reported beside it.
    headline = None
    if rank == 0 and world == 1 and wl != "c3b" and not args.kernels_only:
        hl_clocks = ClockSampler(local)
        hl_clocks.start()
        headline = bench_small("c3b", dev, args)
        headline["c3a"] = bench_small("c3a", dev, args)
        headline["host_us_per_call"] = host_cost_us(dev)
        headline["cuda_graph"] = graph_vs_eager_us(dev)
        headline["clocks"] = hl_clocks.stop()
    mem_c3a = peak_mem_fwd_bwd(dev, 1, 4096, 16, 64, True)
    torch.cuda.empty_cache()
    b0, b1 = rank * B // world, (rank + 1) * B // world
    q, k, v, do = gen_shard(b0, b1, S, H, D, amp, dev)
    q.requires_grad_(); k.requires_grad_(); v.requires_grad_()
    stream = torch.cuda.current_stream(dev)

    det = True if args.deterministic else None

    def step():
        q.grad = k.grad = v.grad = None
        out = flash_attn(q, k, v, causal=causal, deterministic=det)
        out.backward(do)

    torch.cuda.synchronize(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    mem0 = torch.cuda.memory_allocated(dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    check_status(dev)
    # extra device memory of one step beyond its inputs (the output, LSE, the
    # gradients and the backward's workspace), the reference's bench/memory.py metric
    step_peak_mib = (torch.cuda.max_memory_allocated(dev) - mem0) / 2**20
    # power soak: untimed steps until the GPU has run this load for
    # --soak-s seconds, so every GPU count is timed in the same (power-capped)
    # state instead of a short burst at boost clocks
    soak_steps = 0
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_s:
        for _ in range(4):
            step()
        torch.cuda.synchronize(dev)
        soak_steps += 4

    clocks = ClockSampler(local) if rank == 0 else None
    tensor_bytes = q.numel() * q.element_size()
    small = 4 * tensor_bytes < L2_BYTES  # q, k, v, dO fit in L2: flush before every step
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if small else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if clocks:
        clocks.start()
    if small:
        ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            e1.synchronize()
            ms += e0.elapsed_time(e1)
    else:
        ms = time_steps(step, args.steps, stream)
    torch.cuda.synchronize(dev)
    clock_info = clocks.stop() if clocks else None
    if world > 1:
        dist.barrier()
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    check_status(dev)
    total_flops = 2.5 * flops_fwd(B, S, H, D, causal) * args.steps
    value = total_flops / (ms * 1e-3) / 1e12
    l2_note = (f"flushed ({2 * L2_BYTES >> 20} MiB write) before each timed step" if small else
               f"inputs (q, k, v, dO: {4 * tensor_bytes >> 20} MiB) larger than the 126 MB L2")
    if args.kernels_only:
        # profiling mode: only the timed steps ran on the device
        if rank == 0:
            print(json.dumps({"metric": "attention fwd+bwd TFLOP/s", "value": value,
                              "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                              "warmup": args.warmup, "ms_per_step": ms / args.steps,
                              "config": {"workload": wl, "B": B, "S": S, "H": H, "D": D,
                                         "causal": causal, "l2": l2_note,
                                         "deterministic": bool(args.deterministic)},
                              "kernels_only": True}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # ---------------- the same step with the deterministic backward (dQ kernel)
    def step_det():
        q.grad = k.grad = v.grad = None
        flash_attn(q, k, v, causal=causal, deterministic=True).backward(do)

    for _ in range(2):
        step_det()
    det_steps = max(3, min(args.steps, 10))
    det_ms = time_steps(step_det, det_steps, stream) / det_steps
    if world > 1:
        t = torch.tensor([det_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        det_ms = float(t.item())
    q.grad = k.grad = v.grad = None

    # ---------------- e2e: pinned host -> device, step, results -> pinned host
    # Every step copies its inputs (q, k, v, dO) in from pinned host memory and
    # its results (O, dQ, dK, dV) back out, inside the timed region.  Three
    # streams and double-buffered device inputs let step i+1's copy-in and step
    # i-1's copy-out run while step i computes, as a training pipeline would.
    # The pinned buffers are allocated from the GPU's own CPUs so that their
    # pages sit on its NUMA node: with 8 ranks on a two-socket host, buffers
    # placed wherever a rank's thread happened to run would send half of the
    # copies across the socket link.
    with near_gpu(dev.index) as host_local:
        hin = [t.detach().cpu().pin_memory() for t in (q, k, v, do)]
        hout = [[torch.empty_like(hin[0]).pin_memory() for _ in range(4)] for _ in range(2)]
    dbuf = [[torch.empty_like(q) for _ in range(4)] for _ in range(2)]
    for bset in dbuf:
        for t_ in bset[:3]:
            t_.requires_grad_()
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))

    def run_e2e(nsteps):
        ev = lambda: torch.cuda.Event()  # noqa: E731
        in_done = [ev() for _ in range(nsteps)]
        cmp_done = [ev() for _ in range(nsteps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0.record(s_in)
        for i in range(nsteps):
            qd, kd, vd, dod = dbuf[i % 2]
            with torch.cuda.stream(s_in), torch.no_grad():
                if i >= 2:
                    s_in.wait_event(cmp_done[i - 2])  # step i-2 has read this input set
                for d_, h_ in zip(dbuf[i % 2], hin):
                    d_.copy_(h_, non_blocking=True)
                in_done[i].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(in_done[i])
                qd.grad = kd.grad = vd.grad = None
                out = flash_attn(qd, kd, vd, causal=causal)
                out.backward(dod)
                res = (out.detach(), qd.grad, kd.grad, vd.grad)
                cmp_done[i].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(cmp_done[i])
                for h_, d_ in zip(hout[i % 2], res):
                    d_.record_stream(s_out)
                    h_.copy_(d_, non_blocking=True)
        s_out.wait_event(cmp_done[nsteps - 1])
        t1.record(s_out)
        t1.synchronize()
        return t0.elapsed_time(t1)

    # the headline's step count (at least 3, at most 32: ~1.5 s of copies at c4),
    # so the first copy-in and the last copy-out, which nothing overlaps, weigh
    # on e2e as little as they do on a training run of that length
    e2e_steps = max(3, min(args.steps, 32))
    run_e2e(2)
    if world > 1:
        dist.barrier()
    e2e_ms = run_e2e(e2e_steps)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = 2.5 * flops_fwd(B, S, H, D, causal) * e2e_steps / (e2e_ms * 1e-3) / 1e12
    nb = q.numel() * 2
    del hout, hin, dbuf
    dq_, dk_, dv_ = (torch.empty_like(q) for _ in range(3))

    # ---------------- dominant kernel alone: main backward kernel
    lib = _lib.load()
    with torch.no_grad():
        qq, kk_, vv = q.detach(), k.detach(), v.detach()
        o, lse = flash_attn_forward(qq, kk_, vv, causal=causal, return_softmax_lse=True)
        Bl = qq.shape[0]
        nbytes = lib.fa_sm100_bwd_workspace_bytes(Bl, S, H, D)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        status = _lib.status_word(dev)
        scale = 1.0 / math.sqrt(D)

        def phase(p):
            rc = lib.fa_sm100_bwd_phase(p, do.data_ptr(), qq.data_ptr(), kk_.data_ptr(),
                                        vv.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                        dq_.data_ptr(), dk_.data_ptr(), dv_.data_ptr(),
                                        ws.data_ptr(), nbytes, Bl, S, H, D, scale,
                                        1 if causal else 0, status.data_ptr(), _stream_ptr(dev))
            _lib.check(rc, "fa_sm100_bwd_phase")

        phase(0)
        reps = max(5, min(args.steps, 11))

        def timed_median(fn):
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(reps)]
            for e0, e1 in ev:
                e0.record(stream)
                fn()
                e1.record(stream)
            torch.cuda.synchronize(dev)
            return statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)

        phase(1)
        k_ms = timed_median(lambda: phase(1))

        def time_phase(p):
            return timed_median(lambda: phase(p))

        pre_ms, post_ms = time_phase(0), time_phase(2)
        # forward kernel alone: the C ABI on preallocated outputs (no allocation
        # or Python work inside the event window), median of the launches
        o_f = torch.empty_like(qq)
        lse_f = torch.empty((Bl, H, S), dtype=torch.float32, device=dev)

        def fwd_launch():
            rc = lib.fa_sm100_fwd(qq.data_ptr(), kk_.data_ptr(), vv.data_ptr(), o_f.data_ptr(),
                                  lse_f.data_ptr(), Bl, S, H, D, scale, 1 if causal else 0,
                                  status.data_ptr(), _stream_ptr(dev))
            _lib.check(rc, "fa_sm100_fwd")

        fwd_launch()
        f_ms = timed_median(fwd_launch)
        check_status(dev)
        del ws
    peak_burst, peak_sus, peak_kind = load_peaks()
    bwd_alg = 2.5 * flops_fwd(Bl, S, H, D, causal)      # 5 GEMMs of the backward
    fwd_alg = flops_fwd(Bl, S, H, D, causal)            # 2 GEMMs of the forward
    k_tflops = bwd_alg / (k_ms * 1e-3) / 1e12
    traffic, traffic_note = None, "not measured for this workload"
    if wl in BWD_TRAFFIC_PER_LAUNCH:
        t_full, src = BWD_TRAFFIC_PER_LAUNCH[wl]
        traffic = t_full * Bl / B  # this rank's launch covers Bl of the B batches
        traffic_note = src + (f"; x {Bl}/{B} for this rank's batch shard" if Bl != B else "")
    f_tflops = fwd_alg / (f_ms * 1e-3) / 1e12

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(S, D, causal, amp, budget_s=args.cpu_budget)

    if rank == 0:
        line = {
            "metric": "attention fwd+bwd TFLOP/s",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": wl, "B": B, "S": S, "H": H, "D": D, "causal": causal,
                       "global_batch": B, "seq_len": S, "parallelism": f"batch-shard{world}",
                       "flops_per_step": 2.5 * flops_fwd(B, S, H, D, causal),
                       "flop_convention": "4*B*H*S^2*D (/2 causal), fwd+bwd = 2.5x",
                       "l2": l2_note, "power_soak": {"seconds": args.soak_s,
                                                     "untimed_steps": soak_steps}},
            "memory": {"step_peak_extra_mib_per_gpu": step_peak_mib,
                       "inputs_mib_per_gpu": 4 * tensor_bytes / 2**20,
                       "what": "max_memory_allocated during fwd+bwd minus the memory held "
                               "before it (q, k, v, dO); includes O, LSE, dQ/dK/dV and "
                               "the backward workspace",
                       "causal_1x4096x16x64_mib": mem_c3a},
            "pct_of_peak": {"value": value / (world * (peak_sus if peak_sus else peak_burst)),
                            "peak_tflops": world * peak_sus,
                            "kind": f"{peak_kind} bf16 sustained x n_gpus"},
            "gpu_launches": 4 * args.steps,
            "deterministic": {"ms_per_step": det_ms,
                              "tflops": 2.5 * flops_fwd(B, S, H, D, causal) / (det_ms * 1e-3) / 1e12,
                              "what": "same step with deterministic=True (dQ from the "
                                      "query-tile kernel, bit-reproducible)"},
            "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": 4 * nb,
                    "d2h_bytes_per_step": 4 * nb, "steps": e2e_steps,
                    "overlap": "copy-in of step i+1 and copy-out of step i-1 run beside "
                               "step i's compute (three streams, double-buffered inputs)",
                    "host_buffers": ("pinned, on the GPU's NUMA node (allocated from the CPUs "
                                     "NVML reports local to it)") if host_local
                                    else "pinned, default placement (GPU-local CPUs unknown)"},
            "roofline": {"bound": "tensor", "kernel": f"fa_bwd_main_kernel<{D}>",
                         "achieved": k_tflops, "peak": peak_burst, "unit": "TFLOP/s",
                         "frac": k_tflops / peak_burst,
                         "traffic": traffic,
                         "peak_kind": f"{peak_kind} bf16 burst",
                         "flops_per_launch": bwd_alg, "median_ms": k_ms,
                         "traffic_note": traffic_note,
                         "fwd_kernel": {"achieved": f_tflops, "median_ms": f_ms,
                                        "frac": f_tflops / peak_burst},
                         "bwd_pre_ms": pre_ms, "bwd_post_ms": post_ms},
            "clocks": clock_info,
        }
        if headline:
            line["headline_c3b"] = headline
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def peak_mem_fwd_bwd(dev, B, N, H, D, causal):
    """Peak extra allocator memory (MiB) of one fwd+bwd step over the memory held
    before it (q, k, v, dO), measured like the reference's bench/backward.py:69-85
    (one warm step, reset the peak, forward + backward, max_memory_allocated -
    memory_allocated before)."""
    from flash_attn_volta_b200 import flash_attn
    q, k, v, do = gen_shard(0, B, N, H, D, 1.0, dev, seed_base=99)
    for t in (q, k, v):
        t.requires_grad_()
    flash_attn(q, k, v, causal=causal).backward(do)
    q.grad = k.grad = v.grad = None
    torch.cuda.synchronize(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    base = torch.cuda.memory_allocated(dev)
    flash_attn(q, k, v, causal=causal).backward(do)
    torch.cuda.synchronize(dev)
    peak = torch.cuda.max_memory_allocated(dev) - base
    del q, k, v, do
    return peak / 2**20


def host_cost_us(dev, calls=2000):
    """Host time per public-API call (microseconds): flash_attn_forward and
    flash_attn_backward on a tiny shape (1, 128, 1, 64), whose kernels take a
    few microseconds, so the host is the bottleneck of the loop."""
    from flash_attn_volta_b200 import flash_attn_backward, flash_attn_forward
    q, k, v, do = gen_shard(0, 1, 128, 1, 64, 1.0, dev, seed_base=5)
    o, lse = flash_attn_forward(q, k, v, causal=True, return_softmax_lse=True)
    res = {}
    for name, fn in (("fwd", lambda: flash_attn_forward(q, k, v, causal=True)),
                     ("bwd", lambda: flash_attn_backward(do, q, k, v, o, lse, causal=True))):
        for _ in range(50):
            fn()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(calls):
            fn()
        t1 = time.perf_counter()
        torch.cuda.synchronize(dev)
        res[name] = 1e6 * (t1 - t0) / calls
    return res


def graph_vs_eager_us(dev, wl="c1", reps=30):
    """Step time (us) of a small workload's fwd+bwd through the public API,
    eager (host cost per call included) against the same step captured once in
    a CUDA graph and replayed; L2 flushed before each step."""
    from flash_attn_volta_b200 import flash_attn
    B, S, H, D, causal, amp = WORKLOADS[wl]
    q, k, v, do = gen_shard(0, B, S, H, D, amp, dev, seed_base=77)
    for t in (q, k, v):
        t.requires_grad_()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step():
        flash_attn(q, k, v, causal=causal).backward(do)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            q.grad = k.grad = v.grad = None
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    q.grad = k.grad = v.grad = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()

    def timed(fn):
        ts = []
        for i in range(5 + reps):
            flush.zero_()
            torch.cuda.synchronize(dev)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            if i >= 5:
                ts.append(1e3 * e0.elapsed_time(e1))
        return statistics.median(ts)

    def eager():
        q.grad = k.grad = v.grad = None
        step()

    return {"workload": wl, "eager_us": timed(eager), "graph_replay_us": timed(g.replay),
            "what": "one fwd+bwd step from an idle GPU (synchronised before each step): "
                    "eager includes the host time of the two calls"}


def bench_small(wl, dev, args):
    """fwd+bwd of a small workload through the public autograd API, and the
    inference-only forward with LSE, L2 flushed before every step."""
    from flash_attn_volta_b200 import flash_attn, flash_attn_forward
    B, S, H, D, causal, amp = WORKLOADS[wl]
    q, k, v, do = gen_shard(0, B, S, H, D, amp, dev)
    q.requires_grad_(); k.requires_grad_(); v.requires_grad_()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fwd_bwd():
        q.grad = k.grad = v.grad = None
        flash_attn(q, k, v, causal=causal).backward(do)

    def fwd_bwd_det():
        q.grad = k.grad = v.grad = None
        flash_attn(q, k, v, causal=causal, deterministic=True).backward(do)

    def fwd_lse():
        with torch.no_grad():
            flash_attn_forward(q, k, v, causal=causal, return_softmax_lse=True)

    def median_ms(fn):
        ts = []
        for i in range(5 + 20):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            if i >= 5:
                ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    ms, fms, dms = median_ms(fwd_bwd), median_ms(fwd_lse), median_ms(fwd_bwd_det)
    ff = flops_fwd(B, S, H, D, causal)
    return {"B": B, "S": S, "H": H, "D": D, "causal": causal, "ms_per_step": ms,
            "tflops": 2.5 * ff / (ms * 1e-3) / 1e12,
            "tflops_alg": 3.5 * ff / (ms * 1e-3) / 1e12,
            "fwd_lse_ms": fms, "fwd_lse_tflops": ff / (fms * 1e-3) / 1e12,
            "deterministic_ms_per_step": dms,
            "deterministic_tflops": 2.5 * ff / (dms * 1e-3) / 1e12,
            "flop_convention": "tflops: 2.5 x F_fwd; tflops_alg: 3.5 x F_fwd (2 forward + "
                               "5 backward GEMMs); fwd_lse: F_fwd",
            "l2": "flushed (256 MiB write) before each step"}


# ----------------------------------------------------------------------- config 5
C5 = dict(layers=24, hidden=2048, heads=16, head_dim=128, mlp=5504, vocab=32000, batch=8,
          seq=2048)


class _EventMark(torch.autograd.Function):
    """Identity whose backward records a CUDA event (brackets a backward region)."""

    @staticmethod
    def forward(ctx, x, sink):
        ctx.sink = sink
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        ctx.sink.append(e)
        return g, None


def run_c5(args):
    """Config 5: random-init LLaMA-style decoder patched with patch_hf; one step =
    forward + shifted-label cross-entropy + backward + SGD update on 8 x 2048
    uniform token ids.  `value` is the attention fwd+bwd TFLOP/s measured inside
    the step (CUDA events around every attention call and its backward)."""
    import transformers as T
    from flash_attn_volta_b200 import patch_hf
    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = C5
    cfg = T.LlamaConfig(vocab_size=c["vocab"], hidden_size=c["hidden"],
                        intermediate_size=c["mlp"], num_hidden_layers=c["layers"],
                        num_attention_heads=c["heads"], num_key_value_heads=c["heads"],
                        head_dim=c["head_dim"], rope_theta=10000.0, initializer_range=0.02,
                        max_position_embeddings=c["seq"])
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device(dev):
        model = T.LlamaForCausalLM(cfg).to(torch.float16)
    fam, n = patch_hf.patch_model(model)
    assert fam == "llama" and n == c["layers"]
    fwd_ev, bwd_ev = [], []
    base = patch_hf.flash_attn

    def timed_attn(q, k, v, causal=False, sm_scale=None):
        q = _EventMark.apply(q, bwd_ev)      # backward of this runs after attention's backward
        e0 = torch.cuda.Event(enable_timing=True); e0.record()
        out = base(q, k, v, causal=causal, sm_scale=sm_scale)
        e1 = torch.cuda.Event(enable_timing=True); e1.record()
        fwd_ev.append((e0, e1))
        return _EventMark.apply(out, bwd_ev)  # backward of this runs just before it

    patch_hf.flash_attn = timed_attn
    g = torch.Generator().manual_seed(1)
    host_ids = torch.randint(0, c["vocab"], (c["batch"], c["seq"]), generator=g).pin_memory()
    params = [p for p in model.parameters()]
    lr = 1e-4

    def step():
        ids = host_ids.to(dev, non_blocking=True)
        for p in params:
            p.grad = None
        loss = model(ids, labels=ids).loss
        loss.backward()
        with torch.no_grad():
            torch._foreach_add_(params, [p.grad for p in params], alpha=-lr)
        return loss

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    fwd_ev.clear(); bwd_ev.clear()
    clocks = ClockSampler(local)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True); t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    # every step reads its loss back to the host (the step's result)
    losses = [step().item() for _ in range(args.steps)]
    t1.record()
    torch.cuda.synchronize(dev)
    clock_info = clocks.stop()
    step_ms = t0.elapsed_time(t1) / args.steps
    attn_ms = sum(a.elapsed_time(b) for a, b in fwd_ev)
    # bwd events come in pairs per layer: (before attention bwd, after attention bwd)
    attn_ms += sum(bwd_ev[i].elapsed_time(bwd_ev[i + 1]) for i in range(0, len(bwd_ev), 2))
    attn_ms /= args.steps
    f_layer = 2.5 * flops_fwd(c["batch"], c["seq"], c["heads"], c["head_dim"], True)
    value = c["layers"] * f_layer / (attn_ms * 1e-3) / 1e12
    peak_burst, peak_sus, peak_kind = load_peaks()
    line = {
        "metric": "attention fwd+bwd TFLOP/s", "value": value, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (uniform token ids, random-init N(0,0.02) weights)",
        "config": {"workload": "c5", **c, "attention_ms_per_step": attn_ms,
                   "attention_share_of_step": attn_ms / step_ms,
                   "tokens_per_s": c["batch"] * c["seq"] / (step_ms * 1e-3),
                   "loss_first_last": [losses[0], losses[-1]],
                   "flop_convention": "per layer 2.5 x 4*B*H*S^2*D / 2 (causal)"},
        "pct_of_peak": {"value": value / peak_sus, "peak_tflops": peak_sus,
                        "kind": f"{peak_kind} bf16 sustained"},
        "gpu_launches": 4 * c["layers"] * args.steps,
        # the attention FLOPs over the whole training step, token ids copied in
        # and the loss read back every step
        "e2e": {"value": c["layers"] * f_layer / (step_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": host_ids.numel() * 8, "d2h_bytes_per_step": 4,
                "note": "attention FLOPs / full training-step time"},
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def run_ring(args):
    """Config 5, long variant: B=1, S=131072, H=32, D=128, causal; ring context
    parallelism over the N ranks (zigzag shards, NCCL send/recv of K/V blocks).
    Strong scaling: the whole sequence is fixed and split across ranks."""
    import torch.distributed as dist
    from flash_attn_volta_b200 import ring
    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    B, S, H, D, causal = 1, 131072, 32, 128, True
    g = torch.Generator(device=dev).manual_seed(7)
    full = lambda: torch.randn((B, S, H, D), device=dev, generator=g, dtype=torch.float16)
    q, k, v, do = (ring.zigzag_shard(full(), rank, world) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_()

    def step():
        q.grad = k.grad = v.grad = None
        ring.ring_flash_attn(q, k, v, causal=causal).backward(do)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    # count this library's launches in the timed steps: one forward kernel per
    # forward block, three (prep, main, dQ conversion) per backward block
    counts = [0]
    fwd0, bwd0 = ring.block_fwd, ring.block_bwd

    def fwd_counted(*a):
        counts[0] += 2  # the block's forward kernel and its merge kernel
        return fwd0(*a)

    def bwd_counted(*a):
        counts[0] += 3
        return bwd0(*a)

    ring.block_fwd, ring.block_bwd = fwd_counted, bwd_counted
    if world > 1:
        dist.barrier()
    ms = time_steps(step, args.steps, torch.cuda.current_stream(dev))
    ring.block_fwd, ring.block_bwd = fwd0, bwd0
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total = 2.5 * flops_fwd(B, S, H, D, causal) * args.steps
    value = total / (ms * 1e-3) / 1e12
    peak_burst, peak_sus, peak_kind = load_peaks()
    merge = merge_roofline(dev, S // (2 * world), H, D) if rank == 0 else None
    if rank == 0:
        print(json.dumps({
            "metric": "attention fwd+bwd TFLOP/s", "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "merge_roofline": merge,
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "c5long", "B": B, "S": S, "H": H, "D": D, "causal": causal,
                       "parallelism": f"ring-cp{world} (zigzag)",
                       "l2": "inputs (1 GiB per tensor) larger than L2"},
            "pct_of_peak": {"value": value / (world * peak_sus), "peak_tflops": world * peak_sus,
                            "kind": f"{peak_kind} bf16 sustained x n_gpus"},
            "gpu_launches": counts[0],
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_triton(args):
    """Informational leg (not the driver's reference arm): the unmodified
    reference package, installed into baseline/_ref, run on this B200 through its
    own public API (flash_attn_volta.flash_attn: Triton kernels written for
    sm_70, compiled by the installed Triton) at the config-3 shapes, fwd+bwd,
    L2 flushed before each step; its outputs are compared with this library's."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    dev = torch.device("cuda", 0)
    line = {"impl": "reference-triton", "metric": "attention fwd+bwd TFLOP/s", "unit": "TFLOP/s",
            "higher_is_better": True, "n_gpus": 1, "data": "synthetic"}
    try:
        sys.path.insert(0, ref_dir)
        import flash_attn_volta as ref  # noqa: F401
        import triton
        line["triton"] = triton.__version__
        from flash_attn_volta_b200 import flash_attn as ours
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        res = {}
        for wl in ("c3a", "c3b"):
            B, S, H, D, causal, amp = WORKLOADS[wl]
            q, k, v, do = gen_shard(0, B, S, H, D, amp, dev)
            outs = {}
            for name, fn in (("reference", ref.flash_attn), ("ours", ours)):
                qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
                fn(qq, kk, vv, causal=causal).backward(do)  # compile / autotune
                ts = []
                for i in range(3 + max(args.steps, 5)):
                    qq.grad = kk.grad = vv.grad = None
                    flush.zero_()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    o = fn(qq, kk, vv, causal=causal)
                    o.backward(do)
                    e1.record()
                    e1.synchronize()
                    if i >= 3:
                        ts.append(e0.elapsed_time(e1))
                outs[name] = (o.detach(), qq.grad, kk.grad, vv.grad, statistics.median(ts))
            f = 2.5 * flops_fwd(B, S, H, D, causal)
            r, o_ = outs["reference"], outs["ours"]
            res[wl] = {"B": B, "S": S, "H": H, "D": D, "causal": causal,
                       "reference_ms": r[4], "reference_tflops": f / (r[4] * 1e-3) / 1e12,
                       "ours_ms": o_[4], "ours_tflops": f / (o_[4] * 1e-3) / 1e12,
                       "max_abs_diff": {n: float((a.float() - b.float()).abs().max())
                                        for n, a, b in zip(("o", "dq", "dk", "dv"), r[:4], o_[:4])}}
        line["results"] = res
        line["value"] = res["c3b"]["reference_tflops"]
    except Exception as e:  # compile errors of the sm_70 kernels are the result here
        line["unavailable"] = f"{type(e).__name__}: {str(e).splitlines()[0][:300] if str(e) else ''}"
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-triton"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c5", "c5long"], default="c4")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--soak-s", type=float, default=1.0,
                    help="seconds of untimed steps between the warm-up and the timed steps")
    ap.add_argument("--deterministic", action="store_true",
                    help="time the step with the deterministic backward (dQ kernel)")
    ap.add_argument("--kernels-only", action="store_true",
                    help="run only the warm-up and timed steps (for ncu launch lists)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args, args.workload)
    elif args.impl == "reference-triton":
        run_reference_triton(args)
    elif args.workload == "c5":
        run_c5(args)
    elif args.workload == "c5long":
        run_ring(args)
    else:
        run_ours(args, args.workload)


if __name__ == "__main__":
    main()
