"""Benchmark of the B200 FlashAttention-2 forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg3]
                    [--impl ours|reference|reference-kernel] [--sweep]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Metric: attention forward TFLOPS = 4 B H N^2 d / t, halved for causal (the reference's count,
bench/benchmark.py:142), at 1/2/4/8 GPUs, with the fraction of the measured dense fp16/bf16
tensor-core peak.

Workload (every N): BASELINE config 3, B2 H32 N16384 d128 causal, q/k/v N(0,1)*0.5 fp16, the
configuration the metric is quoted on at 1/2/4/8 GPUs. Its B*H = 64 (b,h) heads are split
into contiguous balanced ranges, one per rank (fa.plan_shards; 64/32/16/8 heads per GPU), one
process per GPU, no collective on the data path: strong scaling. A step is one forward pass
over the whole problem (every rank's shard); value = the problem's FLOPs / the max over ranks
of the event-timed duration. The same line carries the non-causal twin (cfg3nc) on the same
shards, at N > 1 the weak-scaling figure (every rank a private copy of config 1), and at N = 1
`per_config`: configs 1 and 2 (fp32 and fp16 accumulation), configs 3 (causal) and 2 with
bfloat16 inputs, config 3 (causal and non-causal) with e4m3 inputs (fa.forward_fp8; its
fraction is of the fp16 peak like every other row, e4m3's tensor peak being twice that), and
rows of the ragged sweep (config 4), each event-timed for K steps with its clocks.

`value` is timed on the device with CUDA events around exactly K steps with inputs resident in
HBM (inputs larger than L2); `e2e` is the same metric through the public API with host
buffers (fa.forward_host: q, k, v copied in from pinned memory and O copied out every step,
inside the timed region), with the measured host<->device link rates beside it. `roofline`
divides the kernel's algorithmic FLOPs per launch by its event-timed duration and by the
measured peak. `cpu_baseline` times the reference's own CPU path (its attention_reference,
compiled from the reference's source into oracle/_ref/ by TorchScript; the numpy restatement
in oracle/ where that file is absent) on a bounded sample of the workload's heads.

Inputs: head h of a workload is drawn on the CPU from its own seeded generator
(fa/synthetic.py make_head_qkv), so any shard is generated alone and every arm and rank sees
the same values for the same head.

--impl reference: the reference's CPU path (above) on the host cores with every thread, on the
same workload and config, rank 0 only; it imports nothing from the product package.
--impl reference-kernel (a context line): the reference's own CUDA kernel compiled for sm_100a
(baseline/build_ref_kernel.py) on the same workload and GPU.
--sweep (context lines): the reference benchmark's FA2-paper shapes (B = 16384/N, H = 2048/d,
bench/benchmark.py:146-192) with PyTorch SDPA's flash and cuDNN backends on the same GPU.
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "flash-attention-from-scratch_b200"

METRIC = "attn fwd TFLOPS (fp16, d=64/128, causal+non) at 1/2/4/8 B200; % of TC peak"
HEADLINE = "cfg3"
PER_CONFIG = ["cfg1", "cfg2", "cfg2acc", "cfg3bf16", "cfg2bf16", "cfg3fp8", "cfg3ncfp8", "cfg4:8191:128:1", "cfg4:12345:128:0", "cfg4:12345:64:1",
              "cfg4:3000:128:0", "cfg4:1000:128:1", "cfg4:1000:64:0"]
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _load_by_path(name: str, path: Path):
    """Imports one source file as a module without importing its package (the product package
    `fa` loads libfa_b200.so on import; the reference arm must not)."""
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def synthetic():
    return _load_by_path("fa_synthetic_bench", PKG / "fa" / "synthetic.py")


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def workload(name: str) -> dict:
    syn = synthetic()
    if name in syn.CONFIGS:
        return dict(syn.CONFIGS[name], outliers=False, variant="opt", name=name)
    if name == "cfg2acc":
        return dict(syn.CONFIGS["cfg2"], outliers=False, variant="fp16acc", name=name)
    if name.endswith("bf16") and name[: -len("bf16")] in syn.CONFIGS:
        # a configuration's shape and values with bfloat16 inputs (an extension of the reference)
        return dict(syn.CONFIGS[name[: -len("bf16")]], outliers=False, variant="opt", dtype="bf16", name=name)
    if name in ("cfg3fp8", "cfg3ncfp8"):
        # config 3 with e4m3 inputs (per-tensor descales; fp16 O), causal / non-causal
        return dict(syn.CONFIGS["cfg3"], causal=(name == "cfg3fp8"), outliers=False, variant="opt", dtype="fp8",
                    name=name)
    if name.startswith("cfg4:"):
        # cfg4:N:d:causal, e.g. cfg4:12345:128:1 (B16 H16, seed 4, outlier channel)
        _, n, d, causal = name.split(":")
        for c in syn.cfg4_cases():
            if c["n"] == int(n) and c["d"] == int(d) and c["causal"] == bool(int(causal)):
                return dict(c, variant="opt", name=name)
    if name.startswith("shape:"):
        # shape:B:H:N:d:causal, seeded N(0,1) inputs (seed 5), e.g. shape:1:4:32768:128:0
        _, b, h, n, d, causal = name.split(":")
        return dict(b=int(b), h=int(h), n=int(n), d=int(d), causal=bool(int(causal)), seed=5, scale=1.0,
                    outliers=False, variant="opt", name=name)
    raise SystemExit(f"unknown workload {name}")


def flops_of(c: dict, heads: int | None = None) -> float:
    h = c["b"] * c["h"] if heads is None else heads
    return 4.0 * h * c["n"] * c["n"] * c["d"] / (2.0 if c["causal"] else 1.0)


def shard_ranges(total: int, world: int) -> list[tuple[int, int]]:
    """Contiguous balanced head ranges (the split of fa.plan_shards, restated here so that the
    reference arm needs nothing from the product package)."""
    base, extra = divmod(total, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def config_dict(c: dict, world: int) -> dict:
    """The `config` of the JSON line; both arms build it the same way from the same inputs."""
    heads = c["b"] * c["h"]
    io_bytes = 4 * heads * c["n"] * c["d"] * 2
    return {
        "workload": c["name"], "B": c["b"], "H": c["h"], "N": c["n"], "d": c["d"], "causal": c["causal"],
        "variant": c["variant"], "value_scale": c["scale"], "outliers": bool(c.get("outliers", False)),
        "heads_total": heads,
        "parallelism": f"heads sharded over {world} GPU(s), contiguous ranges, no collective",
        "heads_per_gpu": [e - s for s, e in shard_ranges(heads, world)],
        "l2": f"inputs larger than L2 ({io_bytes / 1e6:.0f} MB of Q,K,V,O per step)",
    }


def traffic_per_launch(workload_name: str) -> float | None:
    """DRAM bytes (read + write) per launch of the attention kernel, from the committed ncu
    summary profiles/traffic.txt (lines `<workload> <bytes>`), else None."""
    p = REPO / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload_name and not line.startswith("#"):
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Polls SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:  # NVML unavailable: report no samples
            self._h = None

    def sample_once(self):
        if self._h is None:
            return
        try:
            mhz = int(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
            reasons = int(self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            self.samples.append((mhz, reasons))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self.sample_once()
            time.sleep(0.001)

    def start(self):
        self.samples = []
        self._stop.clear()
        if self._h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if not self.samples:
            self.sample_once()
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for bit, name in self.REASONS.items() if bits & bit and name != "gpu_idle"]
        return {
            "sm_mhz": statistics.median(mhz) if mhz else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(mhz),
        }


def pin_to_gpu_numa_node(device_index: int) -> list[int] | None:
    """Restricts this process to the CPUs NVML reports as close to the GPU, so that pinned host
    buffers allocated and first touched afterwards sit on the GPU's NUMA node. Best effort."""
    try:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = [w * 64 + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1]
        cpus = [c for c in cpus if c < os.cpu_count()]
        if cpus:
            os.sched_setaffinity(0, cpus)
            return cpus
    except Exception:
        pass
    return None


def _compiled_reference():
    """The reference's attention_reference as compiled into oracle/_ref/ (None if absent)."""
    return _load_by_path("oracle_build_ref_bench", REPO / "oracle" / "build_ref.py").load()


def cpu_path_timer(c: dict, heads_per_step: int):
    """(step, kind, what): one call of `step` runs the reference's CPU path over heads_per_step
    heads of workload `c` (heads 0 .. heads_per_step-1; every head of a workload has the same
    shape and work). kind is "reference" when the compiled reference is present, else "port"
    (the numpy restatement in oracle/)."""
    import torch

    syn = synthetic()
    q, k, v = syn.make_head_qkv(range(heads_per_step), c["n"], c["d"], c["seed"], scale=c["scale"],
                                outliers=c.get("outliers", False))
    ref = _compiled_reference()
    if ref is not None:
        def step():
            with torch.no_grad():
                for i in range(heads_per_step):
                    ref(q[:, i : i + 1], k[:, i : i + 1], v[:, i : i + 1], c["causal"])

        what = ("the reference's fa/reference.py::attention_reference, compiled unmodified from the "
                "reference source by torch.jit.script (oracle/_ref/attention_reference.pt), torch CPU")
        return step, "reference", what
    oracle = _load_by_path("oracle_attention_bench", REPO / "oracle" / "attention.py")
    qn, kn, vn = q.numpy(), k.numpy(), v.numpy()
    threads = max(1, os.cpu_count() or 1)

    def step():
        oracle.attention(qn, kn, vn, causal=c["causal"], threads=threads, max_chunk_bytes=c["n"] * c["n"] * 4)

    return step, "port", "numpy fp32 restatement of the reference's attention_reference (oracle/attention.py)"


def heads_per_cpu_step(c: dict) -> int:
    """Heads per CPU step: about 1 GiB of fp32 scores (one head at N = 16384)."""
    return max(1, min(c["b"] * c["h"], (1 << 28) // (c["n"] * c["n"])))


def cpu_baseline(c: dict, budget_s: float) -> dict:
    """The reference's CPU path on sampled heads of the workload until budget_s has elapsed."""
    import torch

    threads = max(1, os.cpu_count() or 1)
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        hps = heads_per_cpu_step(c)
        step, kind, what = cpu_path_timer(c, hps)
        step()  # warm-up (allocator, thread pool)
        done, t0 = 0, time.perf_counter()
        while True:
            step()
            done += hps
            if time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
    finally:
        torch.set_num_threads(prev)
    return {
        "value": flops_of(c, done) / dt / 1e12,
        "unit": "TFLOPS",
        "cores": threads,
        "kind": kind,
        "sample": f"{done} heads of {c['name']} ({hps} per call, {dt:.1f} s, {threads} threads): {what}",
    }


def run_reference_arm(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path on rank 0 only (the other ranks exit)."""
    if rank != 0:
        return
    import torch

    c = workload(args.workload)
    threads = max(1, os.cpu_count() or 1)
    torch.set_num_threads(threads)
    hps = heads_per_cpu_step(c)
    step, kind, what = cpu_path_timer(c, hps)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = flops_of(c, hps) * args.steps / dt / 1e12
    sample = (f"{hps} of {c['b'] * c['h']} heads of {c['name']} per step (every head has the same shape "
              f"and work), {threads} threads: {what}")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / max(1, args.steps),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) fp16 inputs per head, CPU generator)",
        "config": config_dict(c, world),
        "sample": sample,
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_kernel_arm(args, rank: int, world: int) -> None:
    """--impl reference-kernel: a context line, not the driver's reference arm. Times the
    reference's own CUDA kernel (mma.sync / ldmatrix / cp.async, written for sm_80+), compiled
    unmodified for sm_100a by baseline/build_ref_kernel.py, on the same workload, GPU and clock
    sampling as --impl ours. Rank 0 only."""
    if rank != 0:
        return
    lib_path = REPO / "baseline" / "_ref" / "libfa_ref_kernel.so"
    if not lib_path.exists():
        print(json.dumps({"impl": "reference-kernel",
                          "unavailable": "baseline/_ref/libfa_ref_kernel.so not built (needs the reference sources)"}))
        return
    import ctypes

    import torch

    sys.path.insert(0, str(PKG))
    from fa import _C

    lib = ctypes.CDLL(str(lib_path))
    lib.fa_ref_kernel_fwd.restype = ctypes.c_int
    lib.fa_ref_kernel_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    c = workload(args.workload)
    variant = args.variant or c["variant"]
    variant_id = {"baseline": 0, "opt": 1, "fp16acc": 2}[variant]
    b, h, n, d, causal = c["b"], c["h"], c["n"], c["d"], c["causal"]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v = synthetic().make_head_qkv(range(b * h), n, d, c["seed"], scale=c["scale"],
                                        outliers=c.get("outliers", False))
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    od = torch.empty_like(qd)
    stream = torch.cuda.current_stream(dev)
    err = ctypes.create_string_buffer(512)
    scale = 1.0 / math.sqrt(d)

    def step():
        rc = lib.fa_ref_kernel_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), 1, b * h, n, d,
                                   scale, int(causal), variant_id, ctypes.c_void_p(stream.cuda_stream), err, 512)
        if rc != 0:
            raise SystemExit(f"reference kernel: {err.value.decode()}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(0)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    stop.synchronize()
    clocks = sampler.stop()
    ms = start.elapsed_time(stop) / args.steps
    ours = _C.forward(qd, kd, vd, causal, None, variant)
    diff = (ours.float() - od.float()).abs()
    peaks, _ = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    value = flops_of(c) / (ms * 1e-3) / 1e12
    print(json.dumps({
        "impl": "reference-kernel", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16 inputs per head, CPU generator)",
        "config": config_dict(dict(c, variant=variant), 1), "pct_tc_peak": value / peak, "clocks": clocks,
        "max_abs_diff_vs_ours": float(diff.max()),
        "kernel": "reference csrc/kernels/flash_fwd.cu (mma.sync m16n8k16) built for sm_100a with the reference's nvcc flags",
    }), flush=True)


def run_sweep(args) -> None:
    """--sweep: the reference benchmark's FA2-paper shapes (bench/benchmark.py:146-192:
    B = 16384 / N, H = 2048 / d, N 512 .. 16384, d 64 / 128, causal and not) on one GPU, with
    PyTorch SDPA's flash and cuDNN backends as context lines. Timing follows
    bench/benchmark.py:108-120 (10 warm-ups, then the median of event-timed launches)."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel

    sys.path.insert(0, str(PKG))
    import fa

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, _ = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))

    def median_ms(fn) -> float:
        for _ in range(10):
            fn()
        torch.cuda.synchronize(dev)
        times = []
        t_end = time.perf_counter() + 1.0
        while len(times) < 20 or (time.perf_counter() < t_end and len(times) < 100):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    for d in (64, 128):
        for causal in (False, True):
            for n in (512, 1024, 2048, 4096, 8192, 16384):
                b, h = 16384 // n, 2048 // d
                g = torch.Generator(device=dev).manual_seed(n * 1000 + d)
                q, k, v = (torch.randn(b, h, n, d, device=dev, generator=g, dtype=torch.float16) for _ in range(3))
                flops = 4.0 * b * h * n * n * d / (2.0 if causal else 1.0)
                row = {"impl": "sweep", "B": b, "H": h, "N": n, "d": d, "causal": causal}
                ours = fa.forward(q, k, v, causal=causal)
                for name, fn in (
                    ("ours", lambda: fa.forward(q, k, v, causal=causal)),
                    ("sdpa_flash", (SDPBackend.FLASH_ATTENTION,)),
                    ("sdpa_cudnn", (SDPBackend.CUDNN_ATTENTION,)),
                ):
                    try:
                        if name != "ours":
                            backend = fn[0]

                            def fn(backend=backend):
                                with sdpa_kernel([backend]):
                                    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)

                            other = fn()
                            row[f"{name}_max_abs_diff"] = float((other.float() - ours.float()).abs().max())
                        ms = median_ms(fn)
                        row[f"{name}_tflops"] = flops / (ms * 1e-3) / 1e12
                    except Exception as exc:  # a backend that does not run this shape here
                        row[f"{name}_tflops"] = None
                        row[f"{name}_error"] = str(exc).splitlines()[0][:160]
                row["ours_pct_tc_peak"] = row["ours_tflops"] / peak
                print(json.dumps(row), flush=True)
                del q, k, v, ours
                torch.cuda.empty_cache()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=HEADLINE)
    ap.add_argument("--variant", default=None, help="override the workload's kernel variant")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-kernel"])
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--sweep", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.impl == "reference-kernel":
        run_reference_kernel_arm(args, rank, world)
        return
    if args.sweep:
        if rank == 0:
            run_sweep(args)
        return
    run_ours(args, rank, world, local_rank)


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(PKG))
    import fa
    from fa import _C

    cpus = pin_to_gpu_numa_node(local_rank)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        # Host-side rendezvous only (a barrier around the timed region and the max over ranks of
        # the durations): gloo, no NCCL, no device collective.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    syn = synthetic()

    def plan_of(qd, causal, variant) -> dict:
        """The schedule fa.forward runs (fa_plan on this device)."""
        return _C.plan_params(_C.make_params(qd, qd, qd, qd, causal, 1.0, _C.parse_variant(variant)), 0)

    def kernels_per_launch(qd, kd, vd, causal, variant) -> int:
        # the attention kernel, plus the combine when the plan splits key ranges
        return 2 if plan_of(qd, causal, variant)["workspace_bytes"] > 0 else 1

    def timed(step, steps: int, warmup: int, sample_clocks: bool):
        """Device time per step (ms) of `step` over exactly `steps` calls after `warmup`,
        CUDA events on this rank's stream, barrier + synchronize on both sides."""
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        sampler = ClockSampler(local_rank) if sample_clocks else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        if sampler:
            sampler.start()
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize(dev)
        clocks = sampler.stop() if sampler else None
        barrier()
        return e0.elapsed_time(e1) / steps, clocks

    def check_status():
        status = _C.device_status(local_rank, clear=True)
        if status != 0:
            raise SystemExit(f"kernel watchdog fired (status {status:#x}); timing invalid")

    # ---- the headline: this rank's shard of the workload ----
    c = workload(args.workload)
    variant = args.variant or c["variant"]
    c["variant"] = variant
    b, h, n, d, causal = c["b"], c["h"], c["n"], c["d"], c["causal"]
    total_heads = b * h
    shard = fa.plan_shards(total_heads, world)[rank]
    heads = range(shard.start, shard.stop)
    q, k, v = syn.make_head_qkv(heads, n, d, c["seed"], scale=c["scale"], outliers=c.get("outliers", False))
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    kpl = kernels_per_launch(qd, kd, vd, causal, variant)

    def step():
        return _C.forward(qd, kd, vd, causal, None, variant)

    ms, clocks = timed(step, args.steps, args.warmup, True)
    ms_max = max_over_ranks(ms)
    check_status()
    shard_flops = flops_of(c, shard.heads)
    value = flops_of(c) / (ms_max * 1e-3) / 1e12
    achieved = shard_flops / (ms * 1e-3) / 1e12

    # ---- the non-causal twin of the headline on the same shards and inputs ----
    twin = None
    if c["name"] in ("cfg3", "cfg3nc"):
        tc = workload("cfg3nc" if causal else "cfg3")
        tc["variant"] = variant

        def twin_step():
            return _C.forward(qd, kd, vd, tc["causal"], None, variant)

        t_ms, t_clocks = timed(twin_step, args.steps, args.warmup, True)
        t_max = max_over_ranks(t_ms)
        check_status()
        t_value = flops_of(tc) / (t_max * 1e-3) / 1e12
        twin = {"workload": tc["name"], "causal": tc["causal"], "value": t_value, "unit": "TFLOPS",
                "ms_per_step": t_max, "frac": t_value / world / peak, "clocks": t_clocks,
                "scaling": "strong", "steps": args.steps, "plan_rank0": plan_of(qd, tc["causal"], variant)}

    # ---- weak scaling (N > 1): every rank a private copy of config 1 ----
    weak = None
    if world > 1:
        wc = workload("cfg1")
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        wq, wk, wv = (torch.randn(wc["b"], wc["h"], wc["n"], wc["d"], device=dev, generator=g,
                                  dtype=torch.float16) for _ in range(3))

        def weak_step():
            return _C.forward(wq, wk, wv, wc["causal"], None, "opt")

        w_ms, _ = timed(weak_step, args.steps, args.warmup, False)
        w_max = max_over_ranks(w_ms)
        check_status()
        weak = {"workload": "cfg1 per GPU", "value": world * flops_of(wc) / (w_max * 1e-3) / 1e12,
                "unit": "TFLOPS", "ms_per_step": w_max, "scaling": "weak"}
        del wq, wk, wv

    # ---- per-config lines (N = 1): the other BASELINE configurations ----
    per_config = None
    if world == 1 and not args.no_per_config:
        per_config = {}
        for name in PER_CONFIG:
            pc = workload(name)
            g = torch.Generator(device=dev).manual_seed(pc["seed"])
            shape = (pc["b"], pc["h"], pc["n"], pc["d"])
            pq, pk, pv = (torch.randn(shape, device=dev, generator=g) * pc["scale"] for _ in range(3))
            if pc.get("outliers"):
                oc = syn.outlier_channels(pc["d"])
                pq[..., :oc] *= 8.0
                pk[..., :oc] *= 8.0
            if pc.get("dtype") == "fp8":
                (pq, qs), (pk, ks), (pv, vs) = (fa.quantize_fp8(t) for t in (pq, pk, pv))

                def pc_step():
                    return _C.forward_fp8(pq, pk, pv, qs, ks, vs, pc["causal"], None, pc["variant"])
            else:
                pdt = torch.bfloat16 if pc.get("dtype") == "bf16" else torch.float16
                pq, pk, pv = pq.to(pdt), pk.to(pdt), pv.to(pdt)

                def pc_step():
                    return _C.forward(pq, pk, pv, pc["causal"], None, pc["variant"])

            p_ms, p_clocks = timed(pc_step, args.steps, args.warmup, True)
            check_status()
            p_val = flops_of(pc) / (p_ms * 1e-3) / 1e12
            io = 4 * pq.numel() * 2 if pc.get("dtype") != "fp8" else pq.numel() * (3 + 2 + 2)  # fp8: q, k, v, V^T out/in, O
            per_config[name] = {
                "B": pc["b"], "H": pc["h"], "N": pc["n"], "d": pc["d"], "causal": pc["causal"],
                "variant": pc["variant"], "dtype": pc.get("dtype", "f16"), "outliers": bool(pc.get("outliers")),
                "value": p_val, "unit": "TFLOPS",
                "ms_per_step": p_ms, "frac": p_val / peak, "hbm_gbs_algorithmic": io / (p_ms * 1e-3) / 1e9,
                "kernels_per_launch": (2 if pc.get("dtype") == "fp8"  # V transpose + attention
                                       else kernels_per_launch(pq, pk, pv, pc["causal"], pc["variant"])),
                "plan": None if pc.get("dtype") == "fp8" else plan_of(pq, pc["causal"], pc["variant"]),
                "traffic": traffic_per_launch(name), "clocks": p_clocks, "steps": args.steps,
            }
            del pq, pk, pv
            torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        qh, kh, vh = q.pin_memory(), k.pin_memory(), v.pin_memory()
        oh = torch.empty_like(qh).pin_memory()
        in_bytes = 3 * qh.numel() * 2
        out_bytes = oh.numel() * 2
        # Link rates of this rank's bytes, outside the timed region (one copy each way).
        scratch = torch.empty(qh.shape, dtype=qh.dtype, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(2):
            e0.record(stream)
            scratch.copy_(qh, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
        h2d_gbs = qh.numel() * 2 / (e0.elapsed_time(e1) * 1e-3) / 1e9
        for _ in range(2):
            e0.record(stream)
            oh.copy_(scratch, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
        d2h_gbs = oh.numel() * 2 / (e0.elapsed_time(e1) * 1e-3) / 1e9
        del scratch

        def e2e_step():
            # host q, k, v in, host O out; copies and kernels pipelined over chunks of heads
            fa.forward_host(qh, kh, vh, causal=causal, variant=variant, out=oh, device=dev)

        e_ms, _ = timed(e2e_step, args.steps, 3, False)
        e_max = max_over_ranks(e_ms)
        check_status()
        rates = gather((h2d_gbs, d2h_gbs))
        e2e = {
            "value": flops_of(c) / (e_max * 1e-3) / 1e12,
            "unit": "TFLOPS",
            "ms_per_step": e_max,
            "h2d_bytes_per_step": in_bytes,
            "d2h_bytes_per_step": out_bytes,
            "per_rank": world > 1,
            "steps": args.steps,
            "h2d_gbs_measured": [round(r[0], 1) for r in rates],
            "d2h_gbs_measured": [round(r[1], 1) for r in rates],
            "link_bound_ms": (in_bytes / (min(r[0] for r in rates) * 1e9) + out_bytes / (min(r[1] for r in rates) * 1e9)) * 1e3,
            "cpu_affinity": f"{len(cpus)} CPUs near the GPU (NVML)" if cpus else "not set",
            "api": "fa.forward_host (pinned host q, k, v and O of this rank's heads; transfers overlapped with the kernels over 8 head chunks)",
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(c, args.cpu_budget_s)

    shards = gather((shard.start, shard.stop, round(ms, 4)))
    if rank == 0:
        smem, threads = _C.kernel_info(d, variant)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded N(0,1) fp16 inputs per head, CPU generator)",
            "config": config_dict(c, world),
            "shards": [{"rank": r, "heads": [s, e], "ms_per_step": t} for r, (s, e, t) in enumerate(shards)],
            "pct_tc_peak": value / world / peak,
            "roofline": {
                "bound": "tensor",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_source": (f"measured bf16/fp16 dense burst (MEASURED_PEAKS.json bf16_tflops)"
                                if peak_kind == "measured" else "fallback 1590 TFLOP/s"),
                "traffic": traffic_per_launch(c["name"]) if world == 1 else None,
                "algorithmic_bytes": 4 * shard.heads * n * d * 2,
                "kernel": f"fa_fwd_sm100_kernel (smem {smem} B, {threads} threads/CTA), rank 0's shard",
            },
            "clocks": clocks,
            "plan_rank0": plan_of(qd, causal, variant),
            "gpu_launches": args.steps * kpl * world,
            "noncausal" if causal else "causal": twin,
            "weak_scaling": weak,
            "per_config": per_config,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
