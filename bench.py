"""Benchmark of the B200 FlashAttention-2 forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg1]
                    [--impl ours|reference|reference-kernel]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Metric: attention forward TFLOPS = 4 B H N^2 d / t, halved for causal (the reference's count,
bench/benchmark.py:142). A step is one forward pass over one batch of the workload:
  * N = 1: the workload is BASELINE config 1 (B4 H16 N4096 d128 causal, seed 1) unless
    --workload names another configuration;
  * N > 1: every rank runs the same per-GPU workload on its own GPU (heads are independent, no
    collective on the data path) -> weak scaling; value = all ranks' FLOPs / max-over-ranks time.

`value` is timed on the device with CUDA events around exactly K launches with inputs resident in
HBM (inputs larger than L2); `e2e` is the same metric through the public API (fa.forward) with
the inputs copied from pinned host memory and O copied back every step. `roofline` divides the
kernel's algorithmic FLOPs per launch by its event-timed duration and by the measured bf16/fp16
dense peak. `cpu_baseline` times the CPU oracle (a numpy restatement of the reference's
fa/reference.py) on a bounded sample of heads of the same workload.

--impl reference times the reference's own CPU path (its attention_reference, as the oracle
port) on the host cores with every thread; under torchrun only rank 0 runs it.
--impl reference-kernel (a context line) times the reference's own CUDA kernel compiled for
sm_100a (baseline/build_ref_kernel.py) on the same workload and GPU.
"""

from __future__ import annotations

import argparse
import datetime
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
for _p in (str(PKG), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def workload(name: str) -> dict:
    from fa.synthetic import CONFIGS, cfg4_cases

    if name in CONFIGS:
        c = dict(CONFIGS[name])
        c.setdefault("outliers", False)
        c["variant"] = "opt"
        c["name"] = name
        return c
    if name == "cfg2acc":
        c = dict(CONFIGS["cfg2"], outliers=False, variant="fp16acc", name=name)
        return c
    if name.startswith("cfg4:"):
        # cfg4:N:d:causal, e.g. cfg4:12345:128:1
        _, n, d, causal = name.split(":")
        for c in cfg4_cases():
            if c["n"] == int(n) and c["d"] == int(d) and c["causal"] == bool(int(causal)):
                return dict(c, variant="opt", name=name)
    if name.startswith("shape:"):
        # shape:B:H:N:d:causal, seeded N(0,1) inputs (seed 5), e.g. shape:1:4:32768:128:0
        _, b, h, n, d, causal = name.split(":")
        return dict(b=int(b), h=int(h), n=int(n), d=int(d), causal=bool(int(causal)), seed=5, scale=1.0,
                    outliers=False, variant="opt", name=name)
    raise SystemExit(f"unknown workload {name}")


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
            time.sleep(0.002)

    def start(self):
        if self._h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
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


def cpu_baseline(c: dict, budget_s: float, threads: int) -> dict:
    """The oracle (numpy restatement of the reference's attention_reference) on heads of the
    workload until budget_s has elapsed (at least one head)."""
    import numpy as np

    from fa.synthetic import attention_flops, make_qkv
    from oracle import attention as oracle

    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    b, h, n, d = c["b"], c["h"], c["n"], c["d"]
    # Heads are independent: the sample draws inputs for at most 64 heads of the same shape,
    # seed and value distribution.
    distinct = min(b * h, threads)
    q, k, v = make_qkv(1, distinct, n, d, c["seed"], scale=c["scale"], outliers=c.get("outliers", False))
    qn, kn, vn = q.numpy(), k.numpy(), v.numpy()
    done, t0 = 0, time.perf_counter()
    ctx = threadpool_limits(limits=1) if threadpool_limits is not None else None
    try:
        if ctx is not None:
            ctx.__enter__()
        # one head per worker in parallel, batch after batch, until the budget is spent (the
        # workload's heads are statistically identical, so the batch is reused)
        while True:
            oracle.attention(qn, kn, vn, causal=c["causal"], threads=threads, max_chunk_bytes=n * n * 4)
            done += distinct
            if time.perf_counter() - t0 >= budget_s or done >= b * h:
                break
    finally:
        if ctx is not None:
            ctx.__exit__(None, None, None)
    dt = time.perf_counter() - t0
    flops = attention_flops(1, done, n, d, c["causal"])
    return {
        "value": flops / dt / 1e12,
        "unit": "TFLOPS",
        "cores": threads,
        "kind": "port",
        "sample": f"{done} of {b * h} heads of {c['name']} ({distinct} at a time, one per core; numpy fp32 "
                  f"restatement of fa/reference.py, {dt:.1f} s)",
    }


def run_reference_arm(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path (oracle port) on rank 0 only."""
    if rank != 0:
        return
    import numpy as np

    from fa.synthetic import attention_flops, make_qkv
    from oracle import attention as oracle

    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    c = workload(args.workload)
    threads = max(1, os.cpu_count() or 1)
    n, d = c["n"], c["d"]
    # One step = the oracle over `per_step` heads of the workload (a bounded sample).
    per_step = max(1, min(threads, 8))
    q, k, v = make_qkv(1, per_step, n, d, c["seed"], scale=c["scale"], outliers=c.get("outliers", False))
    qn, kn, vn = q.numpy(), k.numpy(), v.numpy()

    def step():
        oracle.attention(qn, kn, vn, causal=c["causal"], threads=threads, max_chunk_bytes=n * n * 4)

    ctx = threadpool_limits(limits=1) if threadpool_limits is not None else None
    if ctx is not None:
        ctx.__enter__()
    try:
        for _ in range(args.warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        dt = time.perf_counter() - t0
    finally:
        if ctx is not None:
            ctx.__exit__(None, None, None)
    flops = attention_flops(1, per_step, n, d, c["causal"]) * args.steps
    value = flops / dt / 1e12
    line = {
        "impl": "reference",
        "metric": "attn fwd TFLOPS (fp16, d=64/128, causal+non) at 1/2/4/8 B200; % of TC peak",
        "value": value,
        "unit": "TFLOPS",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / max(1, args.steps),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) fp16 inputs, CPU generator)",
        "config": {"workload": c["name"], "B": c["b"], "H": c["h"], "N": n, "d": d, "causal": c["causal"],
                   "sample_heads_per_step": per_step},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": f"{per_step} heads of {c['name']} per step, numpy fp32 restatement of fa/reference.py"},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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

    from fa import _C
    from fa.synthetic import attention_flops, make_qkv

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
    q, k, v = make_qkv(b, h, n, d, c["seed"], scale=c["scale"], outliers=c.get("outliers", False))
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    od = torch.empty_like(qd)
    stream = torch.cuda.current_stream(dev)
    err = ctypes.create_string_buffer(512)
    scale = 1.0 / math.sqrt(d)

    def step():
        rc = lib.fa_ref_kernel_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), b, h, n, d,
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
    # Same inputs through this repository's kernel, for the difference of the two outputs.
    ours = _C.forward(qd, kd, vd, causal, None, variant)
    diff = (ours.float() - od.float()).abs()
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    flops = attention_flops(b, h, n, d, causal)
    value = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "impl": "reference-kernel",
        "metric": "attn fwd TFLOPS (fp16, d=64/128, causal+non) at 1/2/4/8 B200; % of TC peak",
        "value": value,
        "unit": "TFLOPS",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16 inputs from a CPU generator)",
        "config": {"workload": c["name"], "B": b, "H": h, "N": n, "d": d, "causal": causal, "variant": variant},
        "pct_tc_peak": value / peak,
        "peak_source": peak_kind,
        "clocks": clocks,
        "max_abs_diff_vs_ours": float(diff.max()),
        "kernel": "reference csrc/kernels/flash_fwd.cu (mma.sync m16n8k16) built for sm_100a with the reference's nvcc flags",
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="cfg1")
    ap.add_argument("--variant", default=None, help="override the workload's kernel variant")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-kernel"])
    ap.add_argument("--cpu-budget-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
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

    import torch
    import torch.distributed as dist

    import fa
    from fa import _C
    from fa.synthetic import attention_flops, make_qkv

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    c = workload(args.workload)
    variant = args.variant or c["variant"]
    b, h, n, d, causal = c["b"], c["h"], c["n"], c["d"], c["causal"]
    q, k, v = make_qkv(b, h, n, d, c["seed"], scale=c["scale"], outliers=c.get("outliers", False))
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    flops = attention_flops(b, h, n, d, causal)
    io_bytes = 4 * q.numel() * 2  # read Q, K, V, write O
    stream = torch.cuda.current_stream(dev)

    def step():
        return _C.forward(qd, kd, vd, causal, None, variant)

    # kernels per step: the attention kernel, plus the split-KV combine when the library splits
    splits = _C.choose_splits(_C.make_params(qd, kd, vd, qd, causal, 1.0, _C.parse_variant(variant)), dev)
    kernels_per_step = 1 if splits == 1 else 2

    # ---- device-timed kernel throughput (value, roofline) ----
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local_rank)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    start.record(stream)
    launches = 0
    for _ in range(args.steps):
        step()
        launches += 1
    stop.record(stream)
    stop.synchronize()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms = start.elapsed_time(stop) / args.steps
    ms_max = max_over_ranks(ms)
    status = _C.device_status(local_rank, clear=True)
    if status != 0:
        raise SystemExit(f"kernel watchdog fired (status {status:#x}); timing invalid")

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        qh, kh, vh = q.pin_memory(), k.pin_memory(), v.pin_memory()
        oh = torch.empty_like(qh).pin_memory()
        e_steps = max(1, min(args.steps, 20))

        def e2e_step():
            # fa.forward_host: host q, k, v in, host O out, copies and kernels pipelined over
            # chunks of heads (the copies run inside the timed region every step).
            fa.forward_host(qh, kh, vh, causal=causal, variant=variant, out=oh, device=dev)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        e1.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1) / e_steps)
        e2e = {
            "value": flops * world / (e_ms * 1e-3) / 1e12,
            "unit": "TFLOPS",
            "ms_per_step": e_ms,
            "h2d_bytes_per_step": 3 * q.numel() * 2,
            "d2h_bytes_per_step": q.numel() * 2,
            "steps": e_steps,
            "api": "fa.forward_host (pinned host q, k, v and O; transfers overlapped with the kernels over 8 head chunks)",
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(c, args.cpu_budget_s, max(1, os.cpu_count() or 1))

    if rank == 0:
        peaks, peak_kind = load_peaks()
        achieved = flops / (ms * 1e-3) / 1e12
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        value = flops * world / (ms_max * 1e-3) / 1e12
        traffic = traffic_per_launch(c["name"])
        smem, threads = _C.kernel_info(d, variant)
        line = {
            "metric": "attn fwd TFLOPS (fp16, d=64/128, causal+non) at 1/2/4/8 B200; % of TC peak",
            "value": value,
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded N(0,1) fp16 inputs from a CPU generator)",
            "config": {
                "workload": c["name"], "B": b, "H": h, "N": n, "d": d, "causal": causal,
                "variant": variant, "global_heads": b * h * world, "parallelism": f"heads x{world} (no collective)",
                "kv_splits": splits,
                "l2": f"inputs larger than L2 ({io_bytes / 1e6:.0f} MB of Q,K,V,O per step)",
            },
            "pct_tc_peak": value / world / peak,
            "hbm_gbs_algorithmic": io_bytes / (ms * 1e-3) / 1e9,
            "roofline": {
                "bound": "tensor",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_source": f"{peak_kind} bf16/fp16 dense (MEASURED_PEAKS.json bf16_tflops)" if peak_kind == "measured" else "fallback 1590 TFLOP/s",
                "traffic": traffic,
                "algorithmic_bytes": io_bytes,
                "kernel": f"fa_fwd_sm100_kernel (smem {smem} B, {threads} threads/CTA)",
            },
            "clocks": clocks,
            "gpu_launches": launches * kernels_per_step * world,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
