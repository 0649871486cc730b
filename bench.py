"""Benchmark of the dense-contraction path on B200; prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl choreo|reference]
                    [--workload auto|gemm8192|sharded]

Workloads (inputs are seeded synthetic data of the configuration's shapes and
distributions; nothing is read from disk):
  gemm8192  fp16 GEMM C[8192x8192] = A[8192x8192] B[8192x8192], row-major,
            U[-1,1], fp32 accumulation, fp16 output. The default at N = 1.
  sharded   row-sharded bf16 GEMM M=65536, N=K=8192, U[-0.5,0.5], bias ~N(0,0.1)
            fused with ReLU, bf16 output; rows split across the N ranks
            (strong scaling: total work fixed), B and bias replicated, no
            collective on the data path. The default at N > 1.
One step = one GEMM launch over the whole workload (per rank: its slab).

value : whole-job TFLOP/s with inputs resident in HBM; K steps timed with CUDA
        events on the launching stream between barrier + synchronize, max over
        ranks. A and B together exceed the 126 MB L2, so no flush is needed.
e2e   : the same metric through the C ABI with pinned HOST buffers: every step
        copies A (slab) and B (+bias) host->device, runs the GEMM and copies C
        back, all inside the timed region.
cpu_baseline : the reference's own CPU operator* (include/choreo-ir/choreo-ir.hpp
        :71-101, compiled from its sources into oracle/_ref) on a bounded row
        sample, on the host's cores; the oracle's C restatement when the
        reference library is absent.
--impl reference : that reference CPU path alone, as the comparison arm.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

F16, F32, BF16 = 8, 9, 11
NOMINAL_DENSE_TFLOPS = 2250.0


# ----------------------------------------------------------------- helpers
def load_choreo():
    spec = importlib.util.spec_from_file_location("choreo_b200", ROOT / "choreo-ir_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["choreo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def workload_spec(name: str, world: int, shape: str | None = None, dtype: str = "f16") -> dict:
    if name == "custom":
        m, n, k = (int(x) for x in (shape or "4096x4096x4096").lower().split("x"))
        return dict(workload=f"gemm_{dtype}_{m}x{n}x{k}", m_total=m, n=n, k=k, dtype=dtype,
                    dist="U[-1,1]", bias=False, relu=False, layout="NN")
    if name == "gemm8192":
        return dict(workload="gemm_f16_8192x8192x8192", m_total=8192, n=8192, k=8192, dtype="f16",
                    dist="U[-1,1]", bias=False, relu=False, layout="NN")
    if name == "sharded":
        return dict(workload="rowsharded_gemm_bf16_65536x8192x8192_bias_relu", m_total=65536, n=8192, k=8192,
                    dtype="bf16", dist="U[-0.5,0.5]", bias=True, relu=True, layout="NN")
    raise SystemExit(f"unknown workload {name}")


def measured_peak(timed_seconds: float) -> tuple[float, str]:
    """Dense bf16/fp16 tensor peak to report against: the pool's measured
    cuBLAS figure, burst for a short timed region, sustained for a long one."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if timed_seconds > 2.0 and d.get("bf16_tflops_sustained"):
            return float(d["bf16_tflops_sustained"]), "measured (sustained cuBLAS bf16)"
        return float(d["bf16_tflops"]), "measured (burst cuBLAS bf16)"
    return 1590.0, "fallback"


def profiled_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (a `dram_bytes_per_launch: <n>` line), else None."""
    f = ROOT / "profiles" / f"{workload}.md"
    if f.exists():
        for line in f.read_text().splitlines():
            if line.strip().startswith("dram_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip().split()[0]))
                except ValueError:
                    return None
    return None


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.ids = ",".join(str(i) for i in gpu_indices)
        self.samples: list[list[str]] = []
        self.proc = None
        self.thread = None
        self.marks: list[tuple[float, float]] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", self.ids], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([time.time()] + [x.strip() for x in line.split(",")])

    def mark(self, t0: float, t1: float):
        self.marks.append((t0, t1))

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        inside = [s for s in self.samples if any(a - 0.06 <= s[0] <= b + 0.06 for a, b in self.marks)]
        use = inside or self.samples
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in use:
            try:
                sm.append(float(s[2]))
                mx.append(float(s[3]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, s[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(use), "samples_in_timed_region": len(inside)}


# ----------------------------------------------------------------- reference CPU path
def reference_cpu_sample(spec: dict, seconds_target: float, nthreads: int | None = None) -> dict:
    """Times the reference CPU operator* on a bounded sample of the workload:
    `rows` rows of A (one per thread) against a column slice of B, chosen so
    one call takes about `seconds_target`. Per element the arithmetic is the
    reference's (fp16/bf16 accumulation in k order)."""
    import numpy as np
    from oracle import oracle as orc
    dt = F16 if spec["dtype"] == "f16" else BF16
    lo, hi = (-1.0, 1.0) if spec["dist"] == "U[-1,1]" else (-0.5, 0.5)
    threads = nthreads or orc.threads()
    k, n = spec["k"], spec["n"]
    use_ref = orc.ref is not None
    # calibrate: one row x 256 columns on one thread
    a1 = orc.to_bits(orc.uniform((1, k), lo, hi, 1), dt)
    b1 = orc.to_bits(orc.uniform((k, 256), lo, hi, 2), dt)
    t0 = time.perf_counter()
    orc.ref_matmul(a1, b1, dt, nthreads=1, use_reference_lib=use_ref)
    per_elem = (time.perf_counter() - t0) / 256
    # one row per thread per pass; widen the column slice, then add rows, until
    # a call is expected to take about seconds_target
    elems = max(64.0, seconds_target / max(per_elem, 1e-9))
    cols = int(min(n, elems))
    rows = threads * max(1, int(elems // n))
    a = orc.to_bits(orc.uniform((rows, k), lo, hi, 3), dt)
    b = orc.to_bits(orc.uniform((k, cols), lo, hi, 4), dt)
    return dict(a=a, b=b, dt=dt, rows=rows, cols=cols, threads=threads, use_ref=use_ref,
                flops=2.0 * rows * cols * k)


def run_reference_sample(s: dict) -> float:
    from oracle import oracle as orc
    t0 = time.perf_counter()
    orc.ref_matmul(s["a"], s["b"], s["dt"], nthreads=s["threads"], use_reference_lib=s["use_ref"])
    return time.perf_counter() - t0


def sample_text(s: dict, spec: dict) -> str:
    src = ("reference operator* compiled from its sources (oracle/_ref)" if s["use_ref"]
           else "oracle C restatement of the reference operator*")
    return (f"{s['rows']} rows x {s['cols']} of {spec['n']} columns of C at K={spec['k']} "
            f"({spec['dtype']}, accumulation in {spec['dtype']} as the reference does); {src}; "
            f"{s['threads']} host threads splitting the rows")


# ----------------------------------------------------------------- main arms
def bench_reference(args, spec: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    s = reference_cpu_sample(spec, seconds_target=float(os.environ.get("CHOREO_REF_STEP_SECONDS", "1.0")))
    for _ in range(args.warmup):
        run_reference_sample(s)
    times = [run_reference_sample(s) for _ in range(args.steps)]
    total = sum(times)
    value = s["flops"] * args.steps / total / 1e12
    line = {
        "metric": args.metric, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong" if spec["m_total"] == 65536 else "weak",
        "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
        "config": {**{k: v for k, v in spec.items()}, "timed": "CPU wall clock per step over a bounded sample"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": s["threads"],
                         "kind": "reference" if s["use_ref"] else "port", "sample": sample_text(s, spec)},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_choreo(args, spec: dict, world: int, rank: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    cb = load_choreo()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dt = torch.float16 if spec["dtype"] == "f16" else torch.bfloat16
    lo, hi = (-1.0, 1.0) if spec["dist"] == "U[-1,1]" else (-0.5, 0.5)
    M_total, N, K = spec["m_total"], spec["n"], spec["k"]
    r0, rows = cb.shard_rows(M_total, world, rank)

    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    a = torch.empty(rows, K, device=dev).uniform_(lo, hi, generator=g).to(dt)
    g.manual_seed(99)  # B and bias are replicas: same seed on every rank
    b = torch.empty(K, N, device=dev).uniform_(lo, hi, generator=g).to(dt)
    bias = torch.empty(N, device=dev).normal_(0.0, 0.1, generator=g).to(dt) if spec["bias"] else None
    c = torch.empty(rows, N, device=dev, dtype=dt)
    stream = torch.cuda.current_stream(dev)
    desc = cb.make_gemm_desc(a, b, c, m=rows, n=N, k=K, bias=bias, relu=spec["relu"])
    q = cb.gemm_query(desc)
    assert q.workspace_bytes == 0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def step():
        cb.gemm_desc(desc, stream=stream)

    # ---------------------------------------------------------- device-resident timing
    for _ in range(args.warmup):
        step()
    cb.sync_status(stream)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = [int(x) for x in visible.split(",")] if visible else list(range(max(world, 1)))
    sampler = ClockSampler(phys[:world] if rank == 0 else [phys[local_rank]]) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    t_wall1 = time.time()
    cb.sync_status(stream)
    ms = e0.elapsed_time(e1)
    if sampler:
        sampler.mark(t_wall0, t_wall1)

    # ---------------------------------------------------------- end to end from pinned host buffers
    a_h = torch.empty(rows, K, dtype=dt, pin_memory=True)
    a_h.copy_(a)
    b_h = torch.empty(K, N, dtype=dt, pin_memory=True)
    b_h.copy_(b)
    bias_h = None
    if bias is not None:
        bias_h = torch.empty(N, dtype=dt, pin_memory=True)
        bias_h.copy_(bias)
    c_h = torch.empty(rows, N, dtype=dt, pin_memory=True)
    h2d = a_h.numel() * a_h.element_size() + b_h.numel() * b_h.element_size() + \
        (bias_h.numel() * bias_h.element_size() if bias_h is not None else 0)
    d2h = c_h.numel() * c_h.element_size()

    def e2e_step():
        a.copy_(a_h, non_blocking=True)
        b.copy_(b_h, non_blocking=True)
        if bias is not None:
            bias.copy_(bias_h, non_blocking=True)
        cb.gemm_desc(desc, stream=stream)
        c_h.copy_(c, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 20))
    for _ in range(max(1, min(args.warmup, 3))):
        e2e_step()
    barrier()
    t_wall2 = time.time()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e3.record(stream)
    barrier()
    t_wall3 = time.time()
    cb.sync_status(stream)
    ms_e2e = e2.elapsed_time(e3)
    clocks = None
    if sampler:
        sampler.mark(t_wall2, t_wall3)
        clocks = sampler.stop()

    # ---------------------------------------------------------- max over ranks
    t = torch.tensor([ms, ms_e2e], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, ms_e2e_max = float(t[0]), float(t[1])
    flops_total = 2.0 * M_total * N * K
    value = flops_total * args.steps / (ms_max * 1e-3) / 1e12
    e2e_value = flops_total * e2e_steps / (ms_e2e_max * 1e-3) / 1e12
    # dominant kernel on this rank: one launch per step, back to back on `stream`
    per_launch_ms = ms / args.steps
    achieved = 2.0 * rows * N * K / (per_launch_ms * 1e-3) / 1e12
    peak, peak_src = measured_peak(ms * 1e-3)

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        s = reference_cpu_sample(spec, seconds_target=float(os.environ.get("CHOREO_CPU_BASELINE_SECONDS", "12")))
        secs = run_reference_sample(s)
        cpu = {"value": s["flops"] / secs / 1e12, "unit": "TFLOP/s", "cores": s["threads"],
               "kind": "reference" if s["use_ref"] else "port", "sample": sample_text(s, spec),
               "seconds": round(secs, 2)}
    line = {
        "metric": args.metric,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if spec["m_total"] == 65536 and world > 1 else "weak",
        "vs_baseline": None,
        "dtype": spec["dtype"],
        "data": "synthetic",
        "pct_of_nominal_dense_peak": 100.0 * value / (NOMINAL_DENSE_TFLOPS * world),
        "config": {
            "workload": spec["workload"], "m": M_total, "n": N, "k": K, "layout": spec["layout"],
            "inputs": f"{spec['dist']} seeded on device; fp32 accumulation; {spec['dtype']} output",
            "epilogue": "bias+ReLU" if spec["bias"] else "none",
            "parallelism": f"row-sharded over {world} GPU(s), B replicated, no collective" if world > 1 else "single GPU",
            "rows_per_rank": rows, "tile": f"{q.tile_m}x{q.tile_n}x{q.tile_k}", "stages": q.stages,
            "grid": q.grid_x, "l2": "inputs larger than the 126 MB L2 (no flush needed)",
        },
        "roofline": {
            "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": peak_src, "traffic": profiled_traffic(spec["workload"]),
            "algorithmic_flops_per_launch": 2.0 * rows * N * K,
            "per_launch_ms": per_launch_ms,
        },
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "ms_per_step": ms_e2e_max / e2e_steps},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="choreo", choices=["choreo", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto", "gemm8192", "sharded", "custom"])
    ap.add_argument("--shape", default=None, help="MxNxK for --workload custom")
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16"], help="input/output type for --workload custom")
    ap.add_argument("--tile", default=None,
                    help="force a kernel configuration: pair256, pair128, single256, single128 or single64")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.metric = "fp16 GEMM TFLOP/s @8192^3 and % of B200 dense peak; sharded GEMM at 1/2/4/8 GPU"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = args.workload if args.workload != "auto" else ("gemm8192" if world == 1 else "sharded")
    spec = workload_spec(wl, world, args.shape, args.dtype)
    if args.tile:
        os.environ["CHOREO_GEMM_TILE"] = args.tile

    if args.impl == "reference":
        bench_reference(args, spec, world, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    try:
        bench_choreo(args, spec, world, rank, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
