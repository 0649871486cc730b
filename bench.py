"""Benchmark of the dense-contraction path on B200; prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl choreo|reference]
                    [--workload auto|sharded|gemm8192|custom|smallk|conv|relu]

Workloads (inputs are seeded synthetic data of the configuration's shapes and
distributions; nothing is read from disk):
  sharded   row-sharded bf16 GEMM M=65536, N=K=8192, U[-0.5,0.5], bias ~N(0,0.1)
            fused with ReLU, bf16 output; rows split across the N ranks
            (strong scaling: total work fixed), B and bias replicated, no
            collective on the data path. The default at every N, N = 1
            included, so the 1 -> N curve compares one workload.
  gemm8192  fp16 GEMM C[8192x8192] = A[8192x8192] B[8192x8192], row-major,
            U[-1,1], fp32 accumulation, fp16 output.
  custom    GEMM of --shape MxNxK and --dtype (U[-1,1]), stored as --layout
            (NN default), with a fused bias + ReLU when --bias-relu is given.
  smallk    fp16 GEMM 16384 x 16384 x 128: output-write (HBM) bound.
  conv      implicit-GEMM conv2d NHWC fp16, N=32, 56x56, C=K=256, 3x3, s1 p1,
            activations U[0,1], weights N(0, 1/48), bias N(0, 0.1) + ReLU; at
            N > 1 the 32 images are split across the ranks (strong scaling).
  relu      elementwise ReLU over 2^28 fp16 values (HBM bound).
One step = one launch of the path over the whole workload (per rank: its slab).

value : whole-job throughput with inputs resident in HBM; K steps timed with
        CUDA events on the launching stream between barrier + synchronize,
        max over ranks. Where the inputs fit in the 126 MB L2 (conv, smallk),
        a 256 MB buffer is written between steps and each launch is timed by
        its own event pair; elsewhere the inputs exceed the L2.
e2e   : the same metric through the C ABI's host-buffer plans
        (choreo_host_gemm_run / choreo_host_conv_run) with pinned HOST
        buffers: every step copies the inputs host->device, runs the launches
        and copies the output back, all inside the timed region. For the
        sharded GEMM at N > 1, B crosses PCIe once per step in total: each rank
        copies 1/N of B's rows and an NCCL all-gather over NVLink assembles B
        on every rank (inside the timed region).
configs : at N = 1, every other configuration of the benchmark suite (1024 x
        1024 x 512; 2048/4096/8192 cubes in f16 and bf16; 4097 x 3000 x 1536 in
        NN/NT/TN; the 3x3 conv; small-K) timed the same way, with cuBLAS /
        cuDNN (through torch) on the same GPU as a side reference.
cpu_baseline : the reference's own CPU path (operator*, relu from
        include/choreo-ir/choreo-ir.hpp, compiled from its sources into
        oracle/_ref) on a bounded sample, on all of the host's cores; the
        oracle's C restatement where the reference library is absent or has no
        such entry (conv: the loop of benchmark/kernels/gemm_example.cu:208-253).
--impl reference : that reference CPU path alone, as the comparison arm (rank
        0 only under torchrun; same `config` block as this arm's).
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
HEADLINE_METRIC = "fp16 GEMM TFLOP/s @8192^3 and % of B200 dense peak; sharded GEMM at 1/2/4/8 GPU"
L2_BYTES = 126 * 1024 * 1024


# ----------------------------------------------------------------- helpers
def load_choreo():
    spec = importlib.util.spec_from_file_location("choreo_b200", ROOT / "choreo-ir_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["choreo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def host_cores() -> int:
    """Host threads this process may run on (the affinity mask, not
    OMP_NUM_THREADS, which torchrun sets to 1 for every rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _gemm(workload, m, n, k, dtype, dist, bias, relu, layout="NN"):
    return dict(kind="gemm", workload=workload, m_total=m, n=n, k=k, dtype=dtype, dist=dist, bias=bias,
                relu=relu, layout=layout)


def workload_spec(name: str, shape: str | None = None, dtype: str = "f16", layout: str = "NN",
                  bias_relu: bool = False) -> dict:
    if name == "custom":
        m, n, k = (int(x) for x in (shape or "4096x4096x4096").lower().split("x"))
        suffix = ("" if layout == "NN" else f"_{layout}") + ("_bias_relu" if bias_relu else "")
        return _gemm(f"gemm_{dtype}_{m}x{n}x{k}{suffix}", m, n, k, dtype, "U[-1,1]", bias_relu, bias_relu, layout)
    if name == "gemm8192":
        return _gemm("gemm_f16_8192x8192x8192", 8192, 8192, 8192, "f16", "U[-1,1]", False, False)
    if name == "sharded":
        return _gemm("rowsharded_gemm_bf16_65536x8192x8192_bias_relu", 65536, 8192, 8192, "bf16",
                     "U[-0.5,0.5]", True, True)
    if name == "smallk":
        return _gemm("gemm_f16_16384x16384x128", 16384, 16384, 128, "f16", "U[-1,1]", False, False)
    if name == "conv":
        return dict(kind="conv", workload="conv2d_f16_n32_56x56_c256_k256_3x3_bias_relu", n=32, h=56, w=56,
                    c=256, k=256, r=3, s=3, stride=1, pad=1, dtype="f16", bias=True, relu=True)
    if name == "relu":
        return dict(kind="relu", workload="relu_f16_268435456", numel=1 << 28, dtype="f16")
    raise SystemExit(f"unknown workload {name}")


def spec_flops_bytes(spec: dict, rows: int | None = None) -> tuple[float, float]:
    """Algorithmic FLOPs and HBM bytes of one launch (rows: this rank's slab)."""
    if spec["kind"] == "gemm":
        m = rows if rows is not None else spec["m_total"]
        n, k = spec["n"], spec["k"]
        ob = 2.0
        return 2.0 * m * n * k, 2.0 * (m * k + k * n) + ob * m * n + (2.0 * n if spec["bias"] else 0.0)
    if spec["kind"] == "conv":
        npix = spec["n"] * spec["h"] * spec["w"]          # stride 1, same padding
        red = spec["r"] * spec["s"] * spec["c"]
        return (2.0 * npix * spec["k"] * red,
                2.0 * (npix * spec["c"] + spec["k"] * red + npix * spec["k"] + spec["k"]))
    return 0.0, 4.0 * spec["numel"]


def shard_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Rows of an m-row problem rank `rank` of `world` owns: the partition of
    choreo_shard_rows (whole 128-row tiles, counts differing by at most one
    tile), restated so the reference arm needs no GPU library."""
    tiles = (m + 127) // 128
    base, extra = divmod(tiles, world)
    t0 = rank * base + min(rank, extra)
    nt = base + (1 if rank < extra else 0)
    r0, r1 = min(t0 * 128, m), min((t0 + nt) * 128, m)
    return r0, r1 - r0


def b_rows_share(k: int, world: int, rank: int) -> tuple[int, int, int]:
    """The rows of B (K x N) rank `rank` copies from the host when B crosses
    PCIe once for the whole job: (share, k0, k1) with `share` rows per rank
    (the last ranks' tails empty when world does not divide K) and this rank's
    rows [k0, k1). An all-gather of the `share`-row parts assembles B's K rows
    at the head of a world * share row buffer on every rank."""
    share = -(-k // world)
    return share, min(rank * share, k), min((rank + 1) * share, k)


def conv_images(n: int, world: int, rank: int) -> tuple[int, int]:
    """This rank's contiguous run of images (first, count): the batch split
    evenly, the first n % world ranks taking one extra."""
    base, extra = divmod(n, world)
    count = base + (1 if rank < extra else 0)
    return rank * base + min(rank, extra), count


def flushes_l2(spec: dict, world: int) -> bool:
    """Inputs of rank 0's launch fit in the L2: the timing flushes it."""
    if spec["kind"] == "gemm":
        _, rows = shard_rows(spec["m_total"], world, 0)
        fl, by = spec_flops_bytes(spec, rows)
        return by - 2.0 * rows * spec["n"] <= L2_BYTES
    if spec["kind"] == "conv":
        _, imgs = conv_images(spec["n"], world, 0)
        _, by = spec_flops_bytes({**spec, "n": imgs})
        return by - 2.0 * imgs * spec["h"] * spec["w"] * spec["k"] <= L2_BYTES
    return False


def config_block(spec: dict, world: int) -> dict:
    """The workload's `config`: a function of the workload and the GPU count
    only, so the reference arm prints the very same block."""
    l2 = ("L2 flushed (256 MB written) between timed launches; per-launch events" if flushes_l2(spec, world)
          else "inputs larger than the 126 MB L2 (no flush needed)")
    if spec["kind"] == "gemm":
        _, rows = shard_rows(spec["m_total"], world, 0)
        return {"workload": spec["workload"], "m": spec["m_total"], "n": spec["n"], "k": spec["k"],
                "layout": spec["layout"],
                "inputs": f"{spec['dist']} seeded; fp32 accumulation; {spec['dtype']} output",
                "epilogue": "bias+ReLU" if spec["bias"] else "none",
                "parallelism": (f"row-sharded over {world} GPU(s), B replicated, no collective on the data path"
                                if world > 1 else "single GPU"),
                "rows_per_rank": rows, "l2": l2}
    if spec["kind"] == "conv":
        _, imgs = conv_images(spec["n"], world, 0)
        return {"workload": spec["workload"], "n": spec["n"], "h": spec["h"], "w": spec["w"], "c": spec["c"],
                "k": spec["k"], "rs": f"{spec['r']}x{spec['s']}", "stride": spec["stride"], "pad": spec["pad"],
                "inputs": "activations U[0,1], weights N(0,1/48), bias N(0,0.1), seeded; fp32 accumulation; "
                          "fp16 output",
                "epilogue": "bias+ReLU",
                "parallelism": "single GPU" if world == 1 else
                f"batch split over {world} GPUs, weights replicated, no collective",
                "images_per_rank": imgs, "l2": l2}
    return {"workload": spec["workload"], "numel": spec["numel"], "inputs": "U[-1,1] seeded",
            "parallelism": "single GPU" if world == 1 else f"{world} independent replicas", "l2": l2}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else {}


def measured_peak(timed_seconds: float) -> tuple[float, str]:
    """Dense bf16/fp16 tensor peak to report against: the pool's measured
    cuBLAS figure, burst for a short timed region, sustained for a long one."""
    d = measured_peaks()
    if d:
        if timed_seconds > 2.0 and d.get("bf16_tflops_sustained"):
            return float(d["bf16_tflops_sustained"]), "measured (sustained cuBLAS bf16)"
        return float(d["bf16_tflops"]), "measured (burst cuBLAS bf16)"
    return 1590.0, "fallback"


def measured_hbm() -> tuple[float, str]:
    d = measured_peaks()
    if d.get("hbm_gbs"):
        return float(d["hbm_gbs"]), "measured (copy, read+write bytes)"
    return 6650.0, "fallback"


def profiled_traffic(workload: str, units: float | None = None):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (a `dram_bytes_per_launch: <n>` line). A summary captured on a
    smaller slab than the launch's says so with `captured_units: <rows>`, and
    the figure is scaled by units / captured_units. None without a summary."""
    f = ROOT / "profiles" / f"{workload}.md"
    if not f.exists():
        return None
    vals = {}
    for line in f.read_text().splitlines():
        s = line.strip()
        for key in ("dram_bytes_per_launch:", "captured_units:"):
            if s.startswith(key):
                try:
                    vals[key] = float(s.split(":", 1)[1].strip().split()[0])
                except (ValueError, IndexError):
                    pass
    t = vals.get("dram_bytes_per_launch:")
    if t is None:
        return None
    cu = vals.get("captured_units:")
    if cu and units:
        t = t * units / cu
    return int(t)


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
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in use:
            try:
                sm.append(float(s[2]))
                mx.append(float(s[3]))
                pw.append(float(s[4]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, s[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_median": statistics.median(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(use), "samples_in_timed_region": len(inside)}


# ----------------------------------------------------------------- reference CPU path
def reference_cpu_sample(spec: dict, seconds_target: float, nthreads: int) -> dict:
    """A bounded sample of the workload for the reference CPU path, sized so
    one call takes about `seconds_target` on `nthreads` host threads:
      gemm: `rows` rows of A (a multiple of the thread count) against a column
            slice of B; per element the arithmetic is the reference
            operator*'s (16-bit accumulation in k order);
      conv: a run of output pixels through the reference conv loop;
      relu: a prefix of the tensor through the reference relu.
    Returns the inputs plus `units` (FLOPs, or bytes for relu) per call."""
    from oracle import oracle as orc
    threads = max(1, nthreads)
    if spec["kind"] == "gemm":
        dt = F16 if spec["dtype"] == "f16" else BF16
        lo, hi = (-1.0, 1.0) if spec["dist"] == "U[-1,1]" else (-0.5, 0.5)
        k, n = spec["k"], spec["n"]
        use_ref = orc.ref is not None
        a1 = orc.to_bits(orc.uniform((1, k), lo, hi, 1), dt)
        b1 = orc.to_bits(orc.uniform((k, 256), lo, hi, 2), dt)
        t0 = time.perf_counter()
        orc.ref_matmul(a1, b1, dt, nthreads=1, use_reference_lib=use_ref)
        per_elem = (time.perf_counter() - t0) / 256
        # one row per thread per pass; widen the column slice, then add rows,
        # until a call is expected to take about seconds_target
        elems = max(64.0, seconds_target / max(per_elem, 1e-9))
        cols = int(min(n, elems))
        rows = threads * max(1, int(elems // n))
        a = orc.to_bits(orc.uniform((rows, k), lo, hi, 3), dt)
        b = orc.to_bits(orc.uniform((k, cols), lo, hi, 4), dt)
        return dict(kind="gemm", a=a, b=b, dt=dt, rows=rows, cols=cols, threads=threads, use_ref=use_ref,
                    units=2.0 * rows * cols * k)
    if spec["kind"] == "conv":
        x = orc.to_bits(orc.uniform((1, spec["h"], spec["w"], spec["c"]), 0.0, 1.0, 5), F16)
        w = orc.to_bits(orc.normal((spec["k"], spec["r"], spec["s"], spec["c"]), 0.0, 1.0 / 48, 6), F16)
        t0 = time.perf_counter()
        orc.ref_conv2d_f16(x, w, spec["stride"], spec["pad"], pix=(0, 1), nthreads=1)
        per_pix = time.perf_counter() - t0
        npix = int(min(spec["h"] * spec["w"], max(threads, threads * seconds_target / max(per_pix, 1e-9))))
        red = spec["r"] * spec["s"] * spec["c"]
        return dict(kind="conv", x=x, w=w, npix=npix, threads=threads, use_ref=False,
                    units=2.0 * npix * spec["k"] * red, stride=spec["stride"], pad=spec["pad"])
    # relu: the reference relu is a single-threaded loop
    use_ref = orc.ref is not None
    n1 = 1 << 22
    x = orc.to_bits(orc.uniform((n1,), -1.0, 1.0, 7), F16)
    t0 = time.perf_counter()
    _relu_ref(x, use_ref)
    per = (time.perf_counter() - t0) / n1
    n = int(min(spec["numel"], max(n1, seconds_target / max(per, 1e-12))))
    x = orc.to_bits(orc.uniform((n,), -1.0, 1.0, 8), F16)
    return dict(kind="relu", x=x, n=n, threads=1, use_ref=use_ref, units=4.0 * n)


def _relu_ref(x, use_ref: bool):
    import numpy as np
    from oracle import oracle as orc
    if use_ref:
        out = np.empty_like(x)
        rc = orc.ref.choreo_ref_relu_f16(x.ctypes.data, out.ctypes.data, x.size)
        if rc != 0:
            raise RuntimeError(f"reference relu failed ({rc})")
        return out
    return orc.ref_relu(x, F16)


def run_reference_sample(s: dict) -> float:
    from oracle import oracle as orc
    t0 = time.perf_counter()
    if s["kind"] == "gemm":
        orc.ref_matmul(s["a"], s["b"], s["dt"], nthreads=s["threads"], use_reference_lib=s["use_ref"])
    elif s["kind"] == "conv":
        orc.ref_conv2d_f16(s["x"], s["w"], s["stride"], s["pad"], pix=(0, s["npix"]), nthreads=s["threads"])
    else:
        _relu_ref(s["x"], s["use_ref"])
    return time.perf_counter() - t0


def sample_text(s: dict, spec: dict) -> str:
    if s["kind"] == "gemm":
        src = ("reference operator* compiled from its sources (oracle/_ref)" if s["use_ref"]
               else "oracle C restatement of the reference operator*")
        return (f"{s['rows']} rows x {s['cols']} of {spec['n']} columns of C at K={spec['k']} "
                f"({spec['dtype']}, accumulation in {spec['dtype']} as the reference does); {src}; "
                f"{s['threads']} host threads splitting the rows")
    if s["kind"] == "conv":
        return (f"{s['npix']} output pixels x {spec['k']} channels of image 0 (3x3x{spec['c']} reduction, fp16 "
                f"accumulation as the reference conv loop does); oracle C restatement of the reference's "
                f"conv2d_kernel loop (the reference has no host conv entry to compile); "
                f"{s['threads']} host threads splitting the pixels")
    src = "reference relu compiled from its sources (oracle/_ref)" if s["use_ref"] else "oracle C restatement"
    return f"{s['n']} fp16 values; {src}; single-threaded as the reference loop is"


# ----------------------------------------------------------------- main arms
def metric_of(spec: dict) -> tuple[str, str]:
    if spec["kind"] == "relu":
        return "elementwise ReLU GB/s (fp16, 2^28 values)", "GB/s"
    if spec["kind"] == "conv":
        return "implicit-GEMM conv2d TFLOP/s (NHWC fp16 32x56x56x256, 3x3, bias+ReLU)", "TFLOP/s"
    if spec["workload"] in ("gemm_f16_8192x8192x8192", "rowsharded_gemm_bf16_65536x8192x8192_bias_relu"):
        return HEADLINE_METRIC, "TFLOP/s"
    return f"GEMM TFLOP/s ({spec['workload']})", "TFLOP/s"


def scaling_of(spec: dict, world: int) -> str:
    return "strong" if world > 1 and (spec.get("m_total") == 65536 or spec["kind"] == "conv") else "weak"


def bench_reference(args, spec: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    metric, unit = metric_of(spec)
    s = reference_cpu_sample(spec, float(os.environ.get("CHOREO_REF_STEP_SECONDS", "1.0")), host_cores())
    for _ in range(args.warmup):
        run_reference_sample(s)
    times = [run_reference_sample(s) for _ in range(args.steps)]
    total = sum(times)
    scale = 1e9 if unit == "GB/s" else 1e12
    value = s["units"] * args.steps / total / scale
    line = {
        "metric": metric, "value": value, "unit": unit, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": scaling_of(spec, world),
        "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
        "config": config_block(spec, world),
        "timing": "CPU wall clock per step over a bounded sample of the workload",
        "cpu_baseline": {"value": value, "unit": unit, "cores": s["threads"],
                         "kind": "reference" if s["use_ref"] else "port", "sample": sample_text(s, spec)},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


class Case:
    """Device buffers and the step functions of one workload on one rank."""
    step = None        # one launch on device-resident inputs
    e2e_step = None    # host->device inputs, the launch, device->host output
    floor_step = None  # the same host<->device copies with no kernel
    h2d = d2h = 0
    rows = None        # this rank's slab (GEMM rows)
    units_total = 0.0  # whole-job FLOPs (or bytes) per step
    flops = bytes_ = 0.0  # this rank's algorithmic FLOPs / bytes per launch
    flush = False      # inputs + outputs fit in L2: flush between timed launches
    launches_per_step = 1
    kernel: dict = {}  # what the dispatcher chose
    e2e_info: dict = {}


def _pinned_copy(t):
    import torch
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h


def _copy_floor(stream, dev, ins, outs):
    """The transfers of one end-to-end step and nothing else: every (device,
    pinned host) pair in `ins` copied in on one stream while every (host,
    device) pair in `outs` is copied out on another. Its time is the floor
    the host links put under the end-to-end step (the same bytes, no kernel)."""
    import torch
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step():
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        with torch.cuda.stream(s_in):
            for d, h in ins:
                if d is not None and d.numel():
                    d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            for h, d in outs:
                h.copy_(d, non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)
    return step


def kernel_name(q) -> str:
    if q.kernel == 3 or q.kernel == 1:
        if q.cluster_m == 2 and q.tile_m == 512:
            base = "tc_gemm_pair_wide_kernel"
        elif q.cluster_m == 2:
            base = "tc_gemm_pair_kernel"
        else:
            base = "tc_gemm_kernel"
        return f"{base} ({q.tile_m}x{q.tile_n}x{q.tile_k} tile{', CTA pair' if q.cluster_m == 2 else ''}" + \
               (f", K split {q.split_k} + splitk_reduce_kernel" if q.split_k > 1 else "") + ")"
    return "gemm_f32_kernel"


def setup_gemm(cb, spec, world, rank, dev, stream) -> Case:
    import torch
    import torch.distributed as dist
    dt = torch.float16 if spec["dtype"] == "f16" else torch.bfloat16
    lo, hi = (-1.0, 1.0) if spec["dist"] == "U[-1,1]" else (-0.5, 0.5)
    M_total, N, K = spec["m_total"], spec["n"], spec["k"]
    r0, rows = cb.shard_rows(M_total, world, rank)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    ta, tb = spec["layout"][0] == "T", spec["layout"][1] == "T"   # A stored K x M / B stored N x K
    a = torch.empty((K, rows) if ta else (rows, K), device=dev).uniform_(lo, hi, generator=g).to(dt)
    g.manual_seed(99)  # B and bias are replicas: same seed on every rank
    b = torch.empty((N, K) if tb else (K, N), device=dev).uniform_(lo, hi, generator=g).to(dt)
    bias = torch.empty(N, device=dev).normal_(0.0, 0.1, generator=g).to(dt) if spec["bias"] else None
    c = torch.empty(rows, N, device=dev, dtype=dt)
    desc = cb.make_gemm_desc(a, b, c, m=rows, n=N, k=K, trans_a=ta, trans_b=tb, lda=a.stride(0), ldb=b.stride(0),
                             bias=bias, relu=spec["relu"])
    q = cb.gemm_query(desc)
    case = Case()
    # The workspace holds the repack of an operand whose rows are not 16-byte
    # aligned (each one a launch before the GEMM) and the fp32 partials of a
    # K split (plus its reduction pass).
    ws = torch.empty(max(1, q.workspace_bytes), dtype=torch.uint8, device=dev)
    case.step = lambda: cb.gemm_desc(desc, ws, q.workspace_bytes, stream=stream)
    repacks = int(a.stride(0) * 2 % 16 != 0) + int(b.stride(0) * 2 % 16 != 0)
    case.launches_per_step = 1 + repacks + (1 if q.split_k > 1 else 0)
    if spec["layout"] != "NN":
        # the host-buffer plans stream row-major NN operands only
        case.rows = rows
        case.flops, case.bytes_ = spec_flops_bytes(spec, rows)
        case.units_total = spec_flops_bytes(spec)[0]
        case.flush = flushes_l2(spec, world)
        case.kernel = {"name": kernel_name(q), "tile": f"{q.tile_m}x{q.tile_n}x{q.tile_k}", "repacks": repacks}
        return case
    a_h, b_h = _pinned_copy(a), _pinned_copy(b)
    bias_h = _pinned_copy(bias) if bias is not None else None
    c_h = torch.empty(rows, N, dtype=dt, pin_memory=True)
    plan = cb.HostGemmPlan(rows, N, K, dt, bias=bias is not None, relu=spec["relu"], device=dev)
    if world == 1:
        # one process: the plan copies B and the bias in before the row slabs
        case.e2e_step = lambda: plan.run(a_h, b_h, c_h, bias_h, stream=stream)
        case.h2d = sum(t.numel() * t.element_size() for t in (a_h, b_h, bias_h) if t is not None)
        case.e2e_info = {"path": f"choreo_host_gemm_run: pinned host A/B/bias in, C out; {plan.launches()} row "
                                 "slabs, copies in, GEMMs and copies out overlapped on three streams"}
    else:
        # B crosses PCIe once for the whole job: each rank copies 1/world of
        # B's rows, and an NCCL all-gather over NVLink assembles B everywhere.
        share, k0, k1 = b_rows_share(K, world, rank)
        b_full = torch.empty(share * world, N, device=dev, dtype=dt)
        b_part = torch.empty(share, N, device=dev, dtype=dt)
        bias_d = torch.empty_like(bias) if bias is not None else None

        def e2e():
            if k1 > k0:
                b_part[:k1 - k0].copy_(b_h[k0:k1], non_blocking=True)
            if bias_d is not None:
                bias_d.copy_(bias_h, non_blocking=True)
            dist.all_gather_into_tensor(b_full, b_part)
            plan.run(a_h, b_full, c_h, bias_d, stream=stream, operands_on_device=True)

        case.e2e_step = e2e
        case.h2d = a_h.numel() * a_h.element_size() + (k1 - k0) * N * b_h.element_size() + \
            (bias_h.numel() * bias_h.element_size() if bias_h is not None else 0)
        case.e2e_info = {"path": f"choreo_host_gemm_run with B on the device: pinned host A slab in, C slab out; "
                                 f"{plan.launches()} row slabs overlapped on three streams; B assembled per step "
                                 f"from {share} host rows per rank by an NCCL all-gather (inside the timed "
                                 f"region); bias copied in per step"}
    case.d2h = c_h.numel() * c_h.element_size()
    b_rows = (0, K) if world == 1 else (k0, k1)
    case.floor_step = _copy_floor(stream, dev, [(a, a_h), (b[b_rows[0]:b_rows[1]], b_h[b_rows[0]:b_rows[1]]),
                                                (bias, bias_h)], [(c_h, c)])
    case.rows = rows
    case.b_dev, case.c_dev = b, c
    case.flops, case.bytes_ = spec_flops_bytes(spec, rows)
    case.units_total = spec_flops_bytes(spec)[0]
    case.flush = flushes_l2(spec, world)
    case.kernel = {"name": kernel_name(q), "tile": f"{q.tile_m}x{q.tile_n}x{q.tile_k}", "cluster": q.cluster_m,
                   "stages": q.stages, "grid": q.grid_x, "split_k": int(q.split_k)}
    return case


def setup_conv(cb, spec, world, rank, dev, stream) -> Case:
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rank)
    _, imgs = conv_images(spec["n"], world, rank)
    if imgs == 0:
        raise SystemExit(f"conv: {world} ranks for {spec['n']} images")
    x = torch.empty(imgs, spec["h"], spec["w"], spec["c"], device=dev).uniform_(0, 1, generator=g).half()
    g.manual_seed(6)
    wt = torch.empty(spec["k"], spec["r"], spec["s"], spec["c"], device=dev).normal_(
        0, 1 / 48.0, generator=g).half()
    bias = torch.empty(spec["k"], device=dev).normal_(0, 0.1, generator=g).half()
    out = torch.empty(imgs, spec["h"], spec["w"], spec["k"], device=dev, dtype=torch.float16)
    d = cb.conv_desc(x, wt, out, stride=spec["stride"], padding=spec["pad"], bias=bias, relu=spec["relu"])
    q = cb.conv2d_query(d)
    assert q.workspace_bytes == 0
    case = Case()
    case.step = lambda: cb.conv2d_desc(d, stream=stream)
    x_h, w_h, b_h = _pinned_copy(x), _pinned_copy(wt), _pinned_copy(bias)
    o_h = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    plan = cb.HostConvPlan(imgs, spec["h"], spec["w"], spec["c"], spec["k"], spec["r"], spec["s"], torch.float16,
                           stride=spec["stride"], padding=spec["pad"], bias=True, relu=spec["relu"], device=dev)
    case.e2e_step = lambda: plan.run(x_h, w_h, o_h, b_h, stream=stream)
    case.h2d = sum(t.numel() * t.element_size() for t in (x_h, w_h, b_h))
    case.d2h = o_h.numel() * o_h.element_size()
    case.floor_step = _copy_floor(stream, dev, [(x, x_h), (wt, w_h), (bias, b_h)], [(o_h, out)])
    case.flops, case.bytes_ = spec_flops_bytes({**spec, "n": imgs})
    case.units_total = spec_flops_bytes(spec)[0]
    case.flush = flushes_l2(spec, world)
    case.kernel = {"name": kernel_name(q), "tile": f"{q.tile_m}x{q.tile_n}x{q.tile_k}", "cluster": q.cluster_m,
                   "stages": q.stages, "grid": q.grid_x}
    case.e2e_info = {"path": f"choreo_host_conv_run: pinned host activations/weights/bias in, output out; "
                             f"{plan.launches()} runs of images overlapped on three streams"}
    return case


def setup_relu(cb, spec, world, rank, dev, stream) -> Case:
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    x = torch.empty(spec["numel"], device=dev).uniform_(-1, 1, generator=g).half()
    y = torch.empty_like(x)
    case = Case()
    case.step = lambda: cb.relu(x, y, stream=stream)
    x_h = _pinned_copy(x)
    y_h = torch.empty_like(x_h, pin_memory=True)

    def e2e():
        x.copy_(x_h, non_blocking=True)
        cb.relu(x, y, stream=stream)
        y_h.copy_(y, non_blocking=True)

    case.e2e_step = e2e
    case.h2d = case.d2h = x_h.numel() * 2
    case.flops, case.bytes_ = spec_flops_bytes(spec)
    case.units_total = case.bytes_ * world
    case.kernel = {"name": "map_kernel (relu)"}
    case.e2e_info = {"path": "torch copies around choreo_relu"}
    return case


def time_exchanges(case, world: int, rank: int, dev, stream) -> dict:
    """The two exchanges around a row-sharded GEMM, timed apart from it over
    NCCL (NVLink / NVSwitch): replicating B from rank 0 to every rank, and
    gathering the C slabs onto rank 0. Every rank runs both, in this order;
    times are the max over ranks of CUDA-event time on the launching stream."""
    import torch
    import torch.distributed as dist
    b, c = case.b_dev, case.c_dev
    rows = torch.tensor([c.shape[0]], device=dev, dtype=torch.int64)
    all_rows = [torch.zeros_like(rows) for _ in range(world)]
    dist.all_gather(all_rows, rows)
    equal = len({int(r.item()) for r in all_rows}) == 1
    gather_list = [torch.empty_like(c) for _ in range(world)] if (rank == 0 and equal) else None

    def timed(fn, reps=3):
        fn()  # warm-up (communicator set-up)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    out = {}
    ms_b = timed(lambda: dist.broadcast(b, src=0))
    nbytes_b = b.numel() * b.element_size()
    out["b_broadcast"] = {"ms": ms_b, "bytes": nbytes_b, "GB/s": nbytes_b / (ms_b * 1e-3) / 1e9,
                          "how": "NCCL broadcast from rank 0"}
    if equal:
        ms_c = timed(lambda: dist.gather(c, gather_list=gather_list, dst=0))
        nbytes_c = c.numel() * c.element_size() * (world - 1)
        out["c_gather"] = {"ms": ms_c, "bytes_into_rank0": nbytes_c, "GB/s": nbytes_c / (ms_c * 1e-3) / 1e9,
                           "how": "NCCL gather of the C slabs onto rank 0"}
    return out


class Flusher:
    """Writes a buffer twice the L2's size between timed launches."""

    def __init__(self, dev):
        import torch
        self.buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)


def ab_timing(cb, ours, ref, stream, flush, reps: int, probe, warmup: int = 3) -> dict:
    """Our launch and the side reference's, timed alternately so both see the
    same clocks and power state:
      flushed: median device time of one call, each call bracketed by its own
               events on `stream`, the L2 overwritten before every call
               (outside the events) - the timing rule of the headline;
      back_to_back: mean over `reps` calls issued back to back (warm L2; our
               launches overlap their prologue with the previous one's tail);
      effective_sm_mhz: SM clock during our flushed calls, from the in-kernel
               probe (%clock64 / %globaltimer of CTA 0)."""
    import torch
    for _ in range(warmup):
        ours()
        ref()
    probe.zero_()
    cb.check(cb.lib.choreo_clock_probe_set(probe.data_ptr()))
    ev = lambda: torch.cuda.Event(enable_timing=True)
    mine = [(ev(), ev()) for _ in range(reps)]
    theirs = [(ev(), ev()) for _ in range(reps)]
    for (a0, a1), (b0, b1) in zip(mine, theirs):
        flush()
        a0.record(stream)
        ours()
        a1.record(stream)
        flush()
        b0.record(stream)
        ref()
        b1.record(stream)
    theirs[-1][1].synchronize()
    cb.check(cb.lib.choreo_clock_probe_set(None))
    clk = [int(v) for v in probe.cpu()]
    flushed = statistics.median(a.elapsed_time(b) for a, b in mine)
    flushed_ref = statistics.median(a.elapsed_time(b) for a, b in theirs)
    b2b = []
    for fn in (ours, ref):
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        b2b.append(e0.elapsed_time(e1) / reps)
    return {"ms": flushed, "ms_ref": flushed_ref, "ms_b2b": b2b[0], "ms_ref_b2b": b2b[1],
            "mhz": (1e3 * clk[0] / clk[1]) if clk[1] else None}


def run_configs(cb, dev, stream, reps: int) -> list[dict]:
    """The other configurations of the benchmark suite on this GPU, each timed
    through the C ABI as the median of `reps` L2-flushed launches, alternating
    with cuBLAS / cuDNN (through torch) on the same inputs as a side
    reference; back-to-back means and the effective SM clock beside them."""
    import torch
    import torch.nn.functional as Fn
    peak, peak_src = measured_peak(0.0)
    hbm, _ = measured_hbm()
    flush = Flusher(dev)
    probe = torch.zeros(3, dtype=torch.int64, device=dev)
    out = []

    def gemm_entry(cfg, m, n, k, dt, layout, dist):
        g = torch.Generator(device=dev)
        g.manual_seed(m + 3 * n + 7 * k)
        tdt = torch.float16 if dt == "f16" else torch.bfloat16

        def gen(shape):
            t = torch.empty(shape, device=dev)
            (t.uniform_(-1, 1, generator=g) if dist == "U[-1,1]" else t.normal_(0, 1, generator=g))
            return t.to(tdt)
        ta, tb = layout[0] == "T", layout[1] == "T"
        a = gen((k, m) if ta else (m, k))
        b = gen((n, k) if tb else (k, n))
        c = torch.empty(m, n, device=dev, dtype=tdt)
        d = cb.make_gemm_desc(a, b, c, m=m, n=n, k=k, trans_a=ta, trans_b=tb, lda=a.stride(0), ldb=b.stride(0))
        q = cb.gemm_query(d)
        ws = torch.empty(max(1, q.workspace_bytes), dtype=torch.uint8, device=dev)
        opa = a.t() if ta else a
        opb = b.t() if tb else b
        t = ab_timing(cb, lambda: cb.gemm_desc(d, ws, q.workspace_bytes, stream=stream), lambda: torch.matmul(opa, opb),
                      stream, flush, reps, probe)
        cb.sync_status(stream)
        ms, ms_ref = t["ms"], t["ms_ref"]
        flops = 2.0 * m * n * k
        byts = 2.0 * (m * k + k * n + m * n)
        tf = flops / (ms * 1e-3) / 1e12
        bound = "tensor" if flops / byts > peak * 1e12 / (hbm * 1e9) else "hbm"
        e = {"config": cfg, "workload": f"gemm_{dt}_{m}x{n}x{k}_{layout}", "inputs": dist, "kernel": kernel_name(q),
             "launches": 2 if q.split_k > 1 else 1 + (1 if q.workspace_min_bytes else 0),
             "us": round(ms * 1e3, 2), "tflops": round(tf, 1), "gbs": round(byts / (ms * 1e-3) / 1e9, 1),
             "bound": bound,
             "frac": round(tf / peak, 4) if bound == "tensor" else round(byts / (ms * 1e-3) / 1e9 / hbm, 4),
             "us_back_to_back": round(t["ms_b2b"] * 1e3, 2), "effective_sm_mhz": t["mhz"] and round(t["mhz"]),
             "side_reference": {"what": "cuBLAS via torch.matmul, same inputs and layout", "us": round(ms_ref * 1e3, 2),
                                "tflops": round(flops / (ms_ref * 1e-3) / 1e12, 1),
                                "us_back_to_back": round(t["ms_ref_b2b"] * 1e3, 2)},
             "time_vs_side_reference": round(ms / ms_ref, 3),
             "time_vs_side_reference_back_to_back": round(t["ms_b2b"] / t["ms_ref_b2b"], 3)}
        out.append(e)
        del a, b, c, ws

    gemm_entry("1", 1024, 1024, 512, "f16", "NN", "U[-1,1]")
    for s in (2048, 4096, 8192):
        for dt in ("f16", "bf16"):
            gemm_entry("2", s, s, s, dt, "NN", "U[-1,1]")
    for layout in ("NN", "NT", "TN"):
        gemm_entry("3", 4097, 3000, 1536, "f16", layout, "N(0,1)")
    gemm_entry("small-K", 16384, 16384, 128, "f16", "NN", "U[-1,1]")

    # config 5: the conv, against cuDNN (channels-last fp16 conv with bias; cuDNN's ReLU is a separate op)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x = torch.empty(32, 56, 56, 256, device=dev).uniform_(0, 1, generator=g).half()
    wt = torch.empty(256, 3, 3, 256, device=dev).normal_(0, 1 / 48.0, generator=g).half()
    bias = torch.empty(256, device=dev).normal_(0, 0.1, generator=g).half()
    o = torch.empty(32, 56, 56, 256, device=dev, dtype=torch.float16)
    d = cb.conv_desc(x, wt, o, stride=1, padding=1, bias=bias, relu=True)
    q = cb.conv2d_query(d)
    xc = x.permute(0, 3, 1, 2)       # NCHW view of the NHWC data (channels-last)
    wc = wt.permute(0, 3, 1, 2)      # KCRS view of KRSC
    t = ab_timing(cb, lambda: cb.conv2d_desc(d, stream=stream), lambda: Fn.conv2d(xc, wc, bias, stride=1, padding=1),
                  stream, flush, reps, probe)
    cb.sync_status(stream)
    ms, ms_ref = t["ms"], t["ms_ref"]
    flops = 2.0 * 32 * 56 * 56 * 256 * 2304
    tf = flops / (ms * 1e-3) / 1e12
    out.append({"config": "5", "workload": "conv2d_f16_n32_56x56_c256_k256_3x3_bias_relu", "kernel": kernel_name(q),
                "launches": 1, "us": round(ms * 1e3, 2), "tflops": round(tf, 1), "bound": "tensor",
                "frac": round(tf / peak, 4),
                "us_back_to_back": round(t["ms_b2b"] * 1e3, 2), "effective_sm_mhz": t["mhz"] and round(t["mhz"]),
                "side_reference": {"what": "cuDNN via torch conv2d, channels-last fp16, bias, no ReLU",
                                   "us": round(ms_ref * 1e3, 2), "tflops": round(flops / (ms_ref * 1e-3) / 1e12, 1),
                                   "us_back_to_back": round(t["ms_ref_b2b"] * 1e3, 2)},
                "time_vs_side_reference": round(ms / ms_ref, 3),
                "time_vs_side_reference_back_to_back": round(t["ms_b2b"] / t["ms_ref_b2b"], 3)})
    for e in out:
        e["peak_source"] = peak_src if e["bound"] == "tensor" else "measured (copy)"
    return out


def bench_choreo(args, spec: dict, world: int, rank: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    cb = load_choreo()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)
    if args.tile:
        cb.set_tuning(tile=args.tile)
    setup = {"gemm": setup_gemm, "conv": setup_conv, "relu": setup_relu}[spec["kind"]]
    case = setup(cb, spec, world, rank, dev, stream)
    metric, unit = metric_of(spec)
    hbm_bound = spec["kind"] == "relu"
    if spec["kind"] == "gemm":
        peak_tf = measured_peak(0.0)[0]
        hbm_gbs = measured_hbm()[0]
        hbm_bound = case.flops / case.bytes_ < peak_tf * 1e12 / (hbm_gbs * 1e9)
    flush_buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if case.flush else None
    probe = torch.zeros(3, dtype=torch.int64, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(fn, steps: int) -> float:
        """Device milliseconds of `steps` calls of fn on `stream`. With a
        flush, each call is bracketed by its own events and the L2 is
        overwritten between calls, outside the events."""
        if flush_buf is None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            e1.synchronize()
            return e0.elapsed_time(e1)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for s, e in evs:
            flush_buf.fill_(1.0)
            s.record(stream)
            fn()
            e.record(stream)
        evs[-1][1].synchronize()
        return sum(s.elapsed_time(e) for s, e in evs)

    # ---------------------------------------------------------- device-resident timing
    for _ in range(args.warmup):
        case.step()
    cb.sync_status(stream)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = [int(x) for x in visible.split(",")] if visible else list(range(max(world, 1)))
    sampler = ClockSampler(phys[:world]) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    cb.check(cb.lib.choreo_clock_probe_set(probe.data_ptr()))
    t_wall0 = time.time()
    ms = timed(case.step, args.steps)
    barrier()
    t_wall1 = time.time()
    cb.check(cb.lib.choreo_clock_probe_set(None))
    cb.sync_status(stream)
    if sampler:
        sampler.mark(t_wall0, t_wall1)
    clk = [int(v) for v in probe.cpu()]

    # ---------------------------------------------------------- end to end from pinned host buffers
    e2e_steps = max(1, min(args.steps, 20))
    e2e_fn = case.e2e_step or (lambda: None)
    for _ in range(max(1, min(args.warmup, 3))):
        e2e_fn()
    barrier()
    t_wall2 = time.time()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(e2e_steps):
        e2e_fn()
    e3.record(stream)
    barrier()
    t_wall3 = time.time()
    cb.sync_status(stream)
    ms_e2e = e2.elapsed_time(e3)
    clocks = None
    if sampler:
        sampler.mark(t_wall2, t_wall3)
        clocks = sampler.stop()

    # ---------------------------------------------------------- the end-to-end step's copies alone (its floor)
    ms_floor = 0.0
    if case.floor_step is not None:
        for _ in range(2):
            case.floor_step()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(e2e_steps):
            case.floor_step()
        f1.record(stream)
        barrier()
        ms_floor = f0.elapsed_time(f1)

    # ---------------------------------------------------------- the sharded GEMM's exchanges, timed apart
    exchange = time_exchanges(case, world, rank, dev, stream) if world > 1 and spec["kind"] == "gemm" else None

    # ---------------------------------------------------------- max over ranks
    t = torch.tensor([ms, ms_e2e, ms_floor], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, ms_e2e_max, ms_floor_max = float(t[0]), float(t[1]), float(t[2])
    scale = 1e9 if unit == "GB/s" else 1e12
    value = case.units_total * args.steps / (ms_max * 1e-3) / scale
    e2e_value = case.units_total * e2e_steps / (ms_e2e_max * 1e-3) / scale
    # dominant kernel on this rank: one launch per step on `stream`
    per_launch_ms = ms / args.steps
    if hbm_bound:
        peak, peak_src = measured_hbm()
        roof = {"bound": "hbm", "achieved": case.bytes_ / (per_launch_ms * 1e-3) / 1e9, "peak": peak,
                "unit": "GB/s", "algorithmic_bytes_per_launch": case.bytes_}
    else:
        peak, peak_src = measured_peak(ms * 1e-3)
        roof = {"bound": "tensor", "achieved": case.flops / (per_launch_ms * 1e-3) / 1e12, "peak": peak,
                "unit": "TFLOP/s", "algorithmic_flops_per_launch": case.flops}
    roof["frac"] = roof["achieved"] / peak
    roof["peak_source"] = peak_src
    roof["traffic"] = profiled_traffic(spec["workload"], case.rows)
    roof["per_launch_ms"] = per_launch_ms
    roof["kernel"] = case.kernel.get("name")
    if roof["bound"] == "tensor" and clk[1] > 0:
        # What the SMs could do at the clock the launches actually ran at: 8192
        # dense f16/bf16 FLOP per SM per cycle (a 256 x 256 x 64 k-block of one
        # CTA takes 1024 tensor-pipe cycles), times the SM count.
        mhz = 1e3 * clk[0] / clk[1]
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        roof["clock_limited_peak"] = sms * 8192 * mhz * 1e6 / 1e12
        roof["frac_of_clock_limited_peak"] = roof["achieved"] / roof["clock_limited_peak"]
        roof["clock_limited_how"] = (f"{sms} SMs x 8192 FLOP/cycle x the effective SM clock of the timed launches "
                                     f"({mhz:.0f} MHz, in-kernel %clock64 / %globaltimer)")

    configs = None
    if world == 1 and not args.no_configs:
        configs = run_configs(cb, dev, stream, reps=max(5, min(args.steps, 20)))

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        s = reference_cpu_sample(spec, float(os.environ.get("CHOREO_CPU_BASELINE_SECONDS", "12")), host_cores())
        secs = run_reference_sample(s)
        cpu = {"value": s["units"] / secs / scale, "unit": unit, "cores": s["threads"],
               "kind": "reference" if s["use_ref"] else "port", "sample": sample_text(s, spec),
               "seconds": round(secs, 2)}
    if clocks is not None:
        clocks["effective_sm_mhz"] = (1e3 * clk[0] / clk[1]) if clk[1] > 0 else None
        clocks["effective_sm_mhz_how"] = (f"%clock64 / %globaltimer over the life of CTA 0 of each timed launch "
                                          f"({clk[2]} launches, choreo_clock_probe_set)")
    line = {
        "metric": metric,
        "value": value,
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": scaling_of(spec, world),
        "vs_baseline": None,
        "dtype": spec["dtype"],
        "data": "synthetic",
        "config": config_block(spec, world),
        "kernel": case.kernel,
        "roofline": roof,
        "e2e": None if case.e2e_step is None else {
            "value": e2e_value, "unit": unit, "h2d_bytes_per_step": case.h2d, "d2h_bytes_per_step": case.d2h,
            "steps": e2e_steps, "ms_per_step": ms_e2e_max / e2e_steps,
            "h2d_gbs_per_rank": case.h2d / (ms_e2e_max / e2e_steps * 1e-3) / 1e9,
            "copy_floor_ms_per_step": ms_floor_max / e2e_steps if ms_floor_max else None,
            "copy_floor_gbs_per_rank": ((case.h2d + case.d2h) / (ms_floor_max / e2e_steps * 1e-3) / 1e9
                                        if ms_floor_max else None),
            "frac_of_copy_floor": (ms_floor_max / ms_e2e_max) if ms_floor_max else None,
            "copy_floor_how": "the step's host<->device copies alone (inputs in on one stream, output out on "
                              "another, no kernel), max over ranks",
            **case.e2e_info},
        "gpu_launches": args.steps * case.launches_per_step,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if exchange is not None:
        line["exchanges_outside_timing"] = exchange
    if configs is not None:
        line["configs"] = configs
    if unit == "TFLOP/s":
        line["pct_of_nominal_dense_peak"] = 100.0 * value / (NOMINAL_DENSE_TFLOPS * world)
    emit(line)


_JSON_FD = None


def emit(line: dict) -> None:
    """The one JSON line, on the process's original standard output."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def main() -> None:
    # Library banners (NCCL's version line, warnings) go to stderr: standard
    # output carries the JSON line only.
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="choreo", choices=["choreo", "reference"])
    ap.add_argument("--workload", default="auto",
                    choices=["auto", "sharded", "gemm8192", "custom", "smallk", "conv", "relu"])
    ap.add_argument("--shape", default=None, help="MxNxK for --workload custom")
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16"], help="input/output type for --workload custom")
    ap.add_argument("--bias-relu", action="store_true", help="fused bias + ReLU epilogue for --workload custom")
    ap.add_argument("--layout", default="NN", choices=["NN", "NT", "TN", "TT"],
                    help="storage of A and B for --workload custom (T: A stored K x M / B stored N x K)")
    ap.add_argument("--tile", default=None,
                    help="force a kernel configuration: wide256, pair256, pair128, single256, single128 or single64")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-configuration block at N = 1")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = args.workload if args.workload != "auto" else "sharded"
    spec = workload_spec(wl, args.shape, args.dtype, args.layout, args.bias_relu)

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
