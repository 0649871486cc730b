"""Row-sharded multi-process logic on CPU: world-size-2 and -4 gloo ranks (127.0.0.1).

Each rank takes its slab from choreo_shard_rows (the partition the GPU bench
uses), computes its rows of C with the fp64 oracle, and rank 0 gathers the
slabs and compares them with the unsharded result; the timing reduction the
bench uses (max over ranks) is checked; and a rank that fails before the
collective makes the other rank's collective raise instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from conftest import load_choreo
    from oracle import oracle as orc

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    cb = load_choreo()
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the collective")
        M, N, K = 300, 40, 64
        a = orc.to_bits(orc.uniform((M, K), -0.5, 0.5, 1), orc.BF16)
        b = orc.to_bits(orc.uniform((K, N), -0.5, 0.5, 2), orc.BF16)
        bias = orc.normal((N,), 0, 0.1, 3)
        r0, rows = cb.shard_rows(M, world, rank)
        slab = orc.gemm_f64(a, b, orc.BF16, bias=bias, dtype_bias=orc.F32, relu=True,
                            rows=np.arange(r0, r0 + rows), nthreads=1)
        # gather variable-size slabs: pad to the largest
        max_rows = (M + 127) // 128 * 128
        buf = torch.zeros(max_rows, N, dtype=torch.float64)
        buf[:rows] = torch.from_numpy(slab)
        meta = torch.tensor([r0, rows], dtype=torch.int64)
        bufs = [torch.zeros_like(buf) for _ in range(world)]
        metas = [torch.zeros_like(meta) for _ in range(world)]
        dist.all_gather(bufs, buf)
        dist.all_gather(metas, meta)
        # bench.py's timing reduction: max over ranks
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full = orc.gemm_f64(a, b, orc.BF16, bias=bias, dtype_bias=orc.F32, relu=True, nthreads=1)
            got = np.zeros_like(full)
            covered = 0
            for bb, mm in zip(bufs, metas):
                s0, n = int(mm[0]), int(mm[1])
                got[s0:s0 + n] = bb[:n].numpy()
                covered += n
            ok = covered == M and np.array_equal(got, full) and float(t[0]) == 10.0 + (world - 1)
            Path(out_dir, "result").write_text("ok" if ok else "mismatch")
    except RuntimeError as e:
        if mode == "fail" and rank == 1:
            raise
        Path(out_dir, f"rank{rank}_error").write_text(str(e)[:200])
        dist.destroy_process_group()
        sys.exit(3)
    dist.destroy_process_group()


def _spawn(mode: str, tmp_path, world: int = 2) -> list[int]:
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = []
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            codes.append(-999)
        else:
            codes.append(p.exitcode)
    return codes


def test_row_sharded_slabs_assemble_to_full_result(tmp_path):
    codes = _spawn("ok", tmp_path)
    assert codes == [0, 0]
    assert (tmp_path / "result").read_text() == "ok"


def test_four_ranks_one_with_an_empty_shard(tmp_path):
    """Four ranks over M = 300 rows (three 128-row tiles): the last rank owns
    no rows, takes part in every collective all the same, and the slabs still
    assemble to the full result."""
    codes = _spawn("ok", tmp_path, world=4)
    assert codes == [0, 0, 0, 0]
    assert (tmp_path / "result").read_text() == "ok"


def test_failed_rank_is_detected_not_hung(tmp_path):
    codes = _spawn("fail", tmp_path)
    assert codes[1] != 0                      # the injected failure
    assert codes[0] == 3                      # rank 0's collective raised and it exited cleanly
    assert (tmp_path / "rank0_error").exists()


def _b_once_worker(rank: int, world: int, port: int, k: int, out_dir: str) -> None:
    """bench.py's B-once end-to-end step on gloo ranks: each rank copies its
    rows of the host B (b_rows_share) into a share-row part, and the
    all-gather the bench uses assembles every rank's copy of B."""
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    n = 24
    b_h = (torch.arange(k * n, dtype=torch.float32).reshape(k, n) % 251).to(torch.bfloat16)
    share, k0, k1 = bench.b_rows_share(k, world, rank)
    b_full = torch.full((share * world, n), -1.0, dtype=torch.bfloat16)
    b_part = torch.zeros(share, n, dtype=torch.bfloat16)
    if k1 > k0:
        b_part[:k1 - k0].copy_(b_h[k0:k1])
    dist.all_gather_into_tensor(b_full, b_part)
    ok = torch.equal(b_full[:k], b_h)
    Path(out_dir, f"bonce{rank}").write_text("ok" if ok else "mismatch")
    dist.destroy_process_group()


@pytest.mark.parametrize("world,k", [(2, 8192), (3, 200), (4, 130), (4, 5)])
def test_bench_b_once_assembles_b_on_every_rank(tmp_path, world, k):
    """At N > 1 the bench's end-to-end step brings B over PCIe once for the
    whole job (1/N of its rows per rank) and assembles it by an all-gather:
    every rank ends with B's K rows, also when N does not divide K and the
    last rank's share is short or empty."""
    import torch.multiprocessing as mp
    sys.path.insert(0, str(ROOT))
    import bench
    shares = [bench.b_rows_share(k, world, r) for r in range(world)]
    assert shares[0][1] == 0 and shares[-1][2] == k
    assert all(shares[r][2] == shares[r + 1][1] for r in range(world - 1))
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_b_once_worker, args=(r, world, port, k, str(tmp_path))) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
        if pr.is_alive():
            pr.kill()
            pr.join()
    assert [pr.exitcode for pr in procs] == [0] * world
    assert all((tmp_path / f"bonce{r}").read_text() == "ok" for r in range(world))


def test_bench_workload_specs():
    sys.path.insert(0, str(ROOT))
    import bench
    s = bench.workload_spec("sharded")
    assert (s["m_total"], s["n"], s["k"], s["dtype"], s["bias"], s["relu"]) == (65536, 8192, 8192, "bf16", True, True)
    g = bench.workload_spec("gemm8192")
    assert (g["m_total"], g["n"], g["k"], g["dtype"]) == (8192, 8192, 8192, "f16")


def test_bench_conv_batch_split():
    """bench.py's conv workload splits the 32 images into contiguous runs that
    cover the batch exactly once, sizes differing by at most one."""
    sys.path.insert(0, str(ROOT))
    import bench
    for world in (1, 2, 3, 4, 5, 8):
        runs = [bench.conv_images(32, world, r) for r in range(world)]
        assert sum(c for _, c in runs) == 32
        assert all(runs[i][0] + runs[i][1] == runs[i + 1][0] for i in range(world - 1))
        assert max(c for _, c in runs) - min(c for _, c in runs) <= 1


def test_bench_shard_rows_matches_library(cb):
    """bench.py's restated partition (used by the reference arm, which loads no
    GPU library) is choreo_shard_rows's."""
    sys.path.insert(0, str(ROOT))
    import bench
    for m in (1, 127, 4097, 65536, 65536 + 5):
        for world in (1, 2, 3, 4, 8):
            for r in range(world):
                assert bench.shard_rows(m, world, r) == cb.shard_rows(m, world, r)


def test_bench_reference_arm_line(tmp_path):
    """The reference arm on the CPU: one JSON line whose `config` is exactly the
    block the GPU arm prints for the same workload and GPU count (the default
    workload, the row-sharded GEMM, at every N), and whose core count is the
    host's, not torchrun's OMP_NUM_THREADS=1."""
    import json
    import os
    import subprocess
    sys.path.insert(0, str(ROOT))
    import bench
    env = dict(os.environ, CHOREO_REF_STEP_SECONDS="0.05", OMP_NUM_THREADS="1", WORLD_SIZE="2", RANK="0")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["config"] == bench.config_block(bench.workload_spec("sharded"), 2)
    assert line["config"]["workload"] == "rowsharded_gemm_bf16_65536x8192x8192_bias_relu"
    assert line["cpu_baseline"]["cores"] == bench.host_cores()
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["metric"] == bench.HEADLINE_METRIC
    # rank 1 of the same run does no work and prints nothing
    env["RANK"] = "1"
    r1 = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1"],
                        capture_output=True, text=True, env=env, timeout=120)
    assert r1.returncode == 0 and r1.stdout.strip() == ""
