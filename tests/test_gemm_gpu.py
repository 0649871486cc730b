"""GEMM parity on the GPU through the C ABI (libchoreo_b200.so), checked
against the CPU oracle.

Bar: every output element within 1e-2 relative (floored, see _util.TOL) of
the fp64 oracle over the same rounded inputs; bit-exact where the inputs make
the product exact (identity KATs). Against the reference's own CPU path
(fp16 accumulation) agreement is normwise, and the GPU result must be at
least as close to fp64 as that path is. Full-size configurations are checked
on sampled rows (tile boundaries included) plus row/column checksums that
cover every element.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from _util import (BF16, F16, F32, TOL, as_f64, assert_close, dev_normal, dev_uniform, sample_rows,
                   tdtype, to_dev, to_host)

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def run(cb, a, b, m, n, k, dt_ab, dt_c, **kw):
    import torch
    c = kw.pop("c", None)
    if c is None:
        c = torch.zeros(m, n, device="cuda", dtype=tdtype(dt_c))
    cb.gemm(a, b, c, **kw)
    cb.sync_status()
    return c


# ------------------------------------------------------------------ golden fixtures through the GPU
def test_kat_identity_exact(cb, cuda):
    g = np.load(GOLDEN / "kat_identity_2x2.npz")
    for dt, an, bn, cn in ((F16, "a_f16", "b_f16", "c_f16"), (F32, "a_f32", "b_f32", "c_f32")):
        c = run(cb, to_dev(g[an], dt), to_dev(g[bn], dt), 2, 2, 2, dt, dt)
        assert np.array_equal(to_host(c), g[cn])


def test_kat_wmma_tile(cb, cuda, orc):
    g = np.load(GOLDEN / "wmma_tile_16.npz")
    c = run(cb, to_dev(g["a_f16"], F16), to_dev(g["b_f16"], F16), 16, 16, 16, F16, F32)
    assert np.max(np.abs(to_host(c) - g["c_f32"])) <= float(g["tol"])


def test_kat_baselines_f32(cb, cuda):
    g = np.load(GOLDEN / "baselines_64_f32.npz")
    c = run(cb, to_dev(g["a"], F32), to_dev(g["b"], F32), 64, 64, 64, F32, F32)
    assert np.max(np.abs(to_host(c) - g["c"])) <= float(g["tol"])


def test_kat_end2end_types(cb, cuda, orc):
    g = np.load(GOLDEN / "end2end_types_64x32x48.npz")
    c32 = run(cb, to_dev(g["a_f32"], F32), to_dev(g["b_f32"], F32), 64, 32, 48, F32, F32)
    assert np.max(np.abs(to_host(c32) - g["c_f32"])) <= 1e-4
    c16 = to_host(run(cb, to_dev(g["a_f16"], F16), to_dev(g["b_f16"], F16), 64, 32, 48, F16, F16))
    r64 = orc.gemm_f64(g["a_f16"], g["b_f16"], F16)
    assert_close(as_f64(c16, F16), r64, what="end2end f16")
    ref16 = as_f64(g["c_f16"], F16)
    assert orc.normwise_err(as_f64(c16, F16), ref16) <= TOL
    assert orc.normwise_err(as_f64(c16, F16), r64) <= orc.normwise_err(ref16, r64) + 1e-12


@pytest.mark.parametrize("name", ["ref_matmul_f16_64x48x80.npz", "ref_matmul_bf16_32x24x40.npz",
                                  "ref_matmul_f32_24x16x40.npz"])
def test_golden_reference_outputs(cb, cuda, orc, name):
    g = np.load(GOLDEN / name)
    dt = int(g["dtype"])
    (m, k), n = g["a"].shape, g["b"].shape[1]
    c = to_host(run(cb, to_dev(g["a"], dt), to_dev(g["b"], dt), m, n, k, dt, dt))
    r64 = orc.gemm_f64(g["a"], g["b"], dt)
    assert_close(as_f64(c, dt), r64, what=name)
    ref = as_f64(g["c"], dt)
    # The reference path accumulates in the input type: bf16 (8-bit mantissa)
    # drifts a few 1e-2 normwise from fp64 over K = 40, fp16 stays under 1e-2.
    bar = {F32: 1e-5, F16: TOL, BF16: 4e-2}[dt]
    assert orc.normwise_err(as_f64(c, dt), ref) <= bar
    if dt != F32:
        assert orc.normwise_err(as_f64(c, dt), r64) <= orc.normwise_err(ref, r64)


# ------------------------------------------------------------------ 1024x1024x512 fp16 U[-1,1]
def test_gemm_1024x1024x512_against_fp64_and_reference_path(cb, cuda, orc):
    M, N, K = 1024, 1024, 512
    a = orc.to_bits(orc.uniform((M, K), -1, 1, 42), F16)
    b = orc.to_bits(orc.uniform((K, N), -1, 1, 43), F16)
    c = as_f64(to_host(run(cb, to_dev(a, F16), to_dev(b, F16), M, N, K, F16, F16)), F16)
    r64 = orc.gemm_f64(a, b, F16)
    assert_close(c, r64, what="1024x1024x512")
    ref = as_f64(orc.ref_matmul(a, b, F16, nthreads=orc.threads()), F16)
    assert orc.normwise_err(c, ref) <= TOL
    assert orc.normwise_err(c, r64) < orc.normwise_err(ref, r64)


# ------------------------------------------------------------------ square sweep 2048 / 4096 / 8192
@pytest.mark.parametrize("dt", [F16, BF16])
def test_square_2048_full(cb, cuda, orc, dt):
    n = 2048
    a = orc.to_bits(orc.uniform((n, n), -1, 1, 1), dt)
    b = orc.to_bits(orc.uniform((n, n), -1, 1, 2), dt)
    c = as_f64(to_host(run(cb, to_dev(a, dt), to_dev(b, dt), n, n, n, dt, dt)), dt)
    assert_close(c, orc.gemm_f64(a, b, dt), what=f"2048^3 dt={dt}", k=n)


@pytest.mark.parametrize("dt", [F16, BF16])
@pytest.mark.parametrize("n", [4096, 8192])
def test_square_large_sampled_and_checksums(cb, cuda, orc, dt, n):
    import torch
    a = dev_uniform((n, n), -1, 1, 10 + n, dt)
    b = dev_uniform((n, n), -1, 1, 20 + n, dt)
    c = run(cb, a, b, n, n, n, dt, dt)
    rows = sample_rows(n, 48, seed=n)
    idx = torch.from_numpy(rows).cuda()
    a_h, b_h = to_host(a[idx]), to_host(b)
    r = orc.gemm_f64(a_h, b_h, dt)
    mine = assert_close(as_f64(to_host(c[idx]), dt), r, what=f"{n}^3 rows", k=n)
    # side reference: cuBLAS (torch.matmul) on the same GPU and rows
    theirs = orc.rel_err(as_f64(to_host(torch.matmul(a[idx], b)), dt), r, n)
    assert mine <= max(TOL / 4, 2.0 * theirs), (mine, theirs)
    # every element, in aggregate: 1^T C == (1^T A) B and C 1 == A (B 1)
    c64 = c.double()
    a64, b64 = a.double(), b.double()
    col = (a64.sum(0) @ b64)
    row = (a64 @ b64.sum(1))
    assert torch.allclose(c64.sum(0), col, rtol=0, atol=2e-3 * float(col.abs().max()) + 1e-6 * n)
    assert torch.allclose(c64.sum(1), row, rtol=0, atol=2e-3 * float(row.abs().max()) + 1e-6 * n)


def test_square_deterministic(cb, cuda):
    import torch
    a = dev_uniform((2048, 2048), -1, 1, 5, F16)
    b = dev_uniform((2048, 2048), -1, 1, 6, F16)
    c1 = run(cb, a, b, 2048, 2048, 2048, F16, F16)
    c2 = run(cb, a, b, 2048, 2048, 2048, F16, F16)
    assert torch.equal(c1, c2)


# ------------------------------------------------------------------ ragged 4097x3000x1536 NN/NT/TN
@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "TT"])
def test_ragged_4097x3000x1536_layouts(cb, cuda, orc, layout):
    import torch
    M, N, K = 4097, 3000, 1536
    ta, tb = layout[0] == "T", layout[1] == "T"
    a = dev_normal((K, M) if ta else (M, K), 0, 1, 31, F16)
    b = dev_normal((N, K) if tb else (K, N), 0, 1, 32, F16)
    c = run(cb, a, b, M, N, K, F16, F16, trans_a=ta, trans_b=tb)
    rows = sample_rows(M, 64, seed=3)
    r = orc.gemm_f64(to_host(a), to_host(b), F16, trans_a=ta, trans_b=tb, rows=rows)
    assert_close(as_f64(to_host(c[torch.from_numpy(rows).cuda()]), F16), r, what=f"4097x3000x1536 {layout}", k=K)
    A = a.double().t() if ta else a.double()
    B = b.double().t() if tb else b.double()
    col = A.sum(0) @ B
    assert torch.allclose(c.double().sum(0), col, rtol=0, atol=2e-3 * float(col.abs().max()) + 1e-2)


# ------------------------------------------------------------------ row-sharded 65536x8192x8192 bf16
def test_rowsharded_65536x8192x8192_full_and_slabs(cb, cuda, orc):
    import torch
    M, N, K = 65536, 8192, 8192
    a = dev_uniform((M, K), -0.5, 0.5, 41, BF16)
    b = dev_uniform((K, N), -0.5, 0.5, 42, BF16)
    bias = dev_normal((N,), 0, 0.1, 43, BF16)
    c = run(cb, a, b, M, N, K, BF16, BF16, bias=bias, relu=True)
    rows = sample_rows(M, 40, seed=4, tile=8192)
    r = orc.gemm_f64(to_host(a[torch.from_numpy(rows).cuda()]), to_host(b), BF16, bias=to_host(bias),
                     dtype_bias=BF16, relu=True)
    assert_close(as_f64(to_host(c[torch.from_numpy(rows).cuda()]), BF16), r, what="65536x8192x8192 rows", k=K)
    # Each rank's slab computed on its own equals the same rows of the full GEMM.
    for rank in (0, 3, 7):
        r0, nrows = cb.shard_rows(M, 8, rank)
        cs = run(cb, a[r0:r0 + nrows], b, nrows, N, K, BF16, BF16, bias=bias, relu=True)
        assert torch.equal(cs, c[r0:r0 + nrows])
    del c


@pytest.mark.parametrize("nshards", [1, 2, 3])
def test_rowsharded_driver_on_device0(cb, cuda, orc, nshards):
    """choreo_gemm_rowsharded, the one-process multi-GPU driver, with every
    shard on device 0 (one host thread and one stream per shard): the rows
    match the fp64 oracle, each shard matches the same descriptor run alone
    through choreo_gemm bit for bit, and every shard reports its kernel time."""
    import ctypes as C
    import torch
    M, N, K = 1000, 384, 640
    a = dev_uniform((M, K), -0.5, 0.5, 51, BF16)
    b = dev_uniform((K, N), -0.5, 0.5, 52, BF16)
    bias = dev_normal((N,), 0, 0.1, 53, BF16)
    c = torch.full((M, N), 9.0, device="cuda", dtype=torch.bfloat16)
    spans = [cb.shard_rows(M, nshards, r) for r in range(nshards)]
    descs = (cb.GemmDesc * nshards)(*[cb.make_gemm_desc(a[r0:r0 + rows], b, c[r0:r0 + rows], m=rows, n=N, k=K,
                                                        bias=bias, relu=True) for r0, rows in spans])
    devices = (C.c_int * nshards)(*([0] * nshards))
    streams = [torch.cuda.Stream() for _ in range(nshards)]
    sptrs = (C.c_void_p * nshards)(*[s.cuda_stream for s in streams])
    ms = (C.c_float * nshards)(*([-5.0] * nshards))
    torch.cuda.synchronize()
    cb.check(cb.lib.choreo_gemm_rowsharded(descs, nshards, devices, sptrs, ms))
    torch.cuda.synchronize()
    cb.sync_status()
    assert all(0.0 < v < 1000.0 for v in ms), list(ms)
    r = orc.gemm_f64(to_host(a), to_host(b), BF16, bias=to_host(bias), dtype_bias=BF16, relu=True)
    assert_close(as_f64(to_host(c), BF16), r, what=f"rowsharded x{nshards}", k=K)
    alone = torch.full_like(c, 9.0)
    for r0, rows in spans:
        cb.gemm_desc(cb.make_gemm_desc(a[r0:r0 + rows], b, alone[r0:r0 + rows], m=rows, n=N, k=K, bias=bias,
                                       relu=True))
    cb.sync_status()
    assert torch.equal(c, alone)
    # untimed form (ms_out = NULL) on the default streams
    c.fill_(9.0)
    torch.cuda.synchronize()
    cb.check(cb.lib.choreo_gemm_rowsharded(descs, nshards, devices, None, None))
    torch.cuda.synchronize()
    assert torch.equal(c, alone)


# ------------------------------------------------------------------ the 32x56x56x256 3x3 conv lives in test_conv_gpu.py

# ------------------------------------------------------------------ edge cases
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (1, 300, 70), (300, 1, 70), (129, 257, 65), (7, 9, 17),
                                   (128, 256, 64), (255, 136, 8), (64, 8, 4096), (1000, 1000, 1)])
@pytest.mark.parametrize("dt", [F16, BF16])
def test_odd_shapes(cb, cuda, orc, m, n, k, dt):
    a = orc.to_bits(orc.uniform((m, k), -1, 1, m + k), dt)
    b = orc.to_bits(orc.uniform((k, n), -1, 1, n + k), dt)
    c = as_f64(to_host(run(cb, to_dev(a, dt), to_dev(b, dt), m, n, k, dt, dt)), dt)
    assert_close(c, orc.gemm_f64(a, b, dt), what=f"{m}x{n}x{k}")


@pytest.mark.parametrize("dt_c", [F16, BF16, F32])
@pytest.mark.parametrize("dt_bias", [F16, BF16, F32])
def test_epilogue_alpha_beta_bias_relu(cb, cuda, orc, dt_c, dt_bias):
    import torch
    m, n, k = 300, 200, 100
    a = orc.to_bits(orc.uniform((m, k), -1, 1, 1), BF16)
    b = orc.to_bits(orc.uniform((k, n), -1, 1, 2), BF16)
    c0 = orc.uniform((m, n), -1, 1, 3)
    c0_dev = to_dev(c0, F32).to(tdtype(dt_c))
    c0_h = to_host(c0_dev)
    bias = orc.normal((n,), 0, 0.3, 4)
    bias_dev = to_dev(bias, F32).to(tdtype(dt_bias))
    c = run(cb, to_dev(a, BF16), to_dev(b, BF16), m, n, k, BF16, dt_c, c=c0_dev.clone(), alpha=0.75, beta=-1.25,
            bias=bias_dev, relu=True)
    r = orc.gemm_f64(a, b, BF16, alpha=0.75, beta=-1.25, c0=c0_h, dtype_c0=dt_c, bias=to_host(bias_dev),
                     dtype_bias=dt_bias, relu=True)
    assert_close(as_f64(to_host(c), dt_c), r, what="epilogue")
    assert (to_host(c).astype(np.float64) if dt_c == F32 else as_f64(to_host(c), dt_c)).min() >= 0


def test_batched(cb, cuda, orc):
    import torch
    batch, m, n, k = 5, 200, 136, 72
    a = dev_uniform((batch, m, k), -1, 1, 1, F16)
    b = dev_uniform((batch, k, n), -1, 1, 2, F16)
    c = torch.zeros(batch, m, n, device="cuda", dtype=torch.float16)
    cb.gemm(a, b, c)
    cb.sync_status()
    for i in range(batch):
        r = orc.gemm_f64(to_host(a[i]), to_host(b[i]), F16)
        assert_close(as_f64(to_host(c[i]), F16), r, what=f"batch {i}")


def test_padded_leading_dims_use_workspace(cb, cuda, orc):
    import torch
    m, n, k = 333, 129, 77
    a_full = dev_uniform((m, k + 5), -1, 1, 1, F16)
    b_full = dev_uniform((k, n + 3), -1, 1, 2, F16)
    a, b = a_full[:, :k], b_full[:, :n]
    d = cb.make_gemm_desc(a, b, torch.empty(m, n, device="cuda", dtype=torch.float16), m=m, n=n, k=k,
                          lda=a.stride(0), ldb=b.stride(0))
    q = cb.gemm_query(d)
    assert q.workspace_bytes > 0 and q.workspace_min_bytes > 0
    with pytest.raises(cb.ChoreoError) as e:
        cb.gemm_desc(d)
    assert e.value.code == cb.ERR_WORKSPACE
    ws = torch.empty(q.workspace_bytes + 512, dtype=torch.uint8, device="cuda")
    with pytest.raises(cb.ChoreoError) as e:  # one byte short of the repacks
        cb.gemm_desc(d, ws, q.workspace_min_bytes - 1)
    assert e.value.code == cb.ERR_WORKSPACE
    with pytest.raises(cb.ChoreoError) as e:  # not 256-byte aligned
        cb.gemm_desc(d, ws.data_ptr() + 16, q.workspace_bytes)
    assert e.value.code == cb.ERR_WORKSPACE and "256-byte" in str(e.value)
    cb.gemm_desc(d, ws, q.workspace_min_bytes)  # exactly the repacks
    cb.sync_status()
    c = run(cb, a, b, m, n, k, F16, F16)
    r = orc.gemm_f64(to_host(a), to_host(b), F16)
    assert_close(as_f64(to_host(c), F16), r, what="padded")


def test_output_canary(cb, cuda, orc):
    """C is a window (ldc > N, surrounded by sentinel rows) of a larger buffer:
    nothing outside the M x N window may change."""
    import torch
    m, n, k, ldc = 200, 136, 64, 160
    buf = torch.full((m + 4, ldc), -7.0, device="cuda", dtype=torch.float16)
    view = buf[2:2 + m, :n]
    a = dev_uniform((m, k), -1, 1, 1, F16)
    b = dev_uniform((k, n), -1, 1, 2, F16)
    cb.gemm(a, b, view)
    cb.sync_status()
    host = buf.float().cpu()
    assert (host[:2] == -7).all() and (host[2 + m:] == -7).all() and (host[:, n:] == -7).all()
    r = orc.gemm_f64(to_host(a), to_host(b), F16)
    assert_close(as_f64(to_host(view), F16), r, what="canary window")


def test_host_pointer_rejected(cb, cuda):
    import torch
    a = torch.zeros(64, 64, dtype=torch.float16)
    b = torch.zeros(64, 64, device="cuda", dtype=torch.float16)
    c = torch.zeros(64, 64, device="cuda", dtype=torch.float16)
    d = cb.make_gemm_desc(a, b, c, m=64, n=64, k=64)
    with pytest.raises(cb.ChoreoError) as e:
        cb.gemm_desc(d)
    assert e.value.code == cb.ERR_INVALID_ARG and "host memory" in str(e.value)


def test_query_reports_tcgen05_config(cb, cuda):
    import torch
    x = torch.empty(8192, 8192, device="cuda", dtype=torch.float16)
    q = cb.gemm_query(cb.make_gemm_desc(x, x, x, m=8192, n=8192, k=8192))
    assert q.kernel == 1 and q.tile_n in (64, 128, 256) and q.block_x == 320
    assert (q.tile_m, q.cluster_m) in ((128, 1), (256, 2), (512, 2))
    assert q.grid_x <= cb.device_props(0).sm_count and q.tmem_cols == 2 * q.tile_n
    q32 = cb.gemm_query(cb.make_gemm_desc(x.float(), x.float(), x.float(), m=8192, n=8192, k=8192))
    assert q32.kernel == 2


def test_device_props(cb, cuda):
    p = cb.device_props(0)
    assert (p.cc_major, p.cc_minor) == (10, 0) and p.sm_count >= 100 and p.max_smem_optin >= 200 * 1024


# ------------------------------------------------------------------ every tile configuration
TILES = ["wide256", "pair256", "pair128", "single256", "single128", "single64"]


@pytest.fixture
def force_tile(cb):
    """Forces a tile shape through the tuning API for one test, then restores
    the previous settings."""
    saved = cb.get_tuning()

    def _set(name):
        cb.set_tuning(tile=name)
    yield _set
    cb.check(cb.lib.choreo_tuning_set(cb.C.byref(saved)))


@pytest.mark.parametrize("tile", TILES)
@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("m,n,k", [(517, 390, 200), (1024, 768, 1000), (777, 392, 130)])
def test_forced_tile_configs(cb, cuda, orc, force_tile, tile, layout, m, n, k):
    import torch
    force_tile(tile)
    ta, tb = layout[0] == "T", layout[1] == "T"
    a = dev_uniform((k, m) if ta else (m, k), -1, 1, m + k, BF16)
    b = dev_uniform((n, k) if tb else (k, n), -1, 1, n + k, BF16)
    bias = dev_normal((n,), 0, 0.2, 3, F32)
    c = run(cb, a, b, m, n, k, BF16, BF16, trans_a=ta, trans_b=tb, bias=bias, relu=True)
    desc = cb.make_gemm_desc(a, b, c, m=m, n=n, k=k, trans_a=ta, trans_b=tb, lda=a.stride(0), ldb=b.stride(0))
    q = cb.gemm_query(desc)
    want = {"wide256": (512, 256, 2), "pair256": (256, 256, 2), "pair128": (256, 128, 2),
            "single256": (128, 256, 1), "single128": (128, 128, 1), "single64": (128, 64, 1)}[tile]
    assert (q.tile_m, q.tile_n, q.cluster_m) == want
    r = orc.gemm_f64(to_host(a), to_host(b), BF16, trans_a=ta, trans_b=tb, bias=to_host(bias), relu=True)
    assert_close(as_f64(to_host(c), BF16), r, what=f"{tile} {layout} {m}x{n}x{k}", k=k)


@pytest.mark.parametrize("tile", TILES)
@pytest.mark.parametrize("dt_c", [F16, BF16, F32])
def test_forced_tile_alpha_beta_bias(cb, cuda, orc, force_tile, tile, dt_c):
    """The full epilogue (alpha * acc + beta * C + bias, ReLU) in every kernel
    and output type, with a ragged N so the last 32-column chunk is partial
    (bias lanes past N read nothing) and a 16-byte-aligned C so beta reads C
    with vector loads."""
    import torch
    force_tile(tile)
    m, n, k = 300, 390, 200
    a = dev_uniform((m, k), -1, 1, 21, F16)
    b = dev_uniform((k, n), -1, 1, 22, F16)
    bias = dev_normal((n,), 0, 0.5, 23, BF16)
    c0 = dev_uniform((m, 392), -1, 1, 24, dt_c)[:, :n]
    c = c0.clone()
    cb.gemm(a, b, c, alpha=1.5, beta=0.5, bias=bias, relu=True)
    cb.sync_status()
    c0h = to_host(c0.contiguous())
    r = orc.gemm_f64(to_host(a), to_host(b), F16, alpha=1.5, beta=0.5, c0=c0h, dtype_c0=dt_c, bias=to_host(bias),
                     dtype_bias=BF16, relu=True)
    got = to_host(c.contiguous()).astype(np.float64) if dt_c == F32 else as_f64(to_host(c.contiguous()), dt_c)
    assert_close(got, r, what=f"epilogue {tile} dtype {dt_c}", k=k)


@pytest.mark.parametrize("tile", TILES)
@pytest.mark.parametrize("dt_c", [F16, F32])
def test_forced_tile_canary_and_batch(cb, cuda, orc, force_tile, tile, dt_c):
    """Staged (TMA-store) and direct epilogues write exactly the M x N window of
    a larger buffer, for single and batched problems."""
    import torch
    force_tile(tile)
    m, n, k, ldc = 600, 264, 96, 320
    buf = torch.full((m + 8, ldc), -7.0, device="cuda", dtype=tdtype(dt_c))
    view = buf[3:3 + m, :n]
    a = dev_uniform((m, k), -1, 1, 11, F16)
    b = dev_uniform((k, n), -1, 1, 12, F16)
    cb.gemm(a, b, view)
    cb.sync_status()
    host = buf.float().cpu()
    assert (host[:3] == -7).all() and (host[3 + m:] == -7).all() and (host[:, n:] == -7).all()
    r = orc.gemm_f64(to_host(a), to_host(b), F16)
    got = to_host(view).astype(np.float64) if dt_c == F32 else as_f64(to_host(view), dt_c)
    assert_close(got, r, what=f"canary {tile}")
    batch = 3
    ab = dev_uniform((batch, m, k), -1, 1, 13, F16)
    bb = dev_uniform((batch, k, n), -1, 1, 14, F16)
    cbt = torch.zeros(batch, m, n, device="cuda", dtype=tdtype(dt_c))
    cb.gemm(ab, bb, cbt)
    cb.sync_status()
    for i in range(batch):
        r = orc.gemm_f64(to_host(ab[i]), to_host(bb[i]), F16)
        got = to_host(cbt[i]).astype(np.float64) if dt_c == F32 else as_f64(to_host(cbt[i]), dt_c)
        assert_close(got, r, what=f"batch {i} {tile}")


def test_host_gemm_plan_pipelined(cb, cuda, orc):
    """HostGemmPlan: pinned host A/B/bias in, C out, row slabs overlapped on
    three streams (a ragged last slab included); two runs on the same plan,
    the second with new inputs, each checked against fp64."""
    import torch
    m, n, k = 1500, 384, 256
    plan = cb.HostGemmPlan(m, n, k, torch.bfloat16, bias=True, relu=True, slabs=3)
    assert [rows for _, rows in plan.slabs] == [512, 512, 476]
    for seed in (31, 41):
        a = torch.empty(m, k).uniform_(-1, 1, generator=torch.Generator().manual_seed(seed)).bfloat16().pin_memory()
        b = torch.empty(k, n).uniform_(-1, 1, generator=torch.Generator().manual_seed(seed + 1)).bfloat16().pin_memory()
        bias = torch.empty(n).normal_(0, 0.3, generator=torch.Generator().manual_seed(seed + 2)).bfloat16().pin_memory()
        c = torch.full((m, n), 7.0, dtype=torch.bfloat16).pin_memory()
        plan.run(a, b, c, bias)
        torch.cuda.current_stream().synchronize()
        cb.sync_status()
        ah, bh = a.view(torch.int16).numpy().view(np.uint16), b.view(torch.int16).numpy().view(np.uint16)
        biash = bias.view(torch.int16).numpy().view(np.uint16)
        r = orc.gemm_f64(ah, bh, BF16, bias=biash, dtype_bias=BF16, relu=True)
        got = as_f64(c.view(torch.int16).numpy().view(np.uint16), BF16)
        assert_close(got, r, what=f"host plan seed {seed}", k=k)


def test_nonfinite_inputs_propagate(cb, cuda, orc):
    """A NaN or an Inf in A reaches every element of its output row the way
    fp64 arithmetic says (the tensor cores do not flush or saturate them)."""
    import torch
    m, n, k = 300, 260, 192
    a = orc.to_bits(orc.uniform((m, k), -1, 1, 51), F16)
    b = orc.to_bits(orc.uniform((k, n), 0.25, 1, 52), F16)  # positive B: Inf * b stays +Inf
    a[7, 13] = 0x7E00      # NaN
    a[100, 5] = 0x7C00     # +Inf
    a[250, 0] = 0xFC00     # -Inf
    c = run(cb, to_dev(a, F16), to_dev(b, F16), m, n, k, F16, F32)
    got = to_host(c).astype(np.float64)
    assert np.isnan(got[7]).all()
    assert np.isposinf(got[100]).all() and np.isneginf(got[250]).all()
    rest = np.setdiff1d(np.arange(m), [7, 100, 250])
    r = orc.gemm_f64(a, b, F16, rows=rest)
    assert np.isfinite(got[rest]).all()
    assert_close(got[rest], r, what="finite rows", k=k)


def test_long_reduction(cb, cuda, orc):
    """K = 65536 (1024 k-blocks through the pipeline). The tensor cores'
    fp32 accumulation error grows about linearly with K here (it is no longer
    within the sqrt(K)-scaled per-element floor), so the check is the one that
    holds for any tensor-core GEMM: normwise error <= 1e-3 against fp64, and a
    largest absolute error no worse than cuBLAS's on the same inputs with fp32
    output (+25 %)."""
    import torch
    m, n, k = 256, 512, 65536
    a = orc.to_bits(orc.uniform((m, k), -1, 1, 53), F16)
    b = orc.to_bits(orc.uniform((k, n), -1, 1, 54), F16)
    ad, bd = to_dev(a, F16), to_dev(b, F16)
    c = run(cb, ad, bd, m, n, k, F16, F32)
    r = orc.gemm_f64(a, b, F16)
    got = to_host(c).astype(np.float64)
    assert np.isfinite(got).all()
    assert orc.normwise_err(got, r) <= 1e-3
    e_ours = float(np.max(np.abs(got - r)))
    try:
        ref = torch.mm(ad, bd, out_dtype=torch.float32)
    except (RuntimeError, TypeError):
        pytest.skip("torch.mm(out_dtype=float32) unavailable: cuBLAS side check skipped")
    e_cublas = float(np.max(np.abs(ref.cpu().double().numpy() - r)))
    rms = float(np.sqrt(np.mean(r * r)))
    print(f"K=65536 max |error|: choreo {e_ours:.3e}, cuBLAS {e_cublas:.3e}; rms {rms:.1f}")
    assert e_ours <= 1.25 * e_cublas + 1e-6 * rms, (e_ours, e_cublas, rms)


@pytest.mark.parametrize("layout", ["NN", "NT", "TN"])
@pytest.mark.parametrize("dt_c", [F16, BF16, F32])
def test_split_k(cb, cuda, orc, layout, dt_c):
    """Few output tiles over a long K: the query plans K splits (fp32 partials
    in the workspace, summed by a second pass that applies the epilogue). The
    split result and the unsplit one (no workspace given) both match fp64,
    with alpha, beta, bias and ReLU."""
    import torch
    m, n, k = 300, 200, 8192
    ta, tb = layout[0] == "T", layout[1] == "T"
    a = dev_uniform((k, m) if ta else (m, k), -1, 1, 61, F16)
    b = dev_uniform((n, k) if tb else (k, n), -1, 1, 62, F16)
    bias = dev_normal((n,), 0, 0.5, 63, F32)
    c0 = dev_uniform((m, n), -1, 1, 64, dt_c)
    desc_args = dict(m=m, n=n, k=k, trans_a=ta, trans_b=tb, alpha=0.5, beta=2.0, bias=bias, relu=True)
    c_split, c_plain = c0.clone(), c0.clone()
    d = cb.make_gemm_desc(a, b, c_split, **desc_args)
    q = cb.gemm_query(d)
    assert q.split_k > 1 and q.workspace_bytes >= q.workspace_min_bytes + q.split_k * m * n * 4
    assert (q.workspace_min_bytes > 0) == (layout == "TN")  # K x M A with M = 300: rows not 16-byte aligned
    assert q.tiles <= 148
    ws = torch.empty(q.workspace_bytes, dtype=torch.uint8, device="cuda")
    cb.gemm_desc(d, ws, q.workspace_bytes)
    # the minimum workspace (repacks only) runs the unsplit plan
    cb.gemm_desc(cb.make_gemm_desc(a, b, c_plain, **desc_args), ws, q.workspace_min_bytes)
    cb.sync_status()
    r = orc.gemm_f64(to_host(a), to_host(b), F16, trans_a=ta, trans_b=tb, alpha=0.5, beta=2.0,
                     c0=to_host(c0), dtype_c0=dt_c, bias=to_host(bias), dtype_bias=F32, relu=True)
    for c, what in ((c_split, "split"), (c_plain, "unsplit")):
        got = to_host(c).astype(np.float64) if dt_c == F32 else as_f64(to_host(c), dt_c)
        assert_close(got, r, what=f"{what} {layout} {dt_c}", k=k)


def test_cuda_graph_capture_and_replay(cb, cuda, orc):
    """The C ABI calls capture into a CUDA graph (a plain GEMM, a split-K GEMM
    with its reduction pass, and a conv, each launched with programmatic
    dependent launch) and the replayed graph reproduces the eager results
    bit for bit."""
    import torch
    a1, b1 = dev_uniform((1024, 768), -1, 1, 81, F16), dev_uniform((768, 512), -1, 1, 82, F16)
    a2, b2 = dev_uniform((256, 8192), -1, 1, 83, BF16), dev_uniform((8192, 384), -1, 1, 84, BF16)
    x = dev_uniform((2, 16, 16, 64), 0, 1, 85, F16)
    w = dev_normal((96, 3, 3, 64), 0, 1.0 / 24, 86, F16)
    c1 = torch.empty(1024, 512, device="cuda", dtype=torch.float16)
    c2 = torch.empty(256, 384, device="cuda", dtype=torch.bfloat16)
    o = torch.empty(2, 16, 16, 96, device="cuda", dtype=torch.float16)
    d1 = cb.make_gemm_desc(a1, b1, c1, m=1024, n=512, k=768)
    d2 = cb.make_gemm_desc(a2, b2, c2, m=256, n=384, k=8192, relu=True)
    q2 = cb.gemm_query(d2)
    assert q2.split_k > 1
    ws = torch.empty(q2.workspace_bytes, dtype=torch.uint8, device="cuda")
    dc = cb.conv_desc(x, w, o, relu=True)
    s = torch.cuda.Stream()

    def work():
        cb.gemm_desc(d1, stream=s)
        cb.gemm_desc(d2, ws, q2.workspace_bytes, stream=s)
        cb.conv2d_desc(dc, stream=s)

    with torch.cuda.stream(s):
        work()  # warm-up outside the capture: first-call set-up (kernel attributes, plan cache)
    torch.cuda.synchronize()
    eager = [t.clone() for t in (c1, c2, o)]
    for t in (c1, c2, o):
        t.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        work()
    g.replay()
    torch.cuda.synchronize()
    cb.sync_status()
    for got, want in zip((c1, c2, o), eager):
        assert torch.equal(got, want)
