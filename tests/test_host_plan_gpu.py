"""Host-buffer pipelines (choreo_host_gemm_* / choreo_host_conv_*) on the GPU,
driven through the C ABI with raw pointers (ctypes), checked against the CPU
oracle.

These stand behind the reference's to_device() -> operator* -> to_host() flow
(tensor/tensor.hpp:568-598): inputs and outputs in host memory, the copies
overlapped with the kernels by the library. Cases: pinned and pageable host
memory, B (or the weights) already resident on the device, two runs queued
back to back on one plan without a synchronize between them, a ragged last
part, and the run-time contract errors.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from _util import BF16, F16, as_f64, assert_close

pytestmark = pytest.mark.gpu


def _bits(t):
    import torch
    return t.view(torch.int16).numpy().view(np.uint16)


def _gemm_plan(cb, m, n, k, dt, *, bias, relu, parts=0):
    d = cb.HostGemmDesc()
    d.m, d.n, d.k = m, n, k
    d.dtype_ab = d.dtype_c = d.dtype_bias = dt
    d.alpha = 1.0
    d.has_bias, d.relu, d.parts, d.device = int(bias), int(relu), parts, 0
    h = C.c_void_p()
    cb.check(cb.lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)))
    return h


def test_host_gemm_run_through_c_abi_pinned(cb, cuda, orc):
    """Raw C ABI: create, query parts and info, two runs enqueued back to back
    (new inputs each, no synchronize between them), destroy."""
    import torch
    m, n, k = 2100, 640, 384
    h = _gemm_plan(cb, m, n, k, BF16, bias=True, relu=True, parts=4)
    info = cb.HostPlanInfo()
    cb.check(cb.lib.choreo_host_plan_info_get(h, C.byref(info)))
    # 4 parts asked: 525 rows each, rounded up to whole 512-row tiles -> 3 parts
    assert info.parts == 3 and info.launches_per_run >= 3
    assert info.h2d_bytes == 2 * (m * k + k * n + n) and info.d2h_bytes == 2 * m * n
    assert info.device_bytes >= 2 * (m * k + k * n + m * n)
    spans = []
    for i in range(info.parts):
        f, c = C.c_int64(), C.c_int64()
        cb.check(cb.lib.choreo_host_plan_part(h, i, C.byref(f), C.byref(c)))
        spans.append((f.value, c.value))
    assert spans == [(0, 1024), (1024, 1024), (2048, 52)]
    runs = []
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (11, 21):
        g = torch.Generator().manual_seed(seed)
        a = torch.empty(m, k).uniform_(-1, 1, generator=g).bfloat16().pin_memory()
        b = torch.empty(k, n).uniform_(-1, 1, generator=g).bfloat16().pin_memory()
        bias = torch.empty(n).normal_(0, 0.3, generator=g).bfloat16().pin_memory()
        c = torch.full((m, n), 5.0, dtype=torch.bfloat16).pin_memory()
        cb.check(cb.lib.choreo_host_gemm_run(h, a.data_ptr(), b.data_ptr(), bias.data_ptr(), c.data_ptr(), 0, stream))
        runs.append((a, b, bias, c))
    torch.cuda.current_stream().synchronize()
    cb.sync_status()
    cb.check(cb.lib.choreo_host_plan_destroy(h))
    for a, b, bias, c in runs:
        r = orc.gemm_f64(_bits(a), _bits(b), BF16, bias=_bits(bias), dtype_bias=BF16, relu=True)
        assert_close(as_f64(_bits(c), BF16), r, what="host GEMM plan", k=k)


def test_host_gemm_operands_on_device_and_pageable(cb, cuda, orc):
    """B and bias already on the device (CHOREO_HOST_OPERANDS_ON_DEVICE), A and
    C in pageable (numpy) host memory."""
    import torch
    m, n, k = 1030, 256, 512
    h = _gemm_plan(cb, m, n, k, F16, bias=True, relu=False)
    a = orc.to_bits(orc.uniform((m, k), -1, 1, 61), F16)
    b = orc.to_bits(orc.uniform((k, n), -1, 1, 62), F16)
    bias = orc.to_bits(orc.normal((n,), 0, 0.2, 63), F16)
    bd = torch.from_numpy(b.view(np.int16)).cuda()
    biasd = torch.from_numpy(bias.view(np.int16)).cuda()
    c = np.zeros((m, n), np.uint16)
    stream = torch.cuda.current_stream().cuda_stream
    cb.check(cb.lib.choreo_host_gemm_run(h, a.ctypes.data, bd.data_ptr(), biasd.data_ptr(), c.ctypes.data,
                                         cb.OPERANDS_ON_DEVICE, stream))
    torch.cuda.current_stream().synchronize()
    cb.sync_status()
    r = orc.gemm_f64(a, b, F16, bias=bias, dtype_bias=F16)
    assert_close(as_f64(c, F16), r, what="host GEMM plan, B on device", k=k)
    # contract errors at run time: device memory where host memory belongs,
    # host memory where the flag promises device memory, a missing bias
    assert cb.lib.choreo_host_gemm_run(h, bd.data_ptr(), bd.data_ptr(), biasd.data_ptr(), c.ctypes.data, 0,
                                       stream) == cb.ERR_INVALID_ARG
    assert cb.lib.choreo_host_gemm_run(h, a.ctypes.data, b.ctypes.data, biasd.data_ptr(), c.ctypes.data,
                                       cb.OPERANDS_ON_DEVICE, stream) == cb.ERR_INVALID_ARG
    assert cb.lib.choreo_host_gemm_run(h, a.ctypes.data, b.ctypes.data, None, c.ctypes.data, 0,
                                       stream) == cb.ERR_INVALID_ARG
    assert "with a bias" in cb.lib.choreo_last_error().decode()
    cb.check(cb.lib.choreo_host_plan_destroy(h))


def test_host_conv_weights_on_device(cb, cuda, orc):
    """HostConvPlan with the weights and bias resident on the device, a
    ragged last run of images, against fp64."""
    import torch
    n, hh, ww, c, k = 5, 9, 11, 64, 128
    plan = cb.HostConvPlan(n, hh, ww, c, k, 3, 3, torch.float16, bias=True, relu=True, runs=3)
    assert [cnt for _, cnt in plan.runs] == [2, 2, 1]
    x = orc.to_bits(orc.uniform((n, hh, ww, c), 0, 1, 91), F16)
    wt = orc.to_bits(orc.normal((k, 3, 3, c), 0, 1.0 / 24, 92), F16)
    bias = orc.to_bits(orc.normal((k,), 0, 0.1, 93), F16)
    xh = torch.from_numpy(x.view(np.int16)).view(torch.float16).pin_memory()
    wd = torch.from_numpy(wt.view(np.int16)).view(torch.float16).cuda()
    bd = torch.from_numpy(bias.view(np.int16)).view(torch.float16).cuda()
    out = torch.zeros(n, hh, ww, k, dtype=torch.float16).pin_memory()
    plan.run(xh, wd, out, bd, operands_on_device=True)
    torch.cuda.current_stream().synchronize()
    cb.sync_status()
    ref = orc.conv2d_f64(x, wt, F16, bias=bias, dtype_bias=F16, relu=True)
    assert_close(as_f64(_bits(out), F16).reshape(-1, k), ref, what="host conv plan, weights on device", k=9 * c)
    plan.close()


def test_host_gemm_f32_output_host_bias_many_parts(cb, cuda, orc):
    """f16 inputs with f32 output and a bias of the input type read from the
    host; 7 parts of 512 rows (the last shorter); the plan reused for
    three runs queued back to back, each against fp64."""
    import torch
    m, n, k = 3300, 320, 704
    plan = cb.HostGemmPlan(m, n, k, torch.float16, bias=True, relu=True, slabs=7, dtype_c=torch.float32)
    assert [rows for _, rows in plan.slabs] == [512] * 6 + [228]
    runs = []
    for seed in (5, 6, 7):
        gen = torch.Generator().manual_seed(seed)
        a = torch.empty(m, k).uniform_(-1, 1, generator=gen).half().pin_memory()
        b = torch.empty(k, n).uniform_(-1, 1, generator=gen).half().pin_memory()
        bias = torch.empty(n).normal_(0, 0.5, generator=gen).half().pin_memory()
        c = torch.full((m, n), -9.0, dtype=torch.float32).pin_memory()
        plan.run(a, b, c, bias)
        runs.append((a, b, bias, c))
    torch.cuda.current_stream().synchronize()
    cb.sync_status()
    for a, b, bias, c in runs:
        r = orc.gemm_f64(_bits(a), _bits(b), F16, bias=_bits(bias), dtype_bias=F16, relu=True)
        assert_close(c.numpy().astype(np.float64), r, what="host GEMM plan f32 out", k=k)


def test_clock_probe_counts_launches_and_reads_a_plausible_clock(cb, cuda):
    """choreo_clock_probe_set: every tensor-core launch of this thread adds its
    first CTA's cycles and nanoseconds and counts itself; the ratio is an SM
    clock the B200 can run at; NULL turns it off; host memory is refused."""
    import torch
    probe = torch.zeros(3, dtype=torch.int64, device="cuda")
    a = torch.empty(1024, 2048, device="cuda", dtype=torch.bfloat16).uniform_(-1, 1)
    b = torch.empty(2048, 1024, device="cuda", dtype=torch.bfloat16).uniform_(-1, 1)
    c = torch.empty(1024, 1024, device="cuda", dtype=torch.bfloat16)
    cb.check(cb.lib.choreo_clock_probe_set(probe.data_ptr()))
    try:
        for _ in range(5):
            cb.gemm(a, b, c)
    finally:
        cb.check(cb.lib.choreo_clock_probe_set(None))
    cb.gemm(a, b, c)  # not counted
    cb.sync_status()
    cycles, ns, launches = probe.cpu().tolist()
    assert launches == 5 and cycles > 0 and ns > 0
    assert 200.0 < 1e3 * cycles / ns < 2500.0, 1e3 * cycles / ns
    host = np.zeros(3, np.uint64)
    assert cb.lib.choreo_clock_probe_set(host.ctypes.data) == cb.ERR_INVALID_ARG
    assert cb.lib.choreo_clock_probe_set(probe.data_ptr() + 4) == cb.ERR_INVALID_ARG  # 8-byte alignment


def _half0_rows(m):
    """Rows of a 512 x 256 tile that accumulator half 0 holds: the first 128 of
    each CTA's 256."""
    return np.arange(m) % 256 < 128


def test_handover_window_setting(cb, cuda, orc):
    """The wide tile's hand-over window (choreo_tuning::handover_kb): half 0
    sums k-blocks 0 .. K-1 in order whatever the window, so its rows have the
    same bits for every setting; half 1 sums k-blocks D .. K-1 and then 0 .. D-1,
    so its rows agree with the fp64 product within the tolerance; every setting
    repeats its own bits."""
    import torch
    m, n, k = 1024, 512, 2048
    g = torch.Generator().manual_seed(3)
    a16 = torch.empty(m, k).uniform_(-1, 1, generator=g).half()
    b16 = torch.empty(k, n).uniform_(-1, 1, generator=g).half()
    a, b = a16.cuda(), b16.cuda()
    with cb.tuning(tile="wide256"):
        ref = torch.empty(m, n, device="cuda", dtype=torch.float16)
        cb.gemm(a, b, ref)
    cb.sync_status()
    h0 = torch.from_numpy(_half0_rows(m)).cuda()
    exp = orc.gemm_f64(_bits(a16), _bits(b16), F16)
    for w in (1, 2, 3, 4, 9):
        outs = []
        for _ in range(2):
            with cb.tuning(tile="wide256", handover_kb=w):
                c = torch.empty_like(ref)
                cb.gemm(a, b, c)
            cb.sync_status()
            outs.append(c)
        assert torch.equal(outs[0], outs[1]), w
        assert torch.equal(outs[0][h0], ref[h0]), w
        assert_close(as_f64(_bits(outs[0].cpu()), F16), exp, what=f"GEMM, window {w}", k=k)


def test_handover_window_setting_conv(cb, cuda, orc):
    """The same on the implicit-GEMM conv (36 k-blocks per tile): half-0 pixels
    have the default's bits for every window, and each window's output matches
    the fp64 conv."""
    import torch
    n, hh, ww, c, k = 6, 20, 20, 256, 256
    g = torch.Generator().manual_seed(4)
    x16 = torch.empty(n, hh, ww, c).uniform_(0, 1, generator=g).half()
    w16 = (torch.randn(k, 3, 3, c, generator=g) / 48).half()
    b16 = (torch.randn(k, generator=g) * 0.1).half()
    x, w, bias = x16.cuda(), w16.cuda(), b16.cuda()
    with cb.tuning(tile="wide256"):
        ref = torch.empty(n, hh, ww, k, device="cuda", dtype=torch.float16)
        cb.conv2d(x, w, ref, bias=bias, relu=True)
    cb.sync_status()
    pix = n * hh * ww
    h0 = torch.from_numpy(_half0_rows(pix)).cuda()
    exp = orc.conv2d_f64(_bits(x16), _bits(w16), F16, bias=_bits(b16), dtype_bias=F16, relu=True)
    for win in (1, 2, 3, 4):
        with cb.tuning(tile="wide256", handover_kb=win):
            out = torch.empty_like(ref)
            cb.conv2d(x, w, out, bias=bias, relu=True)
        cb.sync_status()
        assert torch.equal(out.view(pix, k)[h0], ref.view(pix, k)[h0]), win
        assert_close(as_f64(_bits(out.cpu()), F16).reshape(-1, k), exp, what=f"conv, window {win}", k=9 * c)


@pytest.mark.parametrize("kblocks", [1, 2, 3, 4, 5, 6, 9])
def test_wide_tile_handover_paths(cb, cuda, orc, kblocks):
    """The 512 x 256 tile's hand-over paths across K: tiles no longer than the
    window hold and replay their stages (K <= ring depth), longer ones stream
    (head for half 0, body for both, second load of the head for half 1), and
    a window above the ring depth streams with the ring depth; bias + ReLU
    and a ragged M and N edge, each against fp64."""
    import torch
    m, n, k = 1100, 520, 64 * kblocks
    g = torch.Generator().manual_seed(100 + kblocks)
    a = torch.empty(m, k).uniform_(-1, 1, generator=g).bfloat16()
    b = torch.empty(k, n).uniform_(-1, 1, generator=g).bfloat16()
    bias = torch.empty(n).normal_(0, 0.3, generator=g).bfloat16()
    exp = orc.gemm_f64(_bits(a), _bits(b), BF16, bias=_bits(bias), dtype_bias=BF16, relu=True)
    ad, bd, biasd = a.cuda(), b.cuda(), bias.cuda()
    for win in (0, 2, 5, 16):
        with cb.tuning(tile="wide256", handover_kb=win):
            c = torch.full((m, n), 7.0, device="cuda", dtype=torch.bfloat16)
            cb.gemm(ad, bd, c, bias=biasd, relu=True)
        cb.sync_status()
        assert_close(as_f64(_bits(c.cpu()), BF16), exp, what=f"wide tile, {kblocks} k-blocks, window {win}", k=k)


@pytest.mark.parametrize("c_in,r", [(256, 1), (320, 1), (64, 3)])
def test_wide_tile_conv_handover_paths(cb, cuda, orc, c_in, r):
    """The conv's 512 x 256 tile on both sides of the window: 4 k-blocks (1x1,
    256 channels) hold, 5 (1x1, 320 channels: the last block part past C)
    stream with a 3-k-block window, 9 (3x3, 64 channels) stream; against fp64."""
    import torch
    n, hh, ww, k = 3, 14, 14, 256
    g = torch.Generator().manual_seed(c_in + r)
    x = torch.empty(n, hh, ww, c_in).uniform_(0, 1, generator=g).half()
    w = (torch.randn(k, r, r, c_in, generator=g) / np.sqrt(r * r * c_in)).half()
    bias = (torch.randn(k, generator=g) * 0.1).half()
    pad = r // 2
    exp = orc.conv2d_f64(_bits(x), _bits(w), F16, pad=pad, bias=_bits(bias), dtype_bias=F16, relu=True)
    with cb.tuning(tile="wide256"):
        out = torch.empty(n, hh, ww, k, device="cuda", dtype=torch.float16)
        cb.conv2d(x.cuda(), w.cuda(), out, padding=pad, bias=bias.cuda(), relu=True)
    cb.sync_status()
    assert_close(as_f64(_bits(out.cpu()), F16).reshape(-1, k), exp, what=f"wide conv C={c_in} {r}x{r}", k=r * r * c_in)
