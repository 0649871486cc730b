"""Implicit-GEMM conv2d parity on the GPU through the C ABI, against the CPU
oracle: per element within 1e-2 (floored) of the fp64 convolution over the
same rounded inputs; normwise against the reference conv loop's fp16
accumulation (benchmark/kernels/gemm_example.cu:230-247, restated in
oracle/ref_cpu.c)."""
from __future__ import annotations

import numpy as np
import pytest

from _util import BF16, F16, F32, TOL, as_f64, assert_close, tdtype, to_dev, to_host

pytestmark = pytest.mark.gpu


def out_hw(h, w, r, s, stride, pad, dil):
    return (h + 2 * pad - dil * (r - 1) - 1) // stride + 1, (w + 2 * pad - dil * (s - 1) - 1) // stride + 1


def run_conv(cb, x, w, dt_out, stride=1, pad=1, dil=1, bias=None, relu=False, alpha=1.0):
    import torch
    n, h, ww, _ = x.shape
    k, r, s, _ = w.shape
    p, q = out_hw(h, ww, r, s, stride, pad, dil)
    out = torch.full((n, p, q, k), 123.0, device="cuda", dtype=tdtype(dt_out))
    cb.conv2d(x, w, out, stride=stride, padding=pad, dilation=dil, bias=bias, relu=relu, alpha=alpha)
    cb.sync_status()
    return out


@pytest.mark.parametrize("n,h,w,c,k,r,s,stride,pad,dil", [
    (2, 10, 12, 64, 64, 3, 3, 1, 1, 1),
    (3, 9, 7, 128, 192, 3, 3, 1, 1, 1),
    (2, 17, 15, 64, 128, 3, 3, 2, 1, 1),
    (1, 14, 14, 32, 40, 3, 3, 1, 1, 1),      # C < 64: channel block past C reads as zero
    (2, 11, 13, 72, 24, 3, 3, 1, 1, 1),      # C = 72: second channel block partly past C
    (1, 12, 12, 64, 64, 1, 1, 1, 0, 1),      # 1x1
    (1, 16, 16, 64, 64, 5, 5, 1, 2, 1),      # 5x5 pad 2
    (1, 15, 15, 64, 32, 3, 3, 1, 2, 2),      # dilation 2
    (1, 9, 9, 64, 64, 3, 3, 1, 0, 1),        # no padding
    (4, 7, 5, 16, 8, 3, 3, 1, 1, 1),         # tiny
    (1, 10, 10, 16, 3, 3, 3, 2, 0, 1),       # 3 output channels: rows not 16-byte aligned, scalar stores
    (2, 13, 9, 8, 72, 3, 3, 1, 1, 1),        # C = 8, the smallest channel count
])
@pytest.mark.parametrize("dt", [F16, BF16])
def test_conv_small_full(cb, cuda, orc, n, h, w, c, k, r, s, stride, pad, dil, dt):
    x = orc.to_bits(orc.uniform((n, h, w, c), 0, 1, n * h + c), dt)
    wt = orc.to_bits(orc.normal((k, r, s, c), 0, 1.0 / np.sqrt(r * s * c), k + r), dt)
    bias = orc.normal((k,), 0, 0.1, 5)
    out = run_conv(cb, to_dev(x, dt), to_dev(wt, dt), dt, stride, pad, dil, bias=to_dev(bias, F32), relu=True)
    ref = orc.conv2d_f64(x, wt, dt, stride=stride, pad=pad, dil=dil, bias=bias, dtype_bias=F32, relu=True)
    assert_close(as_f64(to_host(out), dt).reshape(-1, k), ref, what="conv")


def test_conv_f32_output_and_alpha(cb, cuda, orc):
    x = orc.to_bits(orc.uniform((2, 8, 8, 64), 0, 1, 1), F16)
    wt = orc.to_bits(orc.normal((64, 3, 3, 64), 0, 0.05, 2), F16)
    out = run_conv(cb, to_dev(x, F16), to_dev(wt, F16), F32, alpha=0.5)
    ref = orc.conv2d_f64(x, wt, F16, alpha=0.5)
    assert_close(to_host(out).reshape(-1, 64).astype(np.float64), ref, what="conv f32 out")


def test_conv_32x56x56x256_3x3_layer(cb, cuda, orc):
    """N=32, 56x56, C=K=256, 3x3, stride 1, pad 1, fp16; activations U[0,1],
    weights N(0, std = 1/sqrt(2304)), bias N(0, 0.1); fused bias + ReLU.
    Checked on 400 sampled output pixels (image borders included) against
    fp64, and normwise against the reference's fp16-accumulating loop."""
    import torch
    N, H, W, Cc, K = 32, 56, 56, 256, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.empty(N, H, W, Cc, device="cuda").uniform_(0, 1, generator=g).half()
    wt = torch.empty(K, 3, 3, Cc, device="cuda").normal_(0, 1 / 48.0, generator=g).half()
    bias = torch.empty(K, device="cuda").normal_(0, 0.1, generator=g).half()
    out = run_conv(cb, x, wt, F16, bias=bias, relu=True)
    rng = np.random.default_rng(0)
    border = [0, 55, 56 * 55, 56 * 56 - 1, 56 * 56 * 31, N * H * W - 1, 56 * 56 * 7 + 56 * 13]
    pix = np.unique(np.concatenate([border, rng.integers(0, N * H * W, 400)])).astype(np.int64)
    xh, wh, bh = to_host(x), to_host(wt), to_host(bias)
    ref = orc.conv2d_f64(xh, wh, F16, bias=bh, dtype_bias=F16, relu=True, pixels=pix)
    got = as_f64(to_host(out.reshape(-1, K)[torch.from_numpy(pix).cuda()]), F16)
    assert_close(got, ref, what="32x56x56x256 3x3", k=9 * Cc)
    # the reference conv loop (fp16 accumulation) on the first 8 pixels of image 0
    ref16 = as_f64(orc.ref_conv2d_f16(xh[:1], wh, 1, 1, pix=(0, 8)), F16)
    pre = orc.conv2d_f64(xh[:1], wh, F16, pixels=np.arange(8))
    mine = orc.conv2d_f64(xh[:1], wh, F16, bias=bh, dtype_bias=F16, relu=True, pixels=np.arange(8))
    gpu8 = as_f64(to_host(out.reshape(-1, K)[:8]), F16)
    assert orc.normwise_err(gpu8, mine) <= TOL
    assert orc.normwise_err(ref16, pre) <= 5e-2


def test_conv_query(cb, cuda):
    import torch
    x = torch.empty(32, 56, 56, 256, device="cuda", dtype=torch.float16)
    w = torch.empty(256, 3, 3, 256, device="cuda", dtype=torch.float16)
    o = torch.empty(32, 56, 56, 256, device="cuda", dtype=torch.float16)
    q = cb.conv2d_query(cb.conv_desc(x, w, o))
    assert q.kernel == 3 and q.workspace_bytes == 0
    assert (q.tile_m, q.cluster_m) in ((128, 1), (256, 2), (512, 2))
    assert q.tiles == -(-32 * 56 * 56 // q.tile_m) * (256 // q.tile_n)


@pytest.mark.parametrize("tile", ["wide256", "pair256", "pair128", "single256", "single128", "single64"])
def test_conv_forced_tiles(cb, cuda, orc, tile):
    x = orc.to_bits(orc.uniform((3, 13, 11, 128), 0, 1, 7), F16)
    wt = orc.to_bits(orc.normal((192, 3, 3, 128), 0, 1.0 / 34, 8), F16)
    bias = orc.normal((192,), 0, 0.1, 9)
    with cb.tuning(tile=tile):
        out = run_conv(cb, to_dev(x, F16), to_dev(wt, F16), F16, bias=to_dev(bias, F32), relu=True)
        q = cb.conv2d_query(cb.conv_desc(to_dev(x, F16), to_dev(wt, F16), out))
    assert q.cluster_m == (2 if tile.startswith(("pair", "wide")) else 1)
    ref = orc.conv2d_f64(x, wt, F16, bias=bias, dtype_bias=F32, relu=True)
    assert_close(as_f64(to_host(out), F16).reshape(-1, 192), ref, what=f"conv {tile}", k=9 * 128)


def test_host_conv_plan_pipelined(cb, cuda, orc):
    """HostConvPlan: pinned host activations, weights and bias in, output out,
    image runs overlapped on three streams (a shorter last run included),
    against fp64 on sampled pixels."""
    import torch
    n, h, w, c, k = 5, 12, 10, 64, 96
    plan = cb.HostConvPlan(n, h, w, c, k, 3, 3, torch.float16, bias=True, relu=True, runs=2)
    assert [cnt for _, cnt in plan.runs] == [3, 2]
    x = orc.to_bits(orc.uniform((n, h, w, c), 0, 1, 71), F16)
    wt = orc.to_bits(orc.normal((k, 3, 3, c), 0, 1.0 / 24, 72), F16)
    bias = orc.to_bits(orc.normal((k,), 0, 0.1, 73), F16)
    as_t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.float16).pin_memory()
    out = torch.zeros(n, h, w, k, dtype=torch.float16).pin_memory()
    plan.run(as_t(x), as_t(wt), out, as_t(bias))
    torch.cuda.current_stream().synchronize()
    cb.sync_status()
    ref = orc.conv2d_f64(x, wt, F16, bias=bias, dtype_bias=F16, relu=True)
    got = as_f64(out.view(torch.int16).numpy().view(np.uint16), F16).reshape(-1, k)
    assert_close(got, ref, what="host conv plan", k=9 * c)
