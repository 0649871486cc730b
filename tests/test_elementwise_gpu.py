"""Device elementwise kernels vs the reference's host arithmetic, bit for bit
(relu: choreo-ir.hpp:196-222, operator+: :150-191, fill: tensor.hpp:530-562),
including unaligned pointers and lengths that are not a multiple of the
vector width."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from _util import BF16, F16, F32, to_dev, to_host

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_relu_golden(cb, cuda):
    import torch
    g = np.load(GOLDEN / "end2end_relu_64x32.npz")
    for dt, xn, yn in ((F32, "x_f32", "y_f32"), (F16, "x_f16", "y_f16")):
        x = to_dev(g[xn], dt)
        y = torch.empty_like(x)
        cb.relu(x, y)
        torch.cuda.synchronize()
        assert np.array_equal(to_host(y), g[yn])


@pytest.mark.parametrize("dt", [F16, F32])
@pytest.mark.parametrize("n,offset", [(1, 0), (7, 1), (1000003, 0), (1000003, 3), (4096, 0)])
def test_relu_add_bitexact(cb, cuda, orc, dt, n, offset):
    import torch
    a = orc.uniform((n + offset,), -2, 2, n)
    b = orc.uniform((n + offset,), -2, 2, n + 1)
    if dt != F32:
        a, b = orc.to_bits(a, dt), orc.to_bits(b, dt)
    ad, bd = to_dev(a, dt)[offset:], to_dev(b, dt)[offset:]
    out = torch.empty_like(to_dev(a, dt))[offset:]
    cb.relu(ad, out)
    torch.cuda.synchronize()
    assert np.array_equal(to_host(out), orc.ref_relu(a[offset:], dt))
    cb.add(ad, bd, out)
    torch.cuda.synchronize()
    assert np.array_equal(to_host(out), orc.ref_add(a[offset:], b[offset:], dt))


def test_bf16_add_and_relu(cb, cuda):
    import torch
    a = torch.randn(100001, device="cuda").bfloat16()
    b = torch.randn(100001, device="cuda").bfloat16()
    o = torch.empty_like(a)
    cb.add(a, b, o)
    torch.cuda.synchronize()
    assert torch.equal(o, (a.float() + b.float()).bfloat16())
    cb.relu(a, o)
    torch.cuda.synchronize()
    assert torch.equal(o, torch.where(a < 0, torch.zeros_like(a), a))


def test_relu_nan_passes_through(cb, cuda):
    import torch
    x = torch.tensor([float("nan"), -1.0, 2.0, -0.0], device="cuda")
    y = torch.empty_like(x)
    cb.relu(x, y)
    torch.cuda.synchronize()
    assert torch.isnan(y[0]) and y[1] == 0 and y[2] == 2


@pytest.mark.parametrize("dt", [F16, BF16, F32])
def test_fill_and_convert(cb, cuda, dt):
    import torch
    from _util import tdtype
    x = torch.empty(12345, device="cuda", dtype=tdtype(dt))
    cb.fill(x, 42.0)
    torch.cuda.synchronize()
    assert (x == 42).all()
    src = torch.randn(12345, device="cuda")
    cb.convert(src, x)
    torch.cuda.synchronize()
    assert torch.equal(x, src.to(tdtype(dt)))
