"""Helpers shared by the GPU parity tests: moving oracle-format arrays
(uint16 bit patterns / float32) to and from torch device tensors, seeded
device-side input generation, and the tolerance checks."""
from __future__ import annotations

import numpy as np

F16, F32, BF16 = 8, 9, 11

# Per-element tolerance against the fp64 oracle: |y - r| <= TOL * max(|r|, tau),
# tau = 1e-3 * rms(r) * sqrt(max(1, K/1024)) (see oracle.rel_err). fp32
# accumulation with fp16/bf16 output rounding gives ~2^-11 / 2^-8 relative;
# 1e-2 is the bar for both.
TOL = 1e-2


def tdtype(dt):
    import torch
    return {F16: torch.float16, BF16: torch.bfloat16, F32: torch.float32}[dt]


def to_dev(arr: np.ndarray, dt: int):
    import torch
    if dt == F32:
        return torch.from_numpy(np.ascontiguousarray(arr, np.float32)).cuda()
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
    return t.view(tdtype(dt))


def to_host(t) -> np.ndarray:
    """Device tensor -> oracle format (uint16 bits for 16-bit types, float32)."""
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def as_f64(arr: np.ndarray, dt: int) -> np.ndarray:
    from oracle import oracle as orc
    if dt == F32:
        return arr.astype(np.float64)
    return orc.bits_to_f32(arr, dt).astype(np.float64)


def dev_uniform(shape, lo, hi, seed, dt):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.empty(shape, device="cuda", dtype=torch.float32).uniform_(lo, hi, generator=g).to(tdtype(dt))


def dev_normal(shape, mean, std, seed, dt):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.empty(shape, device="cuda", dtype=torch.float32).normal_(mean, std, generator=g).to(tdtype(dt))


def sample_rows(m: int, count: int, seed: int, tile: int = 128) -> np.ndarray:
    """First/last rows, tile boundaries around the ends, and random rows."""
    rng = np.random.default_rng(seed)
    fixed = {0, 1, tile - 1, tile, m - 1, m - 2, (m - 1) // tile * tile, max(0, (m - 1) // tile * tile - 1)}
    rows = {r for r in fixed if 0 <= r < m}
    while len(rows) < min(count, m):
        rows.add(int(rng.integers(0, m)))
    return np.array(sorted(rows), dtype=np.int64)


def assert_close(y: np.ndarray, r: np.ndarray, tol: float = TOL, what: str = "", k: int | None = None):
    from oracle import oracle as orc
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    err = orc.rel_err(y, r, k)
    assert err <= tol, f"{what}: max relative error {err:.3e} > {tol:.1e}"
    return err
