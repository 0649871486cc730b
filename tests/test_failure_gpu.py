"""Failure detection on the GPU without faulting it: a pipeline wait that
nothing completes gives up after its bound, the kernel returns, the host sees
CHOREO_ERR_TIMEOUT from choreo_sync_status, and the context keeps working."""
from __future__ import annotations

import time

import pytest

from _util import F16, dev_uniform

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cb, cuda, orc):
    import torch
    cb.sync_status()  # clean slate
    t0 = time.time()
    cb.selftest_wait_timeout(50.0)
    with pytest.raises(cb.ChoreoError) as e:
        cb.sync_status()
    assert e.value.code == cb.ERR_TIMEOUT
    assert time.time() - t0 < 30
    cb.sync_status()  # the record was cleared
    # the context is still usable: a GEMM runs and is correct
    a = dev_uniform((256, 128), -1, 1, 1, F16)
    b = dev_uniform((128, 256), -1, 1, 2, F16)
    c = torch.empty(256, 256, device="cuda", dtype=torch.float16)
    cb.gemm(a, b, c)
    cb.sync_status()
    assert torch.allclose(c.float(), a.float() @ b.float(), rtol=1e-2, atol=1e-2)


def test_selftest_rejects_bad_bound(cb, cuda):
    with pytest.raises(cb.ChoreoError):
        cb.selftest_wait_timeout(0.0)
