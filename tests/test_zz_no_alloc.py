"""choreo_gemm_noalloc: the GEMM entry point for callers that cannot allocate
device memory (a plugin whose host runtime owns every buffer, a loop that must
not call cudaMalloc). It takes no workspace; an operand that needs repacking
is staged in the library's built-in scratch array instead.

Checked through the C ABI against the existing entry point (choreo_gemm with
a caller-allocated workspace), within the suite's tolerance, on two calls in a
row (the second reuses the scratch the first left behind), plus the rejection
of a request whose repack would not fit the scratch. This file is collected
last so a failure here does not hide the rest of the suite; it also passes on
its own in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import pytest

from _util import F16, TOL, dev_normal, dev_uniform

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 * 1024 * 1024


def existing_entry(cb, desc):
    """choreo_gemm with a workspace of the queried size, allocated by the test."""
    import torch
    need = cb.gemm_query(desc).workspace_bytes
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    cb.check(cb.lib.choreo_gemm(C.byref(desc), ws.data_ptr(), need, torch.cuda.current_stream().cuda_stream))
    cb.sync_status()


def noalloc_entry(cb, desc):
    import torch
    cb.check(cb.lib.choreo_gemm_noalloc(C.byref(desc), torch.cuda.current_stream().cuda_stream))
    cb.sync_status()


def compare(orc, got, want):
    g = got.double().cpu().numpy()
    w = want.double().cpu().numpy()
    err = orc.rel_err(g, w)
    assert err <= TOL, err


def test_noalloc_matches_existing_entry_two_calls(cb, cuda, orc):
    import torch
    # call 1: A stored K x M with M = 4097 (lda not 16-byte aligned) -> A is repacked (12.6 MB)
    M, N, K = 4097, 3000, 1536
    a = dev_normal((K, M), 0, 1, 71, F16)
    b = dev_normal((K, N), 0, 1, 72, F16)
    c_new = torch.full((M, N), -3.0, device="cuda", dtype=torch.float16)
    c_old = torch.full((M, N), -3.0, device="cuda", dtype=torch.float16)
    d_new = cb.make_gemm_desc(a, b, c_new, m=M, n=N, k=K, trans_a=True, lda=M, ldb=N)
    d_old = cb.make_gemm_desc(a, b, c_old, m=M, n=N, k=K, trans_a=True, lda=M, ldb=N)
    assert 0 < cb.gemm_query(d_new).workspace_bytes <= SCRATCH_BYTES
    noalloc_entry(cb, d_new)
    existing_entry(cb, d_old)
    compare(orc, c_new, c_old)

    # call 2, right after: different shape, both operands padded (odd leading
    # dimensions) so the scratch still holds call 1's data when it is reused
    m, n, k = 1000, 777, 333
    a2 = dev_uniform((m, k + 3), -1, 1, 73, F16)[:, :k]
    b2 = dev_uniform((k, n + 5), -1, 1, 74, F16)[:, :n]
    c2_new = torch.zeros(m, n, device="cuda", dtype=torch.float16)
    c2_old = torch.zeros(m, n, device="cuda", dtype=torch.float16)
    e_new = cb.make_gemm_desc(a2, b2, c2_new, m=m, n=n, k=k, lda=a2.stride(0), ldb=b2.stride(0))
    e_old = cb.make_gemm_desc(a2, b2, c2_old, m=m, n=n, k=k, lda=a2.stride(0), ldb=b2.stride(0))
    assert cb.gemm_query(e_new).workspace_bytes > 0
    noalloc_entry(cb, e_new)
    existing_entry(cb, e_old)
    compare(orc, c2_new, c2_old)
    # and against the fp64 oracle, so agreement is not agreement on a wrong answer
    from _util import as_f64, to_host
    r = orc.gemm_f64(to_host(a2), to_host(b2), F16)
    assert orc.rel_err(as_f64(to_host(c2_new), F16), r) <= TOL


def test_noalloc_aligned_operands_need_no_scratch(cb, cuda, orc):
    import torch
    a = dev_uniform((512, 256), -1, 1, 75, F16)
    b = dev_uniform((256, 384), -1, 1, 76, F16)
    c_new = torch.zeros(512, 384, device="cuda", dtype=torch.float16)
    c_old = torch.zeros(512, 384, device="cuda", dtype=torch.float16)
    d_new = cb.make_gemm_desc(a, b, c_new, m=512, n=384, k=256)
    assert cb.gemm_query(d_new).workspace_bytes == 0
    noalloc_entry(cb, d_new)
    existing_entry(cb, cb.make_gemm_desc(a, b, c_old, m=512, n=384, k=256))
    compare(orc, c_new, c_old)


def test_noalloc_split_k_partials_in_scratch(cb, cuda, orc):
    """Aligned operands, few output tiles over a long K: the planner splits K
    and the fp32 partial sums live in the built-in scratch. Two calls in a
    row (the second sees the first's partials left in the array) agree with
    choreo_gemm given its own workspace and with the fp64 oracle."""
    import torch
    from _util import as_f64, to_host
    m, n, k = 300, 200, 8192
    for call, seed in enumerate((81, 83)):
        a = dev_uniform((m, k), -1, 1, seed, F16)
        b = dev_uniform((k, n), -1, 1, seed + 1, F16)
        bias = dev_normal((n,), 0, 0.1, seed + 2, F16)
        c_new = torch.full((m, n), 7.0, device="cuda", dtype=torch.float16)
        c_old = torch.full((m, n), 7.0, device="cuda", dtype=torch.float16)
        d_new = cb.make_gemm_desc(a, b, c_new, m=m, n=n, k=k, bias=bias, relu=True)
        d_old = cb.make_gemm_desc(a, b, c_old, m=m, n=n, k=k, bias=bias, relu=True)
        q = cb.gemm_query(d_new)
        assert q.split_k > 1 and q.workspace_min_bytes == 0, (call, q.split_k)
        assert 0 < q.workspace_bytes <= SCRATCH_BYTES
        noalloc_entry(cb, d_new)
        existing_entry(cb, d_old)
        compare(orc, c_new, c_old)
        r = orc.gemm_f64(to_host(a), to_host(b), F16, bias=to_host(bias), dtype_bias=F16, relu=True)
        assert orc.rel_err(as_f64(to_host(c_new), F16), r, k) <= TOL


def test_noalloc_rejects_repack_larger_than_scratch(cb, cuda):
    import torch
    M, N, K = 4097, 64, 8192  # A^T repack: 8192 x 4104 x 2 bytes = 67 MB > 32 MiB
    a = torch.zeros(K, M, device="cuda", dtype=torch.float16)
    b = torch.zeros(K, N, device="cuda", dtype=torch.float16)
    c = torch.full((M, N), 5.0, device="cuda", dtype=torch.float16)
    d = cb.make_gemm_desc(a, b, c, m=M, n=N, k=K, trans_a=True, lda=M, ldb=N)
    assert cb.gemm_query(d).workspace_bytes > SCRATCH_BYTES
    rc = cb.lib.choreo_gemm_noalloc(C.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == cb.ERR_WORKSPACE
    assert "built-in scratch" in cb.lib.choreo_last_error().decode()
    torch.cuda.synchronize()
    assert (c == 5.0).all()
