"""The C ABI boundary, on a host without a GPU.

- libchoreo_b200.so loads and exports every function include/choreo_b200.h
  declares, and nothing of its own beyond them.
- The ctypes mirror of each struct has the size and field offsets a C
  compiler gives the header.
- Host-side logic that needs no device: argument contracts rejected before
  any CUDA call (error codes and messages), the row-shard partition, and the
  multi-GPU driver's failure reporting.
"""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "choreo_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(choreo_\w+)\s*\(", text, flags=re.M))


def exported_functions() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "choreo-ir_b200" / "libchoreo_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T choreo_" in line}


def test_library_exports_every_declared_symbol(cb):
    declared = declared_functions()
    assert len(declared) >= 15
    assert declared == exported_functions()
    for name in declared:
        assert hasattr(cb.lib, name)
        assert name in cb._SIGNATURES


def test_struct_layout_matches_c_compiler(cb, tmp_path):
    structs = {
        "choreo_gemm_desc": cb.GemmDesc,
        "choreo_launch_config": cb.LaunchConfig,
        "choreo_conv_desc": cb.ConvDesc,
        "choreo_device_props": cb.DeviceProps,
        "choreo_tuning": cb.Tuning,
        "choreo_host_gemm_desc": cb.HostGemmDesc,
        "choreo_host_plan_info": cb.HostPlanInfo,
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("  return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {}
    for line in out:
        if line:
            s, f, v = line.split()
            got[(s, f)] = int(v)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_version(cb):
    assert cb.version() == 10000


def test_dtype_codes_equal_reference_enum():
    # include/choreo-ir/core/types.hpp:58-71: FLOAT16 = 8, FLOAT32 = 9, BFLOAT16 = 11
    text = HEADER.read_text()
    assert "CHOREO_DTYPE_F16 = 8" in text and "CHOREO_DTYPE_F32 = 9" in text and "CHOREO_DTYPE_BF16 = 11" in text


# ------------------------------------------------------------------ contracts checked before any CUDA call
def _desc(cb, **kw):
    d = cb.GemmDesc()
    d.m, d.n, d.k = kw.get("m", 64), kw.get("n", 64), kw.get("k", 64)
    d.dtype_ab = kw.get("dtype_ab", cb.F16)
    d.dtype_c = kw.get("dtype_c", cb.F16)
    d.a, d.b, d.c = kw.get("a", 0x1000), kw.get("b", 0x2000), kw.get("c", 0x3000)
    d.lda, d.ldb, d.ldc = kw.get("lda", d.k), kw.get("ldb", d.n), kw.get("ldc", d.n)
    d.alpha, d.beta, d.batch = 1.0, 0.0, kw.get("batch", 1)
    return d


@pytest.mark.parametrize("kw,code,msg", [
    (dict(m=0), -1, "Invalid matrix dimensions"),
    (dict(k=-3), -1, "Invalid matrix dimensions"),
    (dict(a=None), -1, "Input tensor A has null data pointer"),
    (dict(b=None), -1, "Input tensor B has null data pointer"),
    (dict(c=None), -1, "Output tensor C has null data pointer"),
    (dict(dtype_ab=3), -2, "unsupported input dtype"),
    (dict(dtype_ab=9, dtype_c=8), -2, "f32 inputs need an f32 output"),
    (dict(lda=10), -1, "lda=10"),
    (dict(ldc=3), -1, "ldc=3"),
    (dict(batch=0), -1, "batch"),
    (dict(m=1 << 31), -2, "2^31"),
    (dict(batch=1 << 31), -2, "batch above 2^31-1"),
])
def test_gemm_contract_errors(cb, kw, code, msg):
    d = _desc(cb, **kw)
    rc = cb.lib.choreo_gemm(C.byref(d), None, 0, None)
    assert rc == code
    assert msg in cb.lib.choreo_last_error().decode()
    with pytest.raises(cb.ChoreoError):
        cb.gemm_desc(d, stream=0)


def test_null_descriptor(cb):
    assert cb.lib.choreo_gemm(None, None, 0, None) == -1
    assert cb.lib.choreo_conv2d(None, None, 0, None) == -1


def test_conv_contract_errors(cb):
    d = cb.ConvDesc()
    d.n, d.h, d.w, d.c, d.k, d.r, d.s = 1, 8, 8, 12, 8, 3, 3
    d.stride_h = d.stride_w = d.dil_h = d.dil_w = 1
    d.pad_h = d.pad_w = 1
    d.dtype, d.dtype_out = cb.F16, cb.F16
    d.input, d.weight, d.output = 0x1000, 0x2000, 0x3000
    assert cb.lib.choreo_conv2d(C.byref(d), None, 0, None) == -2  # C % 8 != 0
    d.c = 16
    d.stride_h = 0
    assert cb.lib.choreo_conv2d(C.byref(d), None, 0, None) == -1
    d.stride_h = 1
    d.dtype = cb.F32
    assert cb.lib.choreo_conv2d(C.byref(d), None, 0, None) == -2


def test_elementwise_contract_errors(cb):
    assert cb.lib.choreo_relu(42, 0x1000, 0x2000, 10, None) == -2
    assert cb.lib.choreo_relu(cb.F16, None, 0x2000, 10, None) == -1
    assert cb.lib.choreo_add(cb.F16, 0x1000, 0x2000, 0x3000, -1, None) == -1


# ------------------------------------------------------------------ row sharding (host logic)
@pytest.mark.parametrize("m", [1, 127, 128, 129, 4097, 65536, 65536 + 5, 1000003])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shard_rows_partition(cb, m, n):
    spans = [cb.shard_rows(m, n, r) for r in range(n)]
    pos = 0
    for r0, rows in spans:
        assert r0 == pos and rows >= 0
        pos += rows
    assert pos == m
    sizes = [rows for _, rows in spans]
    tiles = [(rows + 127) // 128 for rows in sizes]
    assert max(tiles) - min(tiles) <= 1
    assert sizes == sorted(sizes, reverse=True)
    for r0, rows in spans:
        if rows:  # empty shards (more shards than tiles) start at m
            assert r0 % 128 == 0 and (rows % 128 == 0 or r0 + rows == m)


def test_shard_rows_65536_rows(cb):
    assert [cb.shard_rows(65536, 8, r) for r in range(8)] == [(8192 * r, 8192) for r in range(8)]


def test_shard_rows_bad_args(cb):
    with pytest.raises(cb.ChoreoError):
        cb.shard_rows(100, 0, 0)
    with pytest.raises(cb.ChoreoError):
        cb.shard_rows(100, 2, 2)


def test_rowsharded_driver_reports_failing_shard(cb):
    """Host-side fault injection: shards whose device cannot be selected (ordinal
    999) fail; the driver joins every worker and names the first failing
    shard instead of hanging or crashing."""
    n = 3
    descs = (cb.GemmDesc * n)(*[_desc(cb) for _ in range(n)])
    devices = (C.c_int * n)(999, 998, 997)
    rc = cb.lib.choreo_gemm_rowsharded(descs, n, devices, None, None)
    assert rc == -3
    assert "shard 0 (device 999)" in cb.lib.choreo_last_error().decode()


def test_tensor_map_encode_rejects_bad_arguments(cb):
    """choreo_tensor_map_encode checks its contract on the host, before any
    CUDA call: alignment of the map, base and strides, ranks, box limits and
    the swizzle span."""
    buf = (C.c_uint8 * 256)()
    addr = C.addressof(buf)
    m = addr + (-addr % 64)
    i64 = lambda *v: (C.c_int64 * len(v))(*v)
    u32 = lambda *v: (C.c_uint32 * len(v))(*v)
    enc = cb.lib.choreo_tensor_map_encode
    base = 0x10000
    ok_dims, ok_str, ok_box = i64(72, 100), i64(144), u32(64, 32)
    cases = [
        ((m + 8, cb.F16, 2, base, ok_dims, ok_str, ok_box, 0), "64-byte aligned"),
        ((m, cb.F16, 0, base, ok_dims, ok_str, ok_box, 0), "rank"),
        ((m, cb.F16, 6, base, ok_dims, ok_str, ok_box, 0), "rank"),
        ((m, cb.F16, 2, base + 2, ok_dims, ok_str, ok_box, 0), "16-byte aligned"),
        ((m, cb.F16, 2, base, ok_dims, i64(140), ok_box, 0), "multiple of 16"),
        ((m, cb.F16, 2, base, ok_dims, ok_str, u32(64, 300), 0), "outside 1..256"),
        ((m, cb.F16, 2, base, ok_dims, ok_str, u32(12, 32), 0), "multiple of 16"),
        ((m, cb.F16, 2, base, ok_dims, ok_str, u32(128, 8), 128), "swizzle span"),
        ((m, cb.F16, 2, base, ok_dims, ok_str, ok_box, 48), "swizzle_bytes"),
        ((m, cb.F16, 2, base, i64(0, 100), ok_str, ok_box, 0), "dims[0]"),
        ((m, cb.F16, 2, None, ok_dims, ok_str, ok_box, 0), "null"),
    ]
    for args, msg in cases:
        assert enc(*args) == -1, msg
        assert msg in cb.lib.choreo_last_error().decode(), (msg, cb.lib.choreo_last_error())
    assert enc(m, 3, 2, base, ok_dims, ok_str, ok_box, 0) == -2  # unsupported dtype


# ------------------------------------------------------------------ tuning overrides (explicit API, no environment)
def test_tuning_defaults_roundtrip_and_validation(cb):
    """choreo_tuning_set / _get: NULL restores the defaults, valid settings
    round-trip, invalid ones are refused and leave the previous settings."""
    assert cb.lib.choreo_tuning_set(None) == 0
    d = cb.get_tuning()
    assert (d.tile, d.split_k, d.group_m, d.l2_policy_a, d.l2_policy_b, d.wait_timeout_ms) == (b"", 0, 0, -1, -1, 0.0)
    with cb.tuning(tile="single128", split_k=4, group_m=8, l2_policy_a=2, l2_policy_b=1, wait_timeout_ms=250.0,
                   handover_kb=16):
        t = cb.get_tuning()
        assert (t.tile, t.split_k, t.group_m, t.l2_policy_a, t.l2_policy_b, t.wait_timeout_ms, t.handover_kb) == \
            (b"single128", 4, 8, 2, 1, 250.0, 16)
        for bad, msg in [(dict(tile="huge512"), "unknown tile"), (dict(split_k=65), "split_k"),
                         (dict(group_m=-1), "group_m"), (dict(l2_policy_a=3), "L2 policy"),
                         (dict(wait_timeout_ms=-1.0), "wait_timeout_ms"), (dict(handover_kb=17), "handover_kb"),
                         (dict(handover_kb=-1), "handover_kb")]:
            with pytest.raises(cb.ChoreoError, match=msg):
                cb.set_tuning(**bad)
        assert cb.get_tuning().tile == b"single128"  # unchanged by the refused calls
    assert cb.get_tuning().tile == b""


def test_library_reads_no_environment():
    """The dispatcher's knobs are an explicit API: no source of the library
    calls getenv, so a stray variable in a caller's environment changes
    nothing."""
    for f in (ROOT / "choreo-ir_b200" / "csrc").glob("*.cu*"):
        assert "getenv" not in f.read_text(), f.name


# ------------------------------------------------------------------ host-buffer plans: contracts checked before any CUDA call
def test_host_plan_contract_errors(cb):
    d = cb.HostGemmDesc()
    d.m, d.n, d.k, d.dtype_ab, d.dtype_c = 0, 64, 64, cb.F16, cb.F16
    h = C.c_void_p()
    assert cb.lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)) == -1
    assert "Invalid matrix dimensions" in cb.lib.choreo_last_error().decode() and not h.value
    d.m, d.dtype_ab = 64, 3
    assert cb.lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)) == -2
    d.dtype_ab, d.k = cb.F16, 12  # 24-byte rows of A: not TMA-addressable
    assert cb.lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)) == -2
    assert "multiple of 16 bytes" in cb.lib.choreo_last_error().decode()
    d.k, d.parts = 64, -1
    assert cb.lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)) == -1
    assert cb.lib.choreo_host_gemm_plan_create(None, C.byref(h)) == -1
    cd = cb.ConvDesc()
    cd.n, cd.h, cd.w, cd.c, cd.k, cd.r, cd.s = 2, 8, 8, 16, 16, 3, 3
    cd.stride_h = cd.stride_w = cd.dil_h = cd.dil_w = 0
    assert cb.lib.choreo_host_conv_plan_create(C.byref(cd), 0, 0, C.byref(h)) == -1
    # runs and queries on something that is not a plan of that kind
    assert cb.lib.choreo_host_gemm_run(None, 0x1000, 0x2000, None, 0x3000, 0, None) == -1
    assert cb.lib.choreo_host_conv_run(None, 0x1000, 0x2000, None, 0x3000, 0, None) == -1
    assert cb.lib.choreo_host_plan_info_get(None, None) == -1
    assert cb.lib.choreo_host_plan_destroy(None) == 0
