"""ctypes binding of libchoreo_b200.so (the C ABI in include/choreo_b200.h).

This module is how Python code (tests, bench.py, __graft_entry__) reaches the
CUDA kernels. It calls the C ABI with raw device pointers; torch tensors are
accepted as a convenience for owning device memory and streams, nothing more.
Every non-zero status raises RuntimeError with the library's message, the way
the reference's C++ API throws std::runtime_error.

The library must have been built (choreo-ir_b200/build.py); importing this
module without it raises immediately: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libchoreo_b200.so"

F16, F32, BF16 = 8, 9, 11
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_WORKSPACE = 0, -1, -2, -3, -4, -5


class GemmDesc(C.Structure):
    _fields_ = [
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
        ("dtype_ab", C.c_int32), ("dtype_c", C.c_int32),
        ("a", C.c_void_p), ("lda", C.c_int64), ("trans_a", C.c_int32),
        ("b", C.c_void_p), ("ldb", C.c_int64), ("trans_b", C.c_int32),
        ("c", C.c_void_p), ("ldc", C.c_int64),
        ("alpha", C.c_float), ("beta", C.c_float),
        ("bias", C.c_void_p), ("dtype_bias", C.c_int32),
        ("relu", C.c_int32),
        ("batch", C.c_int64), ("stride_a", C.c_int64), ("stride_b", C.c_int64), ("stride_c", C.c_int64),
    ]


class LaunchConfig(C.Structure):
    _fields_ = [
        ("kernel", C.c_int32), ("tile_m", C.c_int32), ("tile_n", C.c_int32), ("tile_k", C.c_int32),
        ("stages", C.c_int32), ("cluster_m", C.c_int32),
        ("grid_x", C.c_int32), ("grid_y", C.c_int32), ("grid_z", C.c_int32),
        ("block_x", C.c_int32), ("smem_bytes", C.c_int32), ("tmem_cols", C.c_int32),
        ("tiles", C.c_int64), ("workspace_bytes", C.c_int64), ("workspace_min_bytes", C.c_int64),
        ("split_k", C.c_int64),
    ]


class ConvDesc(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("h", C.c_int64), ("w", C.c_int64), ("c", C.c_int64),
        ("k", C.c_int64), ("r", C.c_int64), ("s", C.c_int64),
        ("stride_h", C.c_int32), ("stride_w", C.c_int32),
        ("pad_h", C.c_int32), ("pad_w", C.c_int32),
        ("dil_h", C.c_int32), ("dil_w", C.c_int32),
        ("dtype", C.c_int32), ("dtype_out", C.c_int32),
        ("input", C.c_void_p), ("weight", C.c_void_p), ("output", C.c_void_p),
        ("bias", C.c_void_p), ("dtype_bias", C.c_int32), ("relu", C.c_int32),
        ("alpha", C.c_float),
    ]


class Tuning(C.Structure):
    _fields_ = [
        ("tile", C.c_char * 16), ("split_k", C.c_int32), ("group_m", C.c_int32),
        ("l2_policy_a", C.c_int32), ("l2_policy_b", C.c_int32), ("wait_timeout_ms", C.c_double),
        ("handover_kb", C.c_int32), ("reserved", C.c_int32),
    ]


class DeviceProps(C.Structure):
    _fields_ = [
        ("device", C.c_int32), ("cc_major", C.c_int32), ("cc_minor", C.c_int32),
        ("sm_count", C.c_int32), ("max_smem_optin", C.c_int32), ("cluster_launch", C.c_int32),
        ("total_mem", C.c_int64), ("name", C.c_char * 256),
    ]


# Every symbol include/choreo_b200.h declares, with its ctypes signature.
_SIGNATURES = {
    "choreo_version": (C.c_int, []),
    "choreo_last_error": (C.c_char_p, []),
    "choreo_device_props_get": (C.c_int, [C.c_int, C.POINTER(DeviceProps)]),
    "choreo_sync_status": (C.c_int, [C.c_void_p]),
    "choreo_selftest_wait_timeout": (C.c_int, [C.c_double, C.c_void_p]),
    "choreo_tuning_set": (C.c_int, [C.POINTER(Tuning)]),
    "choreo_tuning_get": (C.c_int, [C.POINTER(Tuning)]),
    "choreo_clock_probe_set": (C.c_int, [C.c_void_p]),
    "choreo_gemm_query": (C.c_int, [C.POINTER(GemmDesc), C.POINTER(LaunchConfig)]),
    "choreo_gemm": (C.c_int, [C.POINTER(GemmDesc), C.c_void_p, C.c_size_t, C.c_void_p]),
    "choreo_gemm_noalloc": (C.c_int, [C.POINTER(GemmDesc), C.c_void_p]),
    "choreo_gemm_rowsharded": (C.c_int, [C.POINTER(GemmDesc), C.c_int, C.POINTER(C.c_int),
                                         C.POINTER(C.c_void_p), C.POINTER(C.c_float)]),
    "choreo_shard_rows": (C.c_int, [C.c_int64, C.c_int, C.c_int, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "choreo_conv2d_query": (C.c_int, [C.POINTER(ConvDesc), C.POINTER(LaunchConfig)]),
    "choreo_host_gemm_plan_create": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "choreo_host_conv_plan_create": (C.c_int, [C.POINTER(ConvDesc), C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "choreo_host_gemm_run": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                       C.c_void_p]),
    "choreo_host_conv_run": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                       C.c_void_p]),
    "choreo_host_plan_info_get": (C.c_int, [C.c_void_p, C.c_void_p]),
    "choreo_host_plan_part": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "choreo_host_plan_destroy": (C.c_int, [C.c_void_p]),
    "choreo_conv2d": (C.c_int, [C.POINTER(ConvDesc), C.c_void_p, C.c_size_t, C.c_void_p]),
    "choreo_relu": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "choreo_add": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "choreo_fill": (C.c_int, [C.c_int32, C.c_void_p, C.c_double, C.c_int64, C.c_void_p]),
    "choreo_convert": (C.c_int, [C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p]),
    "choreo_tensor_map_encode": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.POINTER(C.c_int64),
                                           C.POINTER(C.c_int64), C.POINTER(C.c_uint32), C.c_int32]),
}


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python choreo-ir_b200/build.py`")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class ChoreoError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != 0:
        raise ChoreoError(rc, lib.choreo_last_error().decode())


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


_TORCH_DT = {}


def dtype_code(t) -> int:
    """Library dtype code of a torch tensor."""
    import torch
    if not _TORCH_DT:
        _TORCH_DT.update({torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32})
    return _TORCH_DT[t.dtype]


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def make_gemm_desc(a, b, c, *, m, n, k, trans_a=False, trans_b=False, lda=None, ldb=None, ldc=None,
                   alpha=1.0, beta=0.0, bias=None, relu=False, batch=1,
                   stride_a=0, stride_b=0, stride_c=0, dtype_ab=None, dtype_c=None, dtype_bias=None) -> GemmDesc:
    d = GemmDesc()
    d.m, d.n, d.k = m, n, k
    d.dtype_ab = dtype_ab if dtype_ab is not None else dtype_code(a)
    d.dtype_c = dtype_c if dtype_c is not None else dtype_code(c)
    d.a, d.b, d.c = _ptr(a), _ptr(b), _ptr(c)
    d.trans_a, d.trans_b = int(trans_a), int(trans_b)
    d.lda = lda if lda is not None else (m if trans_a else k)
    d.ldb = ldb if ldb is not None else (k if trans_b else n)
    d.ldc = ldc if ldc is not None else n
    d.alpha, d.beta = alpha, beta
    d.bias = _ptr(bias)
    d.dtype_bias = dtype_bias if dtype_bias is not None else (dtype_code(bias) if bias is not None and not isinstance(bias, int) else F32)
    d.relu = int(relu)
    d.batch, d.stride_a, d.stride_b, d.stride_c = batch, stride_a, stride_b, stride_c
    return d


def gemm_query(d: GemmDesc) -> LaunchConfig:
    out = LaunchConfig()
    check(lib.choreo_gemm_query(C.byref(d), C.byref(out)))
    return out


def gemm_desc(d: GemmDesc, workspace=None, workspace_bytes=0, stream=None) -> None:
    check(lib.choreo_gemm(C.byref(d), _ptr(workspace), workspace_bytes, _stream_ptr(stream)))


def gemm(a, b, c, *, trans_a=False, trans_b=False, alpha=1.0, beta=0.0, bias=None, relu=False,
         workspace=None, stream=None) -> None:
    """C = act(alpha * op(A) op(B) + beta * C + bias) on 2-D (or 3-D batched) torch tensors.

    a is M x K (K x M if trans_a), b is K x N (N x K if trans_b); rows may be
    padded (the row stride is taken as the leading dimension)."""
    batched = a.dim() == 3
    if batched:
        batch = a.shape[0]
        sa, sb, sc = a.stride(0), b.stride(0) if b.dim() == 3 else 0, c.stride(0)
        a2, b2, c2 = a[0], (b[0] if b.dim() == 3 else b), c[0]
    else:
        batch, sa, sb, sc = 1, 0, 0, 0
        a2, b2, c2 = a, b, c
    m = a2.shape[1] if trans_a else a2.shape[0]
    k = a2.shape[0] if trans_a else a2.shape[1]
    n = b2.shape[0] if trans_b else b2.shape[1]
    for t in (a2, b2, c2):
        if t.stride(-1) != 1:
            raise ValueError("innermost dimension must be contiguous")
    d = make_gemm_desc(a, b, c, m=m, n=n, k=k, trans_a=trans_a, trans_b=trans_b,
                       lda=a2.stride(0), ldb=b2.stride(0), ldc=c2.stride(0), alpha=alpha, beta=beta,
                       bias=bias, relu=relu, batch=batch, stride_a=sa, stride_b=sb, stride_c=sc)
    ws_bytes = 0
    if workspace is None:
        need = gemm_query(d).workspace_bytes
        if need:
            import torch
            workspace = torch.empty(need, dtype=torch.uint8, device=c.device)
    if workspace is not None:
        ws_bytes = workspace.numel() * workspace.element_size()
    gemm_desc(d, workspace, ws_bytes, stream)


class HostGemmDesc(C.Structure):
    _fields_ = [
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
        ("dtype_ab", C.c_int32), ("dtype_c", C.c_int32), ("alpha", C.c_float),
        ("has_bias", C.c_int32), ("dtype_bias", C.c_int32), ("relu", C.c_int32),
        ("parts", C.c_int32), ("device", C.c_int32),
    ]


class HostPlanInfo(C.Structure):
    _fields_ = [
        ("parts", C.c_int32), ("launches_per_run", C.c_int32), ("device_bytes", C.c_int64),
        ("h2d_bytes", C.c_int64), ("d2h_bytes", C.c_int64),
    ]


OPERANDS_ON_DEVICE = 1


class _HostPlan:
    """Owner of a choreo_host_plan (the C ABI's host-buffer pipeline)."""

    def __init__(self, handle: C.c_void_p):
        self._h = handle
        self.info = HostPlanInfo()
        check(lib.choreo_host_plan_info_get(self._h, C.byref(self.info)))
        parts = []
        for i in range(self.info.parts):
            f, n = C.c_int64(), C.c_int64()
            check(lib.choreo_host_plan_part(self._h, i, C.byref(f), C.byref(n)))
            parts.append((f.value, n.value))
        self.parts = parts

    def launches(self) -> int:
        return self.info.launches_per_run

    def close(self) -> None:
        if self._h:
            check(lib.choreo_host_plan_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _device_index(device) -> int:
    import torch
    if device is None:
        return torch.cuda.current_device()
    d = torch.device(device)
    return d.index if d.index is not None else torch.cuda.current_device()


class HostGemmPlan(_HostPlan):
    """C = act(A @ B + bias) for row-major tensors in HOST memory through
    choreo_host_gemm_run: A and C are cut into row slabs (whole 512-row
    tiles); the copy of slab i+1 in, the GEMM of slab i and the copy of slab
    i-1 out overlap on two library-owned copy streams and the caller's
    stream. The plan owns its device buffers, made once by
    choreo_host_gemm_plan_create. run() returns with everything enqueued; the
    caller's stream is ordered after the last copy out. Pinned host tensors
    get the overlap."""

    def __init__(self, m, n, k, dtype, *, bias=False, relu=False, slabs=None, device=None, dtype_c=None):
        import torch
        code = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}
        d = HostGemmDesc()
        d.m, d.n, d.k = m, n, k
        d.dtype_ab = code[dtype]
        d.dtype_c = code[dtype_c] if dtype_c is not None else d.dtype_ab
        d.alpha = 1.0
        d.has_bias, d.dtype_bias, d.relu = int(bool(bias)), d.dtype_ab, int(bool(relu))
        d.parts = int(slabs or 0)
        d.device = _device_index(device)
        self.device = d.device
        h = C.c_void_p()
        check(lib.choreo_host_gemm_plan_create(C.byref(d), C.byref(h)))
        super().__init__(h)
        self.slabs = self.parts

    def run(self, a_h, b, c_h, bias=None, stream=None, operands_on_device=False):
        """a_h, c_h: host tensors; b, bias: host tensors, or device tensors of
        the plan's device with operands_on_device=True."""
        check(lib.choreo_host_gemm_run(self._h, _ptr(a_h), _ptr(b), _ptr(bias), _ptr(c_h),
                                       OPERANDS_ON_DEVICE if operands_on_device else 0, _stream_ptr(stream)))


class HostConvPlan(_HostPlan):
    """conv2d for NHWC activations and KRSC weights in HOST memory through
    choreo_host_conv_run: the batch is cut into runs of images, pipelined over
    the PCIe links like HostGemmPlan."""

    def __init__(self, n, h, w, c, k, r, s, dtype, *, stride=1, padding=1, dilation=1, bias=False, relu=False,
                 runs=None, device=None):
        import torch
        code = {torch.float16: F16, torch.bfloat16: BF16}[dtype]
        d = ConvDesc()
        d.n, d.h, d.w, d.c, d.k, d.r, d.s = n, h, w, c, k, r, s
        d.stride_h = d.stride_w = stride
        d.pad_h = d.pad_w = padding
        d.dil_h = d.dil_w = dilation
        d.dtype = d.dtype_out = code
        d.bias = 1 if bias else None  # non-NULL marks a plan with a bias; the pointer is not used
        d.dtype_bias = code
        d.relu = int(bool(relu))
        d.alpha = 1.0
        self.device = _device_index(device)
        hdl = C.c_void_p()
        check(lib.choreo_host_conv_plan_create(C.byref(d), int(runs or 0), self.device, C.byref(hdl)))
        super().__init__(hdl)
        self.runs = self.parts

    def run(self, x_h, w, out_h, bias=None, stream=None, operands_on_device=False):
        check(lib.choreo_host_conv_run(self._h, _ptr(x_h), _ptr(w), _ptr(bias), _ptr(out_h),
                                       OPERANDS_ON_DEVICE if operands_on_device else 0, _stream_ptr(stream)))


def conv_desc(x, w, out, *, stride=1, padding=1, dilation=1, bias=None, relu=False, alpha=1.0) -> ConvDesc:
    """x: NHWC, w: KRSC, out: NHWC (torch tensors, contiguous)."""
    d = ConvDesc()
    d.n, d.h, d.w, d.c = x.shape
    d.k, d.r, d.s = w.shape[0], w.shape[1], w.shape[2]
    d.stride_h = d.stride_w = stride
    d.pad_h = d.pad_w = padding
    d.dil_h = d.dil_w = dilation
    d.dtype, d.dtype_out = dtype_code(x), dtype_code(out)
    d.input, d.weight, d.output = x.data_ptr(), w.data_ptr(), out.data_ptr()
    d.bias = _ptr(bias)
    d.dtype_bias = dtype_code(bias) if bias is not None else F32
    d.relu = int(relu)
    d.alpha = alpha
    return d


def conv2d_query(d: ConvDesc) -> LaunchConfig:
    out = LaunchConfig()
    check(lib.choreo_conv2d_query(C.byref(d), C.byref(out)))
    return out


def conv2d_desc(d: ConvDesc, workspace=None, workspace_bytes=0, stream=None) -> None:
    check(lib.choreo_conv2d(C.byref(d), _ptr(workspace), workspace_bytes, _stream_ptr(stream)))


def conv2d(x, w, out, *, stride=1, padding=1, dilation=1, bias=None, relu=False, alpha=1.0, stream=None) -> None:
    d = conv_desc(x, w, out, stride=stride, padding=padding, dilation=dilation, bias=bias, relu=relu, alpha=alpha)
    conv2d_desc(d, stream=stream)


def relu(x, out, stream=None) -> None:
    check(lib.choreo_relu(dtype_code(x), x.data_ptr(), out.data_ptr(), x.numel(), _stream_ptr(stream)))


def add(a, b, out, stream=None) -> None:
    check(lib.choreo_add(dtype_code(a), a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream_ptr(stream)))


def fill(x, value: float, stream=None) -> None:
    check(lib.choreo_fill(dtype_code(x), x.data_ptr(), float(value), x.numel(), _stream_ptr(stream)))


def convert(src, dst, stream=None) -> None:
    check(lib.choreo_convert(dtype_code(src), src.data_ptr(), dtype_code(dst), dst.data_ptr(), src.numel(),
                             _stream_ptr(stream)))


def sync_status(stream=None) -> None:
    check(lib.choreo_sync_status(_stream_ptr(stream)))


def selftest_wait_timeout(timeout_ms: float, stream=None) -> None:
    check(lib.choreo_selftest_wait_timeout(timeout_ms, _stream_ptr(stream)))


def get_tuning() -> Tuning:
    t = Tuning()
    check(lib.choreo_tuning_get(C.byref(t)))
    return t


def set_tuning(*, tile: str = "", split_k: int = 0, group_m: int = 0, l2_policy_a: int = -1,
               l2_policy_b: int = -1, wait_timeout_ms: float = 0.0, handover_kb: int = 0) -> None:
    """Installs dispatcher overrides (choreo_tuning_set); the defaults leave
    every choice to the library."""
    t = Tuning()
    t.tile = tile.encode()
    t.split_k, t.group_m = split_k, group_m
    t.l2_policy_a, t.l2_policy_b = l2_policy_a, l2_policy_b
    t.wait_timeout_ms = wait_timeout_ms
    t.handover_kb = handover_kb
    check(lib.choreo_tuning_set(C.byref(t)))


class tuning:
    """Context manager: `with tuning(tile="pair256"): ...` applies the
    overrides for the block and restores the previous settings after it."""

    def __init__(self, **kw):
        self.kw = kw
        self.saved = None

    def __enter__(self):
        self.saved = get_tuning()
        set_tuning(**self.kw)
        return self

    def __exit__(self, *exc):
        check(lib.choreo_tuning_set(C.byref(self.saved)))
        return False


def shard_rows(m: int, nshards: int, rank: int) -> tuple[int, int]:
    r0, rows = C.c_int64(), C.c_int64()
    check(lib.choreo_shard_rows(m, nshards, rank, C.byref(r0), C.byref(rows)))
    return r0.value, rows.value


def device_props(device: int = 0) -> DeviceProps:
    p = DeviceProps()
    check(lib.choreo_device_props_get(device, C.byref(p)))
    return p


def version() -> int:
    return lib.choreo_version()
