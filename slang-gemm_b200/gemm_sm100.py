"""Python binding of libgemm_sm100 (include/gemm_sm100.h) over ctypes.

This is the host-side mirror of slang-gemm's cuBLAS-shaped API for Python
callers, tests and bench.py: `Handle` plays the role of `cublas.Context`
(src/cublas.zig:78-90) and its methods take the same arguments as
`cublas.sgemm` / `gemmEx` / `gemmStridedBatchedEx` / `gemmBatchedEx`
(src/cublas.zig:171-241), with device buffers given as raw pointers or torch
CUDA tensors. `host_gemm_ex` mirrors `gemm.gemmEx` (src/gemm.zig:546) over
host numpy buffers.

There is no CPU fallback: importing this module fails if the shared library
has not been built, and every call fails without an sm_100 device.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgemm_sm100.so")
HEADER_PATH = os.path.join(_HERE, "..", "include", "gemm_sm100.h")

# ---- enums (CUDA / cuBLAS integer values; src/gemm.zig:14-113) -------------
OP_N, OP_T, OP_C = 0, 1, 2
R_32F, R_64F, R_16F, R_8I, R_32I, R_16BF = 0, 1, 2, 3, 10, 14
COMPUTE_16F, COMPUTE_16F_PEDANTIC = 64, 65
COMPUTE_32F, COMPUTE_32F_PEDANTIC = 68, 69
COMPUTE_32F_FAST_16F, COMPUTE_32F_FAST_16BF, COMPUTE_32F_FAST_TF32 = 74, 75, 77
COMPUTE_64F, COMPUTE_64F_PEDANTIC = 70, 71
COMPUTE_32I, COMPUTE_32I_PEDANTIC = 72, 73
GEMM_DEFAULT, GEMM_DEFAULT_TENSOR_OP = -1, 99
LAYOUT_ROW_MAJOR, LAYOUT_COL_MAJOR = 0, 1

STATUS_SUCCESS = 0
STATUS_NOT_INITIALIZED = 1
STATUS_ALLOC_FAILED = 3
STATUS_INVALID_VALUE = 7
STATUS_ARCH_MISMATCH = 8
STATUS_EXECUTION_FAILED = 13
STATUS_INTERNAL_ERROR = 14
STATUS_NOT_SUPPORTED = 15

KERNEL_TC_F16 = 1 << 0
KERNEL_TC_BF16 = 1 << 1
KERNEL_TC_I8 = 1 << 2
KERNEL_FFMA = 1 << 3
KERNEL_SIMT = 1 << 4
KERNEL_SCALE = 1 << 5
KERNEL_TMAP = 1 << 6
KERNEL_REDUCE = 1 << 8
KERNEL_TC_TF32 = 1 << 7

ELEM_SIZE = {R_32F: 4, R_64F: 8, R_16F: 2, R_8I: 1, R_32I: 4, R_16BF: 2}
NOALLOC_MAX_BATCH = 256  # GS_NOALLOC_MAX_BATCH
PTR_MAPS_IN_KERNEL_MAX_BATCH = 64  # GS_PTR_MAPS_IN_KERNEL_MAX_BATCH


class GemmError(RuntimeError):
    """A non-success gs_status; `.status` holds the cuBLAS-style code."""

    def __init__(self, status: int, what: str, detail: str = ""):
        self.status = status
        name = status_name(status) if _lib is not None else str(status)
        super().__init__(f"{what}: {name}" + (f" ({detail})" if detail else ""))


class ExDesc(ctypes.Structure):
    """gs_ex_desc: mirrors ExDesc (src/gemm.zig:236-261)."""

    _fields_ = [
        ("op_a", ctypes.c_int), ("op_b", ctypes.c_int),
        ("m", ctypes.c_size_t), ("n", ctypes.c_size_t), ("k", ctypes.c_size_t),
        ("alpha_re", ctypes.c_double), ("alpha_im", ctypes.c_double),
        ("a", ctypes.c_void_p), ("a_len", ctypes.c_size_t), ("a_type", ctypes.c_int), ("lda", ctypes.c_size_t),
        ("b", ctypes.c_void_p), ("b_len", ctypes.c_size_t), ("b_type", ctypes.c_int), ("ldb", ctypes.c_size_t),
        ("beta_re", ctypes.c_double), ("beta_im", ctypes.c_double),
        ("c", ctypes.c_void_p), ("c_len", ctypes.c_size_t), ("c_type", ctypes.c_int), ("ldc", ctypes.c_size_t),
        ("compute_type", ctypes.c_int),
        ("layout", ctypes.c_int),
        ("batch_count", ctypes.c_size_t),
        ("stride_a", ctypes.c_size_t), ("stride_b", ctypes.c_size_t), ("stride_c", ctypes.c_size_t),
        ("algo", ctypes.c_int),
    ]


class PtrBatchedDesc(ctypes.Structure):
    """gs_ptr_batched_desc: mirrors PointerBatchedExDesc (src/gemm.zig:263-284)."""

    _fields_ = [
        ("op_a", ctypes.c_int), ("op_b", ctypes.c_int),
        ("m", ctypes.c_size_t), ("n", ctypes.c_size_t), ("k", ctypes.c_size_t),
        ("alpha_re", ctypes.c_double), ("alpha_im", ctypes.c_double),
        ("a", ctypes.POINTER(ctypes.c_void_p)), ("a_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("a_count", ctypes.c_size_t), ("a_type", ctypes.c_int), ("lda", ctypes.c_size_t),
        ("b", ctypes.POINTER(ctypes.c_void_p)), ("b_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("b_count", ctypes.c_size_t), ("b_type", ctypes.c_int), ("ldb", ctypes.c_size_t),
        ("beta_re", ctypes.c_double), ("beta_im", ctypes.c_double),
        ("c", ctypes.POINTER(ctypes.c_void_p)), ("c_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("c_count", ctypes.c_size_t), ("c_type", ctypes.c_int), ("ldc", ctypes.c_size_t),
        ("compute_type", ctypes.c_int), ("layout", ctypes.c_int), ("algo", ctypes.c_int),
    ]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C slang-gemm_b200` (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i, ll, u32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint32
    st = ctypes.c_int
    sig = {
        "gs_select_device": (st, [ctypes.c_char_p, ctypes.POINTER(i)]),
        "gs_create": (st, [ctypes.POINTER(vp)]),
        "gs_destroy": (st, [vp]),
        "gs_set_stream": (st, [vp, vp]),
        "gs_get_stream": (st, [vp, ctypes.POINTER(vp)]),
        "gs_status_name": (ctypes.c_char_p, [i]),
        "gs_last_error": (ctypes.c_char_p, [vp]),
        "gs_last_kernels": (u32, [vp]),
        "gs_launch_count": (ctypes.c_uint64, [vp]),
        "gs_device_error": (st, [vp, ctypes.POINTER(u32)]),
        "gs_set_wait_limit": (st, [vp, ll]),
        "gs_debug_skip_kblock": (st, [vp, i]),
        "gs_sgemm": (st, [vp, i, i, i, i, i, vp, vp, i, vp, i, vp, vp, i]),
        "gs_sgemm_strided_batched": (st, [vp, i, i, i, i, i, vp, vp, i, ll, vp, i, ll, vp, vp, i, ll, i]),
        "gs_hgemm": (st, [vp, i, i, i, i, i, vp, vp, i, vp, i, vp, vp, i]),
        "gs_gemm_ex": (st, [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i]),
        "gs_gemm_strided_batched_ex": (st, [vp, i, i, i, i, i, vp, vp, i, i, ll, vp, i, i, ll, vp, vp, i, i, ll,
                                            i, i, i]),
        "gs_gemm_batched_ex": (st, [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i, i]),
        "gs_plan_gemm_strided_batched_ex": (st, [i, i, i, i, i, vp, i, i, ll, vp, i, i, ll, vp, i, i, ll, i, i,
                                                 ctypes.POINTER(u32)]),
        "gs_plan_tile": (st, [i, i, i, i, i, i, i, i, i, i, i, ctypes.POINTER(i), ctypes.POINTER(i)]),
        "gs_host_gemm_ex": (st, [vp, ctypes.POINTER(ExDesc)]),
        "gs_host_gemm_batched_ex": (st, [vp, ctypes.POINTER(PtrBatchedDesc)]),
        "gs_plan_shards": (st, [ll, i, ll, ctypes.POINTER(ll)]),
        "gs_gemm_batched_ex_noalloc": (st, [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i]),
        "gs_noalloc_device_error": (st, [vp, ctypes.POINTER(u32)]),
        "gs_multi_create": (st, [ctypes.POINTER(vp), i, ctypes.POINTER(i)]),
        "gs_multi_destroy": (st, [vp]),
        "gs_multi_last_error": (ctypes.c_char_p, [vp]),
        "gs_multi_last_times": (st, [vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)]),
        "gs_gemm_strided_batched_ex_multi": (st, [vp, i, i, i, i, i, vp, ctypes.POINTER(vp), i, i, ll,
                                                  ctypes.POINTER(vp), i, i, ll, vp, ctypes.POINTER(vp), i, i, ll,
                                                  i, i, i, i]),
        "gs_gemm_batched_ex_multi": (st, [vp, i, i, i, i, i, vp, ctypes.POINTER(vp), i, i, ctypes.POINTER(vp), i,
                                          i, vp, ctypes.POINTER(vp), i, i, i, i, i]),
        "gs_gemm_ex_colsplit_multi": (st, [vp, i, i, i, i, i, vp, ctypes.POINTER(vp), i, i, ctypes.POINTER(vp), i,
                                           i, vp, ctypes.POINTER(vp), i, i, i, i, i]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = _load()


def lib() -> ctypes.CDLL:
    return _lib


def status_name(status: int) -> str:
    return _lib.gs_status_name(status).decode()


def declared_symbols(header: str = HEADER_PATH) -> list[str]:
    """Names of the functions include/gemm_sm100.h declares."""
    import re

    text = open(header).read()
    return sorted(set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", text)))


def select_device(name_substr: str | None = None) -> tuple[int, int]:
    """gs_select_device: (status, device index) of the first CUDA device whose name contains `name_substr`
    (made current), as the reference picks its device by name substring (src/vulkan_runner.zig:1273-1299)."""
    dev = ctypes.c_int(-1)
    s = _lib.gs_select_device(name_substr.encode() if name_substr else None, ctypes.byref(dev))
    return s, dev.value


def plan_shards(units: int, parts: int, align: int = 1) -> list[int]:
    """gs_plan_shards: parts+1 cut points of `units` over `parts` devices."""
    out = (ctypes.c_longlong * (parts + 1))()
    s = _lib.gs_plan_shards(units, parts, align, out)
    if s != STATUS_SUCCESS:
        raise GemmError(s, "gs_plan_shards")
    return list(out)


def plan_gemm(transa, transb, m, n, k, A, atype, lda, stride_a, B, btype, ldb, stride_b, C, ctype, ldc, stride_c,
              batch, compute) -> tuple[int, int]:
    """gs_plan_gemm_strided_batched_ex: (status, kernel bit). Pure host logic."""
    kern = ctypes.c_uint32(0)
    s = _lib.gs_plan_gemm_strided_batched_ex(transa, transb, m, n, k, A, atype, lda, stride_a, B, btype, ldb,
                                             stride_b, C, ctype, ldc, stride_c, batch, compute, ctypes.byref(kern))
    return s, kern.value


TILE_1SM, TILE_PAIR, TILE_WIDE = 1, 2, 3


def plan_tile(transa, transb, m, n, k, atype, ctype, compute, batch=1, algo=GEMM_DEFAULT, sm_count=148):
    """gs_plan_tile: (status, tile, k_slices) a tensor-core call of this shape would use (tile 1 = 1-SM
    128x256, 2 = pair 256x256, 3 = wide 256x512; k_slices > 1 = split-K). Pure host logic."""
    tile, parts = ctypes.c_int(0), ctypes.c_int(0)
    s = _lib.gs_plan_tile(transa, transb, m, n, k, atype, ctype, compute, batch, algo, sm_count, ctypes.byref(tile),
                          ctypes.byref(parts))
    return s, tile.value, parts.value


def _ptr(x) -> int | None:
    """Device pointer of a torch tensor, or an int / None passed through."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _scalar(compute: int, v):
    """Host alpha/beta in the representation the compute type selects."""
    if compute in (COMPUTE_32I, COMPUTE_32I_PEDANTIC):
        return ctypes.c_int32(int(v))
    if compute in (COMPUTE_16F, COMPUTE_16F_PEDANTIC):
        import numpy as np

        return ctypes.c_uint16(int(np.array(v, dtype=np.float16).view(np.uint16)))
    return ctypes.c_float(float(v))


def gemm_batched_ex_noalloc(stream, transa, transb, m, n, k, alpha, Aarr, atype, lda, Barr, btype, ldb, beta, Carr,
                            ctype, ldc, batch, compute) -> int:
    """gs_gemm_batched_ex_noalloc: pointer-array batched GEMM that allocates no device memory and needs no
    handle (for callers whose device memory is owned elsewhere). Returns the gs_status; batch is limited to
    NOALLOC_MAX_BATCH. `stream` is a torch.cuda.Stream, a raw cudaStream_t int, or None."""
    a, b = _scalar(compute, alpha), _scalar(compute, beta)
    ptr = getattr(stream, "cuda_stream", stream)
    return _lib.gs_gemm_batched_ex_noalloc(ptr, transa, transb, m, n, k, ctypes.byref(a), _ptr(Aarr), atype, lda,
                                           _ptr(Barr), btype, ldb, ctypes.byref(b), _ptr(Carr), ctype, ldc, batch,
                                           compute)


def noalloc_device_error(stream=None) -> tuple[int, int]:
    """gs_noalloc_device_error: (status, word) -- the device error word of the last
    gs_gemm_batched_ex_noalloc call on the current device, read after synchronising `stream`."""
    w = ctypes.c_uint32(0)
    s = _lib.gs_noalloc_device_error(getattr(stream, "cuda_stream", stream), ctypes.byref(w))
    return s, w.value


@dataclass
class _Stream:
    ptr: int


class Handle:
    """A libgemm_sm100 handle bound to the current CUDA device."""

    def __init__(self, stream=None):
        h = ctypes.c_void_p()
        s = _lib.gs_create(ctypes.byref(h))
        if s != STATUS_SUCCESS:
            raise GemmError(s, "gs_create")
        self._h = h
        if stream is not None:
            self.set_stream(stream)

    def close(self):
        if self._h:
            _lib.gs_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- handle state ----
    def set_stream(self, stream):
        """stream: a torch.cuda.Stream, a raw cudaStream_t int, or None."""
        ptr = getattr(stream, "cuda_stream", stream)
        self._check(_lib.gs_set_stream(self._h, ptr), "gs_set_stream")

    def last_error(self) -> str:
        return _lib.gs_last_error(self._h).decode()

    def last_kernels(self) -> int:
        return _lib.gs_last_kernels(self._h)

    def launch_count(self) -> int:
        return _lib.gs_launch_count(self._h)

    def device_error(self) -> int:
        w = ctypes.c_uint32(0)
        self._check(_lib.gs_device_error(self._h, ctypes.byref(w)), "gs_device_error")
        return w.value

    def set_wait_limit(self, cycles: int):
        """gs_set_wait_limit: SM cycles after which the kernels' bounded waits give up (<= 0: the default)."""
        self._check(_lib.gs_set_wait_limit(self._h, int(cycles)), "gs_set_wait_limit")

    def debug_skip_kblock(self, kblock: int):
        """gs_debug_skip_kblock: test hook that leaves one K block of the first tile unfilled (-1 = off)."""
        self._check(_lib.gs_debug_skip_kblock(self._h, int(kblock)), "gs_debug_skip_kblock")

    def _check(self, s: int, what: str):
        if s != STATUS_SUCCESS:
            raise GemmError(s, what, self.last_error() if self._h else "")

    # ---- cuBLAS-shaped calls (device pointers / torch CUDA tensors) ----
    def sgemm(self, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, check=True) -> int:
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        s = _lib.gs_sgemm(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A), lda, _ptr(B), ldb,
                          ctypes.byref(b), _ptr(C), ldc)
        if check:
            self._check(s, "gs_sgemm")
        return s

    def sgemm_strided_batched(self, transa, transb, m, n, k, alpha, A, lda, sa, B, ldb, sb, beta, C, ldc, sc,
                              batch, check=True) -> int:
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        s = _lib.gs_sgemm_strided_batched(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A), lda, sa,
                                          _ptr(B), ldb, sb, ctypes.byref(b), _ptr(C), ldc, sc, batch)
        if check:
            self._check(s, "gs_sgemm_strided_batched")
        return s

    def hgemm(self, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, check=True) -> int:
        a, b = _scalar(COMPUTE_16F, alpha), _scalar(COMPUTE_16F, beta)
        s = _lib.gs_hgemm(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A), lda, _ptr(B), ldb,
                          ctypes.byref(b), _ptr(C), ldc)
        if check:
            self._check(s, "gs_hgemm")
        return s

    def gemm_ex(self, transa, transb, m, n, k, alpha, A, atype, lda, B, btype, ldb, beta, C, ctype, ldc, compute,
                algo=GEMM_DEFAULT, check=True) -> int:
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_ex(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A), atype, lda, _ptr(B), btype,
                            ldb, ctypes.byref(b), _ptr(C), ctype, ldc, compute, algo)
        if check:
            self._check(s, "gs_gemm_ex")
        return s

    def gemm_strided_batched_ex(self, transa, transb, m, n, k, alpha, A, atype, lda, sa, B, btype, ldb, sb, beta,
                                C, ctype, ldc, sc, batch, compute, algo=GEMM_DEFAULT, check=True) -> int:
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_strided_batched_ex(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A), atype, lda,
                                            sa, _ptr(B), btype, ldb, sb, ctypes.byref(b), _ptr(C), ctype, ldc, sc,
                                            batch, compute, algo)
        if check:
            self._check(s, "gs_gemm_strided_batched_ex")
        return s

    def gemm_batched_ex(self, transa, transb, m, n, k, alpha, Aarr, atype, lda, Barr, btype, ldb, beta, Carr,
                        ctype, ldc, batch, compute, algo=GEMM_DEFAULT, check=True) -> int:
        """Aarr/Barr/Carr: device arrays (torch int64 CUDA tensors) of device pointers."""
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_batched_ex(self._h, transa, transb, m, n, k, ctypes.byref(a), _ptr(Aarr), atype, lda,
                                    _ptr(Barr), btype, ldb, ctypes.byref(b), _ptr(Carr), ctype, ldc, batch, compute,
                                    algo)
        if check:
            self._check(s, "gs_gemm_batched_ex")
        return s

    # ---- host-buffer mirror of gemm.gemmEx ----
    def host_gemm_ex(self, op_a, op_b, m, n, k, alpha, a, a_type, lda, b, b_type, ldb, beta, c, c_type, ldc,
                     compute, layout=LAYOUT_COL_MAJOR, batch=1, stride_a=0, stride_b=0, stride_c=0,
                     algo=GEMM_DEFAULT, check=True) -> int:
        """a, b, c: host buffers (numpy arrays or pinned torch CPU tensors); c is updated in place."""
        def buf(x):
            if hasattr(x, "data_ptr"):
                return x.data_ptr(), x.numel() * x.element_size()
            return x.ctypes.data, x.nbytes

        pa, la = buf(a)
        pb, lb = buf(b)
        pc, lc = buf(c)
        d = ExDesc(op_a, op_b, m, n, k, float(alpha), 0.0, pa, la, a_type, lda, pb, lb, b_type, ldb, float(beta),
                   0.0, pc, lc, c_type, ldc, compute, layout, batch, stride_a, stride_b, stride_c, algo)
        s = _lib.gs_host_gemm_ex(self._h, ctypes.byref(d))
        if check:
            self._check(s, "gs_host_gemm_ex")
        return s

    def host_gemm_batched_ex(self, op_a, op_b, m, n, k, alpha, a_list, a_type, lda, b_list, b_type, ldb, beta,
                             c_list, c_type, ldc, compute, layout=LAYOUT_COL_MAJOR, algo=GEMM_DEFAULT,
                             check=True) -> int:
        """Mirror of gemm.gemmBatchedEx (src/gemm.zig:636-663): lists of host buffers
        (numpy arrays or CPU tensors), one per entry; each c is updated in place."""
        def bufs(xs):
            ptrs, lens = [], []
            for x in xs:
                if hasattr(x, "data_ptr"):
                    ptrs.append(x.data_ptr())
                    lens.append(x.numel() * x.element_size())
                else:
                    ptrs.append(x.ctypes.data)
                    lens.append(x.nbytes)
            return ((ctypes.c_void_p * max(1, len(ptrs)))(*ptrs), (ctypes.c_size_t * max(1, len(lens)))(*lens),
                    len(ptrs))

        pa, la, na = bufs(a_list)
        pb, lb, nb = bufs(b_list)
        pc, lc, nc = bufs(c_list)
        vpp = ctypes.POINTER(ctypes.c_void_p)
        d = PtrBatchedDesc(op_a, op_b, m, n, k, float(alpha), 0.0, ctypes.cast(pa, vpp), la, na, a_type, lda,
                           ctypes.cast(pb, vpp), lb, nb, b_type, ldb, float(beta), 0.0, ctypes.cast(pc, vpp), lc, nc,
                           c_type, ldc, compute, layout, algo)
        s = _lib.gs_host_gemm_batched_ex(self._h, ctypes.byref(d))
        if check:
            self._check(s, "gs_host_gemm_batched_ex")
        return s


GATHER_NONE, GATHER_ALL = -1, -2  # gather_to values besides an index into devs
COLSPLIT_ALIGN = 256              # GS_COLSPLIT_ALIGN


class MultiHandle:
    """gs_multi_create: one handle and stream per device of `devs`, driven from this thread.

    Operand lists hold, per device, the base pointer of the whole problem's buffer on that device
    (torch CUDA tensors or ints); each device reads and writes only its shard (batch range, or
    column block for colsplit). Calls are synchronous."""

    def __init__(self, devs):
        self.devs = list(devs)
        arr = (ctypes.c_int * len(self.devs))(*self.devs)
        h = ctypes.c_void_p()
        s = _lib.gs_multi_create(ctypes.byref(h), len(self.devs), arr)
        if s != STATUS_SUCCESS:
            raise GemmError(s, "gs_multi_create")
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.gs_multi_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return _lib.gs_multi_last_error(self._h).decode()

    def last_times(self) -> tuple[list[float], list[float]]:
        """Per-device (GEMM ms, GEMM + gather ms) of the last call."""
        n = len(self.devs)
        g, t = (ctypes.c_float * n)(), (ctypes.c_float * n)()
        _lib.gs_multi_last_times(self._h, g, t)
        return list(g), list(t)

    def _check(self, s, what):
        if s != STATUS_SUCCESS:
            raise GemmError(s, what, self.last_error())

    def _arr(self, xs):
        if len(xs) != len(self.devs):
            raise ValueError("one operand per device expected")
        return (ctypes.c_void_p * len(xs))(*[_ptr(x) for x in xs])

    def gemm_strided_batched_ex(self, transa, transb, m, n, k, alpha, A, atype, lda, sa, B, btype, ldb, sb, beta,
                                C, ctype, ldc, sc, batch, compute, algo=GEMM_DEFAULT, gather_to=GATHER_NONE,
                                check=True) -> int:
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_strided_batched_ex_multi(self._h, transa, transb, m, n, k, ctypes.byref(a), self._arr(A),
                                                  atype, lda, sa, self._arr(B), btype, ldb, sb, ctypes.byref(b),
                                                  self._arr(C), ctype, ldc, sc, batch, compute, algo, gather_to)
        if check:
            self._check(s, "gs_gemm_strided_batched_ex_multi")
        return s

    def gemm_batched_ex(self, transa, transb, m, n, k, alpha, Aarr, atype, lda, Barr, btype, ldb, beta, Carr, ctype,
                        ldc, batch, compute, algo=GEMM_DEFAULT, check=True) -> int:
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_batched_ex_multi(self._h, transa, transb, m, n, k, ctypes.byref(a), self._arr(Aarr), atype,
                                          lda, self._arr(Barr), btype, ldb, ctypes.byref(b), self._arr(Carr), ctype,
                                          ldc, batch, compute, algo)
        if check:
            self._check(s, "gs_gemm_batched_ex_multi")
        return s

    def gemm_ex_colsplit(self, transa, transb, m, n, k, alpha, A, atype, lda, B, btype, ldb, beta, C, ctype, ldc,
                         compute, algo=GEMM_DEFAULT, gather_to=GATHER_NONE, check=True) -> int:
        a, b = _scalar(compute, alpha), _scalar(compute, beta)
        s = _lib.gs_gemm_ex_colsplit_multi(self._h, transa, transb, m, n, k, ctypes.byref(a), self._arr(A), atype,
                                           lda, self._arr(B), btype, ldb, ctypes.byref(b), self._arr(C), ctype, ldc,
                                           compute, algo, gather_to)
        if check:
            self._check(s, "gs_gemm_ex_colsplit_multi")
        return s
