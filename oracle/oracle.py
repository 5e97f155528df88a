"""ctypes binding of the CPU oracle (liboracle_gemm.so, built from gemm_oracle.c).

TEST INFRASTRUCTURE ONLY. The product library never imports this module;
tests/, __graft_entry__.smoke() and bench.py's CPU legs use it as the checker
and as the timed CPU baseline. It restates slang-gemm's scalar reference
(src/gemm.zig); see gemm_oracle.h for the function-by-function citations.

Parity status: pinned by the reference's own known-answer tests (the
reference itself, Zig 0.16 + Bazel, cannot be built in this image).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle_gemm.so")

ROW_MAJOR, COL_MAJOR = 0, 1
OP_N, OP_T, OP_C = 0, 1, 2
R_32F, R_64F, R_16F, R_8I, R_8U, R_32I, R_16BF = 0, 1, 2, 3, 8, 10, 14
R_8F_E4M3, R_8F_E5M2, R_8F_UE8M0, R_6F_E2M3, R_6F_E3M2, R_4F_E2M1 = 28, 29, 30, 31, 32, 33
OK, ERR_INVALID_BATCH_COUNT, ERR_INVALID_STRIDE, ERR_BUFFER_TOO_SMALL, ERR_INVALID_TYPE, ERR_INVALID_ARGUMENT = range(6)

NP_DTYPE = {R_32F: np.float32, R_64F: np.float64, R_16F: np.uint16, R_16BF: np.uint16, R_8I: np.int8,
            R_8U: np.uint8, R_32I: np.int32}


class Layout(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_size_t), ("row_stride", ctypes.c_size_t), ("col_stride", ctypes.c_size_t)]


class Scalar(ctypes.Structure):
    _fields_ = [("re", ctypes.c_double), ("im", ctypes.c_double)]


class ExDesc(ctypes.Structure):
    _fields_ = [
        ("op_a", ctypes.c_int), ("op_b", ctypes.c_int),
        ("m", ctypes.c_size_t), ("n", ctypes.c_size_t), ("k", ctypes.c_size_t),
        ("alpha", Scalar),
        ("a", ctypes.c_void_p), ("a_len", ctypes.c_size_t), ("a_type", ctypes.c_int), ("lda", ctypes.c_size_t),
        ("b", ctypes.c_void_p), ("b_len", ctypes.c_size_t), ("b_type", ctypes.c_int), ("ldb", ctypes.c_size_t),
        ("beta", Scalar),
        ("c", ctypes.c_void_p), ("c_len", ctypes.c_size_t), ("c_type", ctypes.c_int), ("ldc", ctypes.c_size_t),
        ("compute_type", ctypes.c_int), ("layout", ctypes.c_int), ("batch_count", ctypes.c_size_t),
        ("stride_a", ctypes.c_size_t), ("stride_b", ctypes.c_size_t), ("stride_c", ctypes.c_size_t),
        ("algo", ctypes.c_int),
    ]


class PtrBatchedDesc(ctypes.Structure):
    _fields_ = [
        ("op_a", ctypes.c_int), ("op_b", ctypes.c_int),
        ("m", ctypes.c_size_t), ("n", ctypes.c_size_t), ("k", ctypes.c_size_t),
        ("alpha", Scalar),
        ("a", ctypes.POINTER(ctypes.c_void_p)), ("a_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("a_count", ctypes.c_size_t), ("a_type", ctypes.c_int), ("lda", ctypes.c_size_t),
        ("b", ctypes.POINTER(ctypes.c_void_p)), ("b_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("b_count", ctypes.c_size_t), ("b_type", ctypes.c_int), ("ldb", ctypes.c_size_t),
        ("beta", Scalar),
        ("c", ctypes.POINTER(ctypes.c_void_p)), ("c_lens", ctypes.POINTER(ctypes.c_size_t)),
        ("c_count", ctypes.c_size_t), ("c_type", ctypes.c_int), ("ldc", ctypes.c_size_t),
        ("compute_type", ctypes.c_int), ("layout", ctypes.c_int), ("algo", ctypes.c_int),
    ]


def build() -> str:
    """Compiles liboracle_gemm.so with the committed Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sz, vp, i, f, d = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
    lib.or_f32_to_f16_bits.restype = ctypes.c_uint16
    lib.or_f32_to_f16_bits.argtypes = [f]
    lib.or_f16_bits_to_f32.restype = f
    lib.or_f16_bits_to_f32.argtypes = [ctypes.c_uint16]
    lib.or_f32_to_bf16_bits.restype = ctypes.c_uint16
    lib.or_f32_to_bf16_bits.argtypes = [f]
    lib.or_bf16_bits_to_f32.restype = f
    lib.or_bf16_bits_to_f32.argtypes = [ctypes.c_uint16]
    lib.or_read_scalar.restype = None
    lib.or_read_scalar.argtypes = [vp, i, sz, ctypes.POINTER(Scalar)]
    lib.or_write_scalar.restype = None
    lib.or_write_scalar.argtypes = [vp, i, sz, ctypes.POINTER(Scalar)]
    lib.or_element_size.restype = sz
    lib.or_element_size.argtypes = [i]
    lib.or_gemm_f32.restype = i
    lib.or_gemm_f32.argtypes = [i, i, sz, sz, sz, f, vp, sz, Layout, vp, sz, Layout, f, vp, sz, Layout, sz, sz, sz, sz]
    lib.or_sgemm.restype = i
    lib.or_sgemm.argtypes = [i, i, i, sz, sz, sz, f, vp, sz, sz, vp, sz, sz, f, vp, sz, sz]
    lib.or_sgemm_strided_batched_mt.restype = i
    lib.or_sgemm_strided_batched_mt.argtypes = [i, i, i, sz, sz, sz, f, vp, sz, sz, sz, vp, sz, sz, sz, f, vp, sz, sz,
                                                sz, sz, i]
    lib.or_hgemm.restype = i
    lib.or_hgemm.argtypes = [i, i, i, sz, sz, sz, ctypes.c_uint16, vp, sz, vp, sz, ctypes.c_uint16, vp, sz]
    lib.or_gemm_ex_legacy.restype = i
    lib.or_gemm_ex_legacy.argtypes = [i, i, i, sz, sz, sz, vp, sz, Layout, vp, sz, Layout, vp, sz, Layout, f, f, sz,
                                      sz, sz, sz]
    lib.or_gemm_ex.restype = i
    lib.or_gemm_ex.argtypes = [ctypes.POINTER(ExDesc)]
    lib.or_gemm_ex_mt.restype = i
    lib.or_gemm_ex_mt.argtypes = [ctypes.POINTER(ExDesc), i]
    lib.or_gemm_batched_ex.restype = i
    lib.or_gemm_batched_ex.argtypes = [ctypes.POINTER(PtrBatchedDesc)]
    lib.or_gemm_ex_entries.restype = i
    lib.or_gemm_ex_entries.argtypes = [ctypes.POINTER(ExDesc), sz, vp, vp, vp, vp]
    return lib


lib = _load()


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- codecs ----------------------------------------------------------------

def f32_to_f16_bits(x: float) -> int:
    return lib.or_f32_to_f16_bits(x)


def f16_bits_to_f32(b: int) -> float:
    return lib.or_f16_bits_to_f32(b)


def f32_to_bf16_bits(x: float) -> int:
    return lib.or_f32_to_bf16_bits(x)


def bf16_bits_to_f32(b: int) -> float:
    return lib.or_bf16_bits_to_f32(b)


def bf16_round_array(x: np.ndarray) -> np.ndarray:
    """Vectorised f32ToBf16Bits (src/gemm.zig:924-928): (raw + 0x7fff + lsb) >> 16."""
    raw = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((raw + 0x7FFF + ((raw >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def bf16_bits_to_f32_array(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def read_scalar(data: bytes | np.ndarray, data_type: int, index: int) -> tuple[float, float]:
    buf = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data
    out = Scalar()
    lib.or_read_scalar(_p(buf), data_type, index, ctypes.byref(out))
    return out.re, out.im


# ---- GEMMs -----------------------------------------------------------------

def sgemm(layout, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc) -> int:
    """gemm.sgemm (src/gemm.zig:286-317); c (float32) is updated in place."""
    return lib.or_sgemm(layout, op_a, op_b, m, n, k, alpha, _p(a), a.size, lda, _p(b), b.size, ldb, beta, _p(c),
                        c.size, ldc)


def gemm_f32(op_a, op_b, m, n, k, alpha, a, al, b, bl, beta, c, cl, batch=1, sa=0, sb=0, sc=0) -> int:
    """gemm(f32) with explicit (offset,row_stride,col_stride) layouts (src/gemm.zig:523-544)."""
    return lib.or_gemm_f32(op_a, op_b, m, n, k, alpha, _p(a), a.size, Layout(*al), _p(b), b.size, Layout(*bl),
                           beta, _p(c), c.size, Layout(*cl), batch, sa, sb, sc)


def sgemm_strided_batched_mt(layout, op_a, op_b, m, n, k, alpha, a, lda, sa, b, ldb, sb, beta, c, ldc, sc, batch,
                             threads) -> int:
    return lib.or_sgemm_strided_batched_mt(layout, op_a, op_b, m, n, k, alpha, _p(a), a.size, lda, sa, _p(b),
                                           b.size, ldb, sb, beta, _p(c), c.size, ldc, sc, batch, threads)


def hgemm(layout, op_a, op_b, m, n, k, alpha_bits, a, lda, b, ldb, beta_bits, c, ldc) -> int:
    return lib.or_hgemm(layout, op_a, op_b, m, n, k, alpha_bits, _p(a), lda, _p(b), ldb, beta_bits, _p(c), ldc)


def gemm_ex_legacy(bf16, op_a, op_b, m, n, k, a, al, b, bl, c, cl, alpha, beta, batch=1, sa=0, sb=0, sc=0) -> int:
    return lib.or_gemm_ex_legacy(1 if bf16 else 0, op_a, op_b, m, n, k, _p(a), a.size, Layout(*al), _p(b), b.size,
                                 Layout(*bl), _p(c), c.size, Layout(*cl), alpha, beta, batch, sa, sb, sc)


def make_ex_desc(op_a, op_b, m, n, k, alpha, a, a_type, lda, b, b_type, ldb, beta, c, c_type, ldc,
                 compute_type=68, layout=COL_MAJOR, batch=1, sa=0, sb=0, sc=0) -> ExDesc:
    al = alpha if isinstance(alpha, tuple) else (float(alpha), 0.0)
    be = beta if isinstance(beta, tuple) else (float(beta), 0.0)
    return ExDesc(op_a, op_b, m, n, k, Scalar(*al), a.ctypes.data, a.nbytes, a_type, lda, b.ctypes.data, b.nbytes,
                  b_type, ldb, Scalar(*be), c.ctypes.data, c.nbytes, c_type, ldc, compute_type, layout, batch, sa, sb,
                  sc, -1)


def gemm_ex(*args, threads: int = 1, **kw) -> int:
    """gemm.gemmEx / gemmStridedBatchedEx -> gemmExCuda (src/gemm.zig:546-706); c updated in place.

    threads > 1 splits the output columns over POSIX threads with identical
    per-element arithmetic (bit-identical results)."""
    d = make_ex_desc(*args, **kw)
    if threads > 1:
        return lib.or_gemm_ex_mt(ctypes.byref(d), threads)
    return lib.or_gemm_ex(ctypes.byref(d))


def gemm_ex_entries(desc_args: tuple, desc_kw: dict, batch_idx, rows, cols, out_dtype) -> tuple[int, np.ndarray]:
    """Exact reference values of selected C entries (c_type encoded), without modifying C."""
    d = make_ex_desc(*desc_args, **desc_kw)
    bi = np.ascontiguousarray(batch_idx, dtype=np.int64)
    ri = np.ascontiguousarray(rows, dtype=np.int64)
    ci = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.zeros(len(ri), dtype=out_dtype)
    rc = lib.or_gemm_ex_entries(ctypes.byref(d), len(ri), _p(bi), _p(ri), _p(ci), _p(out))
    return rc, out


def gemm_batched_ex(op_a, op_b, m, n, k, alpha, a_list, a_type, lda, b_list, b_type, ldb, beta, c_list, c_type, ldc,
                    compute_type=68, layout=COL_MAJOR) -> int:
    """gemm.gemmBatchedEx (src/gemm.zig:636-663) over lists of numpy buffers."""
    def arr(lst):
        ptrs = (ctypes.c_void_p * max(1, len(lst)))(*[x.ctypes.data for x in lst])
        lens = (ctypes.c_size_t * max(1, len(lst)))(*[x.nbytes for x in lst])
        return ptrs, lens

    ap, alen = arr(a_list)
    bp, blen = arr(b_list)
    cp, clen = arr(c_list)
    al = alpha if isinstance(alpha, tuple) else (float(alpha), 0.0)
    be = beta if isinstance(beta, tuple) else (float(beta), 0.0)
    d = PtrBatchedDesc(op_a, op_b, m, n, k, Scalar(*al), ctypes.cast(ap, ctypes.POINTER(ctypes.c_void_p)), alen,
                       len(a_list), a_type, lda, ctypes.cast(bp, ctypes.POINTER(ctypes.c_void_p)), blen, len(b_list),
                       b_type, ldb, Scalar(*be), ctypes.cast(cp, ctypes.POINTER(ctypes.c_void_p)), clen, len(c_list),
                       c_type, ldc, compute_type, layout, -1)
    return lib.or_gemm_batched_ex(ctypes.byref(d))


# ---- seeded inputs ---------------------------------------------------------

def value_for(i: np.ndarray | int, bias: float) -> np.ndarray:
    """The reference tests' deterministic fill, in f32:
    ((i*19+7) % 23 - 11) / 7 + bias (tests/gemm_correctness.zig:354-357)."""
    raw = np.asarray((np.asarray(i, dtype=np.int64) * 19 + 7) % 23, dtype=np.float32)
    return (raw - np.float32(11)) / np.float32(7) + np.float32(bias)


def fill_i8(n: int, bias: int = 0) -> np.ndarray:
    """The reference bench's INT8 fill ((i*7+3) % 17) - 8 + bias (bench/gemm_perf.zig:1239-1244)."""
    i = np.arange(n, dtype=np.int64)
    return (((i * 7 + 3) % 17) - 8 + bias).astype(np.int8)


def randn_lowp(rng: np.random.Generator, n: int, dtype: int, scale: float = 0.25) -> np.ndarray:
    """N(0,1)*scale rounded to f16 (IEEE RNE) or bf16 (the reference's rounding); returns uint16 bits."""
    x = (rng.standard_normal(n, dtype=np.float32) * np.float32(scale)).astype(np.float32)
    if dtype == R_16F:
        return x.astype(np.float16).view(np.uint16)
    return bf16_round_array(x)


def decode_lowp(bits: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == R_16F:
        return bits.view(np.float16).astype(np.float32)
    return bf16_bits_to_f32_array(bits)
