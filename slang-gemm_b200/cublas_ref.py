"""cuBLAS as the comparison baseline, called exactly as slang-gemm's src/cublas.zig
does (cublasGemmEx / cublasGemmStridedBatchedEx / cublasSgemm_v2 through the C
API, src/cublas.zig:30-60, :171-241). Used only to time the vendor library next
to libgemm_sm100 for the `shader_cublas_ratio` column; the library itself never
calls cuBLAS.
"""
from __future__ import annotations

import ctypes
import os

_lib = None


def _load():
    global _lib
    if _lib is not None:
        return _lib
    try:
        import torch  # noqa: F401  (makes torch's libcublas.so.12 the one the loader already has)
    except Exception:
        pass
    for name in ("libcublas.so.12", "/usr/local/cuda/lib64/libcublas.so.12", "libcublas.so"):
        try:
            lib = ctypes.CDLL(name)
            break
        except OSError:
            lib = None
    if lib is None:
        raise OSError("libcublas not found")
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.cublasCreate_v2.argtypes = [ctypes.POINTER(vp)]
    lib.cublasDestroy_v2.argtypes = [vp]
    lib.cublasSetStream_v2.argtypes = [vp, vp]
    lib.cublasGetVersion_v2.argtypes = [vp, ctypes.POINTER(i)]
    lib.cublasGemmEx.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i]
    lib.cublasGemmStridedBatchedEx.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, ll, vp, i, i, ll, vp, vp, i, i, ll,
                                               i, i, i]
    lib.cublasSgemm_v2.argtypes = [vp, i, i, i, i, i, vp, vp, i, vp, i, vp, vp, i]
    lib.cublasSgemmStridedBatched.argtypes = [vp, i, i, i, i, i, vp, vp, i, ll, vp, i, ll, vp, vp, i, ll, i]
    lib.cublasGemmBatchedEx.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i, i]
    _lib = lib
    return lib


class Cublas:
    """cublas.Context (src/cublas.zig:78-90) over ctypes."""

    def __init__(self, stream=None):
        lib = _load()
        self._h = ctypes.c_void_p()
        s = lib.cublasCreate_v2(ctypes.byref(self._h))
        if s != 0:
            raise RuntimeError(f"cublasCreate failed: {s}")
        if stream is not None:
            lib.cublasSetStream_v2(self._h, getattr(stream, "cuda_stream", stream))

    def version(self) -> int:
        v = ctypes.c_int(0)
        _load().cublasGetVersion_v2(self._h, ctypes.byref(v))
        return v.value

    def close(self):
        if self._h:
            _load().cublasDestroy_v2(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _scalar(compute, v):
        if compute in (72, 73):
            return ctypes.c_int32(int(v))
        if compute in (64, 65):
            import numpy as np

            return ctypes.c_uint16(int(np.array(v, dtype=np.float16).view(np.uint16)))
        return ctypes.c_float(float(v))

    def gemm_strided_batched_ex(self, ta, tb, m, n, k, alpha, A, at, lda, sa, B, bt, ldb, sb, beta, C, ct, ldc, sc,
                                batch, compute, algo=-1) -> int:
        a, b = self._scalar(compute, alpha), self._scalar(compute, beta)
        p = lambda x: x if isinstance(x, int) else x.data_ptr()  # noqa: E731
        if batch == 1:
            return _load().cublasGemmEx(self._h, ta, tb, m, n, k, ctypes.byref(a), p(A), at, lda, p(B), bt, ldb,
                                        ctypes.byref(b), p(C), ct, ldc, compute, algo)
        return _load().cublasGemmStridedBatchedEx(self._h, ta, tb, m, n, k, ctypes.byref(a), p(A), at, lda, sa, p(B),
                                                  bt, ldb, sb, ctypes.byref(b), p(C), ct, ldc, sc, batch, compute,
                                                  algo)


    def sgemm(self, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, sa=0, sb=0, sc=0, batch=1) -> int:
        """cublas.sgemm / sgemmStridedBatched (src/cublas.zig:171-226)."""
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        p = lambda x: x if isinstance(x, int) else x.data_ptr()  # noqa: E731
        if batch == 1:
            return _load().cublasSgemm_v2(self._h, ta, tb, m, n, k, ctypes.byref(a), p(A), lda, p(B), ldb,
                                          ctypes.byref(b), p(C), ldc)
        return _load().cublasSgemmStridedBatched(self._h, ta, tb, m, n, k, ctypes.byref(a), p(A), lda, sa, p(B), ldb,
                                                 sb, ctypes.byref(b), p(C), ldc, sc, batch)

    def gemm_batched_ex(self, ta, tb, m, n, k, alpha, Aarr, at, lda, Barr, bt, ldb, beta, Carr, ct, ldc, batch,
                        compute, algo=-1) -> int:
        """cublas.gemmBatchedEx (src/cublas.zig:239-241): device arrays of device pointers."""
        a, b = self._scalar(compute, alpha), self._scalar(compute, beta)
        p = lambda x: x if isinstance(x, int) else x.data_ptr()  # noqa: E731
        return _load().cublasGemmBatchedEx(self._h, ta, tb, m, n, k, ctypes.byref(a), p(Aarr), at, lda, p(Barr), bt,
                                           ldb, ctypes.byref(b), p(Carr), ct, ldc, batch, compute, algo)


def version_string() -> str:
    try:
        h = Cublas()
        v = h.version()
        h.close()
        return f"{v // 10000}.{(v // 100) % 100}.{v % 100}"
    except Exception as e:  # pragma: no cover - reporting only
        return f"unavailable ({e})"


if __name__ == "__main__":  # pragma: no cover
    print(os.environ.get("CUDA_VISIBLE_DEVICES"), version_string())
