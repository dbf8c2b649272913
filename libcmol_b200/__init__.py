"""libcmol-b200: a B200-native decode engine behind the libcmol C API.

The product is the shared library ``libcmol_b200/lib/libcmol.so`` (C ABI:
``include/cmol.h``, ``include/cmol_cuda.h``, ``include/cmolcu.h``).  This
package only locates and binds it with ctypes and offers helpers for the
tests and the benchmark.  There is no Python or CPU fallback: if the library
is missing or no GPU is present, the calls that need it raise.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcmol.so")

# GGUF type tags
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14

_lib = None


class CmolError(RuntimeError):
    pass


def lib() -> C.CDLL:
    """The loaded libcmol.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CmolError(f"libcmol.so not built: {LIB_PATH} (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().cmolcu_last_error().decode(errors="replace")


def check(rc: int, what: str):
    if rc != 0:
        raise CmolError(f"{what}: {last_error()}")


_vp = C.c_void_p
_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int32)


def _declare(L):
    def sig(name, res, args):
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args

    sig("cmolcu_last_error", C.c_char_p, [])
    sig("cmolcu_device_count", C.c_int, [])
    sig("cmolcu_weight_upload", C.c_int, [C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)])
    sig("cmolcu_weight_upload_dev", C.c_int, [C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)])
    sig("cmolcu_weight_free", None, [_vp])
    sig("cmolcu_weight_bytes", C.c_size_t, [_vp])
    sig("cmolcu_gemv", C.c_int, [_vp, _vp, C.c_longlong, C.c_int, C.c_int, _vp, C.c_float,
                                 _vp, C.c_longlong, C.c_int, _vp])
    sig("cmolcu_matmul", None, [_fp, _vp, _fp, C.c_int, C.c_int, C.c_int, C.c_int])
    sig("cmolcu_matmul_batched", C.c_int, [_vp, _vp, C.c_int, _vp, C.c_float, _vp, _vp])
    sig("cmolcu_matmul_batched_bench", C.c_int, [C.POINTER(_vp), C.c_int, _vp, C.c_int, _vp, C.c_int, C.c_int,
                                                 C.POINTER(C.c_float)])
    sig("cmolcu_fault_status", C.c_int, [C.c_int, C.POINTER(C.c_uint), C.c_int])
    sig("cmolcu_gemv_bench", C.c_int, [C.POINTER(_vp), C.c_int, _vp, C.c_int, _vp, C.c_int, C.c_int,
                                       C.POINTER(C.c_float)])
    for name, res, args in _EXTRA_SIGS:
        if hasattr(L, name):
            sig(name, res, args)


# Signatures of the engine / public API, filled in by engine.py when present.
_EXTRA_SIGS: list = []


class Weight:
    """A quantised [rows x k] matrix uploaded to one GPU."""

    def __init__(self, gguf_rows, dtype: int, rows: int, k: int, device: int = 0):
        import numpy as np
        self.rows, self.k, self.dtype, self.device = rows, k, dtype, device
        h = _vp()
        if isinstance(gguf_rows, np.ndarray):
            buf = np.ascontiguousarray(gguf_rows)
            check(lib().cmolcu_weight_upload(device, buf.ctypes.data, dtype, rows, k, C.byref(h)),
                  "cmolcu_weight_upload")
        else:  # torch CUDA tensor
            check(lib().cmolcu_weight_upload_dev(device, gguf_rows.data_ptr(), dtype, rows, k, C.byref(h)),
                  "cmolcu_weight_upload_dev")
        self.h = h

    @property
    def nbytes(self) -> int:
        return lib().cmolcu_weight_bytes(self.h)

    def free(self):
        if self.h:
            lib().cmolcu_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def gemv(self, x, y, n: int, x_ld: int, x_inc: int, y_ld: int, y_inc: int,
             norm_w=None, eps: float = 1e-5, stream=None):
        """y(c,r) = W . xn(c) on device tensors (torch); see cmolcu_gemv."""
        check(lib().cmolcu_gemv(self.h, x.data_ptr(), x_ld, x_inc, n,
                                norm_w.data_ptr() if norm_w is not None else None, eps,
                                y.data_ptr(), y_ld, y_inc, stream), "cmolcu_gemv")

    def matmul_batched(self, x, y, n: int, norm_w=None, eps: float = 1e-5, stream=None):
        """y[n][rows] = W . xn on the tensor cores; x [n][k] (torch, device); see cmolcu_matmul_batched."""
        check(lib().cmolcu_matmul_batched(self.h, x.data_ptr(), n,
                                          norm_w.data_ptr() if norm_w is not None else None, eps,
                                          y.data_ptr(), stream), "cmolcu_matmul_batched")


def matmul_batched_bench(weights, x, y, n: int, iters: int = 64, reps: int = 5) -> float:
    """Device milliseconds per tensor-core product over back-to-back launches."""
    arr = (_vp * len(weights))(*[w.h for w in weights])
    ms = C.c_float(0)
    check(lib().cmolcu_matmul_batched_bench(arr, len(weights), x.data_ptr(), n, y.data_ptr(), iters, reps,
                                            C.byref(ms)), "cmolcu_matmul_batched_bench")
    return ms.value


def gemv_bench(weights, x, y, n: int, iters: int = 64, reps: int = 5) -> float:
    """Device milliseconds per GEMV over back-to-back launches (cmolcu_gemv_bench)."""
    arr = (_vp * len(weights))(*[w.h for w in weights])
    ms = C.c_float(0)
    check(lib().cmolcu_gemv_bench(arr, len(weights), x.data_ptr(), n, y.data_ptr(), iters, reps,
                                  C.byref(ms)), "cmolcu_gemv_bench")
    return ms.value
