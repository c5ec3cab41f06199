"""ctypes binding of ``libkvint4.so`` (the C ABI declared in ``include/kvint4.h``).

The shared library is built in-tree by ``kv-cache-triton_b200/build.py`` and
must be present: there is no fallback implementation.  Importing this module
on a machine without a GPU is fine (the library loads; only calls need a
device).
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkvint4.so")

KV4_F32, KV4_F16, KV4_BF16, KV4_U8 = 0, 1, 2, 3
TIE_HALF_AWAY, TIE_HALF_EVEN, TIE_HALF_AWAY_IEEE = 0, 1, 2
KV4_OK = 0
KV4_ERR_INVALID, KV4_ERR_DTYPE, KV4_ERR_SHAPE, KV4_ERR_LAYOUT = 1, 2, 3, 4
KV4_ERR_WORKSPACE, KV4_ERR_CUDA, KV4_ERR_UNSUPPORTED, KV4_ERR_DEVICE = 5, 6, 7, 8
KV4_ERR_SCRATCH_LIMIT = 9

# every function the header declares, for load checks
EXPORTED = (
    "kv4_version", "kv4_strerror", "kv4_last_cuda_error", "kv4_quantize", "kv4_append_kv",
    "kv4_dequantize", "kv4_attention", "kv4_attention_plan", "kv4_attention_partial",
    "kv4_lse_combine", "kv4_device_error", "kv4_attention_noalloc", "kv4_append_attention",
    "kv4_attention_paged", "kv4_attention_paged_plan", "kv4_append_kv_paged",
    "kv4_lse_exchange_bytes", "kv4_lse_exchange", "kv4_prefill_attention",
)


class Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("pad_", ctypes.c_int32),
        ("shape", ctypes.c_int64 * 4),
        ("stride", ctypes.c_int64 * 4),
    ]


class AttnOpts(ctypes.Structure):
    _fields_ = [
        ("force_generic", ctypes.c_int32),
        ("tiles_per_cta", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("debug_drop_last_tile", ctypes.c_int32),
        ("early_start", ctypes.c_int32),
    ]


class AttnPlan(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int32),
        ("ctas", ctypes.c_int32),
        ("tiles_per_cta", ctypes.c_int32),
        ("units", ctypes.c_int32),
        ("max_parts", ctypes.c_int32),
        ("kernels", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
    ]


class Kv4Error(RuntimeError):
    """A libkvint4 entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{fn} failed: {detail or status}")


_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python kv-cache-triton_b200/build.py` "
            "(there is no non-CUDA fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    T = P(Tensor)
    vp, i64, i32, f32, sz = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                             ctypes.c_size_t)
    L.kv4_version.restype = i32
    L.kv4_strerror.restype = ctypes.c_char_p
    L.kv4_strerror.argtypes = [i32]
    L.kv4_last_cuda_error.restype = ctypes.c_char_p
    L.kv4_quantize.argtypes = [T, T, T, i64, i32, i32, vp]
    L.kv4_append_kv.argtypes = [T, T, T, T, T, T, i64, i32, i32, vp]
    L.kv4_dequantize.argtypes = [T, T, T, i32, vp]
    L.kv4_attention.argtypes = [T, T, T, T, T, T, i32, i32, f32, vp, sz, P(AttnOpts), vp]
    L.kv4_attention_plan.argtypes = [T, T, T, T, T, T, i32, i32, P(AttnOpts), P(AttnPlan)]
    L.kv4_attention_partial.argtypes = [T, T, T, T, T, T, T, i64, i64, i32, i32, f32, vp, sz,
                                        P(AttnOpts), vp]
    L.kv4_lse_combine.argtypes = [vp, vp, i64, T, vp]
    L.kv4_device_error.argtypes = [vp, P(ctypes.c_int)]
    L.kv4_attention_noalloc.argtypes = [T, T, T, T, T, T, i32, i32, f32, vp]
    L.kv4_prefill_attention.argtypes = [T, T, T, T, T, T, i32, i32, f32, vp]
    L.kv4_append_attention.argtypes = [T, T, T, T, T, T, T, T, i32, i32, i32, f32, vp, sz,
                                       P(AttnOpts), vp]
    L.kv4_attention_paged.argtypes = [T, T, T, T, T, vp, i64, i64, vp, i64, T, i32, i32, f32, vp,
                                      sz, P(AttnOpts), vp]
    L.kv4_attention_paged_plan.argtypes = [T, T, T, T, T, i64, i64, i32, P(AttnOpts),
                                           P(AttnPlan)]
    L.kv4_append_kv_paged.argtypes = [T, T, T, T, T, T, vp, i32, i32, vp]
    L.kv4_lse_exchange_bytes.restype = i64
    L.kv4_lse_exchange_bytes.argtypes = [i64, i32, i32]
    L.kv4_lse_exchange.argtypes = [vp, vp, i64, i32, vp, i32, i32, vp, T, vp]
    for name in EXPORTED:
        if name not in ("kv4_version", "kv4_strerror", "kv4_last_cuda_error"):
            getattr(L, name).restype = i32
    _lib = L
    return L


def check(fn: str, status: int) -> None:
    if status == KV4_OK:
        return
    L = lib()
    detail = L.kv4_strerror(status).decode()
    if status == KV4_ERR_CUDA:
        detail += ": " + L.kv4_last_cuda_error().decode()
    raise Kv4Error(fn, status, detail)
