"""ctypes binding of libt0b.so (the C ABI declared in include/t0b.h).

The library is the product: there is no Python or CPU fallback.  If the
shared object is missing the import fails loudly with the build command.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libt0b.so")

T0B_OK, T0B_ERR_INVALID, T0B_ERR_FORMAT, T0B_ERR_UNSUPPORTED, T0B_ERR_CUDA, T0B_ERR_OOM, T0B_ERR_DEVICE = range(7)
F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8

# every symbol include/t0b.h declares
EXPORTED = [
    "t0b_last_error", "t0b_engine_create", "t0b_engine_destroy", "t0b_model_load_gguf", "t0b_model_destroy",
    "t0b_model_info_get", "t0b_model_set_stream", "t0b_model_stream", "t0b_model_set_max_tokens", "t0b_model_use_graphs",
    "t0b_forecast", "t0b_forecast_batch", "t0b_forecast_batch_rows", "t0b_forecast_multiseries",
    "t0b_forecast_multiseries_device", "t0b_forecast_rollout", "t0b_model_sync", "t0b_gemm_q", "t0b_swiglu_q", "t0b_gemm_q_noalloc",
    "t0b_qmatrix_create", "t0b_qmatrix_destroy", "t0b_qmatrix_gemm", "t0b_qmatrix_swiglu", "t0b_qmatrix_sync",
    "t0b_gguf_validate",
    "t0b_quantize", "t0b_dequantize", "t0b_row_bytes", "t0b_export_gguf", "t0b_model_profile_enable",
    "t0b_model_profile_read", "t0b_model_launch_count", "t0b_selftest_bounded_wait",
]


class KernelStats(C.Structure):
    _fields_ = [("name", C.c_char * 16), ("launches", C.c_uint64), ("total_ms", C.c_double),
                ("flops", C.c_double), ("bytes", C.c_double)]


class ModelInfo(C.Structure):
    _fields_ = [
        ("embed_dim", C.c_int32), ("num_layers", C.c_int32), ("num_heads", C.c_int32),
        ("mlp_hidden_dim", C.c_int32), ("patch_size", C.c_int32), ("group_every_n", C.c_int32),
        ("dropout", C.c_float), ("n_quantiles", C.c_int32), ("quantile_levels", C.c_float * 32),
        ("scaler_use_arcsinh", C.c_int32), ("scaler_eps", C.c_float), ("variance_offset", C.c_int32),
        ("weight_type", C.c_int32), ("quantizable_gpu_bytes", C.c_uint64), ("total_weight_bytes", C.c_uint64),
    ]


class T0bError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"t0b status {status}: {msg}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m t0_web_b200.build`")
    L = C.CDLL(LIB_PATH)
    vp, sz, st = C.c_void_p, C.c_size_t, C.c_int
    L.t0b_last_error.restype = C.c_char_p
    L.t0b_engine_create.argtypes = [C.c_int, C.POINTER(vp)]
    L.t0b_engine_destroy.argtypes = [vp]
    L.t0b_engine_destroy.restype = None
    L.t0b_model_load_gguf.argtypes = [vp, vp, sz, C.POINTER(vp)]
    L.t0b_model_destroy.argtypes = [vp]
    L.t0b_model_destroy.restype = None
    L.t0b_model_info_get.argtypes = [vp, C.POINTER(ModelInfo)]
    L.t0b_model_set_stream.argtypes = [vp, vp]
    L.t0b_model_stream.argtypes = [vp]
    L.t0b_model_stream.restype = vp
    L.t0b_model_set_max_tokens.argtypes = [vp, sz]
    L.t0b_model_use_graphs.argtypes = [vp, st]
    L.t0b_forecast.argtypes = [vp, vp, sz, sz, sz, vp]
    L.t0b_forecast_batch.argtypes = [vp, vp, sz, sz, sz, sz, vp]
    L.t0b_forecast_batch_rows.argtypes = [vp, vp, vp, sz, sz, sz, vp]
    L.t0b_forecast_multiseries.argtypes = [vp, vp, vp, sz, sz, sz, vp]
    L.t0b_forecast_multiseries_device.argtypes = [vp, vp, vp, sz, sz, sz, vp]
    L.t0b_forecast_rollout.argtypes = [vp, vp, sz, sz, vp, sz, vp]
    L.t0b_model_sync.argtypes = [vp]
    L.t0b_gemm_q.argtypes = [vp, st, vp, st, st, vp, st, vp, vp, vp]
    L.t0b_swiglu_q.argtypes = [vp, st, vp, vp, st, st, st, vp, st, vp, vp, vp, vp, vp]
    L.t0b_qmatrix_create.argtypes = [vp, st, vp, st, st, C.POINTER(vp)]
    L.t0b_qmatrix_destroy.argtypes = [vp]
    L.t0b_qmatrix_destroy.restype = None
    L.t0b_qmatrix_gemm.argtypes = [vp, vp, st, vp, vp, vp]
    L.t0b_qmatrix_swiglu.argtypes = [vp, vp, vp, st, vp, vp, vp, vp, vp]
    L.t0b_qmatrix_sync.argtypes = [vp, vp]
    L.t0b_gemm_q_noalloc.argtypes = [st, vp, st, st, vp, st, vp, vp, vp]
    L.t0b_gguf_validate.argtypes = [vp, sz, C.POINTER(ModelInfo)]
    L.t0b_quantize.argtypes = [st, vp, sz, vp]
    L.t0b_dequantize.argtypes = [st, vp, sz, vp]
    L.t0b_row_bytes.argtypes = [st, sz]
    L.t0b_row_bytes.restype = sz
    L.t0b_export_gguf.argtypes = [sz, vp, vp, vp, vp, st, C.POINTER(ModelInfo), vp, C.POINTER(sz)]
    L.t0b_model_profile_enable.argtypes = [vp, C.c_int]
    L.t0b_model_profile_read.argtypes = [vp, C.POINTER(KernelStats), C.c_int, C.POINTER(C.c_int)]
    L.t0b_model_launch_count.argtypes = [vp]
    L.t0b_model_launch_count.restype = C.c_uint64
    L.t0b_selftest_bounded_wait.argtypes = [vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    _lib = L
    return L


def check(status: int) -> None:
    if status != T0B_OK:
        raise T0bError(status, lib().t0b_last_error().decode(errors="replace"))


def ptr(a) -> C.c_void_p | None:
    """Pointer of a numpy array, or of a torch tensor's data (device or host)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)
