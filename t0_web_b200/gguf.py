"""GGUF codec of the product library (t0-core gguf.rs / weights.rs semantics).

quantize / dequantize: gguf.rs:100-174.  export_gguf: Weights::export_gguf
(weights.rs:187-227).  validate: read_gguf + config_from_gguf_metadata
without a device.  All backed by libt0b.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import F16, Q4_0, Q8_0, ModelInfo, check, lib, ptr

QUANT = {"f16": F16, "q8_0": Q8_0, "q4_0": Q4_0}


def row_bytes(qtype: int, n: int) -> int:
    return int(lib().t0b_row_bytes(qtype, n))


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(row_bytes(qtype, x.size), np.uint8)
    check(lib().t0b_quantize(qtype, ptr(x), x.size, ptr(out)))
    return out


def dequantize(b: np.ndarray, n: int, qtype: int) -> np.ndarray:
    b = np.ascontiguousarray(b, np.uint8)
    out = np.empty(n, np.float32)
    check(lib().t0b_dequantize(qtype, ptr(b), n, ptr(out)))
    return out


def info_struct(cfg: dict) -> ModelInfo:
    m = ModelInfo()
    for k in ("embed_dim", "num_layers", "num_heads", "mlp_hidden_dim", "patch_size", "group_every_n"):
        setattr(m, k, int(cfg[k]))
    m.dropout = float(cfg["dropout"])
    q = list(cfg["quantile_levels"])
    m.n_quantiles = len(q)
    for i, v in enumerate(q):
        m.quantile_levels[i] = v
    m.scaler_use_arcsinh = int(bool(cfg["scaler_use_arcsinh"]))
    m.scaler_eps = float(cfg["scaler_eps"])
    m.variance_offset = int(cfg["scaler_eps_mode"] != "std_clamp")
    return m


def export_gguf(weights: dict[str, np.ndarray], cfg: dict, quant: str) -> bytes:
    names = list(weights)
    arrs = [np.ascontiguousarray(weights[n], np.float32) for n in names]
    cnames = (C.c_char_p * len(names))(*[n.encode() for n in names])
    ndims = np.array([a.ndim for a in arrs], np.int32)
    shapes = np.array([[a.shape[0], a.shape[1] if a.ndim == 2 else 1] for a in arrs], np.int64)
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    info = info_struct(cfg)
    n = C.c_size_t(0)
    check(lib().t0b_export_gguf(len(names), cnames, ptr(ndims), ptr(shapes), ptrs, QUANT[quant], C.byref(info),
                                None, C.byref(n)))
    out = np.empty(n.value, np.uint8)
    check(lib().t0b_export_gguf(len(names), cnames, ptr(ndims), ptr(shapes), ptrs, QUANT[quant], C.byref(info),
                                ptr(out), C.byref(n)))
    return out.tobytes()


def validate(gguf_bytes: bytes) -> ModelInfo:
    buf = np.frombuffer(gguf_bytes, np.uint8)
    info = ModelInfo()
    check(lib().t0b_gguf_validate(ptr(buf), buf.size, C.byref(info)))
    return info
