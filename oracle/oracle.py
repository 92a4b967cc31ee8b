"""ctypes binding of the C oracle (libt0oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py -- never by the product package.
The functions restate the reference engine t0-core; see t0_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libt0oracle.so")

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
QTYPES = {"f16": F16, "q8_0": Q8_0, "q4_0": Q4_0}


class OConfig(C.Structure):
    _fields_ = [
        ("embed_dim", C.c_int), ("num_layers", C.c_int), ("num_heads", C.c_int),
        ("mlp_hidden_dim", C.c_int), ("patch_size", C.c_int), ("group_every_n", C.c_int),
        ("dropout", C.c_float), ("n_quantiles", C.c_int), ("quantile_levels", C.c_float * 32),
        ("scaler_use_arcsinh", C.c_int), ("scaler_eps", C.c_float), ("variance_offset", C.c_int),
    ]


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "t0_oracle.c")):
            build()
        L = C.CDLL(_LIB_PATH)
        vp = C.c_void_p
        L.o_f32_to_f16.restype = C.c_uint16
        L.o_f32_to_f16.argtypes = [C.c_float]
        L.o_f16_to_f32.restype = C.c_float
        L.o_f16_to_f32.argtypes = [C.c_uint16]
        for f in ("o_quantize_q8_0", "o_quantize_q4_0", "o_dequantize_q8_0", "o_dequantize_q4_0"):
            getattr(L, f).argtypes = [vp, C.c_size_t, vp]
            getattr(L, f).restype = None
        L.o_export_gguf.argtypes = [C.c_int, vp, vp, vp, vp, C.c_int, C.POINTER(OConfig),
                                    C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(C.c_size_t)]
        L.o_free.argtypes = [vp]
        L.o_model_load_gguf.argtypes = [vp, C.c_size_t, C.POINTER(vp)]
        L.o_model_free.argtypes = [vp]
        L.o_model_config.argtypes = [vp, C.POINTER(OConfig)]
        L.o_model_tensor.argtypes = [vp, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int64),
                                     C.POINTER(C.c_int64), C.POINTER(C.POINTER(C.c_uint8)),
                                     C.POINTER(C.c_size_t)]
        L.o_forecast.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, vp]
        L.o_forecast_batch.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]
        L.o_interpolate_quantiles.argtypes = [vp, C.c_int, vp, vp, C.c_int, vp]
        L.o_interpolate_quantiles.restype = None
        L.o_weighted_quantile.argtypes = [vp, C.c_int, vp, vp, C.c_int, vp]
        L.o_weighted_quantile.restype = None
        L.o_prob_mass.argtypes = [vp, C.c_int, vp]
        L.o_prob_mass.restype = None
        L.o_forecast_rollout.argtypes = [vp, vp, C.c_int, C.c_int, vp, C.c_int, vp]
        L.o_forecast_batch_rows.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp]
        L.o_forecast_multiseries.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]
        L.o_forward.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp, vp, vp, vp]
        L.o_rmsnorm.argtypes = [vp, C.c_int, C.c_int, vp, C.c_float, vp]
        L.o_rmsnorm.restype = None
        L.o_rope_tables.argtypes = [C.c_int, C.c_int, vp, vp, vp]
        L.o_rope_tables.restype = None
        L.o_scale_input.argtypes = [C.POINTER(OConfig), C.c_int, C.c_int, vp, vp, vp, vp, vp, vp]
        L.o_scale_input.restype = None
        L.o_gemm_q_f64.argtypes = [C.c_int, vp, C.c_int, C.c_int, vp, C.c_int, vp, vp]
        L.o_swiglu_q_f64.argtypes = [C.c_int, vp, C.c_int, C.c_int, vp, C.c_int, vp, C.c_int, vp, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def cfg_struct(cfg: dict) -> OConfig:
    c = OConfig()
    for k in ("embed_dim", "num_layers", "num_heads", "mlp_hidden_dim", "patch_size", "group_every_n"):
        setattr(c, k, int(cfg[k]))
    c.dropout = float(cfg["dropout"])
    q = list(cfg["quantile_levels"])
    c.n_quantiles = len(q)
    for i, v in enumerate(q):
        c.quantile_levels[i] = v
    c.scaler_use_arcsinh = int(bool(cfg["scaler_use_arcsinh"]))
    c.scaler_eps = float(cfg["scaler_eps"])
    c.variance_offset = int(cfg["scaler_eps_mode"] != "std_clamp")
    return c


# ---- codecs -----------------------------------------------------------------
def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, np.float32).ravel()
    return np.array([L.o_f32_to_f16(float(v)) for v in flat], np.uint16).reshape(np.shape(x))


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    bpb = 34 if qtype == Q8_0 else 18
    out = np.zeros(x.size // 32 * bpb, np.uint8)
    fn = lib().o_quantize_q8_0 if qtype == Q8_0 else lib().o_quantize_q4_0
    fn(_p(x), x.size, _p(out))
    return out


def dequantize(b: np.ndarray, n: int, qtype: int) -> np.ndarray:
    b = np.ascontiguousarray(b, np.uint8)
    out = np.zeros(n, np.float32)
    fn = lib().o_dequantize_q8_0 if qtype == Q8_0 else lib().o_dequantize_q4_0
    fn(_p(b), n, _p(out))
    return out


def export_gguf(weights: dict[str, np.ndarray], cfg: dict, quant: str) -> bytes:
    """weights.rs:187-227 `export_gguf` into an in-memory GGUF file."""
    names = list(weights)
    arrs = [np.ascontiguousarray(weights[n], np.float32) for n in names]
    cnames = (C.c_char_p * len(names))(*[n.encode() for n in names])
    ndims = np.array([a.ndim for a in arrs], np.int32)
    shapes = np.array([[a.shape[0], a.shape[1] if a.ndim == 2 else 1] for a in arrs], np.int64)
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    out = C.POINTER(C.c_uint8)()
    n = C.c_size_t()
    c = cfg_struct(cfg)
    rc = lib().o_export_gguf(len(names), cnames, _p(ndims), _p(shapes), ptrs, QTYPES[quant], C.byref(c),
                             C.byref(out), C.byref(n))
    assert rc == 0
    data = C.string_at(out, n.value)
    lib().o_free(out)
    return data


# ---- primitives ---------------------------------------------------------------
def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float = 1e-8) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros_like(x)
    lib().o_rmsnorm(_p(x), rows, dim, _p(np.ascontiguousarray(g, np.float32)), eps, _p(out))
    return out


def rope_tables(seq: int, hd: int):
    cos = np.zeros((seq, hd), np.float32)
    sin = np.zeros((seq, hd), np.float32)
    sc = np.zeros((seq, hd), np.float32)
    lib().o_rope_tables(seq, hd, _p(cos), _p(sin), _p(sc))
    return cos, sin, sc


def scale_input(cfg: dict, variates, mask, group_ids):
    variates = np.ascontiguousarray(variates, np.float32)
    mask = np.ascontiguousarray(mask, np.int8)
    group_ids = np.ascontiguousarray(group_ids, np.int64)
    v, t = variates.shape
    scaled, loc, sc = (np.zeros((v, t), np.float32) for _ in range(3))
    c = cfg_struct(cfg)
    lib().o_scale_input(C.byref(c), v, t, _p(variates), _p(mask), _p(group_ids), _p(scaled), _p(loc), _p(sc))
    return scaled, loc, sc


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


def interpolate_quantiles(query, levels, values) -> np.ndarray:
    """quantile.rs:17-43 (oracle/t0_oracle.c o_interpolate_quantiles)."""
    q, l, v = _f32(query), _f32(levels), _f32(values)
    out = np.zeros(q.size, np.float32)
    lib().o_interpolate_quantiles(_p(q), q.size, _p(l), _p(v), l.size, _p(out))
    return out


def weighted_quantile(query, weights, samples) -> np.ndarray:
    """quantile.rs:47-61."""
    q, w, s = _f32(query), _f32(weights), _f32(samples)
    out = np.zeros(q.size, np.float32)
    lib().o_weighted_quantile(_p(q), q.size, _p(w), _p(s), s.size, _p(out))
    return out


def prob_mass(levels) -> np.ndarray:
    """quantile.rs:66-78."""
    l = _f32(levels)
    out = np.zeros(l.size, np.float32)
    lib().o_prob_mass(_p(l), l.size, _p(out))
    return out


def gemm_q_f64(qtype: int, w_bytes: np.ndarray, N: int, K: int, x: np.ndarray, bias=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0]
    y = np.zeros((M, N), np.float64)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    assert lib().o_gemm_q_f64(qtype, _p(np.ascontiguousarray(w_bytes, np.uint8)), N, K, _p(x), M, _p(b), _p(y)) == 0
    return y


def swiglu_q_f64(qtype: int, w0: np.ndarray, F: int, K: int, w2: np.ndarray, N2: int, x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0]
    z = np.zeros((M, F), np.float64)
    y = np.zeros((M, N2), np.float64)
    assert lib().o_swiglu_q_f64(qtype, _p(np.ascontiguousarray(w0, np.uint8)), F, K,
                                _p(np.ascontiguousarray(w2, np.uint8)), N2, _p(x), M, _p(z), _p(y)) == 0
    return z, y


# ---- model --------------------------------------------------------------------
class OracleModel:
    """t0-core `T0Model` loaded from GGUF bytes (weights dequantized to f32)."""

    def __init__(self, gguf_bytes: bytes):
        self._buf = np.frombuffer(gguf_bytes, np.uint8)
        h = C.c_void_p()
        rc = lib().o_model_load_gguf(_p(self._buf), self._buf.size, C.byref(h))
        if rc != 0:
            raise ValueError("oracle: GGUF parse failed")
        self._h = h
        c = OConfig()
        lib().o_model_config(h, C.byref(c))
        self.n_q = c.n_quantiles
        self.cfg = c

    def __del__(self):
        if getattr(self, "_h", None):
            try:
                lib().o_model_free(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def tensor(self, name: str):
        ty, r, c = C.c_int(), C.c_int64(), C.c_int64()
        ptr, nb = C.POINTER(C.c_uint8)(), C.c_size_t()
        if lib().o_model_tensor(self._h, name.encode(), C.byref(ty), C.byref(r), C.byref(c), C.byref(ptr),
                                C.byref(nb)) != 0:
            raise KeyError(name)
        return ty.value, (r.value, c.value), np.frombuffer(C.string_at(ptr, nb.value), np.uint8)

    def forecast(self, ctx: np.ndarray, horizon: int) -> np.ndarray:
        ctx = np.ascontiguousarray(ctx, np.float32)
        v, t = ctx.shape
        out = np.zeros((v, horizon, self.n_q), np.float32)
        rc = lib().o_forecast(self._h, _p(ctx), v, t, horizon, _p(out))
        if rc:
            raise ValueError(f"oracle forecast failed ({rc})")
        return out

    def forecast_batch(self, ctx: np.ndarray, horizon: int, chunk: int = 16) -> np.ndarray:
        ctx = np.ascontiguousarray(ctx, np.float32)
        n, t = ctx.shape
        out = np.zeros((n, horizon, self.n_q), np.float32)
        rc = lib().o_forecast_batch(self._h, _p(ctx), n, t, horizon, chunk, _p(out))
        if rc:
            raise ValueError(f"oracle forecast_batch failed ({rc})")
        return out

    def forecast_batch_rows(self, rows: list[np.ndarray], horizon: int, chunk: int = 16) -> np.ndarray:
        lengths = np.array([len(r) for r in rows], np.int64)
        ctx = np.ascontiguousarray(np.concatenate(rows).astype(np.float32))
        out = np.zeros((len(rows), horizon, self.n_q), np.float32)
        rc = lib().o_forecast_batch_rows(self._h, _p(ctx), _p(lengths), len(rows), horizon, chunk, _p(out))
        if rc:
            raise ValueError(f"oracle forecast_batch_rows failed ({rc})")
        return out

    def forecast_multiseries(self, ctx: np.ndarray, n_variates: np.ndarray, horizon: int,
                             threads: int = 1) -> np.ndarray:
        ctx = np.ascontiguousarray(ctx, np.float32)
        nv = np.ascontiguousarray(n_variates, np.int32)
        out = np.zeros((ctx.shape[0], horizon, self.n_q), np.float32)
        rc = lib().o_forecast_multiseries(self._h, _p(ctx), _p(nv), nv.size, ctx.shape[1], horizon, threads,
                                          _p(out))
        if rc:
            raise ValueError(f"oracle forecast_multiseries failed ({rc})")
        return out

    def forecast_rollout(self, ctx: np.ndarray, prediction_length: int, query_levels) -> np.ndarray:
        """t0-core model.rs:582-665: [prediction_length, len(query_levels)]."""
        ctx = _f32(ctx).reshape(-1)
        q = _f32(query_levels)
        out = np.zeros((prediction_length, q.size), np.float32)
        rc = lib().o_forecast_rollout(self._h, _p(ctx), ctx.size, prediction_length, _p(q), q.size, _p(out))
        if rc:
            raise ValueError(f"oracle forecast_rollout failed ({rc})")
        return out

    def forward(self, variates, mask, group_ids, variate_type, trace: bool = False):
        variates = np.ascontiguousarray(variates, np.float32)
        v, t = variates.shape
        P = self.cfg.patch_size
        p = t // P
        out = np.zeros((v, p, P, self.n_q), np.float32)
        tr = np.zeros((self.cfg.num_layers + 1, v * p, self.cfg.embed_dim), np.float32) if trace else None
        rc = lib().o_forward(self._h, v, t, _p(variates), _p(np.ascontiguousarray(mask, np.int8)),
                             _p(np.ascontiguousarray(group_ids, np.int64)),
                             _p(np.ascontiguousarray(variate_type, np.int64)), _p(out), _p(tr))
        if rc:
            raise ValueError(f"oracle forward failed ({rc})")
        return (out, tr) if trace else out
