"""Host-side mirror of t0-web's `t0_fast` forecast API over the CUDA engine.

Same entry points, argument meaning and error behaviour as
crates/t0-fast/src/lib.rs (the reference's GPU engine), backed by the
sm_100a kernels of libt0b.so:

=====================================  ======================================
reference (t0_fast)                    here
=====================================  ======================================
Engine::new (engine.rs:109-111)        Engine(device)
load_model_from_gguf (lib.rs:42-44)    load_model_from_gguf(engine, bytes)
forecast (lib.rs:107-109)              forecast(engine, model, ctx, v, t_ctx, horizon)
forecast_batch_chunked (lib.rs:144)    forecast_batch_chunked(...)
forecast_batch_rows_chunked (246)      forecast_batch_rows_chunked(...)
GpuModel::quantizable_gpu_bytes (194)  GpuModel.quantizable_gpu_bytes()
GpuModel::total_weight_bytes (208)     GpuModel.total_weight_bytes()
=====================================  ======================================

plus `forecast_multiseries` (many independent multivariate series in one
call), which the reference expresses as one `forecast` per series.
Outputs are numpy float32 arrays shaped [rows, horizon, n_quantiles].
Invalid arguments raise T0bError (the reference panics / returns anyhow
errors at the same places: horizon > 1024 lib.rs:58-62, malformed GGUF
gguf.rs:350-399).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import KernelStats, ModelInfo, T0bError, check, lib, ptr

DEFAULT_BATCH_CHUNK = 16  # lib.rs:32
MAX_HORIZON = 1024  # model.rs:26


class Engine:
    """A CUDA device context (replaces the wgpu `Engine`)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().t0b_engine_create(int(device), C.byref(h)))
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            try:
                lib().t0b_engine_destroy(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def __del__(self):
        self.close()


class GpuModel:
    """GGUF-resident model: Q8_0/Q4_0 blocks stay in llama.cpp layout on the device."""

    def __init__(self, engine: Engine, gguf_bytes: bytes):
        buf = np.frombuffer(gguf_bytes, np.uint8)
        h = C.c_void_p()
        check(lib().t0b_model_load_gguf(engine.handle, ptr(buf), buf.size, C.byref(h)))
        self._h = h
        self.engine = engine
        info = ModelInfo()
        check(lib().t0b_model_info_get(h, C.byref(info)))
        self.info = info
        self.n_quantiles = info.n_quantiles
        self.quantile_levels = [info.quantile_levels[i] for i in range(info.n_quantiles)]

    @property
    def handle(self):
        return self._h

    def quantizable_gpu_bytes(self) -> int:
        return int(self.info.quantizable_gpu_bytes)

    def total_weight_bytes(self) -> int:
        return int(self.info.total_weight_bytes)

    def set_stream(self, stream_ptr: int) -> None:
        check(lib().t0b_model_set_stream(self._h, C.c_void_p(stream_ptr)))

    def stream(self) -> int:
        return int(lib().t0b_model_stream(self._h) or 0)

    def set_max_tokens(self, n: int) -> None:
        check(lib().t0b_model_set_max_tokens(self._h, int(n)))

    def use_graphs(self, on: bool = True) -> None:
        """Replay forecast passes from cached CUDA graphs (default on)."""
        check(lib().t0b_model_use_graphs(self._h, int(on)))

    def sync(self) -> None:
        check(lib().t0b_model_sync(self._h))

    def profile(self, on: bool = True) -> None:
        """Bracket every kernel launch with CUDA events (resets statistics)."""
        check(lib().t0b_model_profile_enable(self._h, int(on)))

    def profile_read(self) -> dict[str, dict]:
        arr = (KernelStats * 8)()
        n = C.c_int(0)
        check(lib().t0b_model_profile_read(self._h, arr, 8, C.byref(n)))
        return {arr[i].name.decode(): dict(launches=int(arr[i].launches), total_ms=arr[i].total_ms,
                                           flops=arr[i].flops, bytes=arr[i].bytes) for i in range(n.value)}

    def launch_count(self) -> int:
        return int(lib().t0b_model_launch_count(self._h))

    def close(self):
        if getattr(self, "_h", None):
            try:
                lib().t0b_model_destroy(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def __del__(self):
        self.close()


def load_model_from_gguf(engine: Engine, gguf_bytes: bytes) -> GpuModel:
    return GpuModel(engine, gguf_bytes)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def forecast(engine: Engine, model: GpuModel, context, v: int, t_ctx: int, horizon: int) -> np.ndarray:
    """One (joint, possibly multivariate) series of v rows x t_ctx values."""
    ctx = _f32(context).reshape(-1)
    if ctx.size != v * t_ctx:
        raise T0bError(1, f"forecast: context has {ctx.size} values, expected v*t_ctx = {v * t_ctx}")
    out = np.empty((v, horizon, model.n_quantiles), np.float32)
    check(lib().t0b_forecast(model.handle, ptr(ctx), v, t_ctx, horizon, ptr(out)))
    return out


def forecast_rollout(engine: Engine, model: GpuModel, context, t_ctx: int, prediction_length: int,
                     query_quantile_levels) -> np.ndarray:
    """One univariate series, any horizon: [prediction_length, len(levels)]
    (t_ctx values of context; levels ascending inside (0, 1))."""
    ctx = _f32(context).reshape(-1)
    if ctx.size != t_ctx:
        raise T0bError(1, f"forecast_rollout: context has {ctx.size} values, expected t_ctx = {t_ctx}")
    q = _f32(query_quantile_levels).reshape(-1)
    out = np.empty((prediction_length, q.size), np.float32)
    check(lib().t0b_forecast_rollout(model.handle, ptr(ctx), t_ctx, prediction_length, ptr(q), q.size, ptr(out)))
    return out


def forecast_batch_chunked(engine: Engine, model: GpuModel, contexts, n_signals: int, t_ctx: int, horizon: int,
                           chunk_size: int = DEFAULT_BATCH_CHUNK) -> np.ndarray:
    """n_signals independent univariate series, [n_signals, t_ctx]."""
    ctx = _f32(contexts).reshape(-1)
    if ctx.size != n_signals * t_ctx:
        raise T0bError(1, "forecast_batch: contexts.len() must equal n_signals * t_ctx")
    out = np.empty((n_signals, horizon, model.n_quantiles), np.float32)
    check(lib().t0b_forecast_batch(model.handle, ptr(ctx), n_signals, t_ctx, horizon, chunk_size, ptr(out)))
    return out


def forecast_batch_rows_chunked(engine: Engine, model: GpuModel, contexts, lengths, horizon: int,
                                chunk_size: int = DEFAULT_BATCH_CHUNK) -> np.ndarray:
    """Ragged univariate rows concatenated in `contexts` per `lengths`."""
    ctx = _f32(contexts).reshape(-1)
    ln = np.ascontiguousarray(lengths, dtype=np.uint64)
    if int(ln.sum()) != ctx.size:
        raise T0bError(1, "forecast_batch_rows: contexts.len() must equal sum(lengths)")
    out = np.empty((ln.size, horizon, model.n_quantiles), np.float32)
    check(lib().t0b_forecast_batch_rows(model.handle, ptr(ctx), ptr(ln), ln.size, horizon, chunk_size, ptr(out)))
    return out


def forecast_multiseries(engine: Engine, model: GpuModel, contexts, n_variates, t_ctx: int,
                         horizon: int) -> np.ndarray:
    """Independent multivariate series; series i owns n_variates[i] consecutive rows."""
    ctx = _f32(contexts).reshape(-1)
    nv = np.ascontiguousarray(n_variates, dtype=np.int32)
    rows = int(nv.sum())
    if ctx.size != rows * t_ctx:
        raise T0bError(1, "forecast_multiseries: contexts must hold sum(n_variates) * t_ctx values")
    out = np.empty((rows, horizon, model.n_quantiles), np.float32)
    check(lib().t0b_forecast_multiseries(model.handle, ptr(ctx), ptr(nv), nv.size, t_ctx, horizon, ptr(out)))
    return out


def forecast_multiseries_device(model: GpuModel, ctx_dev, n_variates, t_ctx: int, horizon: int, out_dev) -> None:
    """Device-pointer variant (torch CUDA tensors or raw pointers), asynchronous
    on the model's stream."""
    nv = np.ascontiguousarray(n_variates, dtype=np.int32)
    check(lib().t0b_forecast_multiseries_device(model.handle, ptr(ctx_dev), ptr(nv), nv.size, t_ctx, horizon,
                                                ptr(out_dev)))
