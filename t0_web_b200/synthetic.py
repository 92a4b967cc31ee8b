"""Seeded synthetic inputs for the t0-alpha quantized forecast path.

No t0-alpha checkpoint and no benchmark dataset exist on these machines, so
every workload is synthetic:

* weights: random-init tensors with t0-alpha's 303 names and shapes
  (t0-core `model.rs:84-147` names; `docs/reports/t0-alpha-anatomy.md`
  shapes): linear weights, biases and type embeddings ~ N(0, 0.02), norm
  gains 1.0, `head.quantile_levels` = the trained levels.  They are exported
  to GGUF exactly like `t0-cli export-gguf` (weights.rs:187-227), so every
  non-quantized tensor goes through f16.
* contexts: the configurations of the benchmark description (a sine with
  period 24 plus 0.1 N(0,1) noise for the single forecast; sums of 2-3
  sinusoids + trend + N(0, 0.2) with a 5% NaN gap for the multi-series
  forecasts).
"""
from __future__ import annotations

import numpy as np

# t0-alpha config.json (loader.rs:29-41; config.rs serde defaults 24-32)
ALPHA = dict(
    embed_dim=512,
    num_layers=24,
    num_heads=8,
    mlp_hidden_dim=2048,
    patch_size=32,
    group_every_n=3,
    dropout=0.1,
    quantile_levels=[0.1, 0.25, 0.5, 0.75, 0.9],
    scaler_use_arcsinh=True,
    scaler_eps=0.1,
    scaler_eps_mode="variance_offset",
)

# t0-beta's shape (the reference's docs/BENCHMARKS.md:340): embed_dim 1024
# (head_dim 128), 21 quantile levels, `std_clamp` scaler with eps 0.01; the
# other fields as t0-alpha.  The 21 levels are 0.01, 0.05, 0.10, ..., 0.95,
# 0.99 (the documented range; the exact list is this project's choice).
BETA = dict(ALPHA, embed_dim=1024,
            quantile_levels=[0.01] + [round(0.05 * i, 2) for i in range(1, 20)] + [0.99],
            scaler_eps=0.01, scaler_eps_mode="std_clamp")
# a 3-layer (TIME, TIME, GROUP) model of t0-beta's widths, for parity tests
BETA_SMALL = dict(BETA, num_layers=3)

# The smallest model of the same family the engine runs (head_dim 64 or 128,
# embed_dim and mlp_hidden_dim multiples of 256): quick CPU checks and fixtures.
TINY = dict(ALPHA, embed_dim=256, num_layers=3, num_heads=4, mlp_hidden_dim=256)


def tensor_shapes(cfg: dict) -> list[tuple[str, tuple[int, ...]]]:
    """All tensor names and row-major shapes of a t0 model (model.rs:84-147)."""
    E, F, P = cfg["embed_dim"], cfg["mlp_hidden_dim"], cfg["patch_size"]
    hd = E // cfg["num_heads"]
    nq = len(cfg["quantile_levels"])
    out: list[tuple[str, tuple[int, ...]]] = []

    def resblock(prefix, din, dh, dout):
        out.extend([
            (f"{prefix}.mlp.hidden_layer.weight", (dh, din)),
            (f"{prefix}.mlp.hidden_layer.bias", (dh,)),
            (f"{prefix}.mlp.output_layer.weight", (dout, dh)),
            (f"{prefix}.mlp.output_layer.bias", (dout,)),
            (f"{prefix}.residual_layer.weight", (dout, din)),
            (f"{prefix}.residual_layer.bias", (dout,)),
        ])

    resblock("patch_encoder.projection", 3 * P, E, E)
    out.append(("patch_encoder.type_embeddings.weight", (3, E)))
    for i in range(cfg["num_layers"]):
        p = f"transformer.layers.{i}"
        out.extend([
            (f"{p}.attention_block.norm.scale", (E,)),
            (f"{p}.attention_block.attention.wQKV.weight", (3 * E, E)),
            (f"{p}.attention_block.attention.wQKV.bias", (3 * E,)),
            (f"{p}.attention_block.attention.wO.weight", (E, E)),
            (f"{p}.attention_block.attention.wO.bias", (E,)),
            (f"{p}.attention_block.attention.q_norm.scale", (hd,)),
            (f"{p}.attention_block.attention.k_norm.scale", (hd,)),
            (f"{p}.norm.scale", (E,)),
            (f"{p}.mlp.0.weight", (2 * F, E)),
            (f"{p}.mlp.0.bias", (2 * F,)),
            (f"{p}.mlp.2.weight", (E, F)),
            (f"{p}.mlp.2.bias", (E,)),
        ])
    out.append(("transformer.out_norm.scale", (E,)))
    resblock("decoder", E, E, P * nq)
    out.append(("head.quantile_levels", (nq,)))
    return out


def random_weights(cfg: dict = ALPHA, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init f32 weights: N(0, std) everywhere except norm gains (1.0)
    and `head.quantile_levels` (the levels)."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}
    for name, shape in tensor_shapes(cfg):
        if name.endswith(".scale"):
            w[name] = np.ones(shape, np.float32)
        elif name == "head.quantile_levels":
            w[name] = np.asarray(cfg["quantile_levels"], np.float32)
        else:
            w[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return w


def sine_context(t_ctx: int = 512, seed: int = 0, v: int = 1) -> np.ndarray:
    """x_t = sin(2 pi t / 24) + 0.1 N(0,1), shape [v, t_ctx]."""
    rng = np.random.default_rng(seed)
    t = np.arange(t_ctx, dtype=np.float64)
    base = np.sin(2.0 * np.pi * t / 24.0)
    return (base[None, :] + 0.1 * rng.standard_normal((v, t_ctx))).astype(np.float32)


def multiseries(n_series: int, t_ctx: int, seed: int = 0, n_variates: int | tuple[int, int] = 3,
                gap_frac: float = 0.05) -> tuple[np.ndarray, np.ndarray]:
    """Independent multivariate series for the batched configurations.

    Each variate is a sum of 2-3 sinusoids (periods U[7, 168], amplitude
    U[0.5, 2], phase U[0, 2pi]) + a linear trend + N(0, 0.2) noise; every
    series gets one contiguous NaN gap of round(gap_frac * t_ctx) steps at a
    random start (all its variates).  n_variates is a fixed count or an
    inclusive (lo, hi) range drawn uniformly per series.

    Returns (contexts [sum(v_i), t_ctx] f32, n_variates [n_series] int32).
    """
    rng = np.random.default_rng(seed)
    if isinstance(n_variates, tuple):
        nv = rng.integers(n_variates[0], n_variates[1] + 1, size=n_series).astype(np.int32)
    else:
        nv = np.full(n_series, int(n_variates), np.int32)
    rows = int(nv.sum())
    # per-row parameters first, then the values in row chunks (bounded memory)
    k = rng.integers(2, 4, size=(rows, 1))
    period = rng.uniform(7.0, 168.0, size=(3, rows, 1))
    amp = rng.uniform(0.5, 2.0, size=(3, rows, 1)) * (np.arange(3)[:, None, None] < k[None])
    phase = rng.uniform(0.0, 2.0 * np.pi, size=(3, rows, 1))
    slope = rng.uniform(-1.0, 1.0, size=(rows, 1))
    offset = rng.uniform(-1.0, 1.0, size=(rows, 1))
    x = np.empty((rows, t_ctx), np.float32)
    t = np.arange(t_ctx, dtype=np.float64)[None, :]
    for c0 in range(0, rows, 1024):
        c1 = min(rows, c0 + 1024)
        acc = slope[c0:c1] * (t / t_ctx) + offset[c0:c1]
        for j in range(3):
            acc += amp[j, c0:c1] * np.sin((2.0 * np.pi / period[j, c0:c1]) * t + phase[j, c0:c1])
        acc += 0.2 * rng.standard_normal((c1 - c0, t_ctx))
        x[c0:c1] = acc
    gap = int(round(gap_frac * t_ctx))
    if gap > 0:
        r0 = 0
        for s in range(n_series):
            start = int(rng.integers(0, t_ctx - gap + 1))
            x[r0:r0 + nv[s], start:start + gap] = np.nan
            r0 += int(nv[s])
    return x, nv


def gemm_case(N: int, K: int, M: int, seed: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Standalone GEMM inputs: W [N,K] ~ N(0, 0.02), X [M,K] ~ N(0, 1), f32."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    return w, x


def lcg_kernel_case(n: int, k: int, m: int) -> tuple[np.ndarray, np.ndarray]:
    """The hashed-LCG weights / inputs of t0-fast's kernel unit tests
    (crates/t0-fast/src/model.rs:843-848)."""
    i = np.arange(n * k, dtype=np.uint64)
    w = ((((i * np.uint64(2654435761)) % np.uint64(1000)).astype(np.float32) / np.float32(1000.0)
          - np.float32(0.5)) * np.float32(0.6)).astype(np.float32).reshape(n, k)
    j = np.arange(m * k, dtype=np.uint64)
    x = ((((j * np.uint64(40503)) % np.uint64(1000)).astype(np.float32) / np.float32(1000.0)
          - np.float32(0.5)) * np.float32(0.4)).astype(np.float32).reshape(m, k)
    return w, x
