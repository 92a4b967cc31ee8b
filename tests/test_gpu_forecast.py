"""End-to-end forecast parity on the GPU against the C oracle (t0-core
restatement), on the same GGUF bytes and the same seeded inputs.

Tolerance: quantile outputs within 1e-3 max-abs after
the model's own scaling.  Quantiles of the random-init model reach ~200, so
1e-3 is ~5e-6 relative: f32-class arithmetic is required end to end.
"""
import numpy as np
import pytest

from t0_web_b200 import T0bError, synthetic as S, t0_fast

from conftest import max_abs

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
def test_single_forecast_config1(engine, gpu_model, oracle_model, quant):
    """Configuration 1: univariate sine (period 24) + 0.1 N(0,1), ctx 512, h 96."""
    ctx = S.sine_context(512, seed=0)
    got = t0_fast.forecast(engine, gpu_model(quant), ctx, 1, 512, 96)
    ref = oracle_model(quant).forecast(ctx, 96)
    assert got.shape == (1, 96, 5)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_multivariate_joint(engine, gpu_model, oracle_model):
    ctx, _ = S.multiseries(1, 512, seed=1, n_variates=3)
    got = t0_fast.forecast(engine, gpu_model("q8_0"), ctx, 3, 512, 96)
    ref = oracle_model("q8_0").forecast(ctx, 96)
    assert max_abs(got, ref) <= TOL


def test_batch_chunked(engine, gpu_model, oracle_model):
    ctx = np.concatenate([S.sine_context(300, seed=s) for s in range(5)])
    got = t0_fast.forecast_batch_chunked(engine, gpu_model("q8_0"), ctx, 5, 300, 64, chunk_size=2)
    ref = oracle_model("q8_0").forecast_batch(ctx, 64, chunk=2)
    assert max_abs(got, ref) <= TOL


def test_batch_rows_ragged(engine, gpu_model, oracle_model):
    rng = np.random.default_rng(5)
    lengths = [100, 512, 37, 250, 64]
    rows = [rng.standard_normal(n).astype(np.float32).cumsum() * 0.1 for n in lengths]
    rows[2][5:9] = np.nan
    got = t0_fast.forecast_batch_rows_chunked(engine, gpu_model("q8_0"), np.concatenate(rows), lengths, 40,
                                              chunk_size=3)
    ref = oracle_model("q8_0").forecast_batch_rows(rows, 40, chunk=3)
    assert max_abs(got, ref) <= TOL


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
def test_multiseries_gaps_tensor_core_path(engine, gpu_model, oracle_model, quant):
    """Configuration-4 style series (2-3 sinusoids + trend + noise, 5% NaN gap),
    enough tokens (6 x 3 x 67 = 1206) for the tcgen05 GEMM path."""
    ctx, nv = S.multiseries(6, 2048, seed=2, n_variates=3)
    got = t0_fast.forecast_multiseries(engine, gpu_model(quant), ctx, nv, 2048, 96)
    ref = oracle_model(quant).forecast_multiseries(ctx, nv, 96, threads=8)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_multiseries_ragged_variates(engine, gpu_model, oracle_model):
    ctx, nv = S.multiseries(9, 512, seed=3, n_variates=(1, 8))
    got = t0_fast.forecast_multiseries(engine, gpu_model("q8_0"), ctx, nv, 512, 96)
    ref = oracle_model("q8_0").forecast_multiseries(ctx, nv, 96, threads=8)
    assert max_abs(got, ref) <= TOL


@pytest.mark.parametrize("t_ctx", [4000, 4096, 7000])
def test_long_context(engine, gpu_model, oracle_model, t_ctx):
    """p = 128, 131 and 222 patches per row: the tensor-core time attention
    beyond 8 query blocks (the context lengths of the box-wide sweep's 4096
    case and beyond)."""
    ctx, nv = S.multiseries(2, t_ctx, seed=7, n_variates=2)
    got = t0_fast.forecast_multiseries(engine, gpu_model("q8_0"), ctx, nv, t_ctx, 96)
    ref = oracle_model("q8_0").forecast_multiseries(ctx, nv, 96, threads=8)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_unaligned_context_and_horizon(engine, gpu_model, oracle_model):
    ctx = S.sine_context(77, seed=9)
    got = t0_fast.forecast(engine, gpu_model("q8_0"), ctx, 1, 77, 30)
    ref = oracle_model("q8_0").forecast(ctx, 30)
    assert got.shape == (1, 30, 5)
    assert max_abs(got, ref) <= TOL


def test_all_missing_row(engine, gpu_model, oracle_model):
    ctx, _ = S.multiseries(1, 256, seed=4, n_variates=2)
    ctx[1, :] = np.nan
    got = t0_fast.forecast(engine, gpu_model("q8_0"), ctx, 2, 256, 32)
    ref = oracle_model("q8_0").forecast(ctx, 32)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_chunking_is_invisible(engine, gpu_model):
    """Passes split by the token budget give the same result as one pass."""
    m = gpu_model("q8_0")
    ctx, nv = S.multiseries(12, 512, seed=6, n_variates=(1, 4))
    one = t0_fast.forecast_multiseries(engine, m, ctx, nv, 512, 96)
    m.set_max_tokens(64)
    try:
        many = t0_fast.forecast_multiseries(engine, m, ctx, nv, 512, 96)
    finally:
        m.set_max_tokens(393216)
    assert max_abs(one, many) <= TOL


def test_graph_replay_matches_eager_launches(engine, gpu_model):
    """Passes replayed from cached CUDA graphs give the eager launches' outputs
    bit for bit.  The two multiseries cases share every shape and buffer but
    not the largest series (8 vs 12 rows), which selects a different
    group-attention kernel, so a replay keyed too coarsely would show here."""
    m = gpu_model("q8_0")
    ctx16, _ = S.multiseries(2, 512, seed=11, n_variates=8)
    cases = [
        lambda: t0_fast.forecast_multiseries(engine, m, ctx16, np.array([8, 8], np.int32), 512, 96),
        lambda: t0_fast.forecast_multiseries(engine, m, ctx16, np.array([4, 12], np.int32), 512, 96),
        lambda: t0_fast.forecast(engine, m, S.sine_context(512, seed=0), 1, 512, 96),
        lambda: t0_fast.forecast_multiseries(engine, m, *S.multiseries(6, 2048, seed=2, n_variates=3), 2048, 96),
    ]
    m.use_graphs(False)
    try:
        eager = [c() for c in cases]
        n0 = m.launch_count()
        for c in cases:
            c()
        eager_launches = m.launch_count() - n0
    finally:
        m.use_graphs(True)
    for rep in range(2):  # capture, then replay
        n0 = m.launch_count()
        for i, c in enumerate(cases):
            got = c()
            assert np.array_equal(got, eager[i]), (rep, i, max_abs(got, eager[i]))
        assert m.launch_count() - n0 == eager_launches


DECILES = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]


@pytest.mark.parametrize("pred,levels", [(100, DECILES), (1100, DECILES), (1300, [0.1, 0.25, 0.5, 0.75, 0.9])],
                         ids=["one_block", "two_blocks_deciles", "two_blocks_trained_levels"])
def test_rollout_vs_oracle(engine, gpu_model, oracle_model, pred, levels):
    """forecast_rollout (t0-fast lib.rs:259-345): horizons beyond one
    forward pass, every query-level path fed back and re-reduced."""
    ctx = S.sine_context(512, seed=0)
    got = t0_fast.forecast_rollout(engine, gpu_model("q8_0"), ctx, 512, pred, levels)
    ref = oracle_model("q8_0").forecast_rollout(ctx, pred, levels)
    assert got.shape == (pred, len(levels))
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_rollout_rejects_unsorted_levels(engine, gpu_model):
    with pytest.raises(T0bError):
        t0_fast.forecast_rollout(engine, gpu_model("q8_0"), S.sine_context(64), 64, 2000, [0.5, 0.1])


def test_horizon_limit_is_an_error(engine, gpu_model):
    with pytest.raises(T0bError):
        t0_fast.forecast(engine, gpu_model("q8_0"), S.sine_context(64), 1, 64, 1025)


def test_model_bytes(gpu_model):
    m = gpu_model("q8_0")
    assert m.quantizable_gpu_bytes() == 106_954_752  # 100,663,296 values x 34/32
    assert gpu_model("q4_0").quantizable_gpu_bytes() == 56_623_104
    assert m.total_weight_bytes() > m.quantizable_gpu_bytes()


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
def test_tiny_model_matches_golden_fixture(engine, quant):
    """The committed oracle outputs of tests/golden/tiny_forecast.npz (made by
    tests/golden/make_golden.py) for the TINY model: no oracle call at run time."""
    import os
    from t0_web_b200 import gguf
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_forecast.npz"))
    m = t0_fast.load_model_from_gguf(engine, gguf.export_gguf(S.random_weights(S.TINY, seed=0), S.TINY, quant))
    try:
        got = t0_fast.forecast(engine, m, g["sine_ctx"], 1, 77, 30)
        assert max_abs(got, g[quant + "_sine"]) <= TOL
        got = t0_fast.forecast_multiseries(engine, m, g["multi_ctx"], g["multi_nv"], 96, 40)
        assert max_abs(got, g[quant + "_multi"]) <= TOL
    finally:
        m.close()


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
def test_config4_full_batch_sampled(engine, gpu_model, oracle_model, quant):
    """The 256-trivariate-series configuration at its full timed size (ctx
    2048, horizon 96, 51,456 tokens per GEMM, one pass): all 256 series are
    forecast together on the GPU and 8 series spread over the batch are
    checked against the oracle."""
    ctx, nv = S.multiseries(256, 2048, seed=0, n_variates=3)
    got = t0_fast.forecast_multiseries(engine, gpu_model(quant), ctx, nv, 2048, 96)
    assert got.shape == (768, 96, 5)
    assert np.isfinite(got).all()
    series = [0, 37, 73, 110, 146, 183, 219, 255]
    rows = np.concatenate([np.arange(3 * s, 3 * s + 3) for s in series])
    ref = oracle_model(quant).forecast_multiseries(ctx[rows], nv[series], 96, threads=8)
    assert max_abs(got[rows], ref) <= TOL


def _reference_contexts():
    import os
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_contexts.npz"))


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
@pytest.mark.parametrize("case", ["case0_univariate_sine", "case1_trivariate_freqs", "case2_masked_gap"])
def test_reference_fixture_contexts(engine, gpu_model, oracle_model, quant, case):
    """t0-web's own end-to-end fixture inputs (fixtures/manifest.json, made by
    tools/make_fixtures.py:124-146; committed as tests/golden/
    reference_contexts.npz): a univariate sine, three variates of different
    frequencies forecast jointly, and a sine with NaN steps [200, 220).  The
    fixtures' quantiles come from the trained checkpoint, which is absent, so
    the GPU is held to the oracle on the same random-init GGUF."""
    g = _reference_contexts()
    ctx = g[case + "_ctx"]
    h = int(g[case + "_horizon"])
    got = t0_fast.forecast(engine, gpu_model(quant), ctx, ctx.shape[0], ctx.shape[1], h)
    ref = oracle_model(quant).forecast(ctx, h)
    assert got.shape == (ctx.shape[0], h, 5)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL


def test_reference_fixture_long_rollout(engine, gpu_model, oracle_model):
    """fixtures/manifest_long.json's case_long_rollout (tools/
    make_fixtures.py:150-176): ctx 4096, horizon 1200, so one 1024-step block
    and one autoregressive block over the trained levels."""
    g = _reference_contexts()
    ctx = g["case_long_rollout_ctx"]
    h = int(g["case_long_rollout_horizon"])
    levels = [0.1, 0.25, 0.5, 0.75, 0.9]
    got = t0_fast.forecast_rollout(engine, gpu_model("q8_0"), ctx[0], ctx.shape[1], h, levels)
    ref = oracle_model("q8_0").forecast_rollout(ctx[0], h, levels)
    assert got.shape == (h, 5)
    assert np.isfinite(got).all()
    assert max_abs(got, ref) <= TOL
