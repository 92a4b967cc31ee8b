"""Pins the CPU oracle (oracle/t0_oracle.c) to the reference's own known
answers, before anything is checked against it.

Sources of the pinned facts (t0-web, by file:line):
* crates/t0-core/src/gguf.rs:415-433   Q8_0 / Q4_0 round-trip bounds on sin(0.37 i) * 3
* crates/t0-core/src/gguf.rs:100-174   quantizer arithmetic (restated below in numpy)
* crates/t0-fast/src/quant.rs:161-185  word-packed unpack == dequantize_q8_0 exactly
* crates/t0-core/tests/ops_tests.rs:11-72  rmsnorm / RoPE / xpos known answers
* crates/t0-core/src/scaler.rs:44-118  causal Welford scaler (hand-computed case)
* crates/t0-fast/src/model.rs:825-897  hashed-LCG kernel recipe, abs tol 1e-5
* half 2.7.1 (Cargo.lock) f32 -> f16 round-to-nearest-even, pinned against numpy
* tests/golden/quant_blocks.npz: Q8_0 / Q4_0 bytes written by the `gguf`
  Python package (llama.cpp's reference quantizers), see tests/golden/make_golden.py
"""
import os

import numpy as np
import pytest

import oracle as O
from t0_web_b200 import synthetic as S

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sample(n):  # gguf.rs:410-412
    return (np.sin(np.arange(n, dtype=np.float32) * np.float32(0.37)) * np.float32(3.0)).astype(np.float32)


# ---------------------------------------------------------------- quantizers
def test_q8_0_round_trip_bound():
    x = _sample(320)
    y = O.dequantize(O.quantize(x, O.Q8_0), x.size, O.Q8_0)
    assert np.max(np.abs(x - y)) < 0.03


def test_q4_0_round_trip_bound():
    x = _sample(320)
    y = O.dequantize(O.quantize(x, O.Q4_0), x.size, O.Q4_0)
    assert np.max(np.abs(x - y)) < 0.4


def _np_q8_0(x):
    """gguf.rs:100-115 restated in numpy: d = amax/127, q = round-half-away(x * (1/d))."""
    b = x.reshape(-1, 32).astype(np.float32)
    d = (np.max(np.abs(b), axis=1) / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (b * inv[:, None]).astype(np.float32)
    q = np.clip(np.sign(v) * np.floor(np.abs(v) + np.float32(0.5)), -128, 127).astype(np.int8)
    out = np.zeros((b.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.ravel()


def _np_q4_0(x):
    """gguf.rs:133-157: max = signed value of largest |x| (first wins), d = max/-8,
    nibble = clamp(floor(x * (1/d) + 8.5), 0, 15); byte j = lo(x_j) | hi(x_{j+16}) << 4."""
    b = x.reshape(-1, 32).astype(np.float32)
    idx = np.argmax(np.abs(b), axis=1)  # first occurrence of the largest magnitude
    mx = b[np.arange(b.shape[0]), idx]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    n = np.clip(np.floor((b * inv[:, None]).astype(np.float32) + np.float32(8.5)), 0, 15).astype(np.uint8)
    out = np.zeros((b.shape[0], 18), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = n[:, :16] | (n[:, 16:] << 4)
    return out.ravel()


def _quant_inputs():
    rng = np.random.default_rng(3)
    parts = [
        _sample(320),
        rng.standard_normal(32 * 64).astype(np.float32) * np.float32(0.02),
        rng.standard_normal(32 * 16).astype(np.float32) * np.float32(1e4),
        np.zeros(32, np.float32),                                    # d == 0 block
        np.full(32, 1.0, np.float32),
        np.concatenate([np.full(16, 2.0, np.float32), np.full(16, -2.0, np.float32)]),  # magnitude tie
        (np.arange(32, dtype=np.float32) - 16.0) * np.float32(1e-6),  # tiny scales (f16 subnormal d)
        (np.arange(32, dtype=np.float32) - 16.0) * np.float32(0.5) / np.float32(127.0) * np.float32(127.0),
    ]
    return np.concatenate(parts).astype(np.float32)


@pytest.mark.parametrize("qtype,ref", [(O.Q8_0, _np_q8_0), (O.Q4_0, _np_q4_0)], ids=["q8_0", "q4_0"])
def test_quantizer_matches_numpy_restatement(qtype, ref):
    x = _quant_inputs()
    assert np.array_equal(O.quantize(x, qtype), ref(x))


@pytest.mark.parametrize("qtype", [O.Q8_0, O.Q4_0], ids=["q8_0", "q4_0"])
def test_quantizer_matches_golden_blocks(qtype):
    """Bytes pinned by llama.cpp's Python quantizers (the `gguf` package)."""
    g = np.load(os.path.join(GOLDEN, "quant_blocks.npz"))
    key = "q8_0" if qtype == O.Q8_0 else "q4_0"
    x = g["x"]
    assert np.array_equal(O.quantize(x, qtype), g[key])
    assert np.array_equal(O.dequantize(g[key], x.size, qtype), g[key + "_deq"])


def test_q8_word_unpack_is_exact():
    """quant.rs:161-185: u32-word unpack with sign extension == dequantize_q8_0."""
    n = 64
    data = ((np.arange(n, dtype=np.float32) - np.float32(32.0)) * np.float32(0.37)).astype(np.float32)
    b = O.quantize(data, O.Q8_0).reshape(-1, 34)
    deq = O.dequantize(b.ravel(), n, O.Q8_0)
    scales = b[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    words = b[:, 2:].copy().view(np.uint32).ravel()
    out = np.empty(n, np.float32)
    for col in range(n):
        blk, j = divmod(col, 32)
        byte = (int(words[blk * 8 + j // 4]) >> ((j % 4) * 8)) & 0xFF
        sv = byte - 256 if byte >= 128 else byte
        out[col] = np.float32(sv) * scales[blk]
    assert np.max(np.abs(deq - out)) == 0.0


def test_device_int_to_f16_conversions_are_exact():
    """The GPU kernels turn Q8_0 bytes / Q4_0 nibbles into f16 by placing them in
    the mantissa of 1024 (f16 bits 0x6400 | u) and subtracting a bias:
    int8 b -> (1024 + (b ^ 0x80)) - 1152, nibble n -> (1024 + n) - 1032.
    Exhaustive check that both are exact in f16 arithmetic."""
    b = np.arange(256, dtype=np.uint16)
    as_int8 = b.astype(np.uint8).view(np.int8).astype(np.float32)
    h = (np.uint16(0x6400) | (b ^ np.uint16(0x80))).view(np.float16)
    got = (h - np.float16(1152.0)).astype(np.float16)
    assert np.array_equal(got.astype(np.float32), as_int8)
    n = np.arange(16, dtype=np.uint16)
    hn = (np.uint16(0x6400) | n).view(np.float16)
    assert np.array_equal((hn - np.float16(1032.0)).astype(np.float32), n.astype(np.float32) - 8.0)


def test_f16_conversion_matches_numpy_rne():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * (10.0 ** rng.uniform(-9, 5, 4000)).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 2.99e-8, 6.1e-5,
                  np.inf, -np.inf], np.float32),
    ])
    with np.errstate(over="ignore"):
        assert np.array_equal(O.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))


# -------------------------------------------------------------- ops_tests.rs
def test_rmsnorm_hand_computation():
    out = O.rmsnorm(np.array([[3.0, 4.0]], np.float32), np.ones(2, np.float32))
    denom = np.sqrt(12.5)
    assert np.allclose(out[0], [3.0 / denom, 4.0 / denom], atol=1e-5, rtol=0)


def test_rmsnorm_applies_scale_exactly():
    g = np.array([2.0, 0.5, -1.0, 3.0], np.float32)
    out = O.rmsnorm(np.ones((1, 4), np.float32), g)
    assert np.array_equal(out[0], g)


def test_rope_seq1_is_identity():
    cos, sin, sc = O.rope_tables(1, 4)
    assert np.array_equal(cos.ravel(), np.ones(4, np.float32))
    assert np.array_equal(sin.ravel(), np.zeros(4, np.float32))
    assert np.all(np.abs(sc - 1.0) < 1e-6)


def test_xpos_scale_is_halves_concat():
    _, _, sc = O.rope_tables(3, 4)
    row = sc[2]
    assert abs(row[0] - row[2]) < 1e-9 and abs(row[1] - row[3]) < 1e-9
    assert row[0] != row[1]


def test_rope_cos_sin_interleaved():
    """ops.rs:78-115: cos/sin duplicated as f0,f0,f1,f1,..."""
    cos, sin, _ = O.rope_tables(5, 8)
    assert np.array_equal(cos[:, 0::2], cos[:, 1::2]) and np.array_equal(sin[:, 0::2], sin[:, 1::2])
    inv = 10000.0 ** (-np.arange(0, 8, 2) / 8.0)
    ang = np.arange(5)[:, None] * inv[None, :]
    assert np.allclose(cos[:, 0::2], np.cos(ang).astype(np.float32), atol=1e-7)


# ---------------------------------------------------------------- scaler.rs
def test_causal_scaler_hand_computation():
    cfg = dict(S.ALPHA)
    x = np.array([[1.0, 2.0, 3.0, np.nan, 5.0, 0.0]], np.float32)
    mask = np.array([[0, 0, 0, 2, 0, 1]], np.int8)          # missing at 3, pad at 5
    gid = np.array([[0, 0, 0, 0, 0, -1]], np.int64)
    scaled, loc, sc = O.scale_input(cfg, np.nan_to_num(x), mask, gid)
    # Welford over valid steps [1, 2, 3, (skip), 5]
    exp_loc = [1.0, 1.5, 2.0, 2.0, 2.75, 0.0]
    var = [0.0, 0.5, 1.0, 1.0, np.var([1, 2, 3, 5], ddof=1), None]
    exp_sc = [np.sqrt(v + 0.1) for v in var[:5]] + [1.0]
    assert np.allclose(loc[0], exp_loc, atol=1e-6)
    assert np.allclose(sc[0], exp_sc, atol=1e-6)
    xs = np.nan_to_num(x[0])
    assert np.allclose(scaled[0], np.arcsinh((xs - loc[0]) / sc[0]), atol=1e-6)


# ------------------------------------------------------ t0-fast kernel recipe
@pytest.mark.parametrize("qtype", [O.Q8_0, O.Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("m", [1, 40])
def test_lcg_kernel_recipe(qtype, m):
    """model.rs:825-897: N=4, K=512, hashed-LCG inputs, vs a dequant-and-dot
    f32 reference, abs tol 1e-5."""
    n, k = 4, 512
    w, x = S.lcg_kernel_case(n, k, m)
    wb = O.quantize(w, qtype)
    wd = O.dequantize(wb, n * k, qtype).reshape(n, k)
    ref = np.array([[np.float32(np.dot(x[i].astype(np.float32), wd[j])) for j in range(n)] for i in range(m)])
    got = O.gemm_q_f64(qtype, wb, n, k, x)
    assert np.max(np.abs(got - ref)) < 1e-5


# ------------------------------------------------------------ quantile.rs
def _np_interpolate(query, levels, values):
    """quantile.rs:17-43 restated in numpy float32 (stable sort, flat ends)."""
    levels = np.asarray(levels, np.float32)
    values = np.asarray(values, np.float32)
    idx = np.argsort(levels, kind="stable")
    lv, vv = list(levels[idx]), list(values[idx])
    if lv[0] > 0:
        lv.insert(0, np.float32(0.0))
        vv.insert(0, vv[0])
    if lv[-1] < 1:
        lv.append(np.float32(1.0))
        vv.append(vv[-1])
    lv, vv = np.array(lv, np.float32), np.array(vv, np.float32)
    out = []
    for q in np.asarray(query, np.float32):
        upper = min(int(np.searchsorted(lv, q, side="right")), len(lv) - 1)
        lower = max(upper - 1, 0)
        diff = np.float32(lv[upper] - lv[lower])
        w = np.float32(0.0) if diff == 0 else np.float32(np.float32(q - lv[lower]) / diff)
        out.append(np.float32(vv[lower] + np.float32(w * np.float32(vv[upper] - vv[lower]))))
    return np.array(out, np.float32)


def _np_weighted(query, weights, samples):
    """quantile.rs:47-61: running f32 sums in the reference's order."""
    w = np.asarray(weights, np.float32)
    s = np.asarray(samples, np.float32)
    total = np.float32(0.0)
    for x in w:
        total = np.float32(total + x)
    idx = np.argsort(s, kind="stable")
    cum, cw = np.float32(0.0), []
    for i in idx:
        cum = np.float32(cum + np.float32(w[i] / total))
        cw.append(np.float32(min(max(cum, 0.0), 1.0)))
    return _np_interpolate(query, cw, s[idx])


def test_quantile_reference_known_answers():
    """quantile.rs:82-97: identity at the trained levels; probability mass sums to 1."""
    lv = [0.1, 0.25, 0.5, 0.75, 0.9]
    assert np.max(np.abs(O.interpolate_quantiles(lv, lv, [1, 2, 3, 4, 5]) - np.arange(1, 6))) < 1e-6
    assert abs(float(O.prob_mass(lv).sum()) - 1.0) < 1e-6


def test_prob_mass_hand_computed():
    """Trapezoid masses (b[i+2] - b[i]) / 2 over [0, levels, 1], normalised."""
    m = O.prob_mass([0.1, 0.25, 0.5, 0.75, 0.9])
    raw = np.array([0.125, 0.2, 0.25, 0.2, 0.125])
    assert np.allclose(m, raw / raw.sum(), atol=1e-7)


@pytest.mark.parametrize("seed", range(5))
def test_quantile_utilities_match_numpy_restatement(seed):
    rng = np.random.default_rng(seed)
    trained = np.array([0.1, 0.25, 0.5, 0.75, 0.9], np.float32)
    query = np.sort(rng.uniform(0.01, 0.99, 9)).astype(np.float32)
    values = np.sort(rng.standard_normal(5)).astype(np.float32) * np.float32(50)
    assert np.array_equal(O.interpolate_quantiles(query, trained, values), _np_interpolate(query, trained, values))
    w = rng.uniform(0.01, 1.0, 25).astype(np.float32)
    s = rng.standard_normal(25).astype(np.float32)
    s[3] = s[7]  # a tie keeps the stable order
    assert np.array_equal(O.weighted_quantile(query, w, s), _np_weighted(query, w, s))
