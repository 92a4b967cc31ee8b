"""Regenerates the committed golden fixtures of this directory.

quant_blocks.npz   Q8_0 / Q4_0 bytes (and their dequantization) written by
                   the `gguf` Python package 0.19.0 (llama.cpp's reference
                   quantizers, gguf/quants.py), the layout the GGUF files of
                   t0-web carry (t0-core gguf.rs:100-174 produces the same
                   bytes).  Inputs: the reference's own test signal
                   sin(0.37 i) * 3 (gguf.rs:410-412), the quant.rs:166-169
                   ramp, seeded normals at three scales and edge blocks.
reference_contexts.npz
                   The input contexts of t0-web's own end-to-end fixtures
                   (fixtures/manifest.json, fixtures/manifest_long.json, made
                   by tools/make_fixtures.py:124-176): case0_univariate_sine,
                   case1_trivariate_freqs, case2_masked_gap (NaN steps
                   [200, 220)) and case_long_rollout (ctx 4096, horizon
                   1200), with their variate counts and horizons.  Only the
                   contexts are taken: the fixtures' quantiles come from the
                   trained checkpoint, which random-init weights cannot
                   reproduce.  Needs a t0-web checkout:
                   --reference <path to the t0-web repository>.
tiny_forecast.npz  End-to-end quantiles of the CPU oracle for the TINY
                   random-init model (seed 0), Q8_0 and Q4_0: one sine
                   context (ctx 77, horizon 30) and three multivariate series
                   (ctx 96, horizon 40).  A regression pin for the oracle and
                   a fixed target for the GPU tests.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def quant_inputs() -> np.ndarray:
    rng = np.random.default_rng(11)
    parts = [
        (np.sin(np.arange(320, dtype=np.float32) * np.float32(0.37)) * np.float32(3.0)),
        ((np.arange(64, dtype=np.float32) - np.float32(32.0)) * np.float32(0.37)),
        rng.standard_normal(32 * 32).astype(np.float32) * np.float32(0.02),
        rng.standard_normal(32 * 16).astype(np.float32),
        rng.standard_normal(32 * 8).astype(np.float32) * np.float32(300.0),
        np.zeros(32, np.float32),
        np.concatenate([np.full(16, 2.0, np.float32), np.full(16, -2.0, np.float32)]),
        (np.arange(32, dtype=np.float32) - np.float32(16.0)) * np.float32(1e-6),
    ]
    return np.concatenate(parts).astype(np.float32)


def make_quant_blocks():
    from gguf import GGMLQuantizationType as GT, quants
    x = quant_inputs()
    out = {"x": x}
    for key, gt in (("q8_0", GT.Q8_0), ("q4_0", GT.Q4_0)):
        b = quants.quantize(x.reshape(-1, 32), gt)
        out[key] = np.ascontiguousarray(b).view(np.uint8).ravel()
        out[key + "_deq"] = quants.dequantize(b, gt).astype(np.float32).ravel()
    np.savez_compressed(os.path.join(HERE, "quant_blocks.npz"), **out)


def make_tiny_forecast():
    import oracle as O
    from t0_web_b200 import synthetic as S
    w = S.random_weights(S.TINY, seed=0)
    out = {}
    for quant in ("q8_0", "q4_0"):
        m = O.OracleModel(O.export_gguf(w, S.TINY, quant))
        ctx = S.sine_context(77, seed=0)
        out[quant + "_sine"] = m.forecast(ctx, 30)
        ms, nv = S.multiseries(3, 96, seed=5, n_variates=(1, 3))
        out[quant + "_multi"] = m.forecast_multiseries(ms, nv, 40)
    out["sine_ctx"] = S.sine_context(77, seed=0)
    out["multi_ctx"], out["multi_nv"] = S.multiseries(3, 96, seed=5, n_variates=(1, 3))
    np.savez_compressed(os.path.join(HERE, "tiny_forecast.npz"), **out)


def make_reference_contexts(ref_root: str):
    import json
    fx = os.path.join(ref_root, "fixtures")
    out = {}
    names = []
    for man in ("manifest.json", "manifest_long.json"):
        m = json.load(open(os.path.join(fx, man)))
        for c in m["cases"]:
            ctx = np.fromfile(os.path.join(fx, c["context_file"]), dtype="<f4")
            v, t = int(c["v"]), int(c["context_len"])
            assert ctx.size == v * t, (c["name"], ctx.size, v, t)
            out[c["name"] + "_ctx"] = ctx.reshape(v, t).astype(np.float32)
            out[c["name"] + "_horizon"] = np.int64(c["horizon"])
            names.append(c["name"])
    out["names"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "reference_contexts.npz"), **out)


if __name__ == "__main__":
    if "--reference" in sys.argv:
        make_reference_contexts(sys.argv[sys.argv.index("--reference") + 1])
    else:
        make_quant_blocks()
        make_tiny_forecast()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
