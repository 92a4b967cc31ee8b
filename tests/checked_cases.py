"""Runs a fixed set of odd-shaped GEMMs and forecasts through one build of the
library and saves every output, for tests/test_gpu_checked.py.

    python tests/checked_cases.py {product|checked} OUT.npz

`checked` loads libt0b_checked.so (built with -DT0B_CHECKED: every device
index check compiled in, a failed one recorded as T0B_DEVERR_BOUNDS in the
error word and the access skipped).  Each call's status is checked, so an
index check that fails surfaces here as a T0bError (T0B_ERR_DEVICE) and a
non-zero exit.  Outputs are NaN-poisoned before each call: a tile that a
kernel skipped stays NaN.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import t0_web_b200._lib as L  # noqa: E402

if sys.argv[1] == "checked":
    L.LIB_PATH = os.path.join(os.path.dirname(L.LIB_PATH), "libt0b_checked.so")

import torch  # noqa: E402

from t0_web_b200 import gguf, synthetic as S, t0_fast  # noqa: E402
from t0_web_b200._lib import Q4_0, Q8_0, check, lib, ptr  # noqa: E402

# (M, N, K): both GEMM paths (small-M below 128 tokens, tcgen05 above), M off
# every tile boundary, N and K odd multiples of 256
GEMM_SHAPES = [(1, 256, 256), (3, 768, 256), (31, 256, 768), (33, 512, 512), (129, 256, 256), (255, 512, 768),
               (257, 256, 512), (300, 768, 256)]
SWIGLU_M = [3, 33, 200]


def main() -> None:
    out = {}
    eng = t0_fast.Engine(0)
    dev = torch.device("cuda:0")
    for qname, qt in (("q8_0", Q8_0), ("q4_0", Q4_0)):
        for M, N, K in GEMM_SHAPES:
            w, x = S.gemm_case(N, K, M, seed=M + N + K)
            wd = torch.from_numpy(gguf.quantize(w, qt).copy()).to(dev)
            xd = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
            yd = torch.full((M, N), float("nan"), device=dev)
            torch.cuda.synchronize()
            check(lib().t0b_gemm_q(eng.handle, qt, ptr(wd), N, K, ptr(xd), M, None, ptr(yd), None))
            out[f"gemm_{qname}_{M}_{N}_{K}"] = yd.cpu().numpy()
        F, K, N2 = 512, 256, 256
        w0, _ = S.gemm_case(2 * F, K, 1, seed=1)
        w2, _ = S.gemm_case(N2, F, 1, seed=2)
        w0d = torch.from_numpy(gguf.quantize(w0, qt).copy()).to(dev)
        w2d = torch.from_numpy(gguf.quantize(w2, qt).copy()).to(dev)
        for M in SWIGLU_M:
            x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
            xd = torch.from_numpy(x).to(dev)
            zd = torch.full((M, F), float("nan"), device=dev)
            yd = torch.full((M, N2), float("nan"), device=dev)
            torch.cuda.synchronize()
            check(lib().t0b_swiglu_q(eng.handle, qt, ptr(w0d), ptr(w2d), F, K, N2, ptr(xd), M, None, None, ptr(zd),
                                     ptr(yd), None))
            out[f"swiglu_z_{qname}_{M}"] = zd.cpu().numpy()
            out[f"swiglu_y_{qname}_{M}"] = yd.cpu().numpy()
    # forecasts of the TINY model family member (3 layers: TIME, TIME, GROUP):
    # one patch + one horizon step, a single series, ragged rows with a NaN
    # gap, and a multivariate batch on the tensor-core path
    g = gguf.export_gguf(S.random_weights(S.TINY, seed=3), S.TINY, "q8_0")
    m = t0_fast.load_model_from_gguf(eng, g)
    out["fc_tiny"] = t0_fast.forecast(eng, m, S.sine_context(37, seed=1), 1, 37, 1)
    out["fc_single"] = t0_fast.forecast(eng, m, S.sine_context(512, seed=2), 1, 512, 96)
    rng = np.random.default_rng(5)
    lengths = [100, 512, 37, 250, 64]
    rows = [rng.standard_normal(n).astype(np.float32).cumsum() * 0.1 for n in lengths]
    rows[2][5:9] = np.nan
    out["fc_rows"] = t0_fast.forecast_batch_rows_chunked(eng, m, np.concatenate(rows), lengths, 40, chunk_size=3)
    ctx, nv = S.multiseries(6, 1024, seed=2, n_variates=3)
    out["fc_multi"] = t0_fast.forecast_multiseries(eng, m, ctx, nv, 1024, 96)
    m.sync()
    np.savez(sys.argv[2], **out)


if __name__ == "__main__":
    main()
