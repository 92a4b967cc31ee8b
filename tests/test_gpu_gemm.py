"""Dequant-GEMM parity on the GPU, through the C ABI (t0b_gemm_q / t0b_swiglu_q).

Oracle: fp64 product of the f32 inputs with the reference dequantization
(gguf.rs:116-174), oracle/t0_oracle.c o_gemm_q_f64.  Bound (BASELINE): per-GEMM
max relative error <= 2e-3, measured as max|y - y_ref| / max|y_ref|; the
kernels are f32-class, so a tighter REL_TIGHT bound is asserted as well.
"""
import numpy as np
import pytest
import torch

import oracle as O
from t0_web_b200 import gguf, synthetic as S
from t0_web_b200._lib import Q4_0, Q8_0, check, lib, ptr

pytestmark = pytest.mark.gpu

REL_BASELINE = 2e-3
REL_TIGHT = 2e-5


def _gemm(engine, qtype, w_bytes, N, K, x, bias=None):
    dev = torch.device("cuda:0")
    wd = torch.from_numpy(w_bytes.copy()).to(dev)
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    bd = None if bias is None else torch.from_numpy(bias).to(dev)
    yd = torch.full((x.shape[0], N), float("nan"), device=dev)  # poisoned: catches unwritten tiles
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q(engine.handle, qtype, ptr(wd), N, K, ptr(xd), x.shape[0], ptr(bd), ptr(yd), None))
    return yd.cpu().numpy()


def _rel(y, ref):
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [1, 3, 16, 19, 31, 33, 64, 100, 128, 129, 256, 333])
def test_gemm_vs_oracle(engine, qtype, M):
    N, K = 512, 1024
    w, x = S.gemm_case(N, K, M, seed=M)
    wb = gguf.quantize(w, qtype)
    bias = (np.random.default_rng(7).standard_normal(N) * 0.02).astype(np.float32)
    y = _gemm(engine, qtype, wb, N, K, x, bias)
    ref = O.gemm_q_f64(qtype, wb, N, K, x, bias)
    assert np.isfinite(y).all()
    rel = _rel(y, ref)
    assert rel <= REL_BASELINE
    assert rel <= REL_TIGHT, rel


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("K", [256, 768, 1536, 4096, 4352])
@pytest.mark.parametrize("M", [5, 19, 77])
def test_small_m_k_slices(engine, qtype, K, M):
    """Small-M K slicing: one CTA over the whole K (256, with the f32 input
    split inside the kernel; 768), a 6-CTA cluster of 256-wide slices (1536),
    eight slices of 512 (4096), and K = 17 x 256, which has no split into at
    most 8 slices and goes to the tensor-core kernel instead."""
    N = 512
    w, x = S.gemm_case(N, K, M, seed=K + M)
    wb = gguf.quantize(w, qtype)
    bias = (np.random.default_rng(K).standard_normal(N) * 0.02).astype(np.float32)
    y = _gemm(engine, qtype, wb, N, K, x, bias)
    ref = O.gemm_q_f64(qtype, wb, N, K, x, bias)
    assert np.isfinite(y).all()
    assert _rel(y, ref) <= REL_TIGHT


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [16, 256, 4096])
def test_gemm_config2_shape(engine, qtype, M):
    """N=3072, K=1024 (the standalone GEMM configuration); rows sampled for large M."""
    N, K = 3072, 1024
    w, x = S.gemm_case(N, K, M, seed=100 + M)
    wb = gguf.quantize(w, qtype)
    y = _gemm(engine, qtype, wb, N, K, x)
    rows = np.arange(M) if M <= 256 else np.random.default_rng(0).choice(M, 64, replace=False)
    ref = O.gemm_q_f64(qtype, wb, N, K, x[rows])
    assert np.isfinite(y).all()
    assert _rel(y[rows], ref) <= REL_TIGHT


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [1, 40, 200])
def test_kernel_recipe_lcg(engine, qtype, M):
    """t0-fast's kernel unit test recipe (crates/t0-fast/src/model.rs:825-870):
    hashed-LCG weights/inputs, K=512, zero bias, abs tol 1e-5 against a
    dequant-and-dot reference.  N is 256 here (the kernels tile N by 64/256)."""
    N, K = 256, 512
    w, x = S.lcg_kernel_case(N, K, M)
    wb = gguf.quantize(w, qtype)
    y = _gemm(engine, qtype, wb, N, K, x, np.zeros(N, np.float32))
    ref = O.gemm_q_f64(qtype, wb, N, K, x)
    assert float(np.max(np.abs(y - ref))) < 1e-5


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [16, 200])
def test_swiglu_vs_oracle(engine, qtype, M):
    """Fused gate/up + SiLU and down projection (the SwiGLU configuration's
    F=4096, K=1024, N2=1024), z and y checked."""
    F, K, N2 = 4096, 1024, 1024
    rng = np.random.default_rng(M)
    w0 = (rng.standard_normal((2 * F, K), dtype=np.float32) * np.float32(0.02))
    w2 = (rng.standard_normal((N2, F), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((M, K), dtype=np.float32)
    b0, b2 = gguf.quantize(w0, qtype), gguf.quantize(w2, qtype)
    dev = torch.device("cuda:0")
    w0d, w2d = torch.from_numpy(b0).to(dev), torch.from_numpy(b2).to(dev)
    xd = torch.from_numpy(x).to(dev)
    zd = torch.full((M, F), float("nan"), device=dev)
    yd = torch.full((M, N2), float("nan"), device=dev)
    torch.cuda.synchronize()
    check(lib().t0b_swiglu_q(engine.handle, qtype, ptr(w0d), ptr(w2d), F, K, N2, ptr(xd), M, None, None, ptr(zd),
                             ptr(yd), None))
    z, y = zd.cpu().numpy(), yd.cpu().numpy()
    rows = np.arange(M) if M <= 16 else np.arange(0, M, 7)
    zr, yr = O.swiglu_q_f64(qtype, b0, F, K, b2, N2, x[rows])
    assert np.isfinite(z).all() and np.isfinite(y).all()
    assert _rel(z[rows], zr) <= REL_TIGHT
    assert _rel(y[rows], yr) <= REL_TIGHT


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [255, 257, 511, 513])
def test_pair_tile_boundaries(engine, qtype, M):
    """The tensor-core GEMM runs on CTA pairs that own 256 tokens each (128
    per CTA): M just below and above one and two pair tiles leaves the second
    CTA of the last pair partly or wholly past M.  Every row is checked, so
    rows written by the wrong CTA or left unwritten (NaN-poisoned) fail."""
    N, K = 512, 512
    w, x = S.gemm_case(N, K, M, seed=1000 + M)
    wb = gguf.quantize(w, qtype)
    bias = (np.random.default_rng(M).standard_normal(N) * 0.02).astype(np.float32)
    y = _gemm(engine, qtype, wb, N, K, x, bias)
    ref = O.gemm_q_f64(qtype, wb, N, K, x, bias)
    assert np.isfinite(y).all()
    assert _rel(y, ref) <= REL_TIGHT


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [129, 257])
def test_pair_swiglu_boundaries(engine, qtype, M):
    """SwiGLU on CTA pairs (CTA 0 holds the gate rows, CTA 1 the matching up
    rows) at pair-tile boundaries, every row of z and y checked."""
    F, K, N2 = 512, 512, 512
    rng = np.random.default_rng(M + 5)
    w0 = (rng.standard_normal((2 * F, K), dtype=np.float32) * np.float32(0.02))
    w2 = (rng.standard_normal((N2, F), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((M, K), dtype=np.float32)
    b0, b2 = gguf.quantize(w0, qtype), gguf.quantize(w2, qtype)
    dev = torch.device("cuda:0")
    w0d, w2d = torch.from_numpy(b0).to(dev), torch.from_numpy(b2).to(dev)
    xd = torch.from_numpy(x).to(dev)
    zd = torch.full((M, F), float("nan"), device=dev)
    yd = torch.full((M, N2), float("nan"), device=dev)
    torch.cuda.synchronize()
    check(lib().t0b_swiglu_q(engine.handle, qtype, ptr(w0d), ptr(w2d), F, K, N2, ptr(xd), M, None, None, ptr(zd),
                             ptr(yd), None))
    z, y = zd.cpu().numpy(), yd.cpu().numpy()
    zr, yr = O.swiglu_q_f64(qtype, b0, F, K, b2, N2, x)
    assert np.isfinite(z).all() and np.isfinite(y).all()
    assert _rel(z, zr) <= REL_TIGHT
    assert _rel(y, yr) <= REL_TIGHT


def _sampled_rows(M, n=96, seed=0):
    """First and last rows, both sides of every 256-token pair tile near the
    ends, and a seeded spread in between."""
    fixed = [0, 1, 127, 128, 255, 256, M - 257, M - 256, M - 129, M - 128, M - 2, M - 1]
    rest = np.random.default_rng(seed).choice(M, n - len(fixed), replace=False)
    return np.unique(np.clip(np.concatenate([fixed, rest]), 0, M - 1))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
def test_gemm_config2_full_size(engine, qtype):
    """The standalone Q8_0 GEMM configuration at its largest timed size,
    N = 3072, K = 1024, M = 65,536 (805 MB of output): ~96 sampled rows
    against the f64 oracle, every output checked finite."""
    N, K, M = 3072, 1024, 65536
    w, x = S.gemm_case(N, K, M, seed=65536)
    wb = gguf.quantize(w, qtype)
    dev = torch.device("cuda:0")
    wd = torch.from_numpy(wb.copy()).to(dev)
    xd = torch.from_numpy(x).to(dev)
    yd = torch.full((M, N), float("nan"), device=dev)
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q(engine.handle, qtype, ptr(wd), N, K, ptr(xd), M, None, ptr(yd), None))
    rows = _sampled_rows(M)
    assert bool(torch.isfinite(yd).all())
    y = yd[torch.from_numpy(rows).to(dev)].cpu().numpy()
    ref = O.gemm_q_f64(qtype, wb, N, K, x[rows])
    assert _rel(y, ref) <= REL_TIGHT


@pytest.mark.parametrize("qtype,M", [(Q4_0, 1024), (Q8_0, 1024), (Q4_0, 65536)],
                         ids=["q4_0-1024", "q8_0-1024", "q4_0-65536"])
def test_swiglu_config3_timed_sizes(engine, qtype, M):
    """The standalone SwiGLU configuration (F = 4096, K = 1024, N2 = 1024) at
    the timed token counts 1,024 and 65,536: z and y of ~96 sampled rows
    against the f64 oracle, every output checked finite."""
    F, K, N2 = 4096, 1024, 1024
    rng = np.random.default_rng(M + 11)
    w0 = (rng.standard_normal((2 * F, K), dtype=np.float32) * np.float32(0.02))
    w2 = (rng.standard_normal((N2, F), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((M, K), dtype=np.float32)
    b0, b2 = gguf.quantize(w0, qtype), gguf.quantize(w2, qtype)
    dev = torch.device("cuda:0")
    w0d, w2d = torch.from_numpy(b0).to(dev), torch.from_numpy(b2).to(dev)
    xd = torch.from_numpy(x).to(dev)
    zd = torch.full((M, F), float("nan"), device=dev)
    yd = torch.full((M, N2), float("nan"), device=dev)
    torch.cuda.synchronize()
    check(lib().t0b_swiglu_q(engine.handle, qtype, ptr(w0d), ptr(w2d), F, K, N2, ptr(xd), M, None, None, ptr(zd),
                             ptr(yd), None))
    assert bool(torch.isfinite(zd).all()) and bool(torch.isfinite(yd).all())
    rows = _sampled_rows(M)
    idx = torch.from_numpy(rows).to(dev)
    z, y = zd[idx].cpu().numpy(), yd[idx].cpu().numpy()
    zr, yr = O.swiglu_q_f64(qtype, b0, F, K, b2, N2, x[rows])
    assert _rel(z, zr) <= REL_TIGHT
    assert _rel(y, yr) <= REL_TIGHT
