"""Resident-weight GEMMs (t0b_qmatrix_*) on the GPU.

The handle API runs the same kernels as t0b_gemm_q / t0b_swiglu_q with the
prescale found once at creation, so its outputs must equal theirs bit for
bit; it only queues stream work, so a CUDA graph of its calls must replay to
the same outputs.  The fp64 oracle bound (REL_TIGHT, relative to the largest
|y|) is asserted as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from t0_web_b200 import gguf
from t0_web_b200._lib import Q4_0, Q8_0, T0B_ERR_INVALID, check, lib, ptr

pytestmark = pytest.mark.gpu

REL_TIGHT = 2e-5
DEV = torch.device("cuda:0")


def _rel(y, ref):
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


class QMatrix:
    def __init__(self, engine, qtype, wd, N, K):
        h = C.c_void_p()
        check(lib().t0b_qmatrix_create(engine.handle, qtype, ptr(wd), N, K, C.byref(h)))
        self.h, self.wd = h, wd

    def close(self):
        lib().t0b_qmatrix_destroy(self.h)


def _weights(qtype, N, K, seed):
    w = np.random.default_rng(seed).standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    wb = gguf.quantize(w, qtype)
    return wb, torch.from_numpy(wb.copy()).to(DEV)


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [16, 300])
def test_qmatrix_gemm_equals_gemm_q(engine, qtype, M):
    torch.cuda.set_device(0)
    N, K = 768, 1024
    wb, wd = _weights(qtype, N, K, seed=M)
    x = np.random.default_rng(M + 1).standard_normal((M, K), dtype=np.float32)
    bias = (np.random.default_rng(M + 2).standard_normal(N) * 0.02).astype(np.float32)
    xd, bd = torch.from_numpy(x).to(DEV), torch.from_numpy(bias).to(DEV)
    ref = torch.full((M, N), float("nan"), device=DEV)
    got = torch.full((M, N), float("nan"), device=DEV)
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q(engine.handle, qtype, ptr(wd), N, K, ptr(xd), M, ptr(bd), ptr(ref), None))
    q = QMatrix(engine, qtype, wd, N, K)
    try:
        check(lib().t0b_qmatrix_gemm(q.h, ptr(xd), M, ptr(bd), ptr(got), None))
        check(lib().t0b_qmatrix_sync(q.h, None))
    finally:
        q.close()
    g, r = got.cpu().numpy(), ref.cpu().numpy()
    assert np.array_equal(g, r)
    rows = np.arange(0, M, 5)
    yr = O.gemm_q_f64(qtype, wb, N, K, x[rows]) + bias
    assert _rel(g[rows], yr) <= REL_TIGHT


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [16, 200])
def test_qmatrix_swiglu_equals_swiglu_q(engine, qtype, M):
    torch.cuda.set_device(0)
    F, K, N2 = 1024, 512, 512
    _, w0d = _weights(qtype, 2 * F, K, seed=10 + M)
    _, w2d = _weights(qtype, N2, F, seed=20 + M)
    xd = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(M))
    outs = []
    for use_handle in (False, True):
        z = torch.full((M, F), float("nan"), device=DEV)
        y = torch.full((M, N2), float("nan"), device=DEV)
        torch.cuda.synchronize()
        if not use_handle:
            check(lib().t0b_swiglu_q(engine.handle, qtype, ptr(w0d), ptr(w2d), F, K, N2, ptr(xd), M, None, None,
                                     ptr(z), ptr(y), None))
        else:
            q0, q2 = QMatrix(engine, qtype, w0d, 2 * F, K), QMatrix(engine, qtype, w2d, N2, F)
            try:
                check(lib().t0b_qmatrix_swiglu(q0.h, q2.h, ptr(xd), M, None, None, ptr(z), ptr(y), None))
                check(lib().t0b_qmatrix_sync(q0.h, None))
                check(lib().t0b_qmatrix_sync(q2.h, None))
            finally:
                q0.close()
                q2.close()
        outs.append((z.cpu().numpy(), y.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    assert np.isfinite(outs[1][1]).all()


@pytest.mark.parametrize("M", [19, 256])
def test_qmatrix_graph_replay(engine, M):
    """Three matrices' GEMMs captured in one CUDA graph replay to the eager outputs."""
    torch.cuda.set_device(0)
    N, K = 512, 512
    qs = [QMatrix(engine, Q8_0, _weights(Q8_0, N, K, seed=40 + i)[1], N, K) for i in range(3)]
    try:
        xd = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
        ys = [torch.full((M, N), float("nan"), device=DEV) for _ in qs]
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for q, y in zip(qs, ys):
                check(lib().t0b_qmatrix_gemm(q.h, ptr(xd), M, None, ptr(y), C.c_void_p(s.cuda_stream)))
        s.synchronize()
        eager = [y.cpu().numpy() for y in ys]
        for y in ys:
            y.fill_(float("nan"))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
            for q, y in zip(qs, ys):
                check(lib().t0b_qmatrix_gemm(q.h, ptr(xd), M, None, ptr(y), C.c_void_p(s.cuda_stream)))
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        for q in qs:
            check(lib().t0b_qmatrix_sync(q.h, None))
        for y, e in zip(ys, eager):
            assert np.array_equal(y.cpu().numpy(), e)
        del g
    finally:
        for q in qs:
            q.close()


def test_qmatrix_swiglu_rejects_mismatched_shapes(engine):
    torch.cuda.set_device(0)
    _, w0d = _weights(Q8_0, 1024, 512, seed=1)
    _, w2d = _weights(Q8_0, 512, 768, seed=2)  # K = 768 != F = 512
    q0, q2 = QMatrix(engine, Q8_0, w0d, 1024, 512), QMatrix(engine, Q8_0, w2d, 512, 768)
    try:
        x = torch.zeros((4, 512), device=DEV)
        y = torch.zeros((4, 512), device=DEV)
        rc = lib().t0b_qmatrix_swiglu(q0.h, q2.h, ptr(x), 4, None, None, None, ptr(y), None)
        assert rc == T0B_ERR_INVALID
    finally:
        q0.close()
        q2.close()
