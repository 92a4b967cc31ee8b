"""t0b_gemm_q_noalloc (the dequant-GEMM that allocates no device memory)
against the engine entry point t0b_gemm_q, on the GPU.

The no-allocation variant runs the same kernels out of a fixed scratch array
compiled into the library, so on the same inputs it must agree with
t0b_gemm_q within the suite's tight GEMM bound (REL_TIGHT, relative to the
largest |y|).  Every case makes two no-allocation calls in a row, the second
with a different shape, so a call that depended on what the previous one left
in the shared scratch would show up.  This file is named to be collected
last: it must pass alone and after every other GPU test.
"""
import numpy as np
import pytest
import torch

from t0_web_b200 import gguf, synthetic as S
from t0_web_b200._lib import Q4_0, Q8_0, T0B_ERR_INVALID, check, lib, ptr

pytestmark = pytest.mark.gpu

REL_TIGHT = 2e-5
MAX_X = 1 << 22  # T0B_NOALLOC_MAX_X_ELEMENTS


def _device_case(qtype, N, K, M, seed):
    dev = torch.device("cuda:0")
    w, x = S.gemm_case(N, K, M, seed=seed)
    wb = gguf.quantize(w, qtype)
    bias = (np.random.default_rng(seed + 1).standard_normal(N) * 0.02).astype(np.float32)
    return (torch.from_numpy(wb.copy()).to(dev), torch.from_numpy(np.ascontiguousarray(x)).to(dev),
            torch.from_numpy(bias).to(dev))


def _poisoned(M, N):
    return torch.full((M, N), float("nan"), device=torch.device("cuda:0"))


def _engine_gemm(engine, qtype, wd, N, K, xd, M, bd):
    y = _poisoned(M, N)
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q(engine.handle, qtype, ptr(wd), N, K, ptr(xd), M, ptr(bd), ptr(y), None))
    return y.cpu().numpy()


def _noalloc_gemm(qtype, wd, N, K, xd, M, bd):
    y = _poisoned(M, N)
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q_noalloc(qtype, ptr(wd), N, K, ptr(xd), M, ptr(bd), ptr(y), None))
    return y.cpu().numpy()


def _rel(y, ref):
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("shapes", [
    ((512, 1024, 64), (256, 512, 33)),      # small-M path twice
    ((512, 1024, 300), (768, 256, 129)),    # tensor-core path twice
    ((256, 512, 200), (512, 1024, 17)),     # tensor-core then small-M
], ids=["small_small", "tc_tc", "tc_small"])
def test_noalloc_matches_engine_two_calls(engine, qtype, shapes):
    torch.cuda.set_device(0)
    for i, (N, K, M) in enumerate(shapes):
        wd, xd, bd = _device_case(qtype, N, K, M, seed=1000 + 17 * i + M)
        ref = _engine_gemm(engine, qtype, wd, N, K, xd, M, bd)
        y = _noalloc_gemm(qtype, wd, N, K, xd, M, bd)
        assert np.isfinite(y).all(), f"call {i}: unwritten or non-finite outputs"
        assert _rel(y, ref) <= REL_TIGHT, (i, _rel(y, ref))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
def test_noalloc_largest_x_then_repeat(engine, qtype):
    """M*K exactly at the scratch limit, then the same call again."""
    torch.cuda.set_device(0)
    N, K = 256, 1024
    M = MAX_X // K
    wd, xd, bd = _device_case(qtype, N, K, M, seed=77)
    ref = _engine_gemm(engine, qtype, wd, N, K, xd, M, bd)
    y1 = _noalloc_gemm(qtype, wd, N, K, xd, M, bd)
    y2 = _noalloc_gemm(qtype, wd, N, K, xd, M, bd)
    assert np.isfinite(y1).all() and np.isfinite(y2).all()
    assert _rel(y1, ref) <= REL_TIGHT
    assert _rel(y2, ref) <= REL_TIGHT


def test_noalloc_rejects_oversize_x():
    torch.cuda.set_device(0)
    N, K = 256, 1024
    M = MAX_X // K + 1
    dev = torch.device("cuda:0")
    wd = torch.zeros(N * (K // 32) * 34, dtype=torch.uint8, device=dev)
    xd = torch.zeros((1, K), device=dev)  # never read: the size check comes first
    y = torch.full((1, N), 7.0, device=dev)
    rc = lib().t0b_gemm_q_noalloc(Q8_0, ptr(wd), N, K, ptr(xd), M, None, ptr(y), None)
    assert rc == T0B_ERR_INVALID
    assert b"exceeds the fixed scratch" in lib().t0b_last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())
