"""Failure detection on the GPU without a fault: the bounded mbarrier wait.

Every pipeline wait in the kernels (TMA tiles, dequantized tiles, tensor
memory accumulators) is `mbar_wait` (csrc/common.cuh): it gives up after
T0B_WAIT_CYCLES SM cycles, records a device error code and returns, so a
lost arrival surfaces as T0B_ERR_DEVICE rather than a hung GPU.  Here one
warp waits on a barrier that nothing arrives on; the test checks the status,
the recorded code, that the kernel itself ran to its end, and that the
context still runs a GEMM correctly afterwards.  No TMA, tensor memory or
cluster work is started by the self-test kernel.
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

import oracle as O
from t0_web_b200 import gguf, synthetic as S
from t0_web_b200._lib import Q8_0, T0B_ERR_DEVICE, T0B_OK, check, lib, ptr

pytestmark = pytest.mark.gpu

DEVERR_WAIT_X = 1  # T0B_DEVERR_WAIT_X in csrc/common.cuh


def test_bounded_wait_runs_out_and_reports(engine):
    code, outcome = C.c_int(-1), C.c_int(-1)
    t0 = time.perf_counter()
    st = lib().t0b_selftest_bounded_wait(engine.handle, C.byref(code), C.byref(outcome))
    dt = time.perf_counter() - t0
    assert st == T0B_ERR_DEVICE, lib().t0b_last_error()
    assert b"device error code 1" in lib().t0b_last_error()
    assert code.value == DEVERR_WAIT_X
    assert outcome.value == 2  # the wait returned false and the kernel finished
    assert 0.2 < dt < 60.0, dt  # it did wait (about 2 s at B200 clocks), and it ended

    # the context is still usable: a GEMM through the engine matches the oracle
    N, K, M = 256, 512, 40
    w, x = S.gemm_case(N, K, M, seed=3)
    wb = gguf.quantize(w, Q8_0)
    dev = torch.device("cuda:0")
    wd, xd = torch.from_numpy(wb.copy()).to(dev), torch.from_numpy(x).to(dev)
    yd = torch.full((M, N), float("nan"), device=dev)
    torch.cuda.synchronize()
    check(lib().t0b_gemm_q(engine.handle, Q8_0, ptr(wd), N, K, ptr(xd), M, None, ptr(yd), None))
    y = yd.cpu().numpy()
    ref = O.gemm_q_f64(Q8_0, wb, N, K, x)
    assert float(np.max(np.abs(y - ref)) / np.max(np.abs(ref))) <= 2e-5
    assert T0B_OK == 0
