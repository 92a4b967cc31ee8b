"""The index-checked build (libt0b_checked.so, -DT0B_CHECKED).

Every device-side index check of the kernels is compiled in: global-memory
indices of the small-M GEMM (weight rows, epilogue columns, sums of squares),
the TMA coordinates of the tensor-core GEMM and of the time attention
(innermost coordinate on a 16-byte boundary, none negative), and the causal
scaler's feature rows.  A failed check records T0B_DEVERR_BOUNDS and skips
the access; none may fail.  The checks change no arithmetic, so the checked
build's outputs must equal the product build's bit for bit on the same odd
shapes (M off every tile boundary, N and K odd multiples of 256, ragged rows,
a NaN gap), with every output written (NaN-poisoned beforehand).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CHECKED_LIB = os.path.join(os.path.dirname(HERE), "t0_web_b200", "libt0b_checked.so")


def _run(which: str, path: str) -> None:
    r = subprocess.run([sys.executable, os.path.join(HERE, "checked_cases.py"), which, path],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, f"{which} build: {r.stdout[-2000:]}\n{r.stderr[-4000:]}"


def test_checked_build_matches_product_bit_for_bit(tmp_path):
    assert os.path.exists(CHECKED_LIB), "build it with `python -m t0_web_b200.build --checked`"
    prod, chk = tmp_path / "product.npz", tmp_path / "checked.npz"
    _run("product", str(prod))
    _run("checked", str(chk))
    a, b = np.load(prod), np.load(chk)
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        assert np.isfinite(b[k]).all(), k
        assert np.array_equal(a[k], b[k]), k
