import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def alpha_weights():
    from t0_web_b200 import synthetic as S
    return S.random_weights(S.ALPHA, seed=0)


@pytest.fixture(scope="session")
def gguf_bytes(alpha_weights):
    """Product-exported GGUF files of the random-init t0-alpha model."""
    from t0_web_b200 import gguf, synthetic as S
    cache = {}

    def get(quant):
        if quant not in cache:
            cache[quant] = gguf.export_gguf(alpha_weights, S.ALPHA, quant)
        return cache[quant]

    return get


@pytest.fixture(scope="session")
def oracle_model(gguf_bytes):
    import oracle as O
    cache = {}

    def get(quant):
        if quant not in cache:
            cache[quant] = O.OracleModel(gguf_bytes(quant))
        return cache[quant]

    return get


@pytest.fixture(scope="session")
def engine():
    from t0_web_b200 import t0_fast
    e = t0_fast.Engine(0)
    yield e


@pytest.fixture(scope="session")
def gpu_model(engine, gguf_bytes):
    from t0_web_b200 import t0_fast
    cache = {}

    def get(quant):
        if quant not in cache:
            cache[quant] = t0_fast.load_model_from_gguf(engine, gguf_bytes(quant))
        return cache[quant]

    yield get
    for m in cache.values():
        m.close()


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
