"""CPU checks of the product library's host side (no GPU needed):

* libt0b.so loads and exports every function include/t0b.h declares;
* its codecs (t0b_quantize / t0b_dequantize / t0b_export_gguf) are
  byte-identical to the pinned oracle;
* the GGUF files it writes follow t0-core's layout (gguf.rs:299-345:
  reversed ne, 32-aligned offsets, blob right after the tensor infos,
  weights.rs:32-37 quantization policy, weights.rs:208-220 metadata);
* t0b_gguf_validate accepts them and rejects malformed files with
  T0B_ERR_FORMAT instead of crashing;
* the product package never imports the oracle, and fails loudly (a
  T0bError, no CPU fallback) when there is no GPU.
"""
import os
import re
import struct

import numpy as np
import pytest

import oracle as O
from t0_web_b200 import _lib, gguf, synthetic as S
from t0_web_b200._lib import F16, Q4_0, Q8_0, T0bError, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "t0b.h")
GOLDEN = os.path.join(ROOT, "tests", "golden")


# ----------------------------------------------------------------- the ABI
def _header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = re.sub(r"#define[^\n]*", "", src)
    return sorted(set(re.findall(r"\b(t0b_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_header_function():
    names = _header_functions()
    assert len(names) >= 25
    L = lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert sorted(_lib.EXPORTED) == names


def test_header_constants_match_bindings():
    src = open(HEADER).read()
    status = dict((k, int(v)) for k, v in re.findall(r"\b(T0B_(?:OK|ERR_[A-Z]+))\s*=\s*(\d+)", src))
    assert status["T0B_OK"] == _lib.T0B_OK and status["T0B_ERR_INVALID"] == _lib.T0B_ERR_INVALID
    assert status["T0B_ERR_FORMAT"] == _lib.T0B_ERR_FORMAT and status["T0B_ERR_DEVICE"] == _lib.T0B_ERR_DEVICE
    types = dict((k, int(v)) for k, v in re.findall(r"\b(T0B_(?:F32|F16|Q8_0|Q4_0))\s*=\s*(\d+)", src))
    assert (types["T0B_F16"], types["T0B_Q8_0"], types["T0B_Q4_0"]) == (F16, Q8_0, Q4_0)


def test_product_package_never_imports_oracle():
    pkg = os.path.join(ROOT, "t0_web_b200")
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            text = open(os.path.join(pkg, f)).read()
            assert not re.search(r"^\s*(import oracle|from oracle)", text, flags=re.M), f


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU behaviour")
def test_engine_fails_loudly_without_gpu():
    from t0_web_b200 import t0_fast
    with pytest.raises(T0bError):
        t0_fast.Engine(0)


# ---------------------------------------------------------- codecs vs oracle
@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["q8_0", "q4_0"])
def test_quantize_dequantize_match_oracle(qtype):
    g = np.load(os.path.join(GOLDEN, "quant_blocks.npz"))
    rng = np.random.default_rng(5)
    x = np.concatenate([g["x"], rng.standard_normal(32 * 300).astype(np.float32) * np.float32(0.05)])
    b = gguf.quantize(x, qtype)
    assert np.array_equal(b, O.quantize(x, qtype))
    assert np.array_equal(gguf.dequantize(b, x.size, qtype), O.dequantize(b, x.size, qtype))
    key = "q8_0" if qtype == Q8_0 else "q4_0"
    assert np.array_equal(gguf.quantize(g["x"], qtype), g[key])


def test_row_bytes():
    assert gguf.row_bytes(Q8_0, 512) == 16 * 34
    assert gguf.row_bytes(Q4_0, 2048) == 64 * 18
    assert gguf.row_bytes(F16, 10) == 20


@pytest.mark.parametrize("quant", ["f16", "q8_0", "q4_0"])
def test_export_matches_oracle_bytes(quant):
    w = S.random_weights(S.TINY, seed=2)
    assert gguf.export_gguf(w, S.TINY, quant) == O.export_gguf(w, S.TINY, quant)


# ------------------------------------------------------- GGUF file structure
def _read_gguf(b: bytes):
    """Minimal GGUF v3 reader written from the format description
    (gguf.rs:347-405): returns (metadata, infos, blob_start)."""
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, b, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal pos
        n = take("Q")
        s = b[pos:pos + n].decode()
        pos += n
        return s

    assert b[:4] == b"GGUF"
    pos = 4
    assert take("I") == 3
    n_t, n_kv = take("Q"), take("Q")
    meta = {}
    for _ in range(n_kv):
        k = string()
        ty = take("I")
        if ty == 4:
            meta[k] = take("I")
        elif ty == 6:
            meta[k] = take("f")
        elif ty == 7:
            meta[k] = bool(take("B"))
        elif ty == 8:
            meta[k] = string()
        elif ty == 9:
            assert take("I") == 6
            meta[k] = [take("f") for _ in range(take("Q"))]
        else:
            raise AssertionError(f"metadata type {ty}")
    infos = {}
    for _ in range(n_t):
        name = string()
        nd = take("I")
        ne = [take("Q") for _ in range(nd)]
        infos[name] = (ne, take("I"), take("Q"))
    return meta, infos, pos


@pytest.mark.parametrize("quant,qtype", [("q8_0", Q8_0), ("q4_0", Q4_0)])
def test_gguf_layout_policy_and_values(quant, qtype):
    w = S.random_weights(S.TINY, seed=4)
    b = gguf.export_gguf(w, S.TINY, quant)
    meta, infos, blob = _read_gguf(b)
    assert set(meta) == {f"t0.{k}" for k in ("embed_dim", "num_layers", "num_heads", "mlp_hidden_dim",
                                              "patch_size", "group_every_n", "dropout", "quantile_levels",
                                              "scaler_use_arcsinh", "scaler_eps", "scaler_eps_mode")}
    assert meta["t0.embed_dim"] == 256 and meta["t0.scaler_eps_mode"] == "variance_offset"
    assert np.allclose(meta["t0.quantile_levels"], S.TINY["quantile_levels"])
    assert set(infos) == set(w)
    big = (".attention.wQKV.weight", ".attention.wO.weight", ".mlp.0.weight", ".mlp.2.weight")
    end = 0
    for name, (ne, ty, off) in infos.items():
        shape = w[name].shape
        assert ne == list(reversed(shape)), name            # ne is reversed
        assert off % 32 == 0
        quantized = len(shape) == 2 and any(s in name for s in big)
        assert ty == (qtype if quantized else F16), name
        n = int(np.prod(shape))
        size = gguf.row_bytes(ty, n)
        data = np.frombuffer(b, np.uint8, size, blob + off)
        y = gguf.dequantize(data, n, ty).reshape(shape)
        x = w[name]
        if ty == F16:
            assert np.array_equal(y, x.astype(np.float16).astype(np.float32))
        else:
            assert np.max(np.abs(y - x)) <= (0.02 * 5 / (127 if ty == Q8_0 else 7))
        end = max(end, off + size)
    assert blob + end == len(b)  # blob starts right after the infos, no pad


def test_validate_info_tiny():
    w = S.random_weights(S.TINY, seed=4)
    info = gguf.validate(gguf.export_gguf(w, S.TINY, "q8_0"))
    assert (info.embed_dim, info.num_layers, info.num_heads, info.mlp_hidden_dim) == (256, 3, 4, 256)
    assert (info.patch_size, info.group_every_n, info.n_quantiles) == (32, 3, 5)
    assert info.weight_type == Q8_0
    E, F, L = 256, 256, 3
    assert info.quantizable_gpu_bytes == L * (3 * E * E + E * E + 2 * F * E + E * F) // 32 * 34


@pytest.mark.parametrize("quant,expected", [("q8_0", 106_954_752), ("q4_0", 56_623_104)])
def test_validate_alpha_quantizable_bytes(gguf_bytes, quant, expected):
    """t0-alpha: 100,663,296 quantized weights (t0-alpha-anatomy.md:45-54)."""
    info = gguf.validate(gguf_bytes(quant))
    assert info.quantizable_gpu_bytes == expected
    assert (info.embed_dim, info.num_layers, info.mlp_hidden_dim) == (512, 24, 2048)


def test_validate_info_beta_shape():
    """t0-beta's config fields (embed_dim 1024 -> head_dim 128, 21 levels,
    std_clamp scaler with eps 0.01) come through the metadata."""
    info = gguf.validate(gguf.export_gguf(S.random_weights(S.BETA_SMALL, seed=2), S.BETA_SMALL, "q4_0"))
    assert (info.embed_dim, info.num_heads, info.num_layers, info.n_quantiles) == (1024, 8, 3, 21)
    assert info.variance_offset == 0 and abs(info.scaler_eps - 0.01) < 1e-9
    assert np.allclose(list(info.quantile_levels)[:21], S.BETA["quantile_levels"], atol=1e-7)
    assert info.weight_type == Q4_0


@pytest.fixture(scope="module")
def tiny_q8():
    return gguf.export_gguf(S.random_weights(S.TINY, seed=4), S.TINY, "q8_0")


def _rejects(b: bytes):
    with pytest.raises(T0bError) as ei:
        gguf.validate(b)
    assert ei.value.status == _lib.T0B_ERR_FORMAT, str(ei.value)


def test_validate_rejects_bad_magic(tiny_q8):
    _rejects(b"GGUX" + tiny_q8[4:])


def test_validate_rejects_bad_version(tiny_q8):
    _rejects(tiny_q8[:4] + struct.pack("<I", 2) + tiny_q8[8:])


@pytest.mark.parametrize("cut", [0, 3, 8, 23, 100, 1000, -1000, -1])
def test_validate_rejects_truncated(tiny_q8, cut):
    _rejects(tiny_q8[:cut] if cut else b"")


def test_validate_rejects_missing_metadata_key(tiny_q8):
    i = tiny_q8.index(b"t0.num_heads")
    _rejects(tiny_q8[:i] + b"t0.num_heaXs" + tiny_q8[i + 12:])


def test_validate_rejects_missing_tensor():
    w = S.random_weights(S.TINY, seed=4)
    del w["transformer.out_norm.scale"]
    _rejects(gguf.export_gguf(w, S.TINY, "q8_0"))


def test_validate_rejects_wrong_shape():
    w = S.random_weights(S.TINY, seed=4)
    w["transformer.layers.1.mlp.2.weight"] = np.zeros((256, 96), np.float32)
    _rejects(gguf.export_gguf(w, S.TINY, "q8_0"))


def test_validate_unsupported_shapes_and_types():
    """Files that are well-formed but outside what this engine runs give
    T0B_ERR_UNSUPPORTED: head_dim other than 64 and 128, and f16 big matmuls
    (the engine keeps only Q8_0/Q4_0 weights resident)."""
    cfg = dict(S.TINY, num_heads=1)
    with pytest.raises(T0bError) as ei:
        gguf.validate(gguf.export_gguf(S.random_weights(cfg, seed=1), cfg, "q8_0"))
    assert ei.value.status == _lib.T0B_ERR_UNSUPPORTED
    with pytest.raises(T0bError) as ei:
        gguf.validate(gguf.export_gguf(S.random_weights(S.TINY, seed=1), S.TINY, "f16"))
    assert ei.value.status == _lib.T0B_ERR_UNSUPPORTED


def test_validate_rejects_huge_counts(tiny_q8):
    _rejects(tiny_q8[:8] + struct.pack("<Q", 1 << 60) + tiny_q8[16:])
