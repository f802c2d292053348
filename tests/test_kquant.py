"""K-quant weights (Q4_K, Q5_K, Q6_K; the reference's quantizer outputs, src/quantize.cpp:66,
accepted by src/weight_policy.hpp:13-16): the loader's dequantisation (tsb_dequantize_rows,
host only) equals gguf-py's independent implementation of ggml's published one bit for bit,
and the test encoder writes blocks that decode close to their input."""
import ctypes as C

import numpy as np
import pytest

import timestral_b200 as tb
from timestral_b200 import synthetic as sy

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as GT
from gguf import quants

TYPES = {"q4_k": (12, GT.Q4_K, 144), "q5_k": (13, GT.Q5_K, 176), "q6_k": (14, GT.Q6_K, 210), "q8_0": (8, GT.Q8_0, 34)}


def ours(code, raw, rows, ne0):
    out = np.empty((rows, ne0), np.float32)
    raw = np.ascontiguousarray(raw)
    assert tb.lib().tsb_dequantize_rows(code, raw.ctypes.data, rows, ne0, out.ctypes.data) == 0
    return out


def random_blocks(kind, rows, ne0, rng):
    code, gt, nbytes = TYPES[kind]
    per = 256 if kind != "q8_0" else 32
    raw = rng.integers(0, 256, (rows, ne0 // per, nbytes), dtype=np.uint8)
    # finite f16 scale fields, including subnormal and zero ones
    def f16(n):
        v = rng.standard_normal(n).astype(np.float32) * rng.choice([1e-6, 1e-3, 0.05, 2.0], n)
        v[rng.random(n) < 0.05] = 0.0
        return v.astype(np.float16).view(np.uint8).reshape(n, 2)
    n = rows * (ne0 // per)
    flat = raw.reshape(n, nbytes)
    if kind in ("q4_k", "q5_k"):
        flat[:, 0:2] = f16(n)
        flat[:, 2:4] = f16(n)
    elif kind == "q6_k":
        flat[:, 208:210] = f16(n)
    else:
        flat[:, 0:2] = f16(n)
    return raw.reshape(rows, -1)


@pytest.mark.parametrize("kind", ["q4_k", "q5_k", "q6_k", "q8_0"])
def test_dequantize_bitwise_against_gguf_py(kind):
    rng = np.random.default_rng({"q4_k": 1, "q5_k": 2, "q6_k": 3, "q8_0": 4}[kind])
    rows, ne0 = 7, 1024
    raw = random_blocks(kind, rows, ne0, rng)
    code, gt, _ = TYPES[kind]
    want = quants.dequantize(raw, gt).astype(np.float32).reshape(rows, ne0)
    got = ours(code, raw, rows, ne0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", ["q4_k", "q5_k", "q6_k", "q8_0"])
def test_scaled_int8_form_equals_dequantisation(kind):
    """The form the GEMM's dequantising prologue reads (integer values, and per 16 values a
    single-precision scale and offset) gives every value of the loader's dequantisation bit
    for bit as (a * q) - b, each operation rounded in single precision."""
    rng = np.random.default_rng({"q4_k": 5, "q5_k": 6, "q6_k": 7, "q8_0": 8}[kind])
    rows, ne0 = 5, 768
    raw = np.ascontiguousarray(random_blocks(kind, rows, ne0, rng))
    code = TYPES[kind][0]
    q = np.empty((rows, ne0), np.int8)
    a = np.empty((rows, ne0 // 16), np.float32)
    b = np.empty_like(a)
    assert tb.lib().tsb_scaled_int8_rows(code, raw.ctypes.data, rows, ne0, q.ctypes.data, a.ctypes.data,
                                         b.ctypes.data) == 0
    aa, bb = np.repeat(a, 16, axis=1), np.repeat(b, 16, axis=1)
    got = (aa * q.astype(np.float32)).astype(np.float32) - bb
    want = ours(code, raw, rows, ne0)
    assert np.array_equal(got.astype(np.float32).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind,tol", [("q4_k", 0.08), ("q5_k", 0.04), ("q6_k", 0.03)])
def test_encoder_round_trip(kind, tol):
    rng = np.random.default_rng(5)
    a = (rng.standard_normal((6, 768)) * rng.uniform(0.01, 0.1, (6, 1))).astype(np.float32)
    q = sy.quantize_k(a, kind)
    code, gt, nbytes = TYPES[kind]
    assert q.shape == (6, 768 // 256 * nbytes)
    back = quants.dequantize(q, gt).astype(np.float32).reshape(a.shape)
    assert np.array_equal(ours(code, q, 6, 768).view(np.uint32), back.view(np.uint32))
    rel = np.abs(back - a).max(axis=1) / np.abs(a).max(axis=1)
    assert np.all(rel <= tol), rel


def test_rejects_rows_that_are_not_whole_blocks():
    raw = np.zeros(144, np.uint8)
    out = np.empty(200, np.float32)
    assert tb.lib().tsb_dequantize_rows(12, raw.ctypes.data, 1, 200, out.ctypes.data) == tb.TSB_ERR_ARG
    assert tb.lib().tsb_dequantize_rows(2, raw.ctypes.data, 1, 256, out.ctypes.data) == tb.TSB_ERR_ARG


@pytest.mark.parametrize("kind", ["q4_k", "q6_k"])
def test_kquant_gguf_passes_the_loader(kind):
    """A K-quant file passes the schema and storage checks (without a GPU the load stops at the
    device selection, after the model has been read)."""
    path = sy.cached_model(sy.spec_k256(), kind)
    L = tb.lib()
    h = L.timestral_capi_load(str(path).encode(), 1)
    if h:
        L.timestral_capi_free(h)
        return
    msg = L.timestral_capi_last_error(None).decode()
    assert "CUDA" in msg, msg
