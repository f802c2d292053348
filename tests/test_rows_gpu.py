"""Row kernels of the device path against the CPU oracle, through the kernel-level C-ABI
test entries: RMSNorm must match the oracle's restatement of the reference's float sum
cascade (reference src/layers.cpp:262-287, src/torch_sum.hpp:9-23) bit for bit."""
import ctypes as C

import numpy as np
import pytest

import oracle_py as op
import timestral_b200 as tb

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda:0")


@pytest.mark.parametrize("tokens,D", [(1, 32), (37, 96), (300, 128), (129, 768), (64, 1024), (5, 2100)])
def test_rms_bitwise(dev, tokens, D):
    rng = np.random.default_rng(D)
    x = (rng.standard_normal((tokens, D)) * rng.uniform(0.1, 30, (tokens, 1))).astype(np.float32)
    w = rng.uniform(0.5, 1.5, D).astype(np.float32)
    want = op.rms_norm(x, w, 1e-6)
    dx, dw = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
    out = torch.empty(tokens, D, device=dev)
    assert tb.lib().tsb_test_rms(dx.data_ptr(), dw.data_ptr(), tokens, D, C.c_float(1e-6), out.data_ptr(), 0) == 0
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())
    out16 = torch.empty(tokens, D, device=dev, dtype=torch.float16)
    assert tb.lib().tsb_test_rms(dx.data_ptr(), dw.data_ptr(), tokens, D, C.c_float(1e-6), out16.data_ptr(), 1) == 0
    assert np.array_equal(out16.cpu().numpy(), want.astype(np.float16))


@pytest.mark.parametrize("big", [False, True])
def test_split_f16(dev, big):
    """hi + lo reproduces each f32 value to ~2^-22 relative (the tensor-core patch projections
    sum hi*hi + hi*lo + lo*hi), and values beyond 30000 raise the flag that makes the
    CUDA-core kernels recompute the projections."""
    rng = np.random.default_rng(7)
    rows, K = 300, 64
    a = (rng.standard_normal((rows, K)) * rng.uniform(0.01, 100, (rows, 1))).astype(np.float32)
    if big:
        a[123, 5] = 40000.0
    da = torch.from_numpy(a).to(dev)
    out = torch.empty(rows, 3 * K, device=dev, dtype=torch.float16)
    flag = torch.zeros(1, device=dev, dtype=torch.int32)
    assert tb.lib().tsb_test_split_f16(da.data_ptr(), rows, K, out.data_ptr(), flag.data_ptr()) == 0
    o = out.cpu().numpy().astype(np.float64)
    hi, hi2, lo = o[:, :K], o[:, K:2 * K], o[:, 2 * K:]
    assert np.array_equal(hi, hi2)
    assert np.array_equal(hi, a.astype(np.float16).astype(np.float64))
    ok = np.abs(a) <= 30000
    err = np.abs(hi + lo - a.astype(np.float64))[ok]
    assert np.all(err <= 2.0 ** -21 * np.abs(a[ok]) + 2.0 ** -24), float(err.max())
    assert int(flag.item()) == int(big)
