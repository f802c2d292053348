"""CUDA-core GEMM of the F32 path (per-output reference order, reference src/layers.cpp:143-177
linear_f32: f32 FMAs in 192-wide K panels, panel sums added in order): the 64 x 128 tile
kernel that large launches run equals the 64 x 64 kernel bit for bit, so does the panel-split
path of few-row launches, and on small dyadic values, where every partial sum is exact
whatever the order, the result is the exact product."""
import ctypes as C

import numpy as np
import pytest

import timestral_b200 as tb

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda:0")


def run(A, W, order, tiled):
    M, K = A.shape
    N = W.shape[0]
    out = torch.full((M, N), float("nan"), device=A.device)
    rc = tb.lib().tsb_test_simt_gemm(A.data_ptr(), W.data_ptr(), M, N, K, order, tiled, out.data_ptr())
    assert rc == 0, rc
    return out.cpu()


@pytest.mark.parametrize("M,N,K", [(2112, 2304, 768), (2112, 768, 2048), (64, 128, 16), (100, 300, 192),
                                   (1000, 130, 3072), (65, 129, 400), (4096, 4096, 768)])
def test_tiled_equals_64x64(dev, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g).to(dev)
    W = (torch.randn(N, K, generator=g) * 0.05).to(dev)
    a = run(A, W, 0, 1)
    b = run(A, W, 0, 0)
    assert torch.isfinite(a).all()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.parametrize("M,N,K", [(34, 2304, 768), (34, 768, 2048), (64, 4096, 768), (1, 100, 400), (36, 33, 3072),
                                   (300, 768, 768), (512, 130, 384)])
def test_panel_split_equals_one_pass(dev, M, N, K):
    """Launches of at most 512 rows (one decode block of a few series: cfg1 and the reference's
    short benchmark) split K into 192-wide panels run as separate blocks and sum the partials
    in panel order in a second kernel; the result equals the one-pass 64 x 64 kernel bit for bit."""
    g = torch.Generator().manual_seed(M * 3 + N + K)
    A = torch.randn(M, K, generator=g).to(dev)
    W = (torch.randn(N, K, generator=g) * 0.05).to(dev)
    split = run(A, W, 0, 2)
    one = run(A, W, 0, 0)
    assert torch.isfinite(split).all()
    assert torch.equal(split.view(torch.int32), one.view(torch.int32))


def test_panel_order_restatement(dev):
    """Dyadic inputs (multiples of 1/8 and 1/64 in [-1, 1]) over three panels: every product
    and partial sum is exact in f32, so the tiled kernel must return the exact product."""
    M, N, K = 70, 140, 400
    g = torch.Generator().manual_seed(7)
    A = torch.randint(-8, 9, (M, K), generator=g).float() / 8
    W = torch.randint(-8, 9, (N, K), generator=g).float() / 64
    got = run(A.to(dev), W.to(dev), 0, 1)
    # small dyadic values: every product and partial sum is exact in f32, so the order cannot
    # change the result and the float64 dot product is the exact answer
    want = (A.double() @ W.double().T).float()
    assert torch.equal(got, want)
