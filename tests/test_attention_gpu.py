"""Tensor-core time attention against a float64 torch restatement of the reference's masked,
sigmoid-gated sdpa on the time axis (reference src/layers.cpp:578-617, src/masks.cpp:21-26,
src/encoder.cpp:87), through the kernel-level C-ABI test entry.

The kernel rounds probabilities to f16 for the P V product and writes f16 outputs, so the
tolerance is 4e-3 relative to each row's largest |value| plus 2^-10 of the value."""
import ctypes as C

import numpy as np
import pytest

import timestral_b200 as tb
from helpers import time_mask_torch

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda:0")


def allowed_mask(valid, N, S):
    """[rows, S, S] bool: query q may attend key k (no covariates)."""
    rows = valid.shape[0]
    q = torch.arange(S)[:, None]
    k = torch.arange(S)[None, :]
    kv = torch.zeros(rows, S, dtype=torch.bool)
    kv[:, :N] = valid
    kvk = kv[:, None, :].expand(rows, S, S)
    enc = (q < N) & (k < N) & ((kvk & (k <= q)) | (q == k))
    dec = (q >= N) & (((k < N) & kvk) | ((k >= N) & (k <= q)))
    return enc | dec


@pytest.mark.parametrize("S,N,gated,dense", [(1, 1, True, False), (9, 8, True, False), (33, 30, False, False),
                                             (72, 64, True, False), (100, 97, True, False), (128, 120, True, False),
                                             (70, 70, True, False), (72, 64, True, True), (128, 120, False, True),
                                             (40, 32, True, True)])
def test_attention_time_tc(dev, S, N, gated, dense):
    rows, H = 37, 3
    g = torch.Generator().manual_seed(S * 1000 + N)
    q = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    k = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    v = torch.randn(rows, H, S, 64, generator=g).half()
    gate = torch.rand(rows, H, S, 64, generator=g).half() if gated else None
    valid = torch.rand(rows, N, generator=g) > 0.2
    valid[:, 0] = True
    if dense:                        # every key valid: unmasked 16-key chunks below the diagonal
        valid[:] = True
    words = (N + 31) // 32
    bits = np.zeros((rows, words), np.uint32)
    vn = valid.numpy()
    for p in range(N):
        bits[:, p // 32] |= vn[:, p].astype(np.uint32) << np.uint32(p % 32)
    allowed = allowed_mask(valid, N, S)
    s = torch.einsum("rhqd,rhkd->rhqk", q.double(), k.double()) / 8.0
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    want = torch.einsum("rhqk,rhkd->rhqd", p, v.double())
    if gated:
        want = want * gate.double()
    want = want.permute(0, 2, 1, 3).reshape(rows * S, H * 64)
    dq, dk, dv = q.to(dev), k.to(dev), v.to(dev)
    dg = gate.to(dev) if gated else None
    dbits = torch.from_numpy(bits.view(np.int32)).to(dev)
    out = torch.full((rows * S, H * 64), float("nan"), device=dev, dtype=torch.float16)
    err = C.c_int32(0)
    rc = tb.lib().tsb_test_attention_time(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr() if gated else None,
                                          out.data_ptr(), dbits.data_ptr(), rows, H, S, N, C.byref(err))
    assert rc == 0, (rc, err.value)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    scale = want.abs().reshape(rows, S, H, 64).amax(dim=(1, 3), keepdim=True).expand(rows, S, H, 64).reshape(rows * S, H * 64)
    tol = 4e-3 * scale + want.abs() * 2.0 ** -10
    bad = (got - want).abs() > tol
    assert not bad.any(), f"max err {(got - want).abs().max().item():.3e}"


@pytest.mark.parametrize("G,S,N,cov,kernel", [(32, 36, 32, False, 1), (3, 10, 8, False, 1), (18, 70, 35, True, 1),
                                              (64, 20, 16, False, 1), (45, 12, 12, True, 1),
                                              (32, 36, 32, False, 2), (3, 10, 8, False, 2), (18, 70, 35, True, 2),
                                              (7, 5, 3, False, 2), (32, 72, 64, False, 2), (24, 9, 9, True, 2),
                                              (1, 6, 4, False, 2)])
def test_attention_variate(dev, G, S, N, cov, kernel):
    """Variate axis: at each patch slot p a row attends the rows of its series whose patch p is
    observed (every row at decoder slots p >= N), under the covariate role firewall, and
    always itself (reference src/masks.cpp:27). Kernel 1: CUDA cores in f32; kernel 2: tensor
    cores, four (series, head, slot) problems per score tile, probabilities rounded to f16 for
    the P V product (the time kernel's tolerance)."""
    groups, H = 5, 2
    rows = groups * G
    g = torch.Generator().manual_seed(G * 100 + S)
    q = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    k = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    v = torch.randn(rows, H, S, 64, generator=g).half()
    gate = torch.rand(rows, H, S, 64, generator=g).half()
    valid = torch.rand(rows, N, generator=g) > 0.3
    role = torch.randint(0, 3, (rows,), generator=g, dtype=torch.int8) if cov else None
    words = (N + 31) // 32
    bits = np.zeros((rows, words), np.uint32)
    vn = valid.numpy()
    for pp in range(N):
        bits[:, pp // 32] |= vn[:, pp].astype(np.uint32) << np.uint32(pp % 32)
    # allowed[p, i, j] within each group
    usable = torch.ones(rows, S, dtype=torch.bool)
    usable[:, :N] = valid
    want = torch.empty(rows, S, H, 64, dtype=torch.float64)
    for gi in range(groups):
        r = slice(gi * G, (gi + 1) * G)
        qd, kd, vd = q[r].double(), k[r].double(), v[r].double()     # [G,H,S,64]
        s_ = torch.einsum("ihpd,jhpd->hpij", qd, kd) / 8.0
        allow = usable[r].T[None, :, None, :].expand(H, S, G, G).clone()   # key j usable at p
        if cov:
            rq = role[r].long()[:, None]
            rk = role[r].long()[None, :]
            fw = ~(((rq != 0) & (rk == 0)) | ((rq == 2) & (rk != 2)))
            allow &= fw[None, None]
        eye = torch.eye(G, dtype=torch.bool)
        allow |= eye[None, None]
        s_ = s_.masked_fill(~allow, float("-inf"))
        pr = torch.softmax(s_, dim=-1)
        o = torch.einsum("hpij,jhpd->ihpd", pr, vd) * gate[r].double()
        want[r] = o.permute(0, 2, 1, 3)
    want = want.reshape(rows * S, H * 64)
    dq, dk, dv, dg = q.to(dev), k.to(dev), v.to(dev), gate.to(dev)
    dbits = torch.from_numpy(bits.view(np.int32)).to(dev)
    drole = role.to(dev) if cov else None
    out = torch.full((rows * S, H * 64), float("nan"), device=dev, dtype=torch.float16)
    derr = C.c_int32(0)
    rc = tb.lib().tsb_test_attention_variate_ex(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(),
                                                out.data_ptr(), dbits.data_ptr(), drole.data_ptr() if cov else None,
                                                rows, H, S, N, G, kernel, C.byref(derr))
    assert rc == 0, (rc, derr.value)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    scale = want.abs().max().item()
    err = (got - want).abs()
    rel = 2e-3 if kernel == 1 else 4e-3
    assert (err <= rel * scale + want.abs() * 2.0 ** -10).all(), float(err.max())


@pytest.mark.parametrize("S,N,L,cov,kernel,dense", [(1056, 1024, 1024, 0, 2, False), (300, 280, 280, 0, 2, False),
                                                    (129, 128, 128, 0, 2, False), (72, 64, 64, 0, 2, False),
                                                    (1, 1, 1, 0, 2, False), (200, 190, 190, 0, 0, False),
                                                    (140, 70, 64, 1, 2, False), (1200, 600, 560, 1, 2, False),
                                                    (2112, 1056, 1024, 1, 0, False), (72, 36, 32, 1, 2, False),
                                                    (1056, 1024, 1024, 0, 2, True), (1200, 600, 560, 1, 2, True),
                                                    (520, 512, 512, 0, 2, True)])
def test_attention_time_long(dev, S, N, L, cov, kernel, dense):
    """Tiled tensor-core time attention (key tiles of 64, query tiles of 128, lazy rescaling
    of O) against the float64 restatement, with and without the covariate layout."""
    rows, H, bs = 5, 2, 32
    g = torch.Generator().manual_seed(S * 7 + N + cov)
    q = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    k = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    # a few large logits late in the row force the reference maximum to move (rescaling)
    k[:, :, S // 2 :: 97] *= 3
    v = torch.randn(rows, H, S, 64, generator=g).half()
    gate = torch.rand(rows, H, S, 64, generator=g).half()
    valid = torch.rand(rows, N, generator=g) > (0.0 if dense else 0.2)   # dense: unmasked key tiles
    if dense:
        valid[:] = True
    role = torch.tensor([0, 1, 2, 2, 0][:rows], dtype=torch.int8)
    words = (N + 31) // 32
    bits = np.zeros((rows, words), np.uint32)
    vn = valid.numpy()
    for p in range(N):
        bits[:, p // 32] |= vn[:, p].astype(np.uint32) << np.uint32(p % 32)
    allowed = time_mask_torch(valid, role, N, L, S, cov, bs).to(dev)
    qd, kd, vd, gd = (t.to(dev).double() for t in (q, k, v, gate))
    s = torch.einsum("rhqd,rhkd->rhqk", qd, kd) / 8.0
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    want = torch.einsum("rhqk,rhkd->rhqd", torch.softmax(s, dim=-1), vd) * gd
    del s
    want = want.permute(0, 2, 1, 3).reshape(rows * S, H * 64).cpu()
    dbits = torch.from_numpy(bits.view(np.int32)).to(dev)
    drole = role.to(dev)
    out = torch.full((rows * S, H * 64), float("nan"), device=dev, dtype=torch.float16)
    err = C.c_int32(0)
    dq, dk, dv, dg = q.to(dev), k.to(dev), v.to(dev), gate.to(dev)
    rc = tb.lib().tsb_test_attention_time_ex(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), out.data_ptr(),
                                             dbits.data_ptr(), drole.data_ptr(), rows, H, S, N, L, cov, bs, kernel, 0, None,
                                             C.byref(err))
    assert rc == 0, (rc, err.value)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    scale = want.abs().reshape(rows, S, H, 64).amax(dim=(1, 3), keepdim=True).expand(rows, S, H, 64).reshape(rows * S, H * 64)
    tol = 4e-3 * scale + want.abs() * 2.0 ** -10
    bad = (got - want).abs() > tol
    assert not bad.any(), f"max err {(got - want).abs().max().item():.3e} at {bad.nonzero()[:4].tolist()}"


@pytest.mark.parametrize("S,N,L,cov,rows,H", [(36, 32, 32, 0, 37, 3), (9, 8, 8, 0, 5, 3), (64, 60, 60, 0, 7, 12),
                                              (33, 30, 30, 0, 11, 2), (1, 1, 1, 0, 3, 1), (48, 24, 20, 1, 5, 2),
                                              (16, 16, 16, 0, 1, 1), (64, 32, 32, 1, 5, 3)])
def test_attention_time_tc_two_problems_per_tile(dev, S, N, L, cov, rows, H):
    """Rows of S <= 64 tokens run two (row, head) problems per 128-query score tile (their keys
    side by side, each query's key set moved to its problem's block); the outputs equal the
    one-problem-per-tile kernel's bit for bit, including an odd problem count (the last tile
    holds one problem) and the covariate layout, and the float64 restatement within the
    kernel tolerance."""
    bs = 4
    g = torch.Generator().manual_seed(S * 31 + N + cov + rows)
    q = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    k = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    v = torch.randn(rows, H, S, 64, generator=g).half()
    gate = torch.rand(rows, H, S, 64, generator=g).half()
    valid = torch.rand(rows, N, generator=g) > 0.2
    valid[:, 0] = True
    role = torch.tensor([0, 1, 2, 2, 0, 1, 2] * ((rows + 6) // 7), dtype=torch.int8)[:rows]
    words = (N + 31) // 32
    bits = np.zeros((rows, words), np.uint32)
    vn = valid.numpy()
    for p in range(N):
        bits[:, p // 32] |= vn[:, p].astype(np.uint32) << np.uint32(p % 32)
    dq, dk, dv, dg = q.to(dev), k.to(dev), v.to(dev), gate.to(dev)
    dbits = torch.from_numpy(bits.view(np.int32)).to(dev)
    drole = role.to(dev)
    outs = []
    for kernel in (1, 4):
        out = torch.full((rows * S, H * 64), float("nan"), device=dev, dtype=torch.float16)
        err = C.c_int32(0)
        rc = tb.lib().tsb_test_attention_time_ex(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(),
                                                 out.data_ptr(), dbits.data_ptr(), drole.data_ptr(), rows, H, S, N, L,
                                                 cov, bs, kernel, 0, None, C.byref(err))
        assert rc == 0, (kernel, rc, err.value)
        outs.append(out.cpu())
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    allowed = time_mask_torch(valid, role, N, L, S, cov, bs)
    s = torch.einsum("rhqd,rhkd->rhqk", q.double(), k.double()) / 8.0
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    want = (torch.einsum("rhqk,rhkd->rhqd", torch.softmax(s, dim=-1), v.double()) * gate.double())
    want = want.permute(0, 2, 1, 3).reshape(rows * S, H * 64)
    got = outs[0].double()
    assert torch.isfinite(got).all()
    scale = want.abs().reshape(rows, S, H, 64).amax(dim=(1, 3), keepdim=True).expand(rows, S, H, 64).reshape(rows * S, H * 64)
    assert not ((got - want).abs() > 4e-3 * scale + want.abs() * 2.0 ** -10).any()


@pytest.mark.parametrize("S,N,L,cov,rows,H", [(18, 16, 16, 0, 3, 2), (72, 64, 64, 0, 5, 3), (200, 190, 190, 0, 3, 2),
                                              (1056, 1024, 1024, 0, 2, 2), (140, 70, 64, 1, 5, 2),
                                              (2112, 1056, 1024, 1, 2, 1), (33, 33, 33, 0, 4, 1)])
def test_attention_time_simt_tiled_same_bits(dev, S, N, L, cov, rows, H):
    """The tiled CUDA-core time attention (key and value tiles in shared memory, 16 queries per
    block) against the warp-per-query kernel: the reference's operation order in both, so the
    outputs are the same bits, with and without the covariate layout, up to 2,112 tokens."""
    bs = 32
    g = torch.Generator().manual_seed(S * 13 + N + cov)
    q = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    k = (torch.randn(rows, H, S, 64, generator=g) * 2).half()
    v = torch.randn(rows, H, S, 64, generator=g).half()
    gate = torch.rand(rows, H, S, 64, generator=g).half()
    valid = torch.rand(rows, N, generator=g) > 0.2
    valid[:, 0] = True
    role = torch.tensor([0, 1, 2, 2, 0][:rows], dtype=torch.int8)
    words = (N + 31) // 32
    bits = np.zeros((rows, words), np.uint32)
    vn = valid.numpy()
    for p in range(N):
        bits[:, p // 32] |= vn[:, p].astype(np.uint32) << np.uint32(p % 32)
    dq, dk, dv, dg = q.to(dev), k.to(dev), v.to(dev), gate.to(dev)
    dbits = torch.from_numpy(bits.view(np.int32)).to(dev)
    drole = role.to(dev)
    outs = []
    for kernel in (5, 6):
        out = torch.full((rows * S, H * 64), float("nan"), device=dev, dtype=torch.float16)
        err = C.c_int32(0)
        rc = tb.lib().tsb_test_attention_time_ex(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(),
                                                 out.data_ptr(), dbits.data_ptr(), drole.data_ptr(), rows, H, S, N, L,
                                                 cov, bs, kernel, 0, None, C.byref(err))
        assert rc == 0, (kernel, rc, err.value)
        outs.append(out.cpu())
    assert torch.isfinite(outs[0].float()).all()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
