"""tcgen05 GEMM with fused epilogues vs a torch float64 reference of the same op.

Operands are f16 and products of f16 values are exact in f32, so the only difference from
the float64 reference is the f32 accumulation order: tolerance 2e-5 * sqrt(K) relative to
the row scale, plus one f16 rounding (2^-11 relative) for f16 outputs.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import timestral_b200 as tb


def dp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def run(kind, A, B, M, N, K, out=None, ldo=0, bias=None, resid=None, row_group=0, row_stride=0, row_offset=0,
        qkvg=None, S=0, H=0, D=0, rope=0, cos=None, sin=None, rope_row=None, rope_half=32, rope_dup=0,
        a_group=0, a_stride=0, a_offset=0, Bq=None, Bd=None, ldd=0, Bs=None, lds=0):
    t = tb.GemmTest()
    t.kind, t.A, t.lda, t.B, t.ldb = kind, dp(A), A.shape[1], dp(B), B.shape[1]
    t.M, t.N, t.K = M, N, K
    t.out, t.ldo, t.bias, t.resid = dp(out), ldo, dp(bias), dp(resid)
    t.row_group, t.row_stride, t.row_offset = row_group, row_stride, row_offset
    if qkvg is not None:
        for i in range(4):
            t.qkvg[i] = qkvg[i].data_ptr()
    t.S, t.H, t.D, t.rope = S, H, D, rope
    t.cos_tab, t.sin_tab, t.rope_row, t.rope_half = dp(cos), dp(sin), dp(rope_row), rope_half
    t.rope_dup = rope_dup
    t.a_group, t.a_stride, t.a_offset = a_group, a_stride, a_offset
    t.Bq, t.Bd, t.ldd = dp(Bq), dp(Bd), ldd
    t.Bs, t.lds = dp(Bs), lds
    if Bq is not None:
        t.B, t.ldb = None, Bq.shape[1]
    err = C.c_int32(0)
    rc = tb.lib().tsb_test_gemm(C.byref(t), C.byref(err))
    assert rc == 0, (rc, err.value)


def ref_mm(A, B):
    return (A.double() @ B.double().T)


def close(got, want, K, f16=False):
    got = got.double()
    scale = want.abs().max().item() + 1e-30
    tol = 2e-5 * np.sqrt(K) * scale + (want.abs() * 2.0 ** -10 if f16 else 0)
    bad = (got - want).abs() > tol
    assert not bad.any(), f"max err {(got - want).abs().max().item():.3e} scale {scale:.3e}"


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.manual_seed(0)
    return torch.device("cuda:0")


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 768, 768), (77, 96, 32), (1000, 2304, 768), (513, 672, 3072)])
def test_f32_store(dev, M, N, K):
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    bias = torch.randn(N, device=dev)
    out = torch.full((M, N), float("nan"), device=dev)
    run(0, A, B, M, N, K, out=out, ldo=N, bias=bias)
    close(out, ref_mm(A, B) + bias.double(), K)


def test_f16_store(dev):
    M, N, K = 700, 512, 256
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    out = torch.zeros(M, N, device=dev, dtype=torch.float16)
    run(1, A, B, M, N, K, out=out, ldo=N)
    close(out, ref_mm(A, B), K, f16=True)


@pytest.mark.parametrize("group,R", [(8, 300), (1, 517), (32, 9), (4, 1024)])
def test_row_gather_decoder_tokens(dev, group, R):
    """The decoder-token tail: accumulator row m reads A row (m / g) * S + N + m % g (a 3D
    tensor-map gather, g decoder tokens of every S-token row) and writes its residual row at
    the same position; the other rows of the residual stream are untouched."""
    S, Nn, K, N = 72 if group <= 8 else 80, 64 if group <= 8 else 48, 768, 768
    A = torch.randn(R * S, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    x = torch.randn(R * S, N, device=dev)
    x0 = x.clone()
    M = R * group
    run(2, A, B, M, N, K, out=x, ldo=N, resid=x, row_group=group, row_stride=S, row_offset=Nn,
        a_group=group, a_stride=S, a_offset=Nn)
    rows = (torch.arange(M, device=dev) // group) * S + Nn + torch.arange(M, device=dev) % group
    want = x0.clone().double()
    want[rows] += ref_mm(A[rows], B)
    close(x, want, K)
    keep = torch.ones(R * S, dtype=torch.bool, device=dev)
    keep[rows] = False
    assert torch.equal(x[keep], x0[keep])


@pytest.mark.parametrize("K", [768, 2048])
def test_resid_rows_independent_of_tile_schedule(dev, K):
    """Residual add over many tiles per CTA pair (the epilogue prefetches the residual rows
    of its next chunks ahead, across tile boundaries, for K <= 1024; longer K loads them
    into registers): every row equals the same row computed in a launch of 4,096 rows, where
    the pairs take different tiles, bit for bit, and the float64 reference within the
    accumulation tolerance. M is ragged (not a multiple of the 256-row tile)."""
    M, N = 60_001, 768
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    x0 = torch.randn(M, N, device=dev)
    full = x0.clone()
    run(2, A, B, M, N, K, out=full, ldo=N, resid=full)
    sliced = x0.clone()
    for r0 in range(0, M, 4096):
        r1 = min(M, r0 + 4096)
        part = sliced[r0:r1]
        run(2, A[r0:r1], B, r1 - r0, N, K, out=part, ldo=N, resid=part)
    assert torch.equal(full, sliced)
    close(full, x0.double() + ref_mm(A, B), K)


def q8_weights(N, K, dev, seed):
    """Random Q8_0 weights: int8 values [N][K], f16 block scales [N][K/32] (d = amax/127 of
    N(0, 0.02) rows, as the converter writes them), and the f16 weights q * d rounded once."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    d = (torch.rand(N, K // 32, generator=g) * 0.0004 + 1e-5).half()
    w16 = (q.float() * d.float().repeat_interleave(32, dim=1)).half()
    return q.to(dev), d.t().contiguous().to(dev), w16.to(dev)


@pytest.mark.parametrize("kind,M,N,K", [(0, 300, 768, 768), (0, 77, 672, 3072), (1, 700, 512, 256), (2, 513, 768, 3072),
                                        (3, 257, 3072, 768), (4, 1000, 4096, 768), (5, 130, 1536, 768)])
def test_q8_prologue_equals_f16_weights(dev, kind, M, N, K):
    """The Q8_0 prologue (int8 tiles and block scales dequantised in shared memory by the
    converter warps) gives the same bits as the GEMM on the f16 weights q * d."""
    q, dT, w16 = q8_weights(N, K, dev, seed=kind * 7 + M)
    A = torch.randn(M, K, device=dev).half()
    f32 = kind in (0, 2)
    width = N // 2 if kind in (4, 5) else N
    outs = []
    for use_q8 in (False, True):
        out = torch.full((M, width), 0.5, device=dev, dtype=torch.float32 if f32 else torch.float16)
        kw = dict(Bq=q, Bd=dT, ldd=N) if use_q8 else {}
        run(kind, A, w16, M, N, K, out=out, ldo=width, resid=out if kind == 2 else None, **kw)
        outs.append(out.cpu())
    assert torch.equal(outs[0].view(torch.int32 if f32 else torch.int16), outs[1].view(torch.int32 if f32 else torch.int16))
    if kind == 0:
        close(outs[1].to(dev), ref_mm(A, w16), K)


@pytest.mark.parametrize("kind,M,N,K,lo,hi", [(0, 300, 768, 768, -32, 32), (2, 513, 768, 3072, 0, 16),
                                              (4, 1000, 4096, 768, 0, 32), (6, 144, 3072, 768, -32, 32)])
def test_kquant_prologue_equals_f16_weights(dev, kind, M, N, K, lo, hi):
    """The scaled-int8 prologue (K-quant weights: int8 values with an f32 scale and offset per
    16 values, dequantised by the converter warps as (scale * q) - offset, each operation
    rounded in single precision, then once to f16) gives the same bits as the GEMM on those
    f16 weights. Value ranges of Q6_K (-32..31), Q4_K (0..15) and Q5_K (0..31)."""
    g = torch.Generator(device="cpu").manual_seed(kind * 13 + M)
    q = torch.randint(lo, hi, (N, K), generator=g, dtype=torch.int8)
    a = (torch.rand(N, K // 16, generator=g) * 0.003 + 1e-5)
    b = torch.rand(N, K // 16, generator=g) * (0.02 if lo == 0 else 0.0)
    w16 = ((a.repeat_interleave(16, dim=1) * q.float()) - b.repeat_interleave(16, dim=1)).half()
    ab = torch.stack([a.t(), b.t()], dim=-1).contiguous()          # [K/16][N][2]
    q, ab, w16 = q.to(dev), ab.to(dev), w16.to(dev)
    A = torch.randn(M, K, device=dev).half()
    outs = []
    for use in (False, True):
        if kind == 6:
            S, H, D = 72, 12, 768
            qkvg = [torch.zeros((M // S) * H * S * 64, device=dev, dtype=torch.float16) for _ in range(4)]
            kw = dict(Bq=q, Bs=ab, lds=N) if use else {}
            run(kind, A, w16, M, N, K, qkvg=qkvg, S=S, H=H, D=D, **kw)
            outs.append(torch.cat([t.cpu() for t in qkvg]).view(torch.int16))
            continue
        f32 = kind in (0, 2)
        width = N // 2 if kind in (4, 5) else N
        out = torch.full((M, width), 0.5, device=dev, dtype=torch.float32 if f32 else torch.float16)
        kw = dict(Bq=q, Bs=ab, lds=N) if use else {}
        run(kind, A, w16, M, N, K, out=out, ldo=width, resid=out if kind == 2 else None, **kw)
        outs.append(out.cpu().view(torch.int32 if f32 else torch.int16))
    assert torch.equal(outs[0], outs[1])


def test_resid_remap(dev):
    # Patch projection layout: accumulator row m = r*L + p lands on token row r*S + p.
    R, L, S, N, K = 9, 20, 24, 768, 3072
    M = R * L
    A = (torch.randn(M, K, device=dev) * 0.3).half()
    B = (torch.randn(N, K, device=dev) * 0.02).half()
    bias = torch.randn(N, device=dev)
    x = torch.randn(R * S, N, device=dev)
    x0 = x.clone()
    run(2, A, B, M, N, K, out=x, ldo=N, bias=bias, resid=x, row_group=L, row_stride=S)
    want = x0.double().clone()
    idx = (torch.arange(R, device=dev)[:, None] * S + torch.arange(L, device=dev)[None, :]).reshape(-1)
    want[idx] = x0.double()[idx] + (ref_mm(A, B) + bias.double())
    close(x, want, K)


def silu(x):
    return x / (1 + torch.exp(-x))


def test_silu(dev):
    M, N, K = 260, 3072, 768
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    out = torch.zeros(M, N, device=dev, dtype=torch.float16)
    run(3, A, B, M, N, K, out=out, ldo=N)
    close(out, silu(ref_mm(A, B)), K, f16=True)


def interleave_rows(W1, W2, tile=256):
    """Rows of two [F,K] matrices interleaved per tile: [W1 tile half | W2 tile half]."""
    F = W1.shape[0]
    half = tile // 2
    parts = []
    for t in range(F // half):
        parts += [W1[t * half:(t + 1) * half], W2[t * half:(t + 1) * half]]
    return torch.cat(parts, 0).contiguous()


@pytest.mark.parametrize("kind", [4, 5])
def test_paired(dev, kind):
    M, F, K = 333, 2048, 768
    A = torch.randn(M, K, device=dev).half()
    W1 = (torch.randn(F, K, device=dev) * 0.05).half()
    W2 = (torch.randn(F, K, device=dev) * 0.05).half()
    b1, b2 = torch.randn(F, device=dev), torch.randn(F, device=dev)
    W = interleave_rows(W1, W2)
    bias = interleave_rows(b1[:, None], b2[:, None])[:, 0].contiguous()
    out = torch.zeros(M, F, device=dev, dtype=torch.float16)
    run(kind, A, W, M, 2 * F, K, out=out, ldo=F, bias=bias)
    a = ref_mm(A, W1) + b1.double()
    b = ref_mm(A, W2) + b2.double()
    want = a * silu(b) if kind == 4 else a * torch.sigmoid(b)
    close(out, want, K, f16=True)


@pytest.mark.parametrize("rope", [0, 1, 2])
def test_qkvg(dev, rope):
    """rope 1: arbitrary tables (general path); rope 2: tables with equal halves, as
    emb = [freqs, freqs] gives, through the path that reads dims 0..15 only."""
    Rr, S, H, hd = 5, 72, 12, 64
    D = H * hd
    M, N, K = Rr * S, 4 * D, D
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    bias = torch.randn(N, device=dev) * 0.1
    P = 2113
    cos = torch.randn(P, 64, device=dev)
    sin = torch.randn(P, 64, device=dev)
    if rope == 2:
        cos[:, 32:] = cos[:, :32]
        sin[:, 32:] = sin[:, :32]
    rope_row = torch.randint(0, P, (M,), device=dev, dtype=torch.int32)
    bufs = [torch.zeros(Rr, H, S, 64, device=dev, dtype=torch.float16) for _ in range(4)]
    run(6, A, B, M, N, K, bias=bias, qkvg=bufs, S=S, H=H, D=D, rope=int(rope > 0), cos=cos, sin=sin,
        rope_row=rope_row, rope_half=16, rope_dup=int(rope == 2))
    acc = (ref_mm(A, B) + bias.double()).reshape(Rr, S, 4, H, hd).permute(2, 0, 3, 1, 4)  # [4,R,H,S,64]
    c = cos.double()[rope_row.long()].reshape(Rr, S, 64)[:, None]
    s = sin.double()[rope_row.long()].reshape(Rr, S, 64)[:, None]
    for which in range(4):
        want = acc[which].clone()
        if which < 2 and rope:
            x = acc[which]
            rot = torch.cat([-x[..., 32:], x[..., :32]], -1)
            active = torch.zeros(64, dtype=torch.bool, device=dev)
            active[:16] = True
            active[32:48] = True
            want = torch.where(active, x * c + rot * s, x)
        if which == 3:
            want = torch.sigmoid(want)
        close(bufs[which], want, K, f16=True)
