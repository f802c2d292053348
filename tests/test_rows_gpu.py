"""Row kernels of the device path against the CPU oracle, through the kernel-level C-ABI
test entries: RMSNorm must match the oracle's restatement of the reference's float sum
cascade (reference src/layers.cpp:262-287, src/torch_sum.hpp:9-23) bit for bit."""
import ctypes as C

import numpy as np
import pytest

import oracle_py as op
import timestral_b200 as tb
from timestral_b200 import synthetic as sy

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


@pytest.mark.parametrize("R,T,patches,ps", [(64, 2048, 8, 32), (37, 512, 3, 32), (5, 96, 2, 8), (9, 4096, 33, 32)])
def test_refine_bitwise(dev, R, T, patches, ps):
    """Refine of one decode block (reference src/refine.cpp:32-106), with its scratch from the
    allocator as inside a forecast, equals the oracle's float64 restatement bit for bit: the
    warp-parallel kernel keeps every operation and its order."""
    from helpers import unit_config
    Q, mi = 21, 10
    rng = np.random.default_rng(R * 7 + T)
    x = (np.cumsum(rng.standard_normal((R, T)), axis=1) + rng.uniform(-50, 50, (R, 1))).astype(np.float32)
    m = (rng.random((R, T)) > 0.1).astype(np.int8)
    x[m == 0] = 0
    c = unit_config(patch_size=ps, minimum_scale=1e-6)
    _, loc, sc = op.scale_rows(c, x, m, R, T)
    loc0 = np.ascontiguousarray(loc.reshape(R, T)[:, -1])
    sc0 = np.ascontiguousarray(sc.reshape(R, T)[:, -1])
    q = np.sort(rng.standard_normal((R, patches * ps, Q)).astype(np.float32) * sc0[:, None, None] + loc0[:, None, None],
                axis=-1).astype(np.float32)
    role = np.zeros(R, np.int8)
    role[-1] = 2
    want = op.refine_block(c, q, x.reshape(-1), m.reshape(-1), R, T, patches, (role == 0).astype(np.int8))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dx, dm, dr, dl, ds = t(q), t(x), t(m), t(role), t(loc0), t(sc0)
    out = torch.full_like(dq, float("nan"))
    rc = tb.lib().tsb_test_refine(dq.data_ptr(), dx.data_ptr(), dm.data_ptr(), dr.data_ptr(), dl.data_ptr(),
                                  ds.data_ptr(), R, T, patches, ps, Q, mi, C.c_double(1e-6), out.data_ptr())
    assert rc == 0, rc
    got = out.cpu().numpy()
    want = want.reshape(got.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())


@pytest.mark.parametrize("name", ["refine_ps32_T256", "refine_ps8_T40"])
def test_refine_matches_reference_golden(dev, name):
    """The device refine against the reference's own refine_block output (tests/golden,
    written by the reference's compiled src/refine.cpp), bit for bit. The anchor frame it
    takes is the scaler's frame at the last context step (pinned to the same reference)."""
    import json
    from helpers import unit_config
    d = np.load(GOLDEN / f"{name}.npz")
    cfg = json.loads(str(d["config"]))
    R, T, patches, ps = cfg["R"], cfg["T"], cfg["patches"], cfg["patch_size"]
    c = unit_config(patch_size=ps, minimum_scale=cfg["minimum_scale"])
    _, loc, sc = op.scale_rows(c, d["x"], d["m"], R, T)
    loc0 = np.ascontiguousarray(loc.reshape(R, T)[:, -1])
    sc0 = np.ascontiguousarray(sc.reshape(R, T)[:, -1])
    role = (d["targets"] == 0).astype(np.int8)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dx, dm, dr, dl, ds = t(d["q"]), t(d["x"]), t(d["m"]), t(role), t(loc0), t(sc0)
    out = torch.full_like(dq, float("nan"))
    rc = tb.lib().tsb_test_refine(dq.data_ptr(), dx.data_ptr(), dm.data_ptr(), dr.data_ptr(), dl.data_ptr(),
                                  ds.data_ptr(), R, T, patches, ps, 21, 10, C.c_double(cfg["minimum_scale"]), out.data_ptr())
    assert rc == 0, rc
    assert np.array_equal(out.cpu().numpy().view(np.uint32), d["refined"].view(np.uint32))


@pytest.mark.parametrize("R,W,ps,attend", [(5, 3072, 32, 1), (3, 96, 32, 0), (4, 1056, 32, 1), (2, 2400, 48, 1),
                                           (3, 32768, 32, 1), (70, 2048, 32, 1)])
def test_scale_rows_block_form(dev, R, W, ps, attend):
    """The block-per-row scaler (long rows) equals the one-thread-per-row form bit for bit on
    every output, and its anchor frame equals the oracle's causal scaler (reference
    src/scaler.cpp:27-58) at the anchor step."""
    rng = np.random.default_rng(W + R)
    x = (np.cumsum(rng.standard_normal((R, W)), axis=1) * rng.uniform(0.01, 50, (R, 1))).astype(np.float32)
    m = (rng.random((R, W)) > 0.1).astype(np.int8)
    lead = rng.integers(0, W // 2, R)
    for i in range(R):
        m[i, : lead[i]] = 0          # left padding: leading unobserved patches
    x[m == 0] = 0.0
    enc = W // ps - 1
    anchor, ctx_len = (enc * ps) - 1, enc * ps
    dx, dm = torch.from_numpy(x).to(dev), torch.from_numpy(m).to(dev)
    outs = []
    for kernel in (0, 1):
        feat = torch.full((R, W // ps, 2 * ps), float("nan"), device=dev)
        loc, sc, clo, chi, csc = (torch.full((R,), float("nan"), device=dev) for _ in range(5))
        kv = torch.zeros((R, (enc + 31) // 32), dtype=torch.int32, device=dev)
        fo = torch.full((R,), -7, dtype=torch.int32, device=dev)
        rc = tb.lib().tsb_test_scale_rows(dx.data_ptr(), dm.data_ptr(), R, W, ps, C.c_double(1e-6), 1, attend, anchor, enc,
                                          ctx_len, kernel, feat.data_ptr(), loc.data_ptr(), sc.data_ptr(), kv.data_ptr(),
                                          fo.data_ptr(), clo.data_ptr(), chi.data_ptr(), csc.data_ptr())
        assert rc == 0, rc
        outs.append([t.cpu().numpy() for t in (feat, loc, sc, kv, fo, clo, chi, csc)])
    for a, b in zip(*outs):
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    c = op.make_config(sy.spec_209m())
    c.patch_size = ps
    c.minimum_scale = 1e-6
    _, oloc, osc = op.scale_rows(c, x, m, R, W)
    oloc, osc = oloc.reshape(R, W), osc.reshape(R, W)
    assert np.array_equal(outs[1][1].view(np.uint32), oloc[:, anchor].view(np.uint32))
    assert np.array_equal(outs[1][2].view(np.uint32), osc[:, anchor].view(np.uint32))


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("D", [128, 768])
def test_rms_matches_reference_golden(dev, D):
    """Device RMSNorm against the reference's own output (tests/golden, written by the
    reference's compiled src/layers.cpp), bit for bit."""
    d = np.load(GOLDEN / f"rms_norm_D{D}.npz")
    x, w = d["x"], d["w"]
    dx, dw = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
    out = torch.empty(x.shape, device=dev)
    assert tb.lib().tsb_test_rms(dx.data_ptr(), dw.data_ptr(), x.shape[0], D, C.c_float(1e-6), out.data_ptr(), 0) == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint32), d["out"].view(np.uint32))


@pytest.mark.parametrize("kernel", [0, 1])
def test_scaler_matches_reference_golden(dev, kernel):
    """Both device scaler forms: the frame at every patch end equals the reference's own
    running loc/scale there (tests/golden, written by the reference's compiled
    src/scaler.cpp), bit for bit."""
    d = np.load(GOLDEN / "scale_rows_ps32_T256.npz")
    x, m = d["x"], d["m"]
    R, W = x.shape
    ps = 32
    ref_loc, ref_scale = d["loc"].reshape(R, W), d["scale"].reshape(R, W)
    dx, dm = torch.from_numpy(x).to(dev), torch.from_numpy(m).to(dev)
    enc = W // ps
    for anchor in range(ps - 1, W, ps):
        feat = torch.empty((R, W // ps, 2 * ps), device=dev)
        loc, sc = torch.empty(R, device=dev), torch.empty(R, device=dev)
        kv = torch.zeros((R, (enc + 31) // 32), dtype=torch.int32, device=dev)
        fo = torch.empty(R, dtype=torch.int32, device=dev)
        rc = tb.lib().tsb_test_scale_rows(dx.data_ptr(), dm.data_ptr(), R, W, ps, C.c_double(1e-6), 1, 1, anchor, enc,
                                          W, kernel, feat.data_ptr(), loc.data_ptr(), sc.data_ptr(), kv.data_ptr(),
                                          fo.data_ptr(), None, None, None)
        assert rc == 0
        assert np.array_equal(loc.cpu().numpy().view(np.uint32), ref_loc[:, anchor].view(np.uint32)), anchor
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), ref_scale[:, anchor].view(np.uint32)), anchor
