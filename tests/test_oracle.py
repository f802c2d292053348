"""Known-answer tests that pin the CPU oracle to the reference's own unit tests.

Each test restates the expected values of one reference unit test (file:line cited) and
checks the oracle against them. These run without a GPU.
"""
import math

import numpy as np
import pytest

import oracle_py as op
from helpers import unit_config, f32, bits
from timestral_b200 import synthetic as sy

FLT_MAX = np.finfo(np.float32).max


def rejects(f):
    with pytest.raises(RuntimeError):
        f()


# ---- reference tests/test_masks.cpp:5-24 ---------------------------------------------
def test_masks_units():
    c = unit_config(patch_size=2, block_size=2, attend_missing_patches=1, covariate_enabled=0)
    a = op.build_masks(c, [0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0], 2, 6, 1, [9, 9])
    assert a["obs"].tolist() == [0, 1, 0, 0, 0, 0], "patch observation"
    assert a["key_valid"].tolist() == [0, 1, 1, 0, 0, 0], "leading padding versus internal gaps"
    assert a["first_group"].tolist() == [1], "group first observed"
    c.attend_missing_patches = 0
    nm = op.build_masks(c, [0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0], 2, 6, 1, [9, 9])
    assert nm["key_valid"].tolist() == nm["obs"].tolist(), "no missing attention"
    c.attend_missing_patches = 1
    assert a["positions"].tolist() == [-1, 0, 1, 2, -1, 0, 1, 2], "shared negative positions"
    c.covariate_enabled = 1
    b = op.build_masks(c, [1, 1, 0, 0, 1, 1, 1, 1], 2, 4, 1, [5, 5], [0, 2])
    assert b["S"] == 4 and b["time"].size == 32, "covariate layout"
    assert not b["variate"][(2 * 2 + 1) * 2] and b["variate"][(2 * 2) * 2 + 1], "known firewall"
    assert b["anchor"].tolist() == [0, 1, 0, 1] and b["active"].tolist() == [0, 1, 0, 1], "block layout"
    empty = op.build_masks(c, [0, 0], 1, 2, 1, [0])
    assert empty["first_group"].tolist() == [0] and empty["time"].tolist() == [1, 0, 0, 1], "all missing self diagonals"
    multi = op.build_masks(c, [1] * 12, 1, 12, 4, [0], [1])
    assert multi["anchor"].tolist() == [0, 0, 2, 2, 4, 4], "multiple active blocks"
    t = multi["time"]
    assert t[(6 + 4) * 12 + 2] and t[(6 + 4) * 12 + 3] and not t[(6 + 4) * 12 + 4], "block decoder anchor boundary"
    rejects(lambda: op.build_masks(c, [2, 0], 1, 2, 1, [0]))
    rejects(lambda: op.build_masks(c, [1, 0], 1, 2, 1, [0], [3]))


# ---- reference tests/test_scaler.cpp:15-58 --------------------------------------------
def test_scaler_units():
    c = unit_config(patch_size=2, minimum_scale=0.00001, use_asinh=1)
    x = [0, -0.0, 0, 0, 5, 5, 5, 5, 0, 1, 0, 1, -2, 0, 2, 4]
    m = [0, 0, 0, 0] + [1] * 12
    s, loc, sc = op.scale_rows(c, x, m, 4, 4)
    ms = np.float32(c.minimum_scale)
    assert loc[0] == 0 and sc[0] == ms and s[1] == 0 and not math.copysign(1, s[1]) < 0, "masked signed zero"
    assert loc[4] == 5 and sc[4] == ms, "constant floor"
    assert loc[12] == -1 and sc[12] == np.sqrt(np.float32(2)) and loc[15] == 1, "causal patch last sample statistics"
    l2, s2, b2 = op.instance_norm_stats(c, x, m, 4, 4)
    assert b2.tolist() == [0, 0, 1, 0] and l2[2] == 0 and s2[2] == 1, "indicator exact"
    assert l2[3] == 1 and s2[3] == np.sqrt(np.float32(5)), "population variance"
    xn = list(x)
    xn[0] = float("nan")
    s3, l3, _ = op.scale_rows(c, xn, m, 4, 4)
    assert np.isnan(l3[0]) and s3[0] == 0, "unprepared NaN propagates stats, masked output zero"
    cl = op.denormalize([-np.inf, 2, np.inf, np.nan, np.inf, -np.inf, np.nan, np.inf], [0, 0], [1, 1], 4, False)
    assert cl[0] == 2 and cl[2] == 2 and np.isnan(cl[3]) and cl[4] == 0 and cl[5] == 0 and np.isnan(cl[6]), "clamp_nonfinite"
    assert op.denormalize([0, 1, 2], [3], [2], 3, False).tolist() == [3, 5, 7], "inverse affine no asinh"
    rejects(lambda: op.scale_rows(c, [1], [1], 1, 1))
    rejects(lambda: op.scale_rows(c, [1, 2], [1, 2], 1, 2))
    small = unit_config(patch_size=2, minimum_scale=1e-12, use_asinh=1)
    e, _, _ = op.scale_rows(small, [0, 1e-10], [1, 1], 1, 2)
    assert abs(e[0]) < 0.001, "float32 epsilon affine clamp"
    ov = op.denormalize([-1000, 0, 1000, np.nan], [2], [3], 4, True)
    assert ov[0] == 2 and ov[1] == 2 and ov[2] == 2 and np.isnan(ov[3]), "sinh overflow clamp preserves NaN"
    sz, _, _ = op.scale_rows(c, [-0.0, 0.0], [1, 1], 1, 2)
    assert math.copysign(1, sz[0]) < 0, "observed negative zero preserved"


# ---- reference tests/test_refine.cpp:7-50 ---------------------------------------------
def test_refine_units():
    c = unit_config(patch_size=2, minimum_scale=1, knots=[0.1, 0.5, 0.9])
    loc, sc = op.block_frames(c, [0, 0], [1, 1], [2, 2, 0, 0], 1, 2, 2)
    assert loc.tolist() == [0, 1], "causal folding mean"
    assert abs(sc[1] - math.sqrt(4.0 / 3)) < 1e-15, "Bessel scale"
    pair = unit_config(patch_size=8, minimum_scale=1, knots=[0.1, 0.5, 0.9])
    cl, _ = op.block_frames(pair, [2.0 ** 60, 1, -(2.0 ** 60), 1, 1, 1, 1, 1], [1] * 8, [0] * 16, 1, 8, 2)
    assert cl[0] == 0.5, "NumPy pairwise cancellation, not sequential reduction"
    ll, ls = op.block_frames(c, [1e30, 1e30], [1, 1], [1e300, -1e300, 0, 0], 1, 2, 2)
    assert ll[1] == float(np.float32(1e30)) and np.isfinite(ls[1]), "clip relative to offset preserves large level"
    el, es = op.block_frames(c, [99, 99], [0, 0], [0, 0, 0, 0], 1, 2, 2)
    assert el.tolist() == [0, 0] and es.tolist() == [1, 1], "zero weight identity"
    q = np.full(12, 2, np.float32)
    r = op.refine_block(c, q, [0, 0], [1, 1], 1, 2, 2)
    assert r[0] == 2 and r[6] == np.float32(np.float32(2 * np.float32(math.sqrt(4.0 / 3))) + 1), "float32 affine stages"
    mx = FLT_MAX
    ovf = [mx, -mx, -mx, mx, -mx, -mx, mx, -mx, -mx, mx, -mx, -mx]
    sat = op.refine_block(c, ovf, [-mx, -mx], [1, 1], 1, 2, 2)
    assert np.all(sat == -mx), "float32 subtract overflow clamps to finite quantile"
    nq = np.zeros(12, np.float32)
    nq[0] = np.nan
    assert np.isnan(op.refine_block(c, nq, [0, 0], [1, 1], 1, 2, 2)[0]), "refine keeps NaN"
    q2 = q.copy()
    q2[0], q2[1], q2[2] = -0.0, np.inf, np.nan
    unchanged = op.refine_block(c, q2, [0, 0], [1, 1], 1, 2, 2, [0])
    assert np.array_equal(bits(q2), bits(unchanged)), "covariates preserve bits"
    single = np.array([-0.0, np.nan, np.inf, 1, 2, 3], np.float32)
    bypass = op.refine_block(c, single, [], [], 1, 0, 1)
    assert np.array_equal(bits(single), bits(bypass)), "single patch reference early return"
    xl, xs = op.block_frames(c, [0, 0], [1, 1], [np.inf, -np.inf, 0, 0], 1, 2, 2)
    assert np.isfinite(xs[1]) and xs[1] > 1e15, "fold infinities at clip before moments"
    nl, ns = op.block_frames(c, [0, 0], [1, 1], [np.nan, 0, 0, 0], 1, 2, 2)
    assert np.isnan(nl[1]) and np.isnan(ns[1]), "NaN must surface"


# ---- reference tests/test_head.cpp:10-21 (monotone head) -------------------------------
def test_monotone_units():
    c = op.make_config(sy.spec_tiny())
    Q = c.num_quantiles
    mi = [i for i in range(Q) if c.knots[i] == 0.5][0]
    sp = np.zeros(Q, np.float32)
    sp[mi] = np.nan
    rejects(lambda: op.monotone_quantiles(c, sp))
    for v in (np.inf, -np.inf):
        sp = np.full(Q, v, np.float32)
        sp[mi] = 0
        assert np.all(np.isfinite(op.monotone_quantiles(c, sp))), "infinite raw clamped"
    for v in (1000, -1000):
        out = op.monotone_quantiles(c, np.full(Q, v, np.float32))
        assert np.all(np.diff(out) >= 0), "nondecreasing"
    raw = np.zeros(3 * Q, np.float32)
    raw[Q + mi] = -100
    out = op.monotone_quantiles(c, raw).reshape(3, Q)
    assert np.all(np.diff(out, axis=1) >= 0)
    assert out[0, mi] == 0 and out[1, mi] == -100, "median unchanged"
    rejects(lambda: op.monotone_quantiles(c, np.ones(1, np.float32)))


# ---- reference src/numpy_sum.hpp / tests/test_refine.cpp:14 cancellation ---------------
def test_numpy_sum_matches_numpy():
    rng = np.random.default_rng(3)
    for n in (0, 1, 7, 8, 9, 31, 127, 128, 129, 300, 1000, 4097):
        x = np.ascontiguousarray(rng.standard_normal(n) * 10.0 ** rng.integers(-5, 5, n))
        got = op.lib().oracle_numpy_sum(op.ptr(x), n)
        assert got == float(np.add.reduce(x)) or n == 0, n


def test_torch_sum_matches_torch():
    import torch
    rng = np.random.default_rng(4)
    for n in (1, 5, 8, 31, 32, 33, 100, 1000, 2048, 4096, 33000):
        x = f32(rng.standard_normal(n) * 3)
        got = op.lib().oracle_torch_sum_f32(op.ptr(x), n)
        want = torch.from_numpy(x).sum().item()
        assert got == want, (n, got, want)


def test_rms_norm_matches_torch_cascade():
    """The RMSNorm mean follows ATen's float sum cascade (reference src/layers.cpp:257-278)."""
    import torch
    rng = np.random.default_rng(5)
    for D in (32, 64, 96, 128, 768, 800):
        x = f32(rng.standard_normal((3, D)))
        w = f32(rng.standard_normal(D))
        got = op.rms_norm(x, w, 1e-6)
        xt = torch.from_numpy(x)
        mean = (xt * xt).sum(dim=-1, keepdim=True) / np.float32(D)
        inv = 1.0 / torch.sqrt(mean + np.float32(1e-6))
        want = ((xt * inv) * torch.from_numpy(w)).numpy()
        assert np.array_equal(bits(got), bits(want)), D


# ---- reference tests/test_attention.cpp: SDPA sweep, R=1 variate identity --------------
def _sdpa_py(q, k, v, mask, hd, H, S, R, split):
    """Scalar restatement of the reference SDPA (src/layers.cpp:578-617) in numpy float32/64."""
    D = H * hd
    out = np.zeros_like(q)
    scale = np.float32(1 / math.sqrt(hd))
    aexp = op.lib().oracle_attention_exp
    for r in range(R):
        for h in range(H):
            for t in range(S):
                keys = split if (split and t < split) else S
                qv = q[(r * S + t) * D + h * hd:(r * S + t) * D + h * hd + hd].astype(np.float64)
                lg = np.empty(keys, np.float32)
                for j in range(keys):
                    kv = k[(r * S + j) * D + h * hd:(r * S + j) * D + h * hd + hd].astype(np.float64)
                    s = 0.0
                    for d in range(hd):
                        s += qv[d] * kv[d]
                    lg[j] = np.float32(np.float32(s) * scale) + mask[(r * S + t) * S + j]
                mx = lg.max()
                end = keys // 8 * 8
                p = np.empty(keys, np.float32)
                sums = np.zeros(8, np.float32)
                for j in range(keys):
                    p[j] = aexp(float(lg[j] - mx)) if j < end else np.float32(math.exp(float(np.float32(lg[j] - mx))))
                    if j < end:
                        sums[j % 8] = np.float32(sums[j % 8] + p[j])
                a0, a1, a2, a3 = (np.float32(sums[i] + sums[i + 4]) for i in range(4))
                tot = np.float32(np.float32(a0 + a2) + np.float32(a1 + a3))
                for j in range(end, keys):
                    tot = np.float32(tot + p[j])
                rec = np.float32(np.float32(1) / tot)
                for d in range(hd):
                    acc = np.float32(0)
                    for j in range(keys):
                        vv = v[(r * S + j) * D + h * hd + d]
                        if hd < 16:
                            acc = np.float32(acc + np.float32(p[j] * vv))
                        else:
                            acc = np.float32(np.float64(p[j]) * np.float64(vv) + np.float64(acc))
                    out[(r * S + t) * D + h * hd + d] = np.float32(acc * rec)
    return out


@pytest.mark.parametrize("hd,S,split", [(8, 9, 0), (8, 7, 4), (16, 17, 8), (64, 18, 16), (7, 3, 1), (17, 25, 22)])
def test_sdpa_scalar_restatement(hd, S, split):
    rng = np.random.default_rng(821 + hd * 100 + S)
    H, R = 2, 2
    D = H * hd
    q = f32(rng.integers(-1024, 1025, R * S * D) / 1024)
    k = f32(rng.integers(-1024, 1025, R * S * D) / 1024)
    v = f32(rng.integers(-1024, 1025, R * S * D) / 1024)
    mask = np.zeros(R * S * S, np.float32)
    for r in range(R):
        for t in range(S):
            for j in range(S):
                mask[(r * S + t) * S + j] = -np.inf if j > t else 0
    got = op.sdpa(q, k, v, mask, hd, H, S, R, split, threads=3)
    want = _sdpa_py(q, k, v, mask, hd, H, S, R, split)
    # float32 fma in numpy is emulated in float64 then rounded (exact for one fma).
    assert np.array_equal(bits(got), bits(want))


def test_sdpa_single_key_is_v():
    """R=1 variate attention returns v bitwise (reference tests/layer_kind_test.hpp:31-33)."""
    rng = np.random.default_rng(9)
    hd, H = 64, 3
    q, k, v = (f32(rng.standard_normal(H * hd)) for _ in range(3))
    out = op.sdpa(q, k, v, np.zeros(1, np.float32), hd, H, 1, 1)
    assert np.array_equal(bits(out), bits(v))


def test_linear_panels():
    """F32 linear: 192-wide K panels (reference src/layers.cpp:200-219)."""
    rng = np.random.default_rng(11)
    for K in (64, 191, 192, 200, 768):
        w = f32(rng.standard_normal((40, K)))
        x = f32(rng.standard_normal((5, K)))
        b = f32(rng.standard_normal(40))
        got = op.linear_f32(w, x, b)
        want = np.empty_like(got)
        for r in range(5):
            for n in range(40):
                s = np.float32(0)
                for st in range(0, K, 192):
                    p = np.float32(0)
                    for j in range(st, min(K, st + 192)):
                        p = np.float32(np.float64(w[n, j]) * np.float64(x[r, j]) + np.float64(p))
                    s = p if K < 192 else np.float32(s + p)
                want[r, n] = np.float32(s + b[n])
        assert np.array_equal(bits(got), bits(want)), K


# ---- reference tests/test_forecast.cpp:39-53 (invariants I6.4, I6.5, I6.6) --------------
@pytest.fixture(scope="module")
def tiny_oracle(tmp_path_factory):
    p = sy.write_gguf(tmp_path_factory.mktemp("m") / "tiny.gguf", sy.spec_tiny(), "f32")
    return op.OracleModel(p)


def test_forecast_invariants(tiny_oracle):
    m = tiny_oracle
    ctx = (np.arange(44) % 13 - 6).astype(np.float32).reshape(2, 2, 11)
    ctx[0, 0, 0] = np.nan
    ctx[0, 0, 3] = np.nan
    H = 8 + 1
    op.set_per_shot(m, 1)
    try:
        a = m.forecast(ctx, H, clip=0, threads=1)
        again = m.forecast(ctx, H, clip=0, threads=1)
        threaded = m.forecast(ctx, H, clip=0, threads=2)
        assert np.array_equal(bits(a), bits(again)), "I6.5 repeated"
        assert np.array_equal(bits(a), bits(threaded)), "I6.5 threads 1 vs 2"
        neg = m.forecast(-ctx, H, clip=0, threads=1)
        assert np.array_equal(bits(a), bits(-neg[..., ::-1])), "I6.4 bitwise sign symmetry clip off"
        assert np.all(np.isfinite(a)) and np.all(np.diff(a, axis=-1) >= 0), "I6.6"
        clipped = m.forecast(np.abs(ctx), H, clip=1, threads=1)
        assert np.all(clipped >= 0), "nonnegative clipping"
        rejects(lambda: m.forecast(ctx, H, mask=np.full(ctx.shape, 2, np.uint8)))
    finally:
        op.set_per_shot(m, 0)
