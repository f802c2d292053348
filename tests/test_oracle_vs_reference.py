"""Pins the CPU oracle to the reference's own code, bitwise.

oracle/_ref/libtsref.so is compiled by oracle/ref/Makefile from the reference's sources
(src/scaler.cpp, refine.cpp, covariates.cpp, masks.cpp, layers.cpp, head.cpp) where they lie;
these tests feed the same randomised inputs to both and require identical bytes. The
library only exists where the reference sources do (it is built by build() here); without
it the tests skip.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import oracle_py as op
from helpers import unit_config, f32, i8, bits
from timestral_b200 import synthetic as sy

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libtsref.so"
if not REF.exists():
    pytest.skip("oracle/_ref not built (reference sources absent)", allow_module_level=True)
ref = C.CDLL(str(REF))
ref.ref_last_error.restype = C.c_char_p
P = op.ptr
I = C.c_int64


def ok(rc):
    assert rc == 0, ref.ref_last_error().decode()


def oracle():
    return op.lib()


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    if a.dtype == np.float32:
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"max diff {np.nanmax(np.abs(a - b))}"
    elif a.dtype == np.float64:
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    else:
        assert np.array_equal(a, b)


def rows_with_gaps(rng, R, T, nan_frac=0.2):
    x = f32(rng.standard_normal((R, T)) * 10 ** rng.uniform(-3, 3, (R, 1)) + rng.uniform(-100, 100, (R, 1)))
    m = i8(rng.random((R, T)) > nan_frac)
    m[0, :] = 0                                  # an all-missing row
    if R > 2:
        m[2, : T // 2] = 0                       # late start
    x[m == 0] = 0
    x[1, min(3, T - 1)] = -0.0
    return x, m


@pytest.mark.parametrize("ps,T", [(32, 256), (8, 40), (32, 2048)])
def test_scale_rows(ps, T):
    rng = np.random.default_rng(ps + T)
    c = unit_config(patch_size=ps)
    R = 6
    x, m = rows_with_gaps(rng, R, T)
    outs = [np.empty(R * T, np.float32) for _ in range(6)]
    ok(ref.ref_scale_rows(C.byref(c), P(x), P(m), I(R), I(T), P(outs[0]), P(outs[1]), P(outs[2])))
    assert oracle().oracle_scale_rows(C.byref(c), P(x), P(m), I(R), I(T), P(outs[3]), P(outs[4]), P(outs[5])) == 0
    for a, b in zip(outs[:3], outs[3:]):
        same(a, b)


@pytest.mark.parametrize("T", [3, 7, 8, 40, 1056, 33000])
def test_instance_norm_stats(T):
    rng = np.random.default_rng(T)
    c = unit_config()
    R = 4
    x, m = rows_with_gaps(rng, R, T)
    x[3] = (rng.random(T) > 0.5).astype(np.float32)   # an indicator row
    a = [np.empty(R, np.float32), np.empty(R, np.float32), np.empty(R, np.int8)]
    b = [np.empty(R, np.float32), np.empty(R, np.float32), np.empty(R, np.int8)]
    ok(ref.ref_instance_norm_stats(C.byref(c), P(x), P(m), I(R), I(T), P(a[0]), P(a[1]), P(a[2])))
    assert oracle().oracle_instance_norm_stats(C.byref(c), P(x), P(m), I(R), I(T), P(b[0]), P(b[1]), P(b[2])) == 0
    for u, v in zip(a, b):
        same(u, v)


@pytest.mark.parametrize("cov", [False, True])
def test_build_masks(cov):
    rng = np.random.default_rng(5 + cov)
    c = unit_config(patch_size=4, block_size=3, covariate_enabled=1)
    R, T, h = 6, 40, 3
    obs = i8(rng.random((R, T)) > 0.6)
    obs[1, :20] = 0
    groups = np.array([0, 0, 0, 7, 7, 7], np.int64)
    roles = np.array([0, 1, 2, 0, 2, 1], np.int64) if cov else None
    got = op.build_masks(c, obs, R, T, h, groups, roles)
    N, S = got["N"], got["S"]
    out = {k: np.zeros_like(v) for k, v in got.items() if isinstance(v, np.ndarray)}
    out["first_group"] = np.zeros(len(np.unique(groups)), np.int64)
    ok(ref.ref_build_masks(C.byref(c), P(obs), I(R), I(T), I(h), P(groups), P(roles), P(out["obs"]),
                           P(out["key_valid"]), P(out["first_group"]), P(out["positions"]), P(out["time"]),
                           P(out["variate"]), P(out["active"]), P(out["anchor"])))
    for k in out:
        same(out[k], got[k])


@pytest.mark.parametrize("hd,S,split,R", [(64, 72, 64, 3), (64, 18, 16, 2), (8, 9, 0, 2), (16, 33, 30, 2), (7, 5, 2, 3),
                                         (64, 140, 128, 1)])
def test_sdpa(hd, S, split, R):
    """The reference SDPA (AVX2 pair path, src/layers.cpp:578-617) against the oracle's."""
    rng = np.random.default_rng(hd * 1000 + S)
    H = 2
    D = H * hd
    q, k, v = (f32(rng.standard_normal(R * S * D)) for _ in range(3))
    mask = np.where(rng.random((R, S, S)) < 0.3, -np.inf, 0).astype(np.float32)
    for r in range(R):
        for t in range(S):
            mask[r, t, t] = 0
    mask = mask.reshape(-1)
    a = np.empty(R * S * D, np.float32)
    ok(ref.ref_sdpa(P(q), P(k), P(v), P(mask), I(hd), I(H), I(S), I(R), I(split), P(a), C.c_int32(3)))
    b = op.sdpa(q, k, v, mask, hd, H, S, R, split, threads=2)
    same(a, b)


@pytest.mark.parametrize("K,N,rows", [(64, 40, 5), (191, 16, 3), (192, 24, 40), (768, 2304, 36), (3072, 8, 33)])
def test_linear_f32(K, N, rows):
    rng = np.random.default_rng(K + N + rows)
    w, x, b = f32(rng.standard_normal((N, K))), f32(rng.standard_normal((rows, K))), f32(rng.standard_normal(N))
    a = np.empty((rows, N), np.float32)
    ok(ref.ref_linear_f32(P(w), P(x), P(b), I(K), I(N), I(rows), P(a)))
    same(a, op.linear_f32(w, x, b))


def test_head_linear_f64():
    rng = np.random.default_rng(3)
    K, N, rows = 768, 96, 4
    w, x = f32(rng.standard_normal((N, K))), f32(rng.standard_normal((rows, K)))
    a, b = np.empty((rows, N), np.float32), np.empty((rows, N), np.float32)
    ok(ref.ref_head_linear_f64(P(w), P(x), I(K), I(N), I(rows), P(a)))
    assert oracle().oracle_head_linear_f64(P(w), P(x), I(K), I(N), I(rows), P(b)) == 0
    same(a, b)


@pytest.mark.parametrize("D", [32, 128, 768])
def test_rms_norm(D):
    rng = np.random.default_rng(D)
    x, w = f32(rng.standard_normal((7, D)) * 3), f32(rng.standard_normal(D))
    a = np.empty_like(x)
    ok(ref.ref_rms_norm(P(x), P(w), I(7), I(D), C.c_float(1e-6), P(a)))
    same(a, op.rms_norm(x, w, 1e-6))


def test_sigmoid_activation_exp():
    rng = np.random.default_rng(1)
    x = f32(np.concatenate([rng.standard_normal(5000) * 20, [0, -0.0, 87.5, -87.5, 88.5, -88.5, 1e-30, np.inf, -np.inf]]))
    a, b = np.empty_like(x), np.empty_like(x)
    ok(ref.ref_sigmoid(P(x), I(x.size), P(a)))
    oracle().oracle_sigmoid(P(x), I(x.size), P(b))
    same(a, b)


def test_monotone_and_denormalize():
    rng = np.random.default_rng(2)
    c = op.make_config(sy.spec_209m())
    raw = f32(rng.standard_normal(21 * 50) * 5)
    raw[::37] = 25
    a = np.empty_like(raw)
    ok(ref.ref_monotone_quantiles(C.byref(c), P(raw), I(raw.size), P(a)))
    same(a, op.monotone_quantiles(c, raw))
    loc, sc = f32(rng.standard_normal(5) * 100), f32(np.abs(rng.standard_normal(5)) * 10 + 1e-3)
    x = f32(rng.standard_normal(5 * 42) * 30)
    d = np.empty_like(x)
    ok(ref.ref_denormalize(P(x), P(loc), P(sc), I(5), I(42), I(21), C.c_int32(1), P(d)))
    same(d, op.denormalize(x, loc, sc, 21, True))


@pytest.mark.parametrize("ps,T,patches", [(32, 256, 8), (8, 40, 4), (2, 6, 3)])
def test_refine_and_frames(ps, T, patches):
    rng = np.random.default_rng(ps * T)
    c = unit_config(patch_size=ps, minimum_scale=1e-6)
    R, Q = 4, 21
    x, m = rows_with_gaps(rng, R, T)
    q = f32(np.sort(rng.standard_normal((R, patches * ps, Q)) * 5 + 30, axis=-1))
    targets = np.array([1, 1, 0, 1], np.int8)
    a = np.empty_like(q)
    ok(ref.ref_refine_block(C.byref(c), P(q), P(x), P(m), I(R), I(T), I(patches), P(targets), P(a)))
    same(a, op.refine_block(c, q, x.reshape(-1), m.reshape(-1), R, T, patches, targets))
    med = np.ascontiguousarray(rng.standard_normal(R * patches * ps))
    la, sa = np.empty(R * patches), np.empty(R * patches)
    ok(ref.ref_block_frames(C.byref(c), P(x), P(m), P(med), I(R), I(T), I(patches), P(la), P(sa)))
    lb, sb = op.block_frames(c, x, m, med, R, T, patches)
    same(la, lb)
    same(sa, sb)


@pytest.mark.parametrize("V,cov", [(1, False), (3, False), (1, True), (2, True)])
def test_assemble_rows(V, cov):
    rng = np.random.default_rng(V * 10 + cov)
    c = op.make_config(sy.spec_tiny())
    B, T, H = 2, 45, 11
    ctx = f32(rng.standard_normal((B, V, T)))
    ctx[rng.random(ctx.shape) < 0.2] = np.nan
    ctx[0, 0, :7] = np.nan
    keep = [ctx]
    arr = lambda a: (keep.append(a), P(a))[1]
    if cov:
        past = f32(rng.standard_normal((B, 2, T)))
        past[0, 1, 4] = np.nan
        known = f32(rng.standard_normal((B, 1, T + H)))
        cp = np.ascontiguousarray(rng.integers(0, 3, (B, 1, T)).astype(np.float64))
        ck = np.ascontiguousarray(rng.integers(0, 4, (B, 1, T + H)).astype(np.float64))
        cp[0, 0, 2] = np.nan
        ck[1, 0, T + 3] = 17      # unseen in the past
        req = op.OracleRequest(P(ctx), None, B, V, T, H, arr(past), 2, arr(known), 1, arr(cp), 1, arr(ck), 1, -1, -1, 40)
        all_rows = V + 2 + 1 + 1 + 1
    else:
        req = op.OracleRequest(P(ctx), None, B, V, T, H, None, 0, None, 0, None, 0, None, 0, -1, -1, 0)
        all_rows = V
    R = B * all_rows
    ps = c.patch_size
    kept = min(T, req.max_context or c.context_length)
    L = kept + (ps - kept % ps) % ps
    hor = (H + ps - 1) // ps * ps
    res = []
    for lib, fn in ((ref, "ref_assemble_rows"), (oracle(), "oracle_assemble_rows")):
        o = dict(rows=np.zeros((R, L), np.float32), mask=np.zeros((R, L), np.int8), groups=np.zeros(R, np.int64),
                 roles=np.zeros(R, np.int64), future=np.zeros((R, hor), np.float32), fmask=np.zeros((R, hor), np.int8))
        r_, l_, h_ = I(), I(), I()
        rc = getattr(lib, fn)(C.byref(c), C.byref(req), C.byref(r_), C.byref(l_), C.byref(h_), P(o["rows"]), P(o["mask"]),
                              P(o["groups"]), P(o["roles"]), P(o["future"]), P(o["fmask"]))
        assert rc == 0
        assert (r_.value, l_.value, h_.value) == (R, L, hor)
        res.append(o)
    for k in res[0]:
        same(res[0][k], res[1][k])
