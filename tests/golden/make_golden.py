"""Writes the golden fixtures of tests/golden/ from the reference's own code.

Each fixture holds seeded inputs and the outputs of one reference function, computed by
oracle/_ref/libtsref.so (built by oracle/ref/Makefile from the reference's sources:
src/scaler.cpp, masks.cpp, layers.cpp, head.cpp, refine.cpp, covariates.cpp). The tests
(tests/test_golden.py, and the device checks in tests/test_rows_gpu.py) compare against
these files, so the pins hold where the reference sources are not present.

Run from the repository root after `python -c "import __graft_entry__ as g; g.build()"`:
    python tests/golden/make_golden.py
"""
import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT / "tests"), str(ROOT / "oracle"), str(ROOT / "timestral.cpp_b200")]
import oracle_py as op                      # noqa: E402
from helpers import unit_config, f32, i8    # noqa: E402
from timestral_b200 import synthetic as sy  # noqa: E402

OUT = Path(__file__).resolve().parent
REF = ROOT / "oracle" / "_ref" / "libtsref.so"
P = op.ptr
I = C.c_int64


def lib():
    ref = C.CDLL(str(REF))
    ref.ref_last_error.restype = C.c_char_p
    return ref


def ok(ref, rc):
    if rc != 0:
        raise RuntimeError(ref.ref_last_error().decode())


def rows_with_gaps(rng, R, T, nan_frac=0.2):
    x = f32(rng.standard_normal((R, T)) * 10 ** rng.uniform(-3, 3, (R, 1)) + rng.uniform(-100, 100, (R, 1)))
    m = i8(rng.random((R, T)) > nan_frac)
    m[0, :] = 0
    if R > 2:
        m[2, : T // 2] = 0
    x[m == 0] = 0
    x[1, min(3, T - 1)] = -0.0
    return x, m


def save(name, config, **arrays):
    np.savez_compressed(OUT / f"{name}.npz", config=np.array(json.dumps(config)), **arrays)


def main():
    ref = lib()
    # causal scaler (src/scaler.cpp:27-58)
    for ps, T in ((32, 256), (8, 40)):
        rng = np.random.default_rng(ps + T)
        cfg = dict(patch_size=ps)
        c = unit_config(**cfg)
        R = 6
        x, m = rows_with_gaps(rng, R, T)
        outs = [np.empty(R * T, np.float32) for _ in range(3)]
        ok(ref, ref.ref_scale_rows(C.byref(c), P(x), P(m), I(R), I(T), P(outs[0]), P(outs[1]), P(outs[2])))
        save(f"scale_rows_ps{ps}_T{T}", cfg, x=x, m=m, scaled=outs[0], loc=outs[1], scale=outs[2])
    # instance-norm statistics of known covariate rows (src/scaler.cpp:60-107)
    for T in (7, 40, 1056):
        rng = np.random.default_rng(T)
        R = 4
        x, m = rows_with_gaps(rng, R, T)
        x[3] = (rng.random(T) > 0.5).astype(np.float32)
        a = [np.empty(R, np.float32), np.empty(R, np.float32), np.empty(R, np.int8)]
        c = unit_config()
        ok(ref, ref.ref_instance_norm_stats(C.byref(c), P(x), P(m), I(R), I(T), P(a[0]), P(a[1]), P(a[2])))
        save(f"instance_norm_T{T}", {}, x=x, m=m, loc=a[0], scale=a[1], binary=a[2])
    # masks (src/masks.cpp:8-34)
    for cov in (0, 1):
        rng = np.random.default_rng(5 + cov)
        cfg = dict(patch_size=4, block_size=3, covariate_enabled=1)
        c = unit_config(**cfg)
        R, T, h = 6, 40, 3
        obs = i8(rng.random((R, T)) > 0.6)
        obs[1, :20] = 0
        groups = np.array([0, 0, 0, 7, 7, 7], np.int64)
        roles = np.array([0, 1, 2, 0, 2, 1], np.int64) if cov else None
        shape = op.build_masks(c, obs, R, T, h, groups, roles)      # sizes only
        out = {k: np.zeros_like(v) for k, v in shape.items() if isinstance(v, np.ndarray)}
        out["first_group"] = np.zeros(len(np.unique(groups)), np.int64)
        ok(ref, ref.ref_build_masks(C.byref(c), P(obs), I(R), I(T), I(h), P(groups), P(roles), P(out["obs"]),
                                    P(out["key_valid"]), P(out["first_group"]), P(out["positions"]), P(out["time"]),
                                    P(out["variate"]), P(out["active"]), P(out["anchor"])))
        extra = {"roles": roles} if cov else {}
        save(f"masks_cov{cov}", dict(cfg, R=R, T=T, h=h), obs=obs, groups=groups, **extra,
             **{f"out_{k}": v for k, v in out.items()})
    # scaled dot-product attention, AVX2 pair path (src/layers.cpp:578-617)
    for hd, S, split, R in ((64, 18, 16, 2), (16, 33, 30, 2), (7, 5, 2, 3)):
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
        ok(ref, ref.ref_sdpa(P(q), P(k), P(v), P(mask), I(hd), I(H), I(S), I(R), I(split), P(a), C.c_int32(3)))
        save(f"sdpa_hd{hd}_S{S}", dict(hd=hd, H=H, S=S, R=R, split=split), q=q, k=k, v=v, mask=mask, out=a)
    # RMSNorm, ATen float cascade (src/layers.cpp:262-287)
    for D in (128, 768):
        rng = np.random.default_rng(D)
        x, w = f32(rng.standard_normal((7, D)) * 3), f32(rng.standard_normal(D))
        a = np.empty_like(x)
        ok(ref, ref.ref_rms_norm(P(x), P(w), I(7), I(D), C.c_float(1e-6), P(a)))
        save(f"rms_norm_D{D}", dict(eps=1e-6), x=x, w=w, out=a)
    # sigmoid with the SLEEF-style exp (src/layers.cpp:658-667)
    rng = np.random.default_rng(1)
    x = f32(np.concatenate([rng.standard_normal(2000) * 20, [0, -0.0, 87.5, -87.5, 88.5, -88.5, 1e-30, np.inf, -np.inf]]))
    a = np.empty_like(x)
    ok(ref, ref.ref_sigmoid(P(x), I(x.size), P(a)))
    save("sigmoid", {}, x=x, out=a)
    # monotone quantiles and denormalisation (src/head.cpp:61-80, src/scaler.cpp:109-137)
    rng = np.random.default_rng(2)
    c = op.make_config(sy.spec_209m())
    raw = f32(rng.standard_normal(21 * 50) * 5)
    raw[::37] = 25
    a = np.empty_like(raw)
    ok(ref, ref.ref_monotone_quantiles(C.byref(c), P(raw), I(raw.size), P(a)))
    loc, sc = f32(rng.standard_normal(5) * 100), f32(np.abs(rng.standard_normal(5)) * 10 + 1e-3)
    xd = f32(rng.standard_normal(5 * 42) * 30)
    d = np.empty_like(xd)
    ok(ref, ref.ref_denormalize(P(xd), P(loc), P(sc), I(5), I(42), I(21), C.c_int32(1), P(d)))
    save("monotone_denormalize", {"spec": "209m"}, raw=raw, monotone=a, x=xd, loc=loc, scale=sc, denorm=d)
    # refine and block frames (src/refine.cpp)
    for ps, T, patches in ((32, 256, 8), (8, 40, 4)):
        rng = np.random.default_rng(ps * T)
        cfg = dict(patch_size=ps, minimum_scale=1e-6)
        c = unit_config(**cfg)
        R, Q = 4, 21
        x, m = rows_with_gaps(rng, R, T)
        q = f32(np.sort(rng.standard_normal((R, patches * ps, Q)) * 5 + 30, axis=-1))
        targets = np.array([1, 1, 0, 1], np.int8)
        a = np.empty_like(q)
        ok(ref, ref.ref_refine_block(C.byref(c), P(q), P(x), P(m), I(R), I(T), I(patches), P(targets), P(a)))
        med = np.ascontiguousarray(rng.standard_normal(R * patches * ps))
        la, sa = np.empty(R * patches), np.empty(R * patches)
        ok(ref, ref.ref_block_frames(C.byref(c), P(x), P(m), P(med), I(R), I(T), I(patches), P(la), P(sa)))
        save(f"refine_ps{ps}_T{T}", dict(cfg, R=R, T=T, patches=patches), x=x, m=m, q=q, targets=targets,
             refined=a, median=med, frame_loc=la, frame_scale=sa)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
