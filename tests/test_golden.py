"""The CPU oracle against golden fixtures written by the reference's own compiled code
(tests/golden/make_golden.py runs oracle/_ref/libtsref.so, built from the reference's
sources), bit for bit. These run without the reference sources and without a GPU."""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_py as op
from helpers import unit_config
from timestral_b200 import synthetic as sy

GOLDEN = Path(__file__).resolve().parent / "golden"
P = op.ptr
I = C.c_int64


def load(name):
    d = np.load(GOLDEN / f"{name}.npz")
    return json.loads(str(d["config"])), d


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (a.shape, b.shape, a.dtype, b.dtype)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), f"max diff {np.nanmax(np.abs(a.astype(float) - b.astype(float)))}"


@pytest.mark.parametrize("name", ["scale_rows_ps32_T256", "scale_rows_ps8_T40"])
def test_scaler(name):
    cfg, d = load(name)
    R, T = d["x"].shape
    c = unit_config(**cfg)
    outs = [np.empty(R * T, np.float32) for _ in range(3)]
    assert op.lib().oracle_scale_rows(C.byref(c), P(d["x"]), P(d["m"]), I(R), I(T), P(outs[0]), P(outs[1]), P(outs[2])) == 0
    for o, k in zip(outs, ("scaled", "loc", "scale")):
        same(o, d[k])


@pytest.mark.parametrize("T", [7, 40, 1056])
def test_instance_norm(T):
    _, d = load(f"instance_norm_T{T}")
    R = d["x"].shape[0]
    loc, sc, b = op.instance_norm_stats(unit_config(), d["x"], d["m"], R, T)
    same(loc, d["loc"]); same(sc, d["scale"]); same(b, d["binary"])


@pytest.mark.parametrize("cov", [0, 1])
def test_masks(cov):
    cfg, d = load(f"masks_cov{cov}")
    R, T, h = cfg.pop("R"), cfg.pop("T"), cfg.pop("h")
    got = op.build_masks(unit_config(**cfg), d["obs"], R, T, h, d["groups"], d["roles"] if cov else None)
    for k in ("obs", "key_valid", "first_group", "positions", "time", "variate", "active", "anchor"):
        same(got[k], d[f"out_{k}"])


@pytest.mark.parametrize("name", ["sdpa_hd64_S18", "sdpa_hd16_S33", "sdpa_hd7_S5"])
def test_sdpa(name):
    cfg, d = load(name)
    same(op.sdpa(d["q"], d["k"], d["v"], d["mask"], cfg["hd"], cfg["H"], cfg["S"], cfg["R"], cfg["split"], threads=2),
         d["out"])


@pytest.mark.parametrize("D", [128, 768])
def test_rms_norm(D):
    cfg, d = load(f"rms_norm_D{D}")
    same(op.rms_norm(d["x"], d["w"], cfg["eps"]), d["out"])


def test_sigmoid():
    _, d = load("sigmoid")
    out = np.empty_like(d["x"])
    x = np.ascontiguousarray(d["x"])
    op.lib().oracle_sigmoid(P(x), I(x.size), P(out))
    same(out, d["out"])


def test_monotone_and_denormalize():
    _, d = load("monotone_denormalize")
    c = op.make_config(sy.spec_209m())
    same(op.monotone_quantiles(c, d["raw"]), d["monotone"])
    same(op.denormalize(d["x"], d["loc"], d["scale"], 21, True), d["denorm"])


@pytest.mark.parametrize("name", ["refine_ps32_T256", "refine_ps8_T40"])
def test_refine_and_frames(name):
    cfg, d = load(name)
    R, T, patches = cfg.pop("R"), cfg.pop("T"), cfg.pop("patches")
    c = unit_config(**cfg)
    same(op.refine_block(c, d["q"], d["x"].reshape(-1), d["m"].reshape(-1), R, T, patches, d["targets"]), d["refined"])
    la, sa = op.block_frames(c, d["x"], d["m"], d["median"], R, T, patches)
    same(la, d["frame_loc"]); same(sa, d["frame_scale"])
