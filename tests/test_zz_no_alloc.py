"""tsb_refine_static: the refine step of a decode block for callers that may not allocate
device memory (for example a host application that hands this library a fixed set of
buffers and owns every other allocation on the GPU, or a loop that must never enter the
CUDA allocator). The entry point takes its float64 scratch from an array compiled into the
library instead of the allocator.

Its output is checked bit for bit against the refine that takes its scratch from the
allocator (tsb_test_refine, the kernel as the forecast runs it) and against the reference's
own refine output (tests/golden, written by the reference's compiled src/refine.cpp), on
calls in a row with different shapes, so that scratch left over from one call cannot leak
into the next. This file is named to be collected last.
"""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_py as op
import timestral_b200 as tb
from helpers import unit_config

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GOLDEN = Path(__file__).resolve().parent / "golden"
SCRATCH_DOUBLES = 1 << 19       # the library's fixed scratch, in float64 values


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def scratch_per_row(T, patches, ps):
    return 3 * (T // ps + patches) + 2 * ps + 2 * patches


def case(seed, R, T, patches, ps=32, Q=21):
    rng = np.random.default_rng(seed)
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
    role[-1] = 1                        # one non-target row keeps its quantiles
    return x, m, q, role, loc0, sc0


def run(entry, x, m, q, role, loc0, sc0, patches, ps=32, Q=21, mi=10, min_scale=1e-6):
    """Call tsb_refine_static ("static") or the allocating tsb_test_refine ("alloc") on
    device copies of the inputs; returns (status, output)."""
    dev = torch.device("cuda:0")
    R, T = x.shape
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dx, dm, dr, dl, ds = t(q), t(x), t(m), t(role), t(loc0), t(sc0)
    out = torch.full_like(dq, float("nan"))
    args = (dq.data_ptr(), dx.data_ptr(), dm.data_ptr(), dr.data_ptr(), dl.data_ptr(), ds.data_ptr(), R, T, patches, ps,
            Q, mi, C.c_double(min_scale), out.data_ptr())
    if entry == "static":
        rc = tb.lib().tsb_refine_static(*args, None)
    else:
        rc = tb.lib().tsb_test_refine(*args)
    torch.cuda.synchronize()
    return rc, out.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_refine_static_equals_allocating_refine_two_calls_in_a_row():
    for seed, R, T, patches in ((1, 64, 2048, 8), (2, 37, 512, 3)):
        inputs = case(seed, R, T, patches)
        rc, got = run("static", *inputs, patches)
        assert rc == 0, tb.lib().timestral_capi_last_error(None)
        rc, want = run("alloc", *inputs, patches)
        assert rc == 0
        assert np.array_equal(bits(got), bits(want)), float(np.nanmax(np.abs(got - want)))
        assert np.array_equal(got[-1], inputs[2][-1]), "non-target rows keep their quantiles"


def test_refine_static_matches_reference_golden():
    for name in ("refine_ps32_T256", "refine_ps8_T40"):
        d = np.load(GOLDEN / f"{name}.npz")
        cfg = json.loads(str(d["config"]))
        R, T, patches, ps = cfg["R"], cfg["T"], cfg["patches"], cfg["patch_size"]
        c = unit_config(patch_size=ps, minimum_scale=cfg["minimum_scale"])
        _, loc, sc = op.scale_rows(c, d["x"], d["m"], R, T)
        loc0 = np.ascontiguousarray(loc.reshape(R, T)[:, -1])
        sc0 = np.ascontiguousarray(sc.reshape(R, T)[:, -1])
        role = (d["targets"] == 0).astype(np.int8)
        rc, got = run("static", d["x"], d["m"], d["q"], role, loc0, sc0, patches, ps=ps, min_scale=cfg["minimum_scale"])
        assert rc == 0, tb.lib().timestral_capi_last_error(None)
        assert np.array_equal(bits(got), bits(d["refined"])), name


def test_refine_static_rejects_requests_above_its_scratch():
    """Real device buffers of the right sizes on both sides of the limit: one row more than
    the scratch holds is refused (the output is left untouched), the largest request that
    fits runs and equals the allocating refine."""
    T, patches, ps = 2048, 8, 32
    fit = SCRATCH_DOUBLES // scratch_per_row(T, patches, ps)
    inputs = case(5, fit + 1, T, patches)
    rc, out = run("static", *inputs, patches)
    assert rc == tb.TSB_ERR_ARG
    assert b"scratch" in tb.lib().timestral_capi_last_error(None)
    assert np.all(np.isnan(out)), "a refused call writes nothing"
    inputs = tuple(a[:fit] for a in inputs)
    rc, got = run("static", *inputs, patches)
    assert rc == 0, tb.lib().timestral_capi_last_error(None)
    rc, want = run("alloc", *inputs, patches)
    assert rc == 0
    assert np.array_equal(bits(got), bits(want))
