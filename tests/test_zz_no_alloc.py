"""tsb_refine_static: the refine step of a decode block for callers that may not allocate
device memory (for example a host application that hands this library a fixed set of
buffers and owns every other allocation on the GPU). The entry point takes its float64
scratch from an array compiled into the library instead of the allocator.

Its output is checked against the refine of the CPU oracle, the implementation the
device forecast's refine is already held to (the library runs its allocating refine only
inside a whole forecast), at the F32 tolerance of the other GPU tests
(|gpu - oracle| <= 1e-4 + 1e-3 * |oracle|), on two calls in a row with different shapes so
that scratch left over from the first call cannot leak into the second. This file is named
to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_py as op
import timestral_b200 as tb
from helpers import unit_config

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


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
    return c, x, m, q, role, loc0, sc0


def run_static(x, m, q, role, loc0, sc0, patches, ps=32, Q=21, mi=10):
    dev = torch.device("cuda:0")
    R, T = x.shape
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dx, dm, dr, dl, ds = t(q), t(x), t(m), t(role), t(loc0), t(sc0)
    out = torch.full_like(dq, float("nan"))
    rc = tb.lib().tsb_refine_static(dq.data_ptr(), dx.data_ptr(), dm.data_ptr(), dr.data_ptr(), dl.data_ptr(),
                                    ds.data_ptr(), R, T, patches, ps, Q, mi, C.c_double(1e-6), out.data_ptr(), None)
    assert rc == 0, tb.lib().timestral_capi_last_error(None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def check(got, want):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= 1e-4 + 1e-3 * np.abs(want.astype(np.float64))), float(err.max())


def test_refine_static_two_calls_in_a_row():
    for seed, R, T, patches in ((1, 64, 2048, 8), (2, 37, 512, 3)):
        c, x, m, q, role, loc0, sc0 = case(seed, R, T, patches)
        want = op.refine_block(c, q, x.reshape(-1), m.reshape(-1), R, T, patches, (role == 0).astype(np.int8))
        got = run_static(x, m, q, role, loc0, sc0, patches)
        check(got, want.reshape(got.shape))
        assert np.array_equal(got[-1], q[-1]), "non-target rows keep their quantiles"


def test_refine_static_rejects_requests_above_its_scratch():
    c, x, m, q, role, loc0, sc0 = case(3, 2, 64, 2)
    lib = tb.lib()
    rows = 1 << 16     # 65,536 rows x 2,048 steps needs far more than the reserved scratch
    rc = lib.tsb_refine_static(1, 1, 1, None, 1, 1, rows, 2048, 8, 32, 21, 10, C.c_double(1e-6), 1, None)
    assert rc == tb.TSB_ERR_ARG
    assert b"scratch" in lib.timestral_capi_last_error(None)
