"""The reference's own forecast test cases through the C ABI on a B200, against the oracle.

The cases are the ones the reference runs on its tiny checkpoint (its tests/cases.json,
extracted to tests/golden/reference_cases.json by tests/golden/make_reference_cases.py):
short and one-patch contexts, several variates, numeric past and known covariates,
categorical covariates with a code unseen in the context, horizons of many decode blocks
with and without known covariates, leading / scattered / whole-patch gaps, a non-negative
series far from zero (clipping), a constant series, a series with no observation at all, and
a context longer than the model's context length. Inputs follow the reference's generator
(timestral_b200.synthetic.reference_case_inputs). Two models: the tiny checkpoint's
architecture in F32 (CUDA-core path), held to the F32 tolerance of tests/test_forecast_gpu.py
on every value; and a model with the 209M head and patch geometry in F16 (tensor-core path),
held to the F16 bounds of that file against the oracle's F16 restatement. Where the oracle
rejects a request, the device must reject it too.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_py as op
import timestral_b200 as tb
from timestral_b200 import synthetic as sy

pytestmark = pytest.mark.gpu

CASES = json.loads((Path(__file__).resolve().parent / "golden" / "reference_cases.json").read_text())
F32_RTOL, F32_ATOL = 1e-3, 1e-4
F16_MEAN_ND, F16_ROW_FACTOR, F16_VALUE_FACTOR = 1e-3, 3.0, 30.0   # as tests/test_forecast_gpu.py
_models = {}


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def models(spec, weights):
    key = (spec.name, weights)
    if key not in _models:
        path = sy.cached_model(spec, weights)
        _models[key] = (tb.Model(path), op.OracleModel(path))
    return _models[key]


def run_case(case, spec, weights):
    """(context, device forecast, oracle forecast), or None when both reject the request."""
    m, o = models(spec, weights)
    inp = sy.reference_case_inputs(case, spec.patch_size)
    x = inp.pop("context")
    H = case["H"]
    try:
        want = o.forecast(x, H, **inp)
    except Exception as e:                      # the reference rejects the request
        with pytest.raises(Exception):
            m.forecast(x, H, **inp)
        print(f"{case['name']}: rejected by both ({e})")
        return None
    got = m.forecast(x, H, **inp)
    assert got.shape == want.shape == (case["B"], case["V"], H, o.Q)
    assert np.isfinite(got).all()
    # the reference's invariant: quantiles do not cross
    assert np.all(np.diff(got, axis=-1) >= 0)
    return x, got, want


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_case(case):
    r = run_case(case, sy.spec_tiny(), "f32")
    if r is None:
        return
    _, got, want = r
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    tol = F32_ATOL + F32_RTOL * np.abs(want.astype(np.float64))
    print(f"{case['name']}: max|err|={err.max():.3e} worst err/tol={float(np.max(err / tol)):.3e} "
          f"bitwise-equal={np.mean(got == want):.4f}")
    assert np.all(err <= tol), float(np.max(err / tol))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_case_f16_tensor_cores(case):
    spec = sy.spec_small()
    r = run_case(case, spec, "f16")
    if r is None:
        return
    x, got, want = r
    loc, sc = op.anchors(x, spec.patch_size)
    rows_mean, rows_max = op.normalized_deviation_rows(got, want, loc, sc)
    mean, row, mx = float(np.mean(rows_mean)), float(np.max(rows_mean)), float(np.max(rows_max))
    print(f"{case['name']}: normalized deviation mean={mean:.3e} worst row={row:.3e} worst value={mx:.3e}")
    assert mean <= F16_MEAN_ND and row <= F16_ROW_FACTOR * F16_MEAN_ND and mx <= F16_VALUE_FACTOR * F16_MEAN_ND
