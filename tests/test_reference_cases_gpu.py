"""The reference's own forecast test cases through the C ABI on a B200, against the oracle.

The cases are the ones the reference runs on its tiny checkpoint (its tests/cases.json,
extracted to tests/golden/reference_cases.json by tests/golden/make_reference_cases.py):
short and one-patch contexts, several variates, numeric past and known covariates,
categorical covariates with a code unseen in the context, horizons of many decode blocks
with and without known covariates, leading / scattered / whole-patch gaps, a non-negative
series far from zero (clipping), a constant series, a series with no observation at all, and
a context longer than the model's context length. Inputs follow the reference's generator
(timestral_b200.synthetic.reference_case_inputs). The model is the tiny checkpoint's
architecture in F32 (CUDA-core path), held to the F32 tolerance of tests/test_forecast_gpu.py
on every value; where the oracle rejects a request, the device must reject it too.
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
_models = {}


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def models():
    if "tiny" not in _models:
        path = sy.cached_model(sy.spec_tiny(), "f32")
        _models["tiny"] = (tb.Model(path), op.OracleModel(path))
    return _models["tiny"]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_case(case):
    m, o = models()
    ps = sy.spec_tiny().patch_size
    inp = sy.reference_case_inputs(case, ps)
    x = inp.pop("context")
    H = case["H"]
    try:
        want = o.forecast(x, H, **inp)
    except Exception as e:                      # the reference rejects the request
        with pytest.raises(Exception):
            m.forecast(x, H, **inp)
        print(f"{case['name']}: rejected by both ({e})")
        return
    got = m.forecast(x, H, **inp)
    assert got.shape == want.shape == (case["B"], case["V"], H, o.Q)
    assert np.isfinite(got).all()
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    tol = F32_ATOL + F32_RTOL * np.abs(want.astype(np.float64))
    print(f"{case['name']}: max|err|={err.max():.3e} worst err/tol={float(np.max(err / tol)):.3e} "
          f"bitwise-equal={np.mean(got == want):.4f}")
    assert np.all(err <= tol), float(np.max(err / tol))
    # the reference's invariant: quantiles do not cross
    assert np.all(np.diff(got, axis=-1) >= 0)
