"""Synthetic workload generators against the checksums the reference publishes for its own
benchmark input (docs/benchmarks.md: input sums -8.5625 at 32768 steps and -3.234375 at 512)."""
import numpy as np

from timestral_b200 import synthetic as sy


def test_dyadic_input_checksums():
    assert float(sy.series_dyadic(32768).sum(dtype=np.float64)) == -8.5625
    assert float(sy.series_dyadic(512).sum(dtype=np.float64)) == -3.234375


def test_dyadic_input_values():
    x = sy.series_dyadic(300, V=3)
    assert x.shape == (1, 3, 300) and x.dtype == np.float32
    t = np.arange(300)
    for v in range(3):
        want = (((17 * t + 13 * v) % 257) - 128) / 64.0
        assert np.array_equal(x[0, v].astype(np.float64), want)
    assert np.isfinite(x).all()


def test_reference_case_inputs():
    """The reference's test cases (tests/golden/reference_cases.json) build inputs of the
    stated shapes with the stated structure: constant and all-missing series, leading and
    whole-patch gaps on the first row, 0/1 indicator rows, and a categorical code that never
    occurs in the context at step T + H/2 of the known codes."""
    import json
    from pathlib import Path
    cases = {c["name"]: c for c in json.loads((Path(__file__).parent / "golden" / "reference_cases.json").read_text())}
    assert len(cases) == 14
    for c in cases.values():
        d = sy.reference_case_inputs(c, 8)
        assert d["context"].shape == (c["B"], c["V"], c["T"]) and d["context"].dtype == np.float32
        if "known" in d:
            assert d["known"].shape[2] == c["T"] + c["H"]
    assert (sy.reference_case_inputs(cases["const"], 8)["context"] == 5.0).all()
    am = sy.reference_case_inputs(cases["all_missing"], 8)["context"]
    assert np.isnan(am[1]).all() and not np.isnan(am[0]).any()
    nans = sy.reference_case_inputs(cases["nans"], 8)["context"].reshape(-1, 900)
    assert np.isnan(nans[0, :100]).all() and np.isnan(nans[0, 96:104]).all()
    nonneg = sy.reference_case_inputs(cases["nonneg"], 8)["context"]
    assert (nonneg >= 0).all()
    kc = sy.reference_case_inputs(cases["known_cov"], 8)["known"]
    assert set(np.unique(kc[0, 1])) == {0.0, 1.0}
    cu = cases["cat_uni"]
    ck = sy.reference_case_inputs(cu, 8)["cat_known"]
    code = cu["cat_known"]["n_codes"] + 7
    assert ck[0, 0, cu["T"] + cu["H"] // 2] == code and not (ck[0, 0, :cu["T"]] == code).any()
