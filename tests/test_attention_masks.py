"""The torch restatement of the time-axis mask used by the attention kernel tests, pinned to
the oracle's mask builder (reference src/masks.cpp:8-34) on random observation patterns,
with and without the covariate layout. Runs without a GPU."""
import numpy as np
import pytest

import oracle_py as op
from helpers import time_mask_torch, unit_config

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("cov,T,h,bs,seed", [(0, 40, 3, 2, 1), (0, 64, 8, 4, 2), (1, 48, 6, 2, 3), (1, 64, 12, 4, 4),
                                             (1, 40, 2, 2, 5)])
def test_time_mask_matches_oracle(cov, T, h, bs, seed):
    c = unit_config(patch_size=2, block_size=bs, attend_missing_patches=1, covariate_enabled=cov)
    rng = np.random.default_rng(seed)
    R = 4
    observed = (rng.random((R, T)) > 0.3).astype(np.int8)
    roles = [0, 1, 2, 2] if cov else None
    m = op.build_masks(c, observed.ravel(), R, T, h, [0] * R, roles)
    N, S = m["N"], m["S"]
    L = N - h if cov else N
    valid = torch.from_numpy(m["key_valid"].reshape(R, N).astype(bool))
    role = torch.tensor(roles or [0] * R, dtype=torch.int8)
    ours = time_mask_torch(valid, role, N, L, S, cov, bs).numpy()
    ref = m["time"].reshape(R, S, S).astype(bool)
    # encoder queries compute keys < N only (reference src/layers.cpp:591)
    ref[:, :N, N:] = False
    assert ours.shape == ref.shape
    assert np.array_equal(ours, ref), np.argwhere(ours != ref)[:5]
