"""Multi-rank host logic of the series-sharded path on CPU: two gloo ranks, each forecasting
its slice with a deterministic stand-in for the device forecast, must reproduce the
single-process result bit for bit (even and uneven batches, covariates sliced with their
series)."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as td
import torch.multiprocessing as mp

from timestral_b200.shard import forecast_sharded, shard_range


def fake_forecast(context, horizon, past=None):
    """Per-series function of the series' own inputs only, [b, V, H, 3]."""
    b, V, T = context.shape
    base = np.nan_to_num(context).sum(axis=-1, dtype=np.float64)
    if past is not None:
        base = base + past.sum(axis=(1, 2))[:, None]
    steps = np.arange(horizon, dtype=np.float64)
    out = base[:, :, None, None] * 1e-3 + steps[None, None, :, None] + np.array([-1.0, 0.0, 1.0])
    return out.astype(np.float32)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, B, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        x = rng.standard_normal((B, 2, 64)).astype(np.float32)
        past = rng.standard_normal((B, 3, 64)).astype(np.float32)
        got = forecast_sharded(fake_forecast, x, 8, rank, world, td, past=past)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), got)
    finally:
        td.destroy_process_group()


def test_shard_range_covers_the_batch():
    for B in (0, 1, 5, 4096, 4099):
        for world in (1, 2, 3, 8):
            spans = [shard_range(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


@pytest.mark.parametrize("B", [6, 5])
def test_two_gloo_ranks_match_one_process(tmp_path, B):
    world = 2
    mp.start_processes(worker, args=(world, free_port(), B, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    rng = np.random.default_rng(0)
    x = rng.standard_normal((B, 2, 64)).astype(np.float32)
    past = rng.standard_normal((B, 3, 64)).astype(np.float32)
    want = fake_forecast(x, 8, past=past)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert got.shape == want.shape
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
