"""Multi-rank host logic of the series-sharded path on CPU: two gloo ranks, each forecasting
its slice with a deterministic stand-in for the device forecast, must reproduce the
single-process result bit for bit (even and uneven batches, covariates sliced with their
series). Failures are made on the host: a rank whose forecast raises is reported on every
rank, and a rank that exits ends the other's gather with an error instead of a hang."""
import datetime
import os
import socket
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as td
import torch.multiprocessing as mp

from timestral_b200.shard import ShardFailure, forecast_sharded, shard_range


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


def failing_worker(rank, world, port, mode, out_dir):
    """Rank 1 fails: its forecast raises (mode "raise") or the process exits before the
    gather (mode "exit"). Each surviving rank records what it saw."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    x = np.ones((4, 1, 16), np.float32)

    def forecast(context, horizon):
        if rank == 1:
            if mode == "exit":
                os._exit(3)
            raise ValueError("injected shard failure")
        return fake_forecast(context, horizon)
    t0 = time.time()
    try:
        forecast_sharded(forecast, x, 4, rank, world, td)
        seen = "no error"
    except ShardFailure as e:
        seen = f"ShardFailure: {e}"
    except Exception as e:          # the process group's error after a peer exits
        seen = f"{type(e).__name__}: {e}"
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{time.time() - t0:.1f}\n{seen}")
    if mode == "raise":
        td.destroy_process_group()


def test_raising_rank_is_reported_on_every_rank(tmp_path):
    world = 2
    mp.start_processes(failing_worker, args=(world, free_port(), "raise", str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        seconds, seen = (tmp_path / f"rank{r}.txt").read_text().split("\n", 1)
        assert seen.startswith("ShardFailure: rank 1: ValueError: injected shard failure"), seen


def test_exiting_rank_ends_the_gather_with_an_error(tmp_path):
    world = 2
    ctx = mp.start_processes(failing_worker, args=(world, free_port(), "exit", str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    deadline = time.time() + 120
    while time.time() < deadline and any(p.is_alive() for p in ctx.processes):
        time.sleep(0.5)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    codes = [p.exitcode for p in ctx.processes]
    assert codes[1] == 3, codes
    seconds, seen = (tmp_path / "rank0.txt").read_text().split("\n", 1)
    print(f"rank 0 after {seconds} s: {seen}")
    assert seen != "no error" and float(seconds) < 60
