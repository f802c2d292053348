"""Series sharding across GPUs: one process per GPU, each forecasting a contiguous slice of
the batch with its own handle. A series' rows (target, past and known covariates) stay on
one rank, and the forecast of a series does not depend on the other series in its batch,
so the gathered result equals the single-GPU result bit for bit. No collective runs on the
forecast path; the gather of the finished [B, V, H, Q] slices is the only exchange."""
from __future__ import annotations

import numpy as np


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Series [lo, hi) of `rank`: contiguous slices, the first batch % world ranks one longer."""
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"invalid shard request batch={batch} world={world} rank={rank}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class ShardFailure(RuntimeError):
    """The forecast of one or more ranks failed; raised on every rank, with each failed
    rank's error, so that no rank waits for a slice that will not come."""


def forecast_sharded(forecast, context, horizon: int, rank: int, world: int, dist=None, **kw):
    """Forecast this rank's slice of `context` [B, V, T] with `forecast(context, horizon, **kw)`
    and gather every rank's [b, V, H, Q] slice in series order on all ranks. Covariate arrays
    in `kw` with a leading batch axis (past, known, cat_past, cat_known, mask) are sliced too.

    A rank whose forecast raises still takes part in the gather, carrying its error instead of
    a slice, and every rank then raises ShardFailure. A rank that exits instead ends the
    gather of the others with the process group's error (a closed connection, or its
    timeout)."""
    B = context.shape[0]
    lo, hi = shard_range(B, world, rank)
    local_kw = {k: (v[lo:hi] if isinstance(v, np.ndarray) and v.ndim >= 1 and v.shape[0] == B else v)
                for k, v in kw.items()}
    if world == 1 or dist is None:
        return forecast(context[lo:hi], horizon, **local_kw) if hi > lo else None
    part, error = None, None
    try:
        part = forecast(context[lo:hi], horizon, **local_kw) if hi > lo else None
    except Exception as e:          # reported to every rank through the gather
        error = f"rank {rank}: {type(e).__name__}: {e}"
    parts = [None] * world
    dist.all_gather_object(parts, (error, part))
    errors = [e for e, _ in parts if e]
    if errors:
        raise ShardFailure("; ".join(errors))
    return np.concatenate([p for _, p in parts if p is not None], axis=0)
