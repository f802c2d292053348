"""Shared test helpers: oracle configs and small math used by several test files."""
import numpy as np

import oracle_py as op
from timestral_b200 import synthetic as sy


def unit_config(**kw):
    """An oracle config with the 209M defaults, overridable per known-answer test."""
    c = op.make_config(sy.spec_209m())
    for k, v in kw.items():
        if k == "knots":
            c.num_quantiles = len(v)
            for i, x in enumerate(v):
                c.knots[i] = x
        else:
            setattr(c, k, v)
    return c


def f32(x):
    return np.ascontiguousarray(x, np.float32)


def i8(x):
    return np.ascontiguousarray(x, np.int8)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def time_mask_torch(valid, role, N, L, S, cov, bs):
    """[rows, S, S] bool torch mask: query q may attend key k on the time axis (reference
    src/masks.cpp:21-26), restricted to the keys the reference computes (keys < N for encoder
    queries, src/layers.cpp:591). valid: [rows, N] bool key-valid patches; role: [rows] int8
    (0 target, 1 past, 2 known; used on the covariate layout, S = 2N, L context patches,
    decode blocks of bs patches)."""
    import torch
    rows = valid.shape[0]
    q = torch.arange(S)[:, None]
    k = torch.arange(S)[None, :]
    kv = torch.zeros(rows, S, dtype=torch.bool)
    kv[:, :N] = valid
    kvk = kv[:, None, :].expand(rows, S, S)
    if not cov:
        enc = (q < N) & (k < N) & ((kvk & (k <= q)) | (q == k))
        dec = (q >= N) & (((k < N) & kvk) | ((k >= N) & (k <= q)))
        return enc | dec
    known = (role.long() == 2)[:, None, None]

    def anchor(p):
        return torch.where(p >= L, L + bs * torch.div(p - L, bs, rounding_mode="floor"), torch.zeros_like(p))

    enc = (q < N) & (k < N) & ((kvk & (known | (k <= q))) | (q == k))
    qp, kp = q - N, k - N
    qa = qp >= L
    dec_ctx = (q >= N) & (k < N) & kvk & qa & (k < anchor(qp))
    dec_dec = (q >= N) & (k >= N) & ((q == k) | ((k <= q) & qa & (kp >= L) & (anchor(qp) == anchor(kp))))
    return enc | dec_ctx | dec_dec
