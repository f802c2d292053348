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
