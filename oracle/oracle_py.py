"""ctypes binding of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and --impl reference)
as the checker; the product never imports it. The model is read with gguf-py (an
independent reader from the product's C++ GGUF loader) and copied into the oracle.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

LAYER_KIND = {"time": 0, "variate": 1, "time_variate": 2, "variate_time": 3}


class OracleConfig(C.Structure):
    _fields_ = [("patch_size", C.c_int32), ("d_model", C.c_int32), ("num_heads", C.c_int32),
                ("mlp_hidden_dim", C.c_int32), ("n_layers", C.c_int32), ("schedule", C.c_int32 * 256),
                ("num_quantiles", C.c_int32), ("knots", C.c_double * 64), ("block_size", C.c_int32),
                ("context_length", C.c_int32), ("rope_dim", C.c_int32), ("rope_table_pos_min", C.c_int32),
                ("norm_eps", C.c_float), ("attn_bias", C.c_int32), ("mlp_bias", C.c_int32),
                ("time_gate", C.c_int32), ("variate_gate", C.c_int32), ("minimum_scale", C.c_double),
                ("use_asinh", C.c_int32), ("covariate_enabled", C.c_int32),
                ("attend_missing_patches", C.c_int32), ("quantile_width_factor", C.c_double),
                ("per_shot_horizon_patches", C.c_int32), ("quantile_real_cap_k", C.c_double),
                ("extreme_value_threshold", C.c_double), ("symmetric_averaging", C.c_int32),
                ("clip_nonnegative", C.c_int32), ("target_encoding_smooth", C.c_double)]


class OracleRequest(C.Structure):
    _fields_ = [("context", C.c_void_p), ("observation_mask", C.c_void_p), ("B", C.c_int32),
                ("V", C.c_int32), ("T", C.c_int32), ("prediction_length", C.c_int32),
                ("past_cov", C.c_void_p), ("c_past", C.c_int32), ("known_cov", C.c_void_p),
                ("c_known", C.c_int32), ("cat_past", C.c_void_p), ("cc_past", C.c_int32),
                ("cat_known", C.c_void_p), ("cc_known", C.c_int32), ("symmetric_averaging", C.c_int32),
                ("clip_nonnegative", C.c_int32), ("max_context", C.c_int32)]


_lib = None


def build():
    """Compile the oracle library (make in oracle/)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _lib.oracle_last_error.restype = C.c_char_p
        _lib.oracle_model_new.restype = C.c_void_p
        _lib.oracle_model_new.argtypes = [C.POINTER(OracleConfig)]
        _lib.oracle_model_free.argtypes = [C.c_void_p]
        _lib.oracle_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int64]
        _lib.oracle_forecast.argtypes = [C.c_void_p, C.POINTER(OracleRequest), C.c_void_p, C.c_int32]
        _lib.oracle_model_set_per_shot.argtypes = [C.c_void_p, C.c_int32]
        _lib.oracle_model_set_round_attention.argtypes = [C.c_void_p, C.c_int32]
        _lib.oracle_activation_exp.restype = C.c_float
        _lib.oracle_activation_exp.argtypes = [C.c_float]
        _lib.oracle_attention_exp.restype = C.c_float
        _lib.oracle_attention_exp.argtypes = [C.c_float]
        _lib.oracle_numpy_sum.restype = C.c_double
        _lib.oracle_numpy_sum.argtypes = [C.c_void_p, C.c_int64]
        _lib.oracle_torch_sum_f32.restype = C.c_float
        _lib.oracle_torch_sum_f32.argtypes = [C.c_void_p, C.c_int64]
    return _lib


def _check(rc):
    if rc != 0:
        raise RuntimeError(lib().oracle_last_error().decode())


def ptr(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _field(reader, key):
    f = reader.fields[key]
    t = f.types[0]
    import gguf
    if t == gguf.GGUFValueType.STRING:
        return bytes(f.parts[f.data[0]]).decode()
    if t == gguf.GGUFValueType.ARRAY:
        if f.types[1] == gguf.GGUFValueType.STRING:
            return [bytes(f.parts[i]).decode() for i in f.data]
        return [f.parts[i][0].item() for i in f.data]
    return f.parts[f.data[0]][0].item()


def config_from_reader(reader) -> OracleConfig:
    g = lambda k: _field(reader, k)
    c = OracleConfig()
    c.patch_size = g("timestral.patch_size"); c.d_model = g("timestral.embedding_length")
    c.num_heads = g("timestral.attention.head_count"); c.mlp_hidden_dim = g("timestral.feed_forward_length")
    sched = g("timestral.block_schedule"); c.n_layers = len(sched)
    for i, s in enumerate(sched):
        c.schedule[i] = LAYER_KIND[s]
    knots = g("timestral.quantile_knots"); c.num_quantiles = len(knots)
    for i, k in enumerate(knots):
        c.knots[i] = k
    c.block_size = g("timestral.block_size"); c.context_length = g("timestral.context_length")
    c.rope_dim = g("timestral.rope.dimension_count"); c.rope_table_pos_min = g("timestral.rope.table_pos_min")
    c.norm_eps = g("timestral.attention.layer_norm_rms_epsilon")
    c.attn_bias = int(g("timestral.attention.bias")); c.mlp_bias = int(g("timestral.mlp.bias"))
    c.time_gate = int(g("timestral.attention.time_gate") == "sdpa_sigmoid")
    c.variate_gate = int(g("timestral.attention.variate_gate") == "sdpa_sigmoid")
    c.minimum_scale = g("timestral.scaler.minimum_scale"); c.use_asinh = int(g("timestral.scaler.use_asinh"))
    c.covariate_enabled = int(g("timestral.covariate_enabled"))
    c.attend_missing_patches = int(g("timestral.attend_missing_patches"))
    c.quantile_width_factor = g("timestral.quantile_width_factor")
    c.per_shot_horizon_patches = g("timestral.forecaster.per_shot_horizon_patches")
    c.quantile_real_cap_k = g("timestral.forecaster.quantile_real_cap_k")
    c.extreme_value_threshold = g("timestral.forecaster.extreme_value_threshold")
    c.symmetric_averaging = int(g("timestral.forecaster.symmetric_averaging"))
    c.clip_nonnegative = int(g("timestral.forecaster.clip_nonnegative"))
    c.target_encoding_smooth = g("timestral.target_encoding.smooth")
    return c


def make_config(spec) -> OracleConfig:
    """Config struct from a synthetic ModelSpec (no file needed)."""
    c = OracleConfig()
    c.patch_size = spec.patch_size; c.d_model = spec.d_model; c.num_heads = spec.num_heads
    c.mlp_hidden_dim = spec.mlp_hidden_dim; c.n_layers = len(spec.block_schedule)
    for i, s in enumerate(spec.block_schedule):
        c.schedule[i] = LAYER_KIND[s]
    c.num_quantiles = spec.num_quantiles
    for i, k in enumerate(spec.quantile_knots):
        c.knots[i] = k
    c.block_size = spec.block_size; c.context_length = spec.context_length
    c.rope_dim = spec.rope_dim; c.rope_table_pos_min = spec.pos_min; c.norm_eps = np.float32(spec.norm_eps)
    c.attn_bias = int(spec.attn_bias); c.mlp_bias = int(spec.mlp_bias)
    c.time_gate = int(spec.time_gate == "sdpa_sigmoid"); c.variate_gate = int(spec.variate_gate == "sdpa_sigmoid")
    c.minimum_scale = spec.minimum_scale; c.use_asinh = int(spec.use_asinh)
    c.covariate_enabled = int(spec.covariate_enabled); c.attend_missing_patches = int(spec.attend_missing_patches)
    c.quantile_width_factor = spec.quantile_width_factor; c.per_shot_horizon_patches = spec.per_shot_horizon_patches
    c.quantile_real_cap_k = spec.quantile_real_cap_k; c.extreme_value_threshold = spec.extreme_value_threshold
    c.symmetric_averaging = int(spec.symmetric_averaging); c.clip_nonnegative = int(spec.clip_nonnegative)
    c.target_encoding_smooth = spec.target_encoding_smooth
    return c


class OracleModel:
    """The oracle's copy of one GGUF model."""

    def __init__(self, path):
        import gguf
        reader = gguf.GGUFReader(str(path))
        self.config = config_from_reader(reader)
        self.knots = list(self.config.knots[: self.config.num_quantiles])
        L = lib()
        self.h = L.oracle_model_new(C.byref(self.config))
        types = {gguf.GGMLQuantizationType.F32: 0, gguf.GGMLQuantizationType.F16: 1,
                 gguf.GGMLQuantizationType.Q8_0: 8}
        for t in reader.tensors:
            ne = [int(x) for x in t.shape]
            ne0 = ne[0]
            ne1 = int(np.prod(ne[1:])) if len(ne) > 1 else 1
            data = np.ascontiguousarray(np.asarray(t.data))
            _check(L.oracle_model_set(self.h, t.name.encode(), ptr(data), types[t.tensor_type], ne0, ne1))

    def __del__(self):
        try:
            lib().oracle_model_free(self.h)
        except Exception:
            pass

    @property
    def Q(self):
        return self.config.num_quantiles

    def forecast(self, context, H, mask=None, past=None, known=None, cat_past=None, cat_known=None,
                 symmetric=-1, clip=-1, max_context=0, threads=None):
        context = np.ascontiguousarray(context, np.float32)
        B, V, T = context.shape
        keep = []

        def arr(a, dt):
            if a is None:
                return None, 0
            a = np.ascontiguousarray(a, dt)
            keep.append(a)
            return a, a.shape[1]
        m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        p, cp = arr(past, np.float32)
        k, ck = arr(known, np.float32)
        qp, ccp = arr(cat_past, np.float64)
        qk, cck = arr(cat_known, np.float64)
        r = OracleRequest(ptr(context), ptr(m), B, V, T, H, ptr(p), cp, ptr(k), ck, ptr(qp), ccp,
                          ptr(qk), cck, symmetric, clip, max_context)
        out = np.empty((B, V, H, self.Q), np.float32)
        _check(lib().oracle_forecast(self.h, C.byref(r), ptr(out), threads or os.cpu_count()))
        return out

    def predict_block(self, rows, observed, h, groups, roles=None, future=None, future_mask=None, threads=None):
        rows = np.ascontiguousarray(rows, np.float32)
        R, T = rows.shape
        obs = np.ascontiguousarray(observed, np.int8)
        g = np.ascontiguousarray(groups, np.int64)
        ro = None if roles is None else np.ascontiguousarray(roles, np.int64)
        f = None if future is None else np.ascontiguousarray(future, np.float32)
        fm = None if future_mask is None else np.ascontiguousarray(future_mask, np.int8)
        n = h * self.config.patch_size
        out = np.empty((R, n, self.Q), np.float32)
        norm = np.empty_like(out)
        loc = np.empty(R, np.float32)
        sc = np.empty(R, np.float32)
        _check(lib().oracle_predict_block(self.h, ptr(rows), ptr(obs), C.c_int64(R), C.c_int64(T), C.c_int64(h),
                                          ptr(g), ptr(ro), ptr(f), ptr(fm), ptr(out), ptr(norm), ptr(loc),
                                          ptr(sc), C.c_int32(threads or os.cpu_count())))
        return out, norm, loc, sc


def normalized_deviation(actual, ref, loc, scale):
    """Per-row normalized deviation of the reference's quantisation quality metric
    (scripts/quant_metrics.py:50-69): z = asinh((ref-loc)/scale), w = scale*cosh(z),
    e = |actual-ref| / (w * rms(z)). Returns (mean, max) over all rows."""
    means, maxs = normalized_deviation_rows(actual, ref, loc, scale)
    return float(np.mean(means)), float(np.max(maxs))


def normalized_deviation_rows(actual, ref, loc, scale):
    """The same metric per target row: (mean over the row's values, max over them), each
    an array of one entry per row."""
    ref = np.asarray(ref, np.float64)
    act = np.asarray(actual, np.float64)
    R = loc.shape[0]
    ref = ref.reshape(R, -1)
    act = act.reshape(R, -1)
    means, maxs = [], []
    for r in range(R):
        z = np.arcsinh((ref[r] - loc[r]) / scale[r])
        w = scale[r] * np.cosh(z)
        rms = float(np.sqrt(np.mean(z * z)))
        if rms == 0:
            same = np.array_equal(ref[r], act[r])
            means.append(0.0 if same else np.inf)
            maxs.append(0.0 if same else np.inf)
            continue
        e = np.abs(act[r] - ref[r]) / (w * rms)
        means.append(float(np.mean(e)))
        maxs.append(float(np.max(e)))
    return np.array(means), np.array(maxs)


# ---------------------------------------------------------------------------------------
# Component wrappers (known-answer tests).

def _i64(x):
    return np.ascontiguousarray(x, np.int64)


def scale_rows(cfg, x, mask, rows, length):
    x = np.ascontiguousarray(x, np.float32); m = np.ascontiguousarray(mask, np.int8)
    s, l, c = (np.empty(rows * length, np.float32) for _ in range(3))
    _check(lib().oracle_scale_rows(C.byref(cfg), ptr(x), ptr(m), C.c_int64(rows), C.c_int64(length), ptr(s), ptr(l), ptr(c)))
    return s, l, c


def instance_norm_stats(cfg, x, mask, rows, length):
    x = np.ascontiguousarray(x, np.float32); m = np.ascontiguousarray(mask, np.int8)
    loc, sc = np.empty(rows, np.float32), np.empty(rows, np.float32)
    b = np.empty(rows, np.int8)
    _check(lib().oracle_instance_norm_stats(C.byref(cfg), ptr(x), ptr(m), C.c_int64(rows), C.c_int64(length), ptr(loc), ptr(sc), ptr(b)))
    return loc, sc, b


def build_masks(cfg, observed, R, T, h, groups, roles=None):
    obs_in = np.ascontiguousarray(observed, np.int8)
    g = _i64(groups)
    ro = None if roles is None else _i64(roles)
    cov = int(bool(cfg.covariate_enabled and ro is not None and np.any(ro != 0)))
    N, S, L = C.c_int64(), C.c_int64(), C.c_int64()
    lib().oracle_mask_sizes(C.byref(cfg), C.c_int64(R), C.c_int64(T), C.c_int64(h), cov, C.byref(N), C.byref(S), C.byref(L))
    N, S = N.value, S.value
    ng = len(np.unique(g))
    out = dict(obs=np.zeros(R * N, np.int8), key_valid=np.zeros(R * N, np.int8), first_group=np.zeros(max(ng, 1), np.int64),
               positions=np.zeros(R * S, np.int64), time=np.zeros(R * S * S, np.int8), variate=np.zeros(S * R * R, np.int8),
               active=np.zeros(R * N, np.int8), anchor=np.zeros(R * N, np.int64))
    _check(lib().oracle_build_masks(C.byref(cfg), ptr(obs_in), C.c_int64(R), C.c_int64(T), C.c_int64(h), ptr(g), ptr(ro),
                                    ptr(out["obs"]), ptr(out["key_valid"]), ptr(out["first_group"]), ptr(out["positions"]),
                                    ptr(out["time"]), ptr(out["variate"]), ptr(out["active"]), ptr(out["anchor"])))
    out["first_group"] = out["first_group"][:ng]
    out["N"], out["S"] = N, S
    return out


def sdpa(q, k, v, mask, hd, H, S, R, split=0, threads=1):
    q, k, v, mask = (np.ascontiguousarray(a, np.float32) for a in (q, k, v, mask))
    out = np.empty_like(q)
    _check(lib().oracle_sdpa(ptr(q), ptr(k), ptr(v), ptr(mask), C.c_int64(hd), C.c_int64(H), C.c_int64(S), C.c_int64(R),
                             C.c_int64(split), ptr(out), C.c_int32(threads)))
    return out


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    _check(lib().oracle_rms_norm(ptr(x), ptr(w), C.c_int64(x.shape[0]), C.c_int64(x.shape[1]), C.c_float(eps), ptr(out)))
    return out


def linear_f32(w, x, b=None):
    w = np.ascontiguousarray(w, np.float32); x = np.ascontiguousarray(x, np.float32)
    b = None if b is None else np.ascontiguousarray(b, np.float32)
    N, K = w.shape
    y = np.empty((x.shape[0], N), np.float32)
    _check(lib().oracle_linear_f32(ptr(w), ptr(x), ptr(b), C.c_int64(K), C.c_int64(N), C.c_int64(x.shape[0]), ptr(y)))
    return y


def monotone_quantiles(cfg, raw):
    raw = np.ascontiguousarray(raw, np.float32)
    out = np.empty_like(raw)
    _check(lib().oracle_monotone_quantiles(C.byref(cfg), ptr(raw), C.c_int64(raw.size), ptr(out)))
    return out


def denormalize(x, loc, scale, Q, use_asinh):
    x = np.ascontiguousarray(x, np.float32); loc = np.ascontiguousarray(loc, np.float32); scale = np.ascontiguousarray(scale, np.float32)
    out = np.empty_like(x)
    rows = loc.size
    _check(lib().oracle_denormalize(ptr(x), ptr(loc), ptr(scale), C.c_int64(rows), C.c_int64(x.size // rows), C.c_int64(Q),
                                    C.c_int32(int(use_asinh)), ptr(out)))
    return out


def refine_block(cfg, q, x, mask, rows, length, patches, targets=None):
    q = np.ascontiguousarray(q, np.float32)
    x = np.ascontiguousarray(x if len(x) else np.zeros(1), np.float32)
    m = np.ascontiguousarray(mask if len(mask) else np.zeros(1), np.int8)
    t = None if targets is None else np.ascontiguousarray(targets, np.int8)
    out = np.empty_like(q)
    _check(lib().oracle_refine_block(C.byref(cfg), ptr(q), ptr(x), ptr(m), C.c_int64(rows), C.c_int64(length),
                                     C.c_int64(patches), ptr(t), ptr(out)))
    return out


def block_frames(cfg, x, mask, median, rows, length, patches):
    x = np.ascontiguousarray(x, np.float32); m = np.ascontiguousarray(mask, np.int8); md = np.ascontiguousarray(median, np.float64)
    loc, sc = np.empty(rows * patches), np.empty(rows * patches)
    _check(lib().oracle_block_frames(C.byref(cfg), ptr(x), ptr(m), ptr(md), C.c_int64(rows), C.c_int64(length),
                                     C.c_int64(patches), ptr(loc), ptr(sc)))
    return loc, sc


def set_per_shot(model, n):
    lib().oracle_model_set_per_shot(model.h, C.c_int32(n))


def set_round_attention(model, on):
    """Round q/k/v and sigmoid(gate) to f16 before attention (the device's storage)."""
    lib().oracle_model_set_round_attention(model.h, C.c_int32(int(on)))


def anchors(context, ps, minimum_scale=1e-6):
    """First-pass anchor frame of each target row (the causal loc/scale at the last step of
    the forward-filled, left-padded context), used to normalise forecast comparisons."""
    B, V, T = context.shape
    pad = (ps - T % ps) % ps
    rows = np.zeros((B * V, T + pad), np.float32)
    mask = np.zeros((B * V, T + pad), np.int8)
    for r, x in enumerate(np.asarray(context, np.float32).reshape(B * V, T)):
        obs = np.isfinite(x)
        idx = np.where(obs, np.arange(T), -1)
        idx = np.maximum.accumulate(idx)
        rows[r, pad:] = np.where(idx >= 0, x[np.maximum(idx, 0)], 0.0)
        mask[r, pad:] = obs
    cfg = OracleConfig()
    cfg.patch_size = ps
    cfg.minimum_scale = minimum_scale
    cfg.use_asinh = 1
    _, loc, sc = scale_rows(cfg, rows, mask, B * V, T + pad)
    L = T + pad
    return loc.reshape(B * V, L)[:, -1].copy(), sc.reshape(B * V, L)[:, -1].copy()
