"""Random-init Timestral models in the reference GGUF schema, and seeded synthetic series.

No trained weights or datasets exist on this machine, so every model the tests and the
benchmark use is written here: the tensor list and KV set of the reference loader
(src/model_loader.cpp:72-160 for the KVs, :166-207 for the tensor schema), the storage
policy of the converter (scripts/convert_timestral_to_gguf.py:123-142: F16 or Q8_0 only on
the projection weights of the allowlist, everything else F32), and the rope tables of the
reference class (scripts/convert_timestral_to_gguf.py:153-167, docs/PLAN.md A.5.4).

Weights: seed 0, linear weights N(0, 0.02), norm gains 1, biases 0, forecast_query
N(0, 0.02), drawn from one numpy Generator in schema order.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import re
from pathlib import Path

import numpy as np

KNOTS_21 = (0.01, 0.05, 0.1, 0.15, 0.2, 0.25, 0.3, 0.35, 0.4, 0.45, 0.5,
            0.55, 0.6, 0.65, 0.7, 0.75, 0.8, 0.85, 0.9, 0.95, 0.99)


@dataclasses.dataclass(frozen=True)
class ModelSpec:
    """The architecture KVs of one model (reference src/config.hpp:25-71)."""
    name: str
    patch_size: int
    d_model: int
    num_heads: int
    mlp_hidden_dim: int
    block_schedule: tuple
    quantile_knots: tuple
    block_size: int
    context_length: int
    rope_theta: float = 10000.0
    rope_partial_factor: float = 0.5
    norm_eps: float = 1e-6
    attn_bias: bool = False
    mlp_bias: bool = False
    time_gate: str = "sdpa_sigmoid"
    variate_gate: str = "sdpa_sigmoid"
    minimum_scale: float = 1e-6
    use_asinh: bool = True
    covariate_enabled: bool = True
    split_context_horizon: bool = True
    attend_missing_patches: bool = True
    quantile_width_factor: float = 3.0
    per_shot_horizon_patches: int = 32
    quantile_real_cap_k: float = 1e4
    extreme_value_threshold: float = 1e30
    symmetric_averaging: bool = True
    clip_nonnegative: bool = True
    target_encoding_smooth: float = 1.0
    norm_gain_spread: float = 0.0     # > 0: RMSNorm gains drawn from 1 + U(-spread, spread)

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.rope_partial_factor)

    @property
    def pos_min(self) -> int:
        return -(self.context_length // self.patch_size + self.block_size)

    @property
    def num_quantiles(self) -> int:
        return len(self.quantile_knots)


def spec_209m() -> ModelSpec:
    """Released Timestral-209M hyper-parameters (reference docs/PLAN.md:37-59)."""
    return ModelSpec(name="Timestral-209M-random", patch_size=32, d_model=768, num_heads=12,
                     mlp_hidden_dim=2048,
                     block_schedule=("time", "time", "time", "time_variate") * 6,
                     quantile_knots=KNOTS_21, block_size=32, context_length=32768)


def spec_tiny(bias: bool = False) -> ModelSpec:
    """The tiny test checkpoint of the reference (scripts/make_tiny_checkpoint.py:33-38)."""
    return ModelSpec(name="timestral-tiny" + ("-bias" if bias else ""), patch_size=8, d_model=32,
                     num_heads=4, mlp_hidden_dim=64,
                     block_schedule=("time", "variate", "time_variate", "variate_time"),
                     quantile_knots=(0.05, 0.1, 0.25, 0.4, 0.5, 0.6, 0.75, 0.9, 0.95),
                     block_size=4, context_length=2048, attn_bias=bias, mlp_bias=bias)


def spec_k256() -> ModelSpec:
    """spec_small with 256-wide rows (D = 256, four heads, F = 512), so that every reduced
    weight row is a whole number of 256-value K-quant super-blocks."""
    return ModelSpec(name="timestral-k256", patch_size=32, d_model=256, num_heads=4, mlp_hidden_dim=512,
                     block_schedule=("time", "variate", "time_variate", "variate_time"),
                     quantile_knots=KNOTS_21, block_size=32, context_length=4096)


def spec_small(bias: bool = False) -> ModelSpec:
    """A model with the 209M head and patch geometry (head_dim 64, patch 32, 21 knots) but
    two heads and four layers, one of each kind, so that tensor-core shapes are exercised
    at test sizes the CPU oracle finishes in seconds."""
    return ModelSpec(name="timestral-small" + ("-bias" if bias else ""), patch_size=32, d_model=128,
                     num_heads=2, mlp_hidden_dim=256,
                     block_schedule=("time", "variate", "time_variate", "variate_time"),
                     quantile_knots=KNOTS_21, block_size=32, context_length=4096,
                     attn_bias=bias, mlp_bias=bias)


def spec_small_long() -> ModelSpec:
    """spec_small with the 209M context length (32768 steps, 1024 context patches), so rows
    reach the long-row attention kernel (S up to 1056, 2112 with covariates)."""
    return ModelSpec(name="timestral-small-long", patch_size=32, d_model=128, num_heads=2, mlp_hidden_dim=256,
                     block_schedule=("time", "variate", "time_variate", "variate_time"),
                     quantile_knots=KNOTS_21, block_size=32, context_length=32768)


def spec_small_gains() -> ModelSpec:
    """spec_small with RMSNorm gains in [0.5, 1.5] (the random init of the others is 1), so
    that the norm weights folded into the consuming GEMM weights are not a no-op."""
    return dataclasses.replace(spec_small(), name="timestral-small-gains", norm_gain_spread=0.5)


LAYER_AXES = {"time": (True,), "variate": (False,), "time_variate": (True, False),
              "variate_time": (False, True)}

REDUCED = re.compile(r"blk\.[0-9]+\.(?:attn\.[0-9]+\.(?:qkv|gate|out)|ffn_w12|ffn_w3)\.weight")


def reduced_weight_name(name: str) -> bool:
    """The allowlist of weights that may be stored as F16/Q8_0
    (reference src/weight_policy.hpp:8-12)."""
    return name in {"patch.out.weight", "head.hidden.weight", "head.out.weight",
                    "head.res.weight"} or bool(REDUCED.fullmatch(name))


def schema(s: ModelSpec):
    """[(gguf name, numpy shape (torch order), kind)] in file order; kind is one of
    'linear', 'bias', 'norm', 'query', 'rope' (reference src/model_loader.cpp:166-207)."""
    D, F, ps, Q, hd = s.d_model, s.mlp_hidden_dim, s.patch_size, s.num_quantiles, s.head_dim
    out = [("patch.hidden.weight", (4 * D, 2 * ps), "linear"), ("patch.hidden.bias", (4 * D,), "bias"),
           ("patch.out.weight", (D, 4 * D), "linear"), ("patch.out.bias", (D,), "bias"),
           ("patch.res.weight", (D, 2 * ps), "linear"), ("patch.res.bias", (D,), "bias"),
           ("patch.forecast_query", (D,), "query")]
    for i, kind in enumerate(s.block_schedule):
        b = f"blk.{i}."
        for j, is_time in enumerate(LAYER_AXES[kind]):
            a = f"{b}attn.{j}."
            out.append((f"{b}attn_norm.{j}.weight", (D,), "norm"))
            out.append((a + "qkv.weight", (3 * D, D), "linear"))
            if s.attn_bias:
                out.append((a + "qkv.bias", (3 * D,), "bias"))
            if (s.time_gate if is_time else s.variate_gate) == "sdpa_sigmoid":
                out.append((a + "gate.weight", (D, D), "linear"))
                if s.attn_bias:
                    out.append((a + "gate.bias", (D,), "bias"))
            out.append((a + "out.weight", (D, D), "linear"))
            if s.attn_bias:
                out.append((a + "out.bias", (D,), "bias"))
        out.append((b + "ffn_norm.weight", (D,), "norm"))
        out.append((b + "ffn_w12.weight", (2 * F, D), "linear"))
        if s.mlp_bias:
            out.append((b + "ffn_w12.bias", (2 * F,), "bias"))
        out.append((b + "ffn_w3.weight", (D, F), "linear"))
        if s.mlp_bias:
            out.append((b + "ffn_w3.bias", (D,), "bias"))
    out += [("out_norm.weight", (D,), "norm"), ("head.hidden.weight", (4 * D, D), "linear"),
            ("head.out.weight", (ps * Q, 4 * D), "linear"), ("head.res.weight", (ps * Q, D), "linear")]
    P = 2 * (-s.pos_min) + 1
    out += [("rope.inv_freq", (hd // 2,), "rope"), ("rope.cos", (P, hd), "rope"), ("rope.sin", (P, hd), "rope")]
    return out


def rope_tables(s: ModelSpec):
    """inv_freq, cos, sin as float32, computed with torch float32 arithmetic: inv_freq[i] =
    1/theta**(2i/rope_dim) for i < rope_dim/2 else 0; emb = [pos*inv_freq, pos*inv_freq];
    tables cos(emb), sin(emb) for pos_min..-pos_min (reference docs/PLAN.md A.5.4, P9, P10)."""
    import torch
    hd, rd = s.head_dim, s.rope_dim
    inv = torch.zeros(hd // 2, dtype=torch.float32)
    inv[: rd // 2] = 1.0 / (s.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.int64).float() / rd))
    pos = torch.arange(s.pos_min, -s.pos_min + 1, dtype=torch.int64).float()
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return inv.numpy().copy(), torch.cos(emb).numpy().copy(), torch.sin(emb).numpy().copy()


def init_weights(s: ModelSpec, seed: int = 0):
    """Dict name -> float32 array (torch shape), random-init as documented in the module."""
    rng = np.random.default_rng(seed)
    inv, cos, sin = rope_tables(s)
    w = {}
    for name, shape, kind in schema(s):
        if kind == "linear" or kind == "query":
            w[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        elif kind == "bias":
            w[name] = np.zeros(shape, np.float32)
        elif kind == "norm":
            w[name] = np.ones(shape, np.float32)
            if s.norm_gain_spread > 0:
                w[name] += rng.uniform(-s.norm_gain_spread, s.norm_gain_spread, shape).astype(np.float32)
    w["rope.inv_freq"], w["rope.cos"], w["rope.sin"] = inv, cos, sin
    # The converter stores qkv rows head-major (docs/PLAN.md B.3); a random init has no
    # torch order to permute from, so the draw above is already taken as head-major.
    return w


# ---------------------------------------------------------------------------------------
# K-quant encoders for test models. They write valid ggml Q4_K / Q5_K / Q6_K super-blocks of
# 256 values (layouts as ggml publishes them) with simple min/max scales; they are not ggml's
# quantiser (which searches the scales), only a way to produce K-quant GGUFs to load.

def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def quantize_k(a, kind: str) -> np.ndarray:
    """a: [N][K] float32 with K % 256 == 0 -> uint8 [N][K/256 * block bytes]."""
    a = np.ascontiguousarray(a, np.float32)
    N, K = a.shape
    assert K % 256 == 0, K
    x = a.reshape(-1, 256)
    nb = x.shape[0]
    if kind in ("q4_k", "q5_k"):
        levels = 15 if kind == "q4_k" else 31
        sub = x.reshape(nb, 8, 32)
        mn = np.minimum(sub.min(axis=2), 0.0)
        mx = sub.max(axis=2)
        scale = (mx - mn) / levels
        mins = -mn
        d16 = _f16(scale.max(axis=1) / 63.0)
        m16 = _f16(mins.max(axis=1) / 63.0)
        d = d16.astype(np.float32)[:, None]
        dm = m16.astype(np.float32)[:, None]
        sc = np.where(d > 0, np.clip(np.rint(scale / np.where(d > 0, d, 1)), 0, 63), 0).astype(np.int32)
        mq = np.where(dm > 0, np.clip(np.rint(mins / np.where(dm > 0, dm, 1)), 0, 63), 0).astype(np.int32)
        step = (d * sc)[:, :, None]
        off = (dm * mq)[:, :, None]
        q = np.where(step > 0, np.clip(np.rint((sub + off) / np.where(step > 0, step, 1)), 0, levels), 0).astype(np.int32)
        scales = np.zeros((nb, 12), np.uint8)
        scales[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
        scales[:, 4:8] = (mq[:, 0:4] & 63) | ((mq[:, 4:8] >> 4) << 6)
        scales[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mq[:, 4:8] & 0xF) << 4)
        lo = (q & 0xF).astype(np.uint8).reshape(nb, 4, 2, 32)
        qs = (lo[:, :, 0, :] | (lo[:, :, 1, :] << 4)).reshape(nb, 128)
        parts = [d16.reshape(nb, 1).view(np.uint8), m16.reshape(nb, 1).view(np.uint8), scales]
        if kind == "q5_k":
            hi = ((q >> 4) & 1).astype(np.uint8)                       # [nb, 8, 32]
            qh = np.zeros((nb, 32), np.uint8)
            for j in range(8):
                qh |= hi[:, j, :] << j
            parts.append(qh)
        parts.append(qs)
        out = np.concatenate(parts, axis=1)
    elif kind == "q6_k":
        sub = x.reshape(nb, 16, 16)
        scale = np.abs(sub).max(axis=2) / 31.0
        d16 = _f16(scale.max(axis=1) / 127.0)
        d = d16.astype(np.float32)[:, None]
        sc = np.where(d > 0, np.clip(np.rint(scale / np.where(d > 0, d, 1)), 0, 127), 0).astype(np.int32)
        step = (d * sc)[:, :, None]
        q = np.where(step > 0, np.clip(np.rint(sub / np.where(step > 0, step, 1)), -32, 31), 0).astype(np.int32) + 32
        q = q.reshape(nb, 2, 4, 32)                                    # [half][t][l]: value l + 32 t
        ql = np.zeros((nb, 2, 64), np.uint8)
        ql[:, :, 0:32] = (q[:, :, 0, :] & 0xF) | ((q[:, :, 2, :] & 0xF) << 4)
        ql[:, :, 32:64] = (q[:, :, 1, :] & 0xF) | ((q[:, :, 3, :] & 0xF) << 4)
        qh = ((q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4) |
              ((q[:, :, 3, :] >> 4) << 6)).astype(np.uint8)
        out = np.concatenate([ql.reshape(nb, 128), qh.reshape(nb, 64), sc.astype(np.int8).view(np.uint8),
                              d16.reshape(nb, 1).view(np.uint8)], axis=1)
    else:
        raise ValueError(kind)
    return np.ascontiguousarray(out.reshape(N, -1))


K_QUANT_TYPES = {"q4_k": 12, "q5_k": 13, "q6_k": 14}


def write_gguf(path, s: ModelSpec, outtype: str = "f32", seed: int = 0, weights=None) -> Path:
    """Write one model file. outtype: f32, f16, q8_0, q4_k, q5_k or q6_k (reduced weights only)."""
    import gguf
    from gguf import GGUFValueType as VT
    if outtype not in ("f32", "f16", "q8_0", "q4_k", "q5_k", "q6_k"):
        raise ValueError(outtype)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    w = weights if weights is not None else init_weights(s, seed)
    wr = gguf.GGUFWriter(str(path), "timestral")
    S = lambda k, v: wr.add_key_value(k, v, VT.STRING)
    U = lambda k, v: wr.add_key_value(k, int(v), VT.UINT32)
    F64 = lambda k, v: wr.add_key_value(k, float(v), VT.FLOAT64)
    B = lambda k, v: wr.add_key_value(k, bool(v), VT.BOOL)
    S("general.name", s.name)
    S("general.license", "Random weights written by the timestral-b200 test generator.")
    S("general.license.name", "none")
    S("general.license.link", "")
    S("general.source.url", "")
    S("timestral.source.hf_revision", "")
    S("timestral.source.code_sha", "")
    S("timestral.source.weights_sha256", "")
    U("timestral.converter_version", 1)
    if outtype != "f32":
        S("timestral.conversion.outtype", outtype)
    U("timestral.patch_size", s.patch_size)
    U("timestral.embedding_length", s.d_model)
    U("timestral.attention.head_count", s.num_heads)
    U("timestral.feed_forward_length", s.mlp_hidden_dim)
    U("timestral.block_count", len(s.block_schedule))
    wr.add_key_value("timestral.block_schedule", list(s.block_schedule), VT.ARRAY, VT.STRING)
    wr.add_key_value("timestral.quantile_knots", [float(q) for q in s.quantile_knots], VT.ARRAY, VT.FLOAT64)
    U("timestral.block_size", s.block_size)
    U("timestral.context_length", s.context_length)
    F64("timestral.rope.freq_base", s.rope_theta)
    F64("timestral.rope.partial_factor", s.rope_partial_factor)
    U("timestral.rope.dimension_count", s.rope_dim)
    wr.add_key_value("timestral.rope.table_pos_min", int(s.pos_min), VT.INT32)
    wr.add_key_value("timestral.attention.layer_norm_rms_epsilon", float(np.float32(s.norm_eps)), VT.FLOAT32)
    B("timestral.attention.bias", s.attn_bias)
    B("timestral.mlp.bias", s.mlp_bias)
    S("timestral.attention.time_gate", s.time_gate)
    S("timestral.attention.variate_gate", s.variate_gate)
    B("timestral.attention.split_context_horizon", s.split_context_horizon)
    B("timestral.attention.qkv_head_major", True)
    F64("timestral.scaler.minimum_scale", s.minimum_scale)
    B("timestral.scaler.use_asinh", s.use_asinh)
    B("timestral.scaler.stabilize_with_global", False)
    B("timestral.covariate_enabled", s.covariate_enabled)
    B("timestral.attend_missing_patches", s.attend_missing_patches)
    F64("timestral.quantile_width_factor", s.quantile_width_factor)
    U("timestral.forecaster.per_shot_horizon_patches", s.per_shot_horizon_patches)
    F64("timestral.forecaster.quantile_real_cap_k", s.quantile_real_cap_k)
    F64("timestral.forecaster.extreme_value_threshold", s.extreme_value_threshold)
    B("timestral.forecaster.symmetric_averaging", s.symmetric_averaging)
    B("timestral.forecaster.clip_nonnegative", s.clip_nonnegative)
    F64("timestral.target_encoding.smooth", s.target_encoding_smooth)
    for name, shape, kind in schema(s):
        a = np.ascontiguousarray(w[name], dtype=np.float32)
        assert a.shape == tuple(shape), (name, a.shape, shape)
        if outtype == "f16" and reduced_weight_name(name):
            wr.add_tensor(name, np.ascontiguousarray(a.astype(np.float16)),
                          raw_dtype=gguf.GGMLQuantizationType.F16)
        elif outtype == "q8_0" and reduced_weight_name(name):
            from gguf.quants import quantize
            q = quantize(a, gguf.GGMLQuantizationType.Q8_0)
            wr.add_tensor(name, np.ascontiguousarray(q), raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif outtype in K_QUANT_TYPES and reduced_weight_name(name):
            q = quantize_k(a.reshape(a.shape[0], -1), outtype)
            wr.add_tensor(name, q, raw_dtype=gguf.GGMLQuantizationType(K_QUANT_TYPES[outtype]))
        else:
            wr.add_tensor(name, a, raw_dtype=gguf.GGMLQuantizationType.F32)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return path


def cached_model(s: ModelSpec, outtype: str, seed: int = 0, root=None) -> Path:
    """Write (once) and return the path of a model file under a scratch directory."""
    root = Path(root or os.environ.get("TSB200_MODEL_DIR", "/tmp/tsb200_models"))
    key = hashlib.sha1(json.dumps([dataclasses.asdict(s), outtype, seed, 1], sort_keys=True,
                                  default=list).encode()).hexdigest()[:12]
    path = root / f"{s.name}-{outtype}-{key}.gguf"
    if not path.exists():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        write_gguf(tmp, s, outtype, seed)
        os.replace(tmp, path)
    return path


# ---------------------------------------------------------------------------------------
# Seeded synthetic series with the shapes and value distributions of each workload.

def series_sine(T: int, seed: int = 0):
    """x_t = sin(2*pi*t/24) + 0.1*N(0,1); B=V=1."""
    rng = np.random.default_rng(seed)
    t = np.arange(T)
    return (np.sin(2 * np.pi * t / 24) + 0.1 * rng.standard_normal(T)).astype(np.float32)[None, None, :]


def series_dyadic(T: int, V: int = 1):
    """The reference benchmark's input (named dyadic-v1 there): x[v, t] = (((17 t + 13 v) mod
    257) - 128) / 64, exact in f32, no missing values; shape [1, V, T]. Its sum is -8.5625 at
    T = 32768 and -3.234375 at T = 512 (V = 1), the input checksums the reference reports."""
    t = np.arange(T, dtype=np.int64)[None, :]
    v = np.arange(V, dtype=np.int64)[:, None]
    return ((((17 * t + 13 * v) % 257) - 128) / 64.0).astype(np.float32)[None]


def reference_case_inputs(case: dict, patch_size: int) -> dict:
    """Inputs of one case of the reference's forecast tests (its tests/cases.json), built as
    its generator builds them (reference scripts/gen_reference_baseline.py:675-745): one
    numpy default_rng(seed); per series b and variate v a Gaussian random walk plus
    10 sin(2 pi t / (period (1 + v/4)) + 0.3 b), a level and a linear trend (absolute values
    when `positive`, every step `constant` when given); missing steps: the first `leading`
    steps and the listed whole patches of the first row, a scattered fraction, and whole rows;
    numeric covariates 5 sin(2 pi t / (period + 7 + 5 c) + b / 2) + N(0, 1/4) (known ones over
    T + H), 0/1 indicator rows alternating every 5 + 2 c steps, categorical codes drawn
    uniformly (a code unseen in the context at step T + H/2 of the known ones when asked).
    Returns {"context": [B,V,T] float32, "past", "known": float32, "cat_past", "cat_known":
    float64 (NaN = missing)} with the keys the case uses."""
    rng = np.random.default_rng(case["seed"])
    B, V, T, H = case["B"], case["V"], case["T"], case["H"]
    s = case.get("series", {})
    period = s.get("period", 24)
    t = np.arange(T, dtype=np.float64)
    x = np.empty((B, V, T))
    for b in range(B):
        for v in range(V):
            walk = np.cumsum(rng.normal(0.0, s.get("noise_std", 1.0), T))
            wave = 10.0 * np.sin(2.0 * np.pi * t / (period * (1.0 + 0.25 * v)) + 0.3 * b)
            x[b, v] = s.get("level", 0.0) + s.get("trend", 0.0) * t + wave + walk
    if s.get("positive"):
        x = np.abs(x)
    if s.get("constant") is not None:
        x[:] = s["constant"]
    x = x.astype(np.float32)
    rows = x.reshape(B * V, T)
    miss = case.get("missing", {})
    if miss.get("leading"):
        rows[0, :miss["leading"]] = np.nan
    for p in miss.get("missing_patches", []):
        rows[0, p * patch_size:(p + 1) * patch_size] = np.nan
    if miss.get("scattered_frac"):
        rows[rng.random(rows.shape) < miss["scattered_frac"]] = np.nan
    for i in miss.get("all_missing_series", []):
        rows[i, :] = np.nan
    out = {"context": x}

    def numeric_rows(n, length, nan_frac):
        tt = np.arange(length, dtype=np.float64)
        r = np.empty((B, n, length))
        for b in range(B):
            for c in range(n):
                r[b, c] = 5.0 * np.sin(2 * np.pi * tt / (period + 7 + 5 * c) + 0.5 * b) + 0.5 * rng.normal(size=length)
        r = r.astype(np.float32)
        if nan_frac:
            r[rng.random(r.shape) < nan_frac] = np.nan
        return r

    pc = case.get("past", {})
    if pc.get("numeric"):
        out["past"] = numeric_rows(pc["numeric"], T, pc.get("nan_frac", 0.0))
    kc = case.get("known", {})
    if kc.get("numeric") or kc.get("indicator"):
        parts = []
        if kc.get("numeric"):
            parts.append(numeric_rows(kc["numeric"], T + H, kc.get("nan_frac", 0.0)))
        if kc.get("indicator"):
            tt = np.arange(T + H)
            ind = np.empty((B, kc["indicator"], T + H), np.float32)
            for c in range(kc["indicator"]):
                ind[:, c, :] = ((tt // (5 + 2 * c)) % 2 == 0).astype(np.float32)
            parts.append(ind)
        out["known"] = np.concatenate(parts, axis=1)
    cp = case.get("cat_past", {})
    if cp.get("rows"):
        codes = rng.integers(0, cp["n_codes"], size=(B, cp["rows"], T)).astype(np.float64)
        if cp.get("nan_frac"):
            codes[rng.random(codes.shape) < cp["nan_frac"]] = np.nan
        out["cat_past"] = codes
    ck = case.get("cat_known", {})
    if ck.get("rows"):
        codes = rng.integers(0, ck["n_codes"], size=(B, ck["rows"], T + H)).astype(np.float64)
        if ck.get("unseen_in_horizon"):
            codes[:, :, T + H // 2] = ck["n_codes"] + 7
        if ck.get("nan_frac"):
            codes[rng.random(codes.shape) < ck["nan_frac"]] = np.nan
        out["cat_known"] = codes
    return out


def series_random_walk(B: int, T: int, nan_frac: float = 0.05, seed0: int = 0):
    """Gaussian random walk (step N(0,1), seed = i) plus a level offset U(-100, 100), with
    a fraction of context steps set to NaN; shape [B,1,T]."""
    out = np.empty((B, 1, T), np.float32)
    for i in range(B):
        rng = np.random.default_rng(seed0 + i)
        x = np.cumsum(rng.standard_normal(T)) + rng.uniform(-100, 100)
        x[rng.random(T) < nan_frac] = np.nan
        out[i, 0] = x
    return out


def series_var1(B: int, V: int, T: int, seed: int = 0):
    """VAR(1) x_t = 0.9 x_{t-1} + eps, eps ~ N(0, Sigma), Sigma_ij = 0.5^|i-j|; [B,V,T]."""
    rng = np.random.default_rng(seed)
    idx = np.arange(V)
    L = np.linalg.cholesky(0.5 ** np.abs(idx[:, None] - idx[None, :]))
    out = np.empty((B, V, T), np.float32)
    for b in range(B):
        x = np.zeros(V)
        eps = rng.standard_normal((T, V)) @ L.T
        for t in range(T):
            x = 0.9 * x + eps[t]
            out[b, :, t] = x
    return out


def series_covariates(B: int, V: int, T: int, H: int, seed: int = 0):
    """Targets, 8 past AR(1) covariates, 4 known sinusoidal covariates (periods
    7/24/168/365 plus noise), 2 categorical known covariates in [0, 16)."""
    rng = np.random.default_rng(seed)
    past = np.empty((B, 8, T), np.float32)
    for b in range(B):
        e = rng.standard_normal((8, T))
        x = np.zeros(8)
        for t in range(T):
            x = 0.7 * x + e[:, t]
            past[b, :, t] = x
    t = np.arange(T + H)
    known = np.empty((B, 4, T + H), np.float32)
    for b in range(B):
        for j, p in enumerate((7, 24, 168, 365)):
            known[b, j] = np.sin(2 * np.pi * t / p + rng.uniform(0, 2 * np.pi)) + 0.1 * rng.standard_normal(T + H)
    cat = rng.integers(0, 16, size=(B, 2, T + H)).astype(np.float64)
    walk = np.cumsum(rng.standard_normal((B, V, T)), axis=-1)
    target = (0.5 * known[:, :, :T].sum(axis=1, keepdims=True) + walk).astype(np.float32)
    return target, past, known, cat


def series_seasonal(B: int, T: int, nan_frac: float = 0.01, seed0: int = 0):
    """Seasonal sine (period U[12,200]) + trend + noise, with NaNs; seeded per series."""
    out = np.empty((B, 1, T), np.float32)
    t = np.arange(T, dtype=np.float64)
    for i in range(B):
        rng = np.random.default_rng(seed0 + i)
        period = rng.uniform(12, 200)
        amp = rng.uniform(0.5, 10)
        x = amp * np.sin(2 * np.pi * t / period + rng.uniform(0, 2 * np.pi))
        x += rng.uniform(-0.01, 0.01) * t + rng.uniform(-50, 50) + 0.2 * rng.standard_normal(T)
        x[rng.random(T) < nan_frac] = np.nan
        out[i, 0] = x
    return out
