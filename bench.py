"""Forecast throughput benchmark (series/sec) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg5] [--weights f16|q8_0|q6_k|q5_k|q4_k]
                    [--batch B] [--no-cpu] [--no-e2e]
    python bench.py --impl reference ...   # the CPU reference arm (rank 0 only)
    python bench.py --compare-cublas       # the fused GEMMs against cuBLAS at the cfg5 shapes

Workloads (209M architecture, random init seed 0, synthetic series of each config's shape;
symmetric averaging and clipping on):
  cfg1  f32  B=1    V=1   T=512   H=64   sin(2 pi t / 24) + 0.1 N(0,1)
  cfg2  f16  B=64   V=1   T=2048  H=256  random walks + U(-100,100) offset, 5% NaN
  cfg3  f16  B=16   V=32  T=1024  H=128  VAR(1), Sigma_ij = 0.5^|i-j|
  cfg4  f16  B=32   V=4   T=1024  H=96   + 8 past, 4 known, 2 categorical known covariates
  cfg5  f16 (or --weights q8_0 / K-quants)  B=4096  V=1  T=2048  H=256  seasonal sine + trend, 1% NaN
  cfg6  f16  B=64   V=1   T=32768 H=1024 long context, seasonal + 1% NaN
  pub32k / pub512  f32  B=1  T=32768 / 512, H=1024 / 32: the reference's published benchmark
        shapes on its dyadic-v1 input, with the ratio to its published seconds as vs_baseline
The default is cfg5, the throughput configuration the headline metric is quoted on. The
batch is sharded across GPUs with no collective on the forecast path; each rank runs its
slice through its own handle.

Printed JSON (rank 0): `value` is whole-job series/sec with the context already in device
memory (tsb_forecast_device, CUDA events on the engine stream, max over ranks; cfg4's
covariates have no device-resident entry, so its `value` goes through the C ABI); `e2e` is
the same metric through timestral_capi_forecast with host buffers (upload and download
inside the timed region); `roofline` is the time-attention kernel timed with CUDA events
around each of its launches over K more steps run right after the (uninstrumented) timed
region; `roofline_gemm` the tensor-core GEMMs of one extra evented step;
`cpu_baseline` the CPU oracle on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "timestral.cpp_b200"))

D_MODEL, D_FF, HEADS, HEAD_DIM, PATCH, N_Q = 768, 2048, 12, 64, 32, 21
TIME_SUBLAYERS, VARIATE_SUBLAYERS, MLPS = 24, 6, 24

CONFIGS = {
    "cfg1": dict(weights="f32", B=1, V=1, T=512, H=64, cpu_sample=1,
                 desc="cfg1: 209M f32 random-init, B=1, V=1, T=512, H=64, sine + noise"),
    "cfg2": dict(weights="f16", B=64, V=1, T=2048, H=256, cpu_sample=8,
                 desc="cfg2: 209M f16 random-init, B=64, V=1, T=2048, H=256, random walks, 5% NaN"),
    "cfg3": dict(weights="f16", B=16, V=32, T=1024, H=128, cpu_sample=1,
                 desc="cfg3: 209M f16 random-init, B=16, V=32, T=1024, H=128, VAR(1)"),
    "cfg4": dict(weights="f16", B=32, V=4, T=1024, H=96, cpu_sample=1,
                 desc="cfg4: 209M f16 random-init, B=32, V=4, T=1024, H=96, 8 past + 4 known + 2 categorical covariates"),
    "cfg5": dict(weights=None, B=4096, V=1, T=2048, H=256, cpu_sample=16,
                 desc="cfg5 throughput: 209M {w} random-init, B={B} series ({per} per GPU), V=1, T=2048, H=256, symmetric+clip"),
    # The reference's own published benchmark shape (its docs/benchmarks.md measurement
    # contract): F32 weights, one series, context 32768, horizon 1024, the dyadic-v1 input,
    # symmetric averaging and clipping on. The oracle takes tens of seconds per call here,
    # so its CPU line is one call after one warm-up on all threads, with no one-thread run.
    "pub32k": dict(weights="f32", B=1, V=1, T=32768, H=1024, cpu_sample=1, cpu_sample_1t=0, cpu_repeats=1,
                   desc="pub32k: the reference's published benchmark shape: 209M f32 random-init, B=1, V=1, "
                        "T=32768, H=1024 (S=1056, one 32-patch block), dyadic-v1 input "
                        "((17t+13v) mod 257 - 128)/64, symmetric+clip",
                   published={"seconds_per_forecast": 18.281547354, "threads": 6,
                              "what": "timestral.cpp standalone-MKL profile 68a5a53, 209M F32, context 32768, "
                                      "horizon 1024, B=1, median of 5 after one warm-up",
                              "one_thread_seconds": 36.392652770,
                              "pytorch_reference_seconds": {"1": 14.379144, "6": 4.443924},
                              "cpu": "AMD Ryzen 5 7430U (6 cores)", "source": "docs/benchmarks.md of the reference"}),
    "pub512": dict(weights="f32", B=1, V=1, T=512, H=32, cpu_sample=1,
                   desc="pub512: the reference's published short benchmark shape: 209M f32 random-init, B=1, V=1, "
                        "T=512, H=32, dyadic-v1 input ((17t+13v) mod 257 - 128)/64, symmetric+clip",
                   published={"seconds_per_forecast": 0.405898183, "threads": 6,
                              "what": "timestral.cpp native with the optimized linear kernels, 209M F32, context 512, "
                                      "horizon 32, B=1",
                              "one_thread_seconds": 1.541307288,
                              "pytorch_reference_seconds": {"1": 0.419565},
                              "cpu": "AMD Ryzen 5 7430U (6 cores)", "source": "docs/m6c-linear.md and docs/benchmarks.md of the reference"}),
    "cfg6": dict(weights="f16", B=64, V=1, T=32768, H=1024, cpu_sample=1,
                 desc="cfg6 long context: 209M f16 random-init, B=64, V=1, T=32768 (the full 1024-patch context), "
                      "H=1024 (one 32-patch decode block, S=1056), seasonal + 1% NaN"),
}

# DRAM bytes (read + write) of one time-attention (row, head) problem at S = 72: a constant
# taken from ncu captures of the kernel (B = 1024, dram__bytes_read.sum +
# dram__bytes_write.sum over 24,576 problems, mean of two launches), not measured by this
# script; traffic per launch scales with the problems. The bench line says so in
# roofline.traffic_source.
ATTN_DRAM_BYTES_PER_PROBLEM = 45220
# The same for the long-row kernel at S = 1056 (cfg6), per (row, head) plane (B = 8: 119.4 MB
# over 192 planes).
ATTN_LONG_DRAM_BYTES_PER_PLANE = 621760


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg5", choices=sorted(CONFIGS))
    ap.add_argument("--weights", default="f16", choices=["f16", "q8_0", "q6_k", "q5_k", "q4_k"],
                    help="cfg5 weight type")
    ap.add_argument("--batch", type=int, default=0, help="override the config's batch")
    ap.add_argument("--cpu-sample", type=int, default=0, help="series timed on the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--compare-cublas", action="store_true",
                    help="time each fused GEMM kind and cuBLAS (torch.mm, f16 in/out) at the cfg5 token count")
    a = ap.parse_args()
    c = dict(CONFIGS[a.config])
    c.setdefault("cpu_sample_1t", 1)
    if c["weights"] is None:
        c["weights"] = a.weights
    if a.batch:
        c["B"] = a.batch
    if a.cpu_sample:
        c["cpu_sample"] = a.cpu_sample
    return a, c


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            hbm, burst = float(d["hbm_gbs"]), float(d["bf16_tflops"])
            return hbm, burst, float(d.get("bf16_tflops_sustained", burst)), "measured"
        except (ValueError, KeyError, TypeError):
            pass                  # unreadable: the fallback figures below, labelled as such
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU during the timed region, read
    through NVML every 20 ms from a thread (reading only; nothing is set). Falls back to
    `nvidia-smi -lms 200` when NVML is not importable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.samples = []         # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self.stop_flag = threading.Event()
        self.thread = None
        self.nvml = None

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nvml = nv
            handle = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)),
                                             int(nv.nvmlDeviceGetCurrentClocksEventReasons(handle))))
                    except Exception:
                        pass
                    self.stop_flag.wait(0.02)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            reasons = set()
            for _, mask in self.samples:
                for name, attr in self.REASONS:
                    if mask & getattr(self.nvml, attr, 0):
                        reasons.add(name)
            sm = [mhz for mhz, _ in self.samples]
            return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml, 20 ms"}
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = [n for n, _ in self.REASONS]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def workload(cfg: str, c: dict, lo: int, hi: int):
    """Inputs of series [lo, hi) of the config: (context [b,V,T], covariate kwargs)."""
    from timestral_b200 import synthetic as sy
    T, H, V = c["T"], c["H"], c["V"]
    if cfg == "cfg1":
        return np.repeat(sy.series_sine(T, seed=0), hi - lo, axis=0), {}
    if cfg == "cfg2":
        return sy.series_random_walk(hi - lo, T, nan_frac=0.05, seed0=lo), {}
    if cfg == "cfg3":
        return sy.series_var1(c["B"], V, T, seed=0)[lo:hi], {}
    if cfg == "cfg4":
        target, past, known, cat = sy.series_covariates(c["B"], V, T, H, seed=0)
        return target[lo:hi], {"past": past[lo:hi], "known": known[lo:hi], "cat_known": cat[lo:hi]}
    if cfg in ("pub32k", "pub512"):
        return np.repeat(sy.series_dyadic(T, V), hi - lo, axis=0), {}
    out = np.empty((hi - lo, 1, T), np.float32)
    for k, i in enumerate(range(lo, hi)):
        out[k] = sy.series_seasonal(1, T, nan_frac=0.01, seed0=i)[0]
    return out, {}


def model_path(weights: str, rank: int, dist):
    from timestral_b200 import synthetic as sy
    if rank == 0:
        sy.cached_model(sy.spec_209m(), weights)
    if dist is not None:
        dist.barrier()
    return sy.cached_model(sy.spec_209m(), weights)


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def oracle_runs(cfg: str, c: dict, sample: int, threads: int, repeats: int):
    """Seconds of `repeats` timed calls of the CPU oracle (the port of the reference's
    forecast path) on the first `sample` series of the workload, after one untimed call."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle_py as op
    from timestral_b200 import synthetic as sy
    m = op.OracleModel(sy.cached_model(sy.spec_209m(), c["weights"]))
    x, kw = workload(cfg, c, 0, sample)
    m.forecast(x[:1], c["H"], threads=threads, **{k: v[:1] for k, v in kw.items()})   # warm caches
    out = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        m.forecast(x, c["H"], threads=threads, **kw)
        out.append(time.perf_counter() - t0)
    return out


def _cpu_child(cfg, c, plan, q):
    import resource
    res = []
    for sample, threads, repeats in plan:
        res.append((sample, threads, oracle_runs(cfg, c, sample, threads, repeats)))
    q.put((res, resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * 1024))


def cpu_baseline(cfg: str, c: dict, repeats: int = 5):
    """The CPU oracle on a bounded sample of the same workload, timed in a spawned child
    process (its own peak RSS, no GPU state): all host threads on `cpu_sample` series and one
    thread on `cpu_sample_1t` series, each the median of `repeats` calls after one warm-up."""
    import multiprocessing as mp
    threads = os.cpu_count() or 1
    repeats = c.get("cpu_repeats", repeats)
    plan = [(c["cpu_sample"], threads, repeats)]
    if c["cpu_sample_1t"]:
        plan.append((c["cpu_sample_1t"], 1, repeats))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_cpu_child, args=(cfg, c, plan, q))
    p.start()
    res, rss = q.get()
    p.join()
    (s_all, t_all, d_all) = res[0]
    med_all = float(np.median(d_all))
    out = {"value": s_all / med_all, "unit": "series/s", "cores": t_all, "kind": "port",
           "sample": f"{s_all} series of the same workload ({c['weights']} 209M, V={c['V']}, T={c['T']}, "
                     f"H={c['H']}) per call, median of {repeats} calls ({med_all:.2f} s) after one warm-up",
           "peak_rss_bytes": int(rss), "cpu_model": cpu_model()}
    if len(res) > 1:
        s_one, _, d_one = res[1]
        med_one = float(np.median(d_one))
        out["one_thread"] = {"value": s_one / med_one, "unit": "series/s", "cores": 1,
                             "sample": f"{s_one} series per call, median of {repeats} calls ({med_one:.2f} s)"}
    return out


def gemm_flops(rows: int, S: int, L: int, V_rows: int, decoder_tokens: int) -> int:
    """Tensor-core GEMM FLOPs of one decode block: per token 24 time sublayers
    (q|k|v|gate + out: 5 D^2 MACs), 6 variate sublayers (3 D^2 when a series has one row:
    v|gate + out; else 5 D^2), 24 MLPs (3 D F); the context-patch projections (K = 64:
    4 D + D outputs, then 4 D -> D); the head per decoder token (D -> 4D -> 21*32, plus
    the D -> 21*32 residual)."""
    D, F = D_MODEL, D_FF
    var = 3 * D * D if V_rows == 1 else 5 * D * D
    per_token = TIME_SUBLAYERS * 5 * D * D + VARIATE_SUBLAYERS * var + MLPS * 3 * D * F
    patch = 2 * PATCH * 5 * D + 4 * D * D
    head = D * 4 * D + 4 * D * N_Q * PATCH + D * N_Q * PATCH
    return 2 * rows * (S * per_token + L * patch + decoder_tokens * head)


def compare_cublas(seconds: float = 2.0):
    """The production GEMM kinds of the 209M layer (tsb_test_gemm, one tcgen05 launch each)
    and cuBLAS (torch.mm, f16 operands, f16 output, no epilogue) on the same operands at the
    cfg5 token count (M = 4096 series x 2 passes x 72 tokens), each looped for `seconds` so
    that the power cap settles; one JSON line per op with its SM clock. The test entry
    synchronizes after each launch (a few microseconds of idle per launch are included)."""
    import ctypes as C
    import torch
    import timestral_b200 as tb
    M, S, H, D, F = 589_824, 72, 12, 768, 2048
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape):
        return (torch.randn(*shape, device=dev, generator=g) * 0.05).to(torch.float16)

    def ptr(t):
        return C.c_void_p(t.data_ptr()) if t is not None else None

    def ours(kind, A, B, N, K, out=None, resid=None, qkvg=None, rope=None):
        t = tb.GemmTest()
        t.kind, t.A, t.lda, t.B, t.ldb, t.M, t.N, t.K = kind, ptr(A), A.shape[1], ptr(B), B.shape[1], M, N, K
        t.out, t.ldo, t.resid = ptr(out), (out.shape[1] if out is not None else 0), ptr(resid)
        if qkvg is not None:
            for i in range(4):
                t.qkvg[i] = qkvg[i].data_ptr()
            t.S, t.H, t.D, t.rope = S, H, D, 1
            t.cos_tab, t.sin_tab, t.rope_row = ptr(rope[0]), ptr(rope[1]), ptr(rope[2])
            t.rope_half, t.rope_dup = 16, 1
        err = C.c_int32(0)

        def call():
            rc = tb.lib().tsb_test_gemm(C.byref(t), C.byref(err))
            if rc != 0:
                raise RuntimeError(f"tsb_test_gemm kind {kind}: {rc} ({err.value})")
        return call

    A768, A2048 = rnd(M, D), rnd(M, F)
    Wqkvg, W12, Wout, W3 = rnd(4 * D, D), rnd(2 * F, D), rnd(D, D), rnd(D, F)
    ang = torch.rand(2113, 16, device=dev, generator=g) * 6.283
    cos, sin = torch.ones(2113, 64, device=dev), torch.zeros(2113, 64, device=dev)
    for lo in (0, 32):   # rotated dims 0-15 and 32-47 (the 209M table), equal halves
        cos[:, lo:lo + 16], sin[:, lo:lo + 16] = torch.cos(ang), torch.sin(ang)
    rope_row = (torch.arange(M, device=dev, dtype=torch.int32) % S) + 1000
    qkvg = [torch.empty(M, D, device=dev, dtype=torch.float16) for _ in range(4)]
    swi = torch.empty(M, F, device=dev, dtype=torch.float16)
    res = torch.zeros(M, D, device=dev, dtype=torch.float32)
    o3072 = torch.empty(M, 4 * D, device=dev, dtype=torch.float16)
    o4096 = torch.empty(M, 2 * F, device=dev, dtype=torch.float16)
    o768 = torch.empty(M, D, device=dev, dtype=torch.float16)
    ops = [
        ("fused q/k/v/gate + RoPE + sigmoid(gate), head-major", ours(6, A768, Wqkvg, 4 * D, D, qkvg=qkvg, rope=(cos, sin, rope_row)), 4 * D, D),
        ("cuBLAS, same operands, plain f16 output", lambda: torch.mm(A768, Wqkvg.t(), out=o3072), 4 * D, D),
        ("fused MLP up + SwiGLU", ours(4, A768, W12, 2 * F, D, out=swi), 2 * F, D),
        ("cuBLAS, same operands, plain f16 output", lambda: torch.mm(A768, W12.t(), out=o4096), 2 * F, D),
        ("fused out projection + f32 residual add", ours(2, A768, Wout, D, D, out=res, resid=res), D, D),
        ("cuBLAS, same operands, plain f16 output", lambda: torch.mm(A768, Wout.t(), out=o768), D, D),
        ("fused MLP down + f32 residual add", ours(2, A2048, W3, D, F, out=res, resid=res), D, F),
        ("cuBLAS, same operands, plain f16 output", lambda: torch.mm(A2048, W3.t(), out=o768), D, F),
    ]
    for name, fn, N, K in ops:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        n = max(5, int(seconds / max(time.perf_counter() - t0, 1e-4)))
        clk = ClockSampler(0)
        clk.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = e0.elapsed_time(e1) / n
        print(json.dumps({"op": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                          "tflops": round(2.0 * M * N * K / ms / 1e9, 1), "launches": n, "clocks": clocks}), flush=True)
    return 0


def main():
    a, c = parse()
    if a.compare_cublas:
        return compare_cublas()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        a.gpus = world
    metric = f"forecast series/sec at T={c['T']},H={c['H']}"
    if a.impl == "reference":
        if rank != 0:
            return 0
        threads = os.cpu_count() or 1
        secs = oracle_runs(a.config, c, c["cpu_sample"], threads, max(a.steps, 1))
        v = c["cpu_sample"] / float(np.median(secs))
        b = {"value": v, "unit": "series/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
             "sample": f"{c['cpu_sample']} series of the same workload per step, median of {len(secs)} steps"}
        # The port computes what the reference computes on this GGUF: F16 weights with
        # activations rounded to F16 and F32 accumulation (ggml's F16 mul_mat), f32 elsewhere.
        print(json.dumps({"impl": "reference", "metric": metric, "value": v, "unit": "series/s", "n_gpus": a.gpus,
                          "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "strong",
                          "dtype": c["weights"], "data": "synthetic",
                          "config": {"workload": f"{a.config} 209M {c['weights']} B={c['B']} V={c['V']} T={c['T']} "
                                                 f"H={c['H']} (CPU sample)"},
                          "cpu_baseline": b,
                          "e2e": {"value": v, "unit": "series/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return 0

    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as td
        torch.cuda.set_device(local)
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        dist = td
    else:
        torch.cuda.set_device(local)
    import timestral_b200 as tb
    from timestral_b200.shard import shard_range
    dev = torch.device("cuda", local)
    B, V, T, H = c["B"], c["V"], c["T"], c["H"]
    lo, hi = shard_range(B, world, rank)
    per = hi - lo
    path = model_path(c["weights"], rank, dist)
    model = tb.Model(path, device=local)
    Q = model.num_quantiles
    x, kw = workload(a.config, c, lo, hi)
    covariates = bool(kw)
    stream = torch.cuda.ExternalStream(model.stream(), device=dev)
    hx = torch.from_numpy(np.ascontiguousarray(x)).pin_memory().numpy()

    if covariates:
        def step():
            model.forecast(hx, H, **kw)
    else:
        d_ctx = torch.from_numpy(x).to(dev)
        d_out = torch.empty((per, V, H, Q), device=dev, dtype=torch.float32)

        def step():
            model.forecast_device(d_ctx.data_ptr(), None, per, V, T, H, d_out.data_ptr(), asynchronous=True)

    for _ in range(a.warmup):
        step()
    if tb.lib().tsb_sync(model.h) != 0:
        raise RuntimeError(model.last_error)
    launches_per_step = model.last_launch_count()
    rows, S, L, blocks = model.last_geometry()
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    # The timed region runs the forecasts as a caller does (no per-kernel events, so repeated
    # single-block forecasts replay their CUDA graph).
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    clk = clocks.stop()
    if tb.lib().tsb_sync(model.h) != 0:
        raise RuntimeError(model.last_error)
    ms = e0.elapsed_time(e1) / a.steps
    # Attention launch durations: the same K steps again with CUDA events around every
    # attention launch on the engine stream (plain launches).
    model.timing_reset()
    model.timing(True, attention_only=True)
    for _ in range(a.steps):
        step()
    if tb.lib().tsb_sync(model.h) != 0:
        raise RuntimeError(model.last_error)
    att_ms, att_n = model.timing_read("attention")
    model.timing(False)
    # GEMM share of a step: one extra step with every launch bracketed by events.
    model.timing_reset()
    model.timing(True)
    step()
    tb.lib().tsb_sync(model.h)
    gemm_ms, gemm_n = model.timing_read("gemm")
    all_ms, all_n = model.timing_read("all")
    model.timing(False)
    # End to end through the public C ABI with host buffers: the context from page-locked
    # memory (e2e) and from ordinary pageable memory (e2e_pageable); the result lands in the
    # buffer the library returns. One GPU: this rank's handle. Several GPUs: rank 0 alone
    # forecasts the whole batch through one handle over every rank's GPU (tsb_load_devices:
    # series shards, one host thread and stream per GPU, each shard's result copied into its
    # slice of the one output), while the other ranks wait on the host.
    e2e = e2e_pageable = None
    multi_note = None
    if not a.no_e2e:
        def timed(fn):
            fn()                              # sizes the staging buffers once, untimed
            t0 = time.perf_counter()
            for _ in range(a.steps):
                fn()
            return (time.perf_counter() - t0) / a.steps
        if world == 1:
            px = np.ascontiguousarray(x)
            e2e = timed(lambda: model.forecast(hx, H, **kw))
            e2e_pageable = timed(lambda: model.forecast(px, H, **kw))
        else:
            import datetime
            host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
            dist.barrier(group=host_group)
            if rank == 0:
                full_x, full_kw = workload(a.config, c, 0, B)
                full_hx = torch.from_numpy(np.ascontiguousarray(full_x)).pin_memory().numpy()
                multi = tb.Model(path, devices=list(range(world)))
                e2e = timed(lambda: multi.forecast(full_hx, H, **full_kw))
                e2e_pageable = timed(lambda: multi.forecast(np.ascontiguousarray(full_x), H, **full_kw))
                multi.close()
                multi_note = (f"one process, one handle over {world} GPUs (tsb_load_devices), wall clock around "
                              "timestral_capi_forecast: H2D of every shard, forecasts, D2H into one buffer")
            dist.barrier(group=host_group)
    stats = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max = stats[0].item()
    if rank == 0:
        hbm, tf, tf_sus, kind = peaks()
        # Attention: per (row, head) problem q, k, v, sigmoid(gate) read and the output
        # written (5 S hd f16 values); FLOPs 4 hd sum_q keys(q), keys = L for encoder queries
        # and S for decoder queries (the reference's computed set); one launch per time
        # sublayer and block.
        # Two byte counts per (row, head) problem: the survey's (q, k, v read and the output
        # written, 4 S hd f16 values: the bytes any unfused attention must move) and the
        # kernel's own (also sigmoid(gate), which it reads to apply the gate in its epilogue).
        problems = rows * HEADS
        att_bytes = 4 * S * HEAD_DIM * 2 * problems
        att_kernel_bytes = 5 * S * HEAD_DIM * 2 * problems
        att_flops = 4 * HEAD_DIM * (L * L + (S - L) * S) * problems
        att_avg = att_ms / max(att_n, 1)
        achieved_gbs = att_bytes / (att_avg / 1e3) / 1e9
        achieved_kernel_gbs = att_kernel_bytes / (att_avg / 1e3) / 1e9
        achieved_tf = att_flops / (att_avg / 1e3) / 1e12
        roof_tf = min(tf, (att_flops / att_bytes) * hbm / 1e3)
        tc_path = model.tensor_core_path
        gflops = gemm_flops(rows, S, L, V, S - L) * blocks
        value = B / (ms_max / 1e3)
        cdesc = c["desc"].format(w=c["weights"], B=B, per=per) if a.config == "cfg5" else c["desc"]
        out = {
            "metric": metric, "value": value, "unit": "series/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16" if c["weights"] != "f32" else "f32", "data": "synthetic",
            "config": {"workload": cdesc, "global_batch": B, "seq_len": S,
                       "parallelism": f"series-sharded x{world}",
                       "l2": "per-step working set far above the 126 MB L2" if a.config in ("cfg5", "cfg6")
                             else "steps run back to back without an L2 flush (small working set)",
                       "path": "device-resident context" if not covariates else "C ABI with host buffers (covariates)"},
            "roofline": {"kernel": ("attention_time_tc" if S <= 128 else "attention_time_tc_long") if tc_path
                                   else "attention_time_simt",
                         **({"bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s",
                             "frac": achieved_gbs / hbm} if roof_tf < tf else
                            {"bound": "tensor", "achieved": achieved_tf, "peak": tf_sus, "unit": "TFLOP/s",
                             "frac": achieved_tf / tf_sus}),
                         "traffic": (ATTN_DRAM_BYTES_PER_PROBLEM * problems if a.config == "cfg5" else
                                     ATTN_LONG_DRAM_BYTES_PER_PLANE * problems if a.config == "cfg6" else None),
                         "traffic_unit": "bytes per launch",
                         "traffic_source": ("a constant per (row, head) problem from one ncu capture of this kernel "
                                            "(dram__bytes_read.sum + dram__bytes_write.sum), scaled by the problems "
                                            "of a launch; not measured in this run"),
                         "algorithmic_bytes": att_bytes,
                         "bytes_convention": "q, k, v read + output written (4 x S x 64 f16 per row and head)",
                         "kernel_bytes": att_kernel_bytes, "kernel_bytes_achieved_gbs": achieved_kernel_gbs,
                         "kernel_bytes_frac": achieved_kernel_gbs / hbm,
                         "kernel_bytes_convention": "also sigmoid(gate) read (5 x S x 64 f16 per row and head)",
                         "achieved_tflops": achieved_tf, "roofline_tflops": roof_tf,
                         "frac_of_dense_contraction_roofline": achieved_tf / roof_tf,
                         "launch_ms": att_avg, "launches_per_step": att_n / max(a.steps, 1), "peak_kind": kind},
            "clocks": clk,
            "gpu_launches": launches_per_step * a.steps,
        }
        if tc_path:
            out["roofline_gemm"] = {"bound": "tensor",
                                    "achieved": gflops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None,
                                    "peak": tf_sus, "unit": "TFLOP/s",
                                    "frac": (gflops / (gemm_ms / 1e3) / 1e12) / tf_sus if gemm_ms else None,
                                    "gemm_ms_per_step": gemm_ms, "share_of_step": gemm_ms / all_ms if all_ms else None,
                                    "peak_kind": kind + " sustained"}
        if e2e:
            cov_bytes = sum(int(v.nbytes) for v in kw.values()) * B // max(per, 1)
            out["e2e"] = {"value": B / e2e, "unit": "series/s",
                          "h2d_bytes_per_step": B * V * T * 4 + cov_bytes, "d2h_bytes_per_step": B * V * H * Q * 4,
                          "input": "page-locked host buffer", "output": "the library's result buffer"}
            if multi_note:
                out["e2e"]["how"] = multi_note
            if e2e_pageable:
                out["e2e_pageable"] = {"value": B / e2e_pageable, "unit": "series/s",
                                       "input": "pageable host buffer (numpy)"}
        if "published" in c:
            # The reference publishes this exact metric (one series per forecast): the ratio
            # to its published median, with what that number measured.
            out["vs_baseline"] = value * c["published"]["seconds_per_forecast"]
            out["published"] = c["published"]
        if world == 1 and not a.no_cpu:
            out["cpu_baseline"] = cpu_baseline(a.config, c)
        print(json.dumps(out), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
