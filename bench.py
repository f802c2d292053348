"""Forecast throughput benchmark (series/sec at T=2048, H=256) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--weights f16|q8_0] [--batch B]
    python bench.py --impl reference ...   # the CPU reference arm (rank 0 only)

Workload: the 209M-architecture forecaster (random init, seed 0) on B=4096 synthetic series
(seasonal sine with period U[12,200], trend, 1% NaN, seeded per series), V=1, T=2048,
H=256, symmetric averaging and clipping on. The batch is sharded B/N series per GPU with
no collective on the forecast path; each rank runs its shard through its own engine.

Printed JSON (rank 0): `value` is whole-job series/sec with the context already in device
memory (tsb_forecast_device, CUDA events on the engine stream, max over ranks); `e2e` is the
same metric through timestral_capi_forecast with host buffers (upload and download inside
the timed region); `roofline` is the attention kernel measured live; `cpu_baseline` is the
CPU oracle on a bounded sample of the same workload.
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

T_CTX, H_OUT, B_TOTAL = 2048, 256, 4096


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--weights", default="f16", choices=["f16", "q8_0"])
    ap.add_argument("--batch", type=int, default=B_TOTAL)
    ap.add_argument("--cpu-sample", type=int, default=48, help="series timed on the CPU baseline (about 15-20 s)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU, sampled every 200 ms."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
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
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
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
                "samples": len(sm)}


def workload(lo: int, hi: int):
    from timestral_b200 import synthetic as sy
    out = np.empty((hi - lo, 1, T_CTX), np.float32)
    for k, i in enumerate(range(lo, hi)):
        out[k] = sy.series_seasonal(1, T_CTX, nan_frac=0.01, seed0=i)[0]
    return out


def model_path(weights: str, rank: int, dist):
    from timestral_b200 import synthetic as sy
    if rank == 0:
        p = sy.cached_model(sy.spec_209m(), weights)
    if dist is not None:
        dist.barrier()
    return sy.cached_model(sy.spec_209m(), weights)


def cpu_baseline(sample: int, weights: str):
    """The CPU oracle on `sample` series of the same workload, all host threads."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle_py as op
    from timestral_b200 import synthetic as sy
    m = op.OracleModel(sy.cached_model(sy.spec_209m(), weights))
    x = workload(0, sample)
    threads = os.cpu_count() or 1
    m.forecast(x[:1], H_OUT, threads=threads)   # warm caches
    t0 = time.perf_counter()
    m.forecast(x, H_OUT, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "series/s", "cores": threads, "kind": "port",
            "sample": f"{sample} series of the same workload (T={T_CTX}, H={H_OUT}, {weights} 209M), "
                      f"one forecast call, {dt:.2f} s"}


# DRAM bytes (read + write) of one time-attention (row, head) problem at S = 72, from the
# ncu capture summarised in profiles/attention_time_tc_cfg5.md (B = 1024, dram__bytes_read.sum
# + dram__bytes_write.sum over 24,576 problems); traffic per launch scales with the problems.
ATTN_DRAM_BYTES_PER_PROBLEM = 45384


def attention_algorithmic(rows: int, S: int, L: int, heads: int = 12, hd: int = 64):
    """FLOPs and bytes of one time-attention launch over `rows` rows: 4*hd*sum_q keys(q) per
    (row, head) with keys = L for encoder queries and S for decoder queries; bytes = q, k, v,
    sigmoid-gate read and output written, f16."""
    flops = 4 * hd * (L * L + (S - L) * S)
    nbytes = 5 * S * hd * 2
    return flops * rows * heads, nbytes * rows * heads


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        a.gpus = world
    if a.impl == "reference":
        if rank != 0:
            return 0
        b = cpu_baseline(a.cpu_sample, a.weights)
        vals = [b["value"]]
        for _ in range(max(a.steps, 1) - 1):
            vals.append(cpu_baseline(a.cpu_sample, a.weights)["value"])
        v = float(np.median(vals))
        b["value"] = v
        print(json.dumps({"impl": "reference", "metric": "forecast series/sec at T=2048,H=256", "value": v,
                          "unit": "series/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
                          "higher_is_better": True, "scaling": "strong", "dtype": "f32", "data": "synthetic",
                          "config": {"workload": f"209M {a.weights} B={a.batch} V=1 T={T_CTX} H={H_OUT} (CPU sample)"},
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
    dev = torch.device("cuda", local)
    from timestral_b200.shard import shard_range
    lo, hi = shard_range(a.batch, world, rank)
    per = hi - lo
    path = model_path(a.weights, rank, dist)
    model = tb.Model(path, device=local)
    Q = model.num_quantiles
    x = workload(lo, hi)
    d_ctx = torch.from_numpy(x).to(dev)
    d_out = torch.empty((per, 1, H_OUT, Q), device=dev, dtype=torch.float32)
    stream = torch.cuda.ExternalStream(model.stream(), device=dev)

    def step():
        model.forecast_device(d_ctx.data_ptr(), None, per, 1, T_CTX, H_OUT, d_out.data_ptr(), asynchronous=True)

    for _ in range(a.warmup):
        step()
    if tb.lib().tsb_sync(model.h) != 0:
        raise RuntimeError(model.last_error)
    launches_per_step = model.last_launch_count()
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    # Attention launches are bracketed by CUDA events on the engine stream inside the timed
    # region (two events per launch, 24 launches per step).
    model.timing_reset()
    model.timing(True, attention_only=True)
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
    # End to end through the public C ABI with host buffers.
    e2e = None
    if not a.no_e2e:
        hx = torch.from_numpy(x).pin_memory().numpy()
        model.forecast(hx[:1], H_OUT)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(a.steps):
            model.forecast(hx, H_OUT)
        e2e_s = (time.perf_counter() - t0) / a.steps
        e2e = e2e_s
    stats = torch.tensor([ms, e2e or 0.0], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max, e2e_max = stats[0].item(), stats[1].item()
    if rank == 0:
        hbm, tf, tf_sus, kind = peaks()
        L = T_CTX // 32
        S = L + H_OUT // 32
        rows = 2 * per
        fl, by = attention_algorithmic(rows, S, L)
        att_avg = att_ms / max(att_n, 1)
        achieved_gbs = by / (att_avg / 1e3) / 1e9
        achieved_tf = fl / (att_avg / 1e3) / 1e12
        roof_tf = min(tf, (fl / by) * hbm / 1e3)
        # Tensor-core GEMM work per step on this rank, as the kernels compute it: patch
        # output projection per context patch, per token 24 time sublayers (q|k|v|gate and
        # out: 5*D^2), 6 variate sublayers of one-row series (v|gate and out: 3*D^2), 24 MLPs
        # (3*D*F), and the head per decoder token.
        D, F = 768, 2048
        per_token = 24 * 5 * D * D + 6 * 3 * D * D + 24 * 3 * D * F
        gemm_flops = 2 * rows * (L * 4 * D * D + S * per_token + (S - L) * (D * 4 * D + 4 * D * 672 + D * 672))
        value = a.batch / (ms_max / 1e3)
        out = {
            "metric": "forecast series/sec at T=2048,H=256", "value": value, "unit": "series/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"cfg5 throughput: 209M {a.weights} random-init, B={a.batch} series "
                                   f"({per} per GPU), V=1, T={T_CTX}, H={H_OUT}, symmetric+clip",
                       "global_batch": a.batch, "seq_len": S, "parallelism": f"series-sharded x{world}",
                       "l2": "per-step working set (~13 GB at B=4096) far above the 126 MB L2"},
            "roofline": {"kernel": "attention_time_tc", "bound": "hbm", "achieved": achieved_gbs, "peak": hbm,
                         "unit": "GB/s", "frac": achieved_gbs / hbm,
                         "traffic": (ATTN_DRAM_BYTES_PER_PROBLEM * rows * 12 if ATTN_DRAM_BYTES_PER_PROBLEM else None),
                         "traffic_unit": "bytes per launch", "algorithmic_bytes": by,
                         "achieved_tflops": achieved_tf, "roofline_tflops": roof_tf,
                         "frac_of_dense_contraction_roofline": achieved_tf / roof_tf,
                         "launch_ms": att_avg, "launches_per_step": att_n, "peak_kind": kind},
            "roofline_gemm": {"bound": "tensor", "achieved": gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None,
                              "peak": tf_sus, "unit": "TFLOP/s",
                              "frac": (gemm_flops / (gemm_ms / 1e3) / 1e12) / tf_sus if gemm_ms else None,
                              "gemm_ms_per_step": gemm_ms, "share_of_step": gemm_ms / all_ms if all_ms else None,
                              "peak_kind": kind + " sustained"},
            "clocks": clk,
            "gpu_launches": launches_per_step * a.steps,
        }
        if e2e:
            out["e2e"] = {"value": a.batch / e2e_max, "unit": "series/s",
                          "h2d_bytes_per_step": a.batch * T_CTX * 4, "d2h_bytes_per_step": a.batch * H_OUT * Q * 4}
        if world == 1 and not a.no_cpu:
            out["cpu_baseline"] = cpu_baseline(a.cpu_sample, a.weights)
        print(json.dumps(out), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
