"""ctypes binding of libtimestral_b200.so: the reference's C ABI (timestral_capi.h) plus the
device seam (timestral_b200.h). There is no CPU fallback: importing `lib()` fails loudly
when the CUDA library has not been built.
"""
from __future__ import annotations

import ctypes as C
import weakref
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = PKG / "lib" / "libtimestral_b200.so"

TSB_OK, TSB_ERR_ARG, TSB_ERR_CUDA, TSB_ERR_DEVICE, TSB_ERR_MODEL, TSB_ERR_NAN = range(6)


class ForecastRequest(C.Structure):
    """timestral_forecast_request (include/timestral_capi.h), field order is ABI."""
    _fields_ = [("context", C.c_void_p), ("observation_mask", C.c_void_p), ("B", C.c_int32),
                ("V", C.c_int32), ("T", C.c_int32), ("prediction_length", C.c_int32),
                ("past_cov", C.c_void_p), ("c_past", C.c_int32), ("known_cov", C.c_void_p),
                ("c_known", C.c_int32), ("cat_past", C.c_void_p), ("cc_past", C.c_int32),
                ("cat_known", C.c_void_p), ("cc_known", C.c_int32), ("symmetric_averaging", C.c_int32),
                ("clip_nonnegative", C.c_int32), ("max_context", C.c_int32)]


class GemmTest(C.Structure):
    _fields_ = [("kind", C.c_int32), ("A", C.c_void_p), ("lda", C.c_int64), ("B", C.c_void_p),
                ("ldb", C.c_int64), ("M", C.c_int32), ("N", C.c_int32), ("K", C.c_int32),
                ("out", C.c_void_p), ("ldo", C.c_int64), ("bias", C.c_void_p), ("resid", C.c_void_p),
                ("row_group", C.c_int32), ("row_stride", C.c_int32), ("row_offset", C.c_int32),
                ("qkvg", C.c_void_p * 4), ("S", C.c_int32), ("H", C.c_int32), ("D", C.c_int32),
                ("rope", C.c_int32), ("cos_tab", C.c_void_p), ("sin_tab", C.c_void_p),
                ("rope_row", C.c_void_p), ("rope_half", C.c_int32),
                ("rope_dup", C.c_int32), ("a_group", C.c_int32), ("a_stride", C.c_int32),
                ("a_offset", C.c_int32), ("Bq", C.c_void_p), ("Bd", C.c_void_p), ("ldd", C.c_int64),
                ("Bs", C.c_void_p), ("lds", C.c_int64)]


_lib = None

# Every symbol the headers in include/ declare, with (restype, argtypes).
SIGNATURES = {
    "timestral_capi_abi_version": (C.c_int, []),
    "timestral_capi_load": (C.c_void_p, [C.c_char_p, C.c_int]),
    "timestral_capi_free": (None, [C.c_void_p]),
    "timestral_capi_last_error": (C.c_char_p, [C.c_void_p]),
    "timestral_capi_num_quantiles": (C.c_int, [C.c_void_p]),
    "timestral_capi_quantile_level": (C.c_double, [C.c_void_p, C.c_int]),
    "timestral_capi_forecast": (C.c_void_p, [C.c_void_p, C.POINTER(ForecastRequest), C.POINTER(C.c_int32)]),
    "timestral_capi_free_buffer": (None, [C.c_void_p]),
    "tsb_forecast_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                      C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32]),
    "tsb_sync": (C.c_int, [C.c_void_p]),
    "tsb_load_devices": (C.c_void_p, [C.c_char_p, C.c_int, C.POINTER(C.c_int32), C.c_int32]),
    "tsb_device_count": (C.c_int32, [C.c_void_p]),
    "tsb_set_device": (C.c_int, [C.c_int32]),
    "tsb_stream": (C.c_void_p, [C.c_void_p]),
    "tsb_timing_enable": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_timing_read": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "tsb_timing_reset": (None, [C.c_void_p]),
    "tsb_last_launch_count": (C.c_int64, [C.c_void_p]),
    "tsb_model_path": (C.c_int, [C.c_void_p]),
    "tsb_dequantize_rows": (C.c_int, [C.c_uint32, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]),
    "tsb_scaled_int8_rows": (C.c_int, [C.c_uint32, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    "tsb_last_geometry": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)] + [C.POINTER(C.c_int32)] * 3),
    "tsb_test_gemm": (C.c_int, [C.POINTER(GemmTest), C.POINTER(C.c_int32)]),
    "tsb_test_attention_time": (C.c_int, [C.c_void_p] * 6 + [C.c_int32] * 4 + [C.POINTER(C.c_int32)]),
    "tsb_covariate_assembly": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_graph_replay": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_fused_norm": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_attention_kernels": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_decoder_tail": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_dequant_prologue": (C.c_int, [C.c_void_p, C.c_int32]),
    "tsb_test_scale_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_double] + [C.c_int32] * 6
                            + [C.c_void_p] * 8),
    "tsb_test_attention_time_ex": (C.c_int, [C.c_void_p] * 7 + [C.c_int32] * 9 + [C.POINTER(C.c_float), C.POINTER(C.c_int32)]),
    "tsb_test_split_f16": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p]),
    "tsb_test_attention_variate": (C.c_int, [C.c_void_p] * 7 + [C.c_int32] * 5),
    "tsb_test_attention_variate_ex": (C.c_int, [C.c_void_p] * 7 + [C.c_int32] * 6 + [C.POINTER(C.c_int32)]),
    "tsb_test_rms": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_float, C.c_void_p, C.c_int32]),
    "tsb_test_simt_gemm": (C.c_int, [C.c_void_p, C.c_void_p] + [C.c_int32] * 5 + [C.c_void_p]),
    "tsb_test_refine": (C.c_int, [C.c_void_p] * 6 + [C.c_int32] * 6 + [C.c_double, C.c_void_p]),
    "tsb_test_wait_expiry": (C.c_int, [C.c_int32, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "tsb_test_fail_workspace_allocations": (C.c_int, [C.c_int32]),
    "tsb_test_device_reset": (C.c_int, []),
    "tsb_refine_static": (C.c_int, [C.c_void_p] * 6 + [C.c_int32] * 6 + [C.c_double, C.c_void_p, C.c_void_p]),
}


def lib():
    """Load the CUDA library; raises if it was not built (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python timestral.cpp_b200/build.py` "
                               "(the forecast path has no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name, None)
            if f is None:
                continue
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class TimestralError(RuntimeError):
    pass


def _vp(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


class Model:
    """A loaded model handle (timestral_capi_load) with the reference's C ABI semantics."""

    def __init__(self, path, n_threads: int = 1, device: int | None = None, devices=None):
        """devices: a list of GPU ordinals to shard every request's series over (one handle,
        tsb_load_devices); device: the one GPU of a single-device handle."""
        L = lib()
        if devices is not None:
            arr = (C.c_int32 * len(devices))(*devices)
            self.h = L.tsb_load_devices(str(path).encode(), n_threads, arr, len(devices))
        else:
            if device is not None:
                L.tsb_set_device(device)
            self.h = L.timestral_capi_load(str(path).encode(), n_threads)
        if not self.h:
            raise TimestralError(L.timestral_capi_last_error(None).decode())

    @property
    def device_count(self) -> int:
        return lib().tsb_device_count(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().timestral_capi_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def num_quantiles(self) -> int:
        return lib().timestral_capi_num_quantiles(self.h)

    def quantile_levels(self):
        return [lib().timestral_capi_quantile_level(self.h, i) for i in range(self.num_quantiles)]

    @property
    def last_error(self) -> str:
        e = lib().timestral_capi_last_error(self.h)
        return e.decode() if e else ""

    def forecast(self, context, H, mask=None, past=None, known=None, cat_past=None, cat_known=None,
                 symmetric=-1, clip=-1, max_context=0):
        """timestral_capi_forecast on host arrays; returns [B,V,H,Q] float32."""
        context = np.ascontiguousarray(context, np.float32)
        B, V, T = context.shape
        keep = [context]

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
        r = ForecastRequest(_vp(context), _vp(m), B, V, T, H, _vp(p), cp, _vp(k), ck, _vp(qp), ccp,
                            _vp(qk), cck, symmetric, clip, max_context)
        q = C.c_int32(0)
        L = lib()
        ptr = L.timestral_capi_forecast(self.h, C.byref(r), C.byref(q))
        if not ptr:
            raise TimestralError(self.last_error)
        # The array views the library's buffer (no copy); the buffer is released with
        # timestral_capi_free_buffer when the last view of it goes away.
        buf = (C.c_float * (B * V * H * q.value)).from_address(ptr)
        weakref.finalize(buf, L.timestral_capi_free_buffer, C.c_void_p(ptr))
        return np.ctypeslib.as_array(buf).reshape(B, V, H, q.value)

    def forecast_device(self, d_context: int, d_mask: int | None, B, V, T, H, d_out: int,
                        symmetric=-1, clip=-1, max_context=0, asynchronous=False):
        rc = lib().tsb_forecast_device(self.h, d_context, d_mask, B, V, T, H, symmetric, clip, max_context,
                                       d_out, int(asynchronous))
        if rc != TSB_OK:
            raise TimestralError(f"tsb_forecast_device failed ({rc}): {self.last_error}")

    def stream(self) -> int:
        return lib().tsb_stream(self.h) or 0

    def fused_norm(self, mode: int):
        """RMSNorm carried by the GEMMs: 1 (default), 0 off, 2 on with a forced fallback run."""
        if lib().tsb_fused_norm(self.h, int(mode)) != 0:
            raise RuntimeError("tsb_fused_norm failed")

    def attention_kernels(self, mode: int):
        """Tensor-core path attention: 0 tensor-core kernels (default), 1 CUDA-core kernels with
        the reference's float64 q.k dots and f32 softmax on the same f16 q/k/v."""
        if lib().tsb_attention_kernels(self.h, int(mode)) != 0:
            raise RuntimeError("tsb_attention_kernels failed")

    def dequant_prologue(self, on: bool):
        """Block-quantised weights (Q8_0, K-quants) dequantised in the GEMM prologue (on) or
        read as the f16 copies made at load (off, the default)."""
        rc = lib().tsb_dequant_prologue(self.h, int(on))
        if rc != 0:
            raise TimestralError(f"tsb_dequant_prologue failed ({rc}): {self.last_error}")

    def decoder_tail(self, on: bool):
        """Last layer's per-token work on the decoder tokens alone (default on; same bits)."""
        if lib().tsb_decoder_tail(self.h, int(on)) != 0:
            raise RuntimeError("tsb_decoder_tail failed")

    def graph_replay(self, on: bool):
        """CUDA-graph replay of repeated single-block forecasts (on by default)."""
        if lib().tsb_graph_replay(self.h, int(on)) != 0:
            raise RuntimeError("tsb_graph_replay failed")

    def covariate_assembly(self, on_device: bool):
        """Assemble covariate requests on the device (default) or on the host."""
        if lib().tsb_covariate_assembly(self.h, int(on_device)) != 0:
            raise RuntimeError("tsb_covariate_assembly failed")

    def timing(self, enable: bool, attention_only: bool = False):
        lib().tsb_timing_enable(self.h, 2 if (enable and attention_only) else int(enable))

    def timing_read(self, cls: str):
        ms = C.c_double(0)
        n = C.c_int64(0)
        lib().tsb_timing_read(self.h, cls.encode(), C.byref(ms), C.byref(n))
        return ms.value, n.value

    def timing_reset(self):
        lib().tsb_timing_reset(self.h)

    def last_launch_count(self) -> int:
        return lib().tsb_last_launch_count(self.h)

    def last_geometry(self):
        """(rows, S, L, blocks) of the last decode block of the last forecast."""
        rows, S, L, blocks = C.c_int64(0), C.c_int32(0), C.c_int32(0), C.c_int32(0)
        lib().tsb_last_geometry(self.h, C.byref(rows), C.byref(S), C.byref(L), C.byref(blocks))
        return rows.value, S.value, L.value, blocks.value

    @property
    def tensor_core_path(self) -> bool:
        return lib().tsb_model_path(self.h) == 1
