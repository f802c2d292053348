"""The C-ABI library loads without a GPU, exports every symbol include/*.h declares, keeps
the reference's request layout, and reports load errors the reference's way (no GPU needed).
"""
import ctypes as C
import re
from pathlib import Path

import pytest

import timestral_b200 as tb

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = []
    for h in sorted((REPO / "include").glob("*.h")):
        text = h.read_text()
        names += re.findall(r"TIMESTRAL_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return names


def test_library_exports_every_declared_symbol():
    lib = tb.lib()
    names = declared_symbols()
    assert "timestral_capi_forecast" in names and "tsb_forecast_device" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(tb.SIGNATURES), set(names) - set(tb.SIGNATURES)


def test_request_layout_matches_reference():
    # Field offsets of timestral_forecast_request (reference include/timestral_capi.h:29-40).
    R = tb.ForecastRequest
    assert [f[0] for f in R._fields_] == ["context", "observation_mask", "B", "V", "T", "prediction_length",
                                          "past_cov", "c_past", "known_cov", "c_known", "cat_past", "cc_past",
                                          "cat_known", "cc_known", "symmetric_averaging", "clip_nonnegative",
                                          "max_context"]
    assert R.context.offset == 0 and R.observation_mask.offset == 8 and R.B.offset == 16
    assert R.prediction_length.offset == 28 and R.past_cov.offset == 32 and R.c_past.offset == 40
    assert R.max_context.offset == 100 and C.sizeof(R) == 104


def test_header_compiles_as_c99(tmp_path):
    """The public header is strict C99 and its layout agrees with the binding."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    src = tmp_path / "t.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "timestral_capi.h"\n#include "timestral_b200.h"\n'
                   'int main(void){printf("%zu %zu %zu\\n", offsetof(timestral_forecast_request, c_past),'
                   ' offsetof(timestral_forecast_request, max_context), sizeof(timestral_forecast_request));return 0;}\n')
    exe = tmp_path / "t"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-pedantic", f"-I{REPO / 'include'}", str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    R = tb.ForecastRequest
    assert [int(x) for x in out] == [R.c_past.offset, R.max_context.offset, C.sizeof(R)]


def test_abi_version_and_load_errors(tmp_path):
    lib = tb.lib()
    assert lib.timestral_capi_abi_version() == 1
    assert not lib.timestral_capi_load(None, 1)
    assert lib.timestral_capi_last_error(None) == b"model path is required"
    assert not lib.timestral_capi_load(b"x.gguf", 0)
    assert lib.timestral_capi_last_error(None) == b"invalid CPU thread count"
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf at all")
    assert not lib.timestral_capi_load(str(bad).encode(), 1)
    assert lib.timestral_capi_last_error(None)
    # NULL-handle queries set the thread-local error and return their sentinels.
    assert lib.timestral_capi_num_quantiles(None) == 0
    assert lib.timestral_capi_last_error(None) == b"null handle"
    q = C.c_int32(7)
    assert not lib.timestral_capi_forecast(None, None, C.byref(q)) and q.value == 0


def test_model_loader_rejects_schema_violations(tmp_path):
    """Loader checks (reference src/model_loader.cpp:264-287) run before any GPU work."""
    import gguf
    import numpy as np
    from timestral_b200 import synthetic as sy
    good = sy.write_gguf(tmp_path / "tiny.gguf", sy.spec_tiny(), "f32")
    lib = tb.lib()
    # Missing tensor: rewrite without out_norm.weight.
    r = gguf.GGUFReader(str(good))
    w = gguf.GGUFWriter(str(tmp_path / "missing.gguf"), "timestral")
    for f in r.fields.values():
        if f.name.startswith("GGUF.") or f.name == "general.architecture":
            continue
        t = f.types[0]
        if t == gguf.GGUFValueType.ARRAY:
            vals = [bytes(f.parts[i]).decode() if f.types[1] == gguf.GGUFValueType.STRING else f.parts[i][0].item()
                    for i in f.data]
            w.add_key_value(f.name, vals, t, f.types[1])
        elif t == gguf.GGUFValueType.STRING:
            w.add_key_value(f.name, bytes(f.parts[f.data[0]]).decode(), t)
        else:
            w.add_key_value(f.name, f.parts[f.data[0]][0].item(), t)
    for t in r.tensors:
        if t.name != "out_norm.weight":
            w.add_tensor(t.name, np.asarray(t.data), raw_dtype=t.tensor_type)
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    assert not lib.timestral_capi_load(str(tmp_path / "missing.gguf").encode(), 1)
    assert lib.timestral_capi_last_error(None) == b"missing tensor: out_norm.weight"


def _rewrite_gguf(src, dst, drop=(), retype=None):
    """A copy of the GGUF at src without the tensors in drop and with the tensors in retype
    ({name: "f16" | "q8_0"}) stored in that type."""
    import gguf
    import numpy as np
    retype = retype or {}
    r = gguf.GGUFReader(str(src))
    w = gguf.GGUFWriter(str(dst), "timestral")
    for f in r.fields.values():
        if f.name.startswith("GGUF.") or f.name == "general.architecture":
            continue
        t = f.types[0]
        if t == gguf.GGUFValueType.ARRAY:
            vals = [bytes(f.parts[i]).decode() if f.types[1] == gguf.GGUFValueType.STRING else f.parts[i][0].item()
                    for i in f.data]
            w.add_key_value(f.name, vals, t, f.types[1])
        elif t == gguf.GGUFValueType.STRING:
            w.add_key_value(f.name, bytes(f.parts[f.data[0]]).decode(), t)
        else:
            w.add_key_value(f.name, f.parts[f.data[0]][0].item(), t)
    for t in r.tensors:
        if t.name in drop:
            continue
        data = np.asarray(t.data)
        if retype.get(t.name) == "f16":
            w.add_tensor(t.name, data.astype(np.float16), raw_dtype=gguf.GGMLQuantizationType.F16)
        elif retype.get(t.name) == "q8_0":
            q = gguf.quants.quantize(data.astype(np.float32), gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(t.name, q, raw_shape=q.shape, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(t.name, data, raw_dtype=t.tensor_type)
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    return dst


def test_model_loader_enforces_the_storage_policy(tmp_path):
    """Reduced types only on the projection weights the reference's policy names, and a
    Q8_0 row length a multiple of its 32-value block (reference src/model_loader.cpp:275-281,
    src/weight_policy.hpp:13-30; tests/test_f16.cpp and tests/test_q8.cpp rejections). The
    loader refuses before any GPU work, with the reference's message (ggml's type names)."""
    from timestral_b200 import synthetic as sy
    good = sy.write_gguf(tmp_path / "tiny.gguf", sy.spec_tiny(), "f32")
    lib = tb.lib()
    for name, kind in (("out_norm.weight", "f16"), ("rope.cos", "f16"), ("out_norm.weight", "q8_0")):
        bad = _rewrite_gguf(good, tmp_path / f"bad_{kind}.gguf", retype={name: kind})
        assert not lib.timestral_capi_load(str(bad).encode(), 1)
        assert lib.timestral_capi_last_error(None).decode() == \
            f"tensor {name} has type {kind}, forbidden by the storage policy"
    # Reduced projection weights pass the loader (on a machine without a GPU the load then
    # stops at the device).
    ok = _rewrite_gguf(good, tmp_path / "reduced.gguf",
                       retype={"blk.0.attn.0.qkv.weight": "q8_0", "head.out.weight": "f16"})
    h = lib.timestral_capi_load(str(ok).encode(), 1)
    if h:
        lib.timestral_capi_free(h)
    else:
        assert "storage policy" not in lib.timestral_capi_last_error(None).decode()


def test_device_switches_reject_bad_arguments():
    """The device-seam switches refuse a null handle (and tsb_fused_norm an unknown mode)
    without touching a GPU."""
    import timestral_b200 as tb
    L = tb.lib()
    err_arg = 1                      # TSB_ERR_ARG
    assert L.tsb_fused_norm(None, 1) == err_arg
    assert L.tsb_graph_replay(None, 1) == err_arg
    assert L.tsb_covariate_assembly(None, 1) == err_arg
