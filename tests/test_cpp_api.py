"""The library's C++ API (ts::Model::load, ts::Forecaster::forecast with a ForecastTrace,
ts::Forecaster::decode; reference src/forecaster.hpp:24-56, src/model_loader.hpp:33-65)
driven by a compiled C++ program, tests/cpp/forecaster_api_test.cpp, against the C ABI and
itself on a B200. The CPU part checks that the program builds against the exported API."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

from timestral_b200 import LIB_PATH
from timestral_b200 import synthetic as sy

REPO = Path(__file__).resolve().parents[1]
SRC = REPO / "tests" / "cpp" / "forecaster_api_test.cpp"


def build(tmp: Path) -> Path:
    cxx = shutil.which("g++") or "g++"
    exe = tmp / "forecaster_api_test"
    cmd = [cxx, "-std=c++17", "-O1", str(SRC), "-I", str(REPO / "timestral.cpp_b200" / "host"),
           "-I", str(REPO / "include"), str(LIB_PATH), f"-Wl,-rpath,{LIB_PATH.parent}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_api_builds_against_the_exported_symbols(tmp_path):
    if not LIB_PATH.exists():
        pytest.skip("library not built")
    assert build(tmp_path).exists()


@pytest.mark.gpu
def test_cpp_api_on_the_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    exe = build(tmp_path)
    model = sy.cached_model(sy.spec_small(True), "f16")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0"))
    p = subprocess.run([str(exe), str(model)], capture_output=True, text=True, timeout=600, env=env)
    print(p.stdout, p.stderr)
    assert p.returncode == 0, p.stderr
    assert p.stdout.startswith("OK ")
