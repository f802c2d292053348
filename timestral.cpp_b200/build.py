"""Build libtimestral_b200.so in-tree (timestral.cpp_b200/lib/).

CUDA sources are compiled for sm_100a only; host C++17 sources with the same nvcc driver.
Objects are rebuilt when their source or any header of the package is newer.

    python timestral.cpp_b200/build.py [-j N] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "lib" / "obj"
LIB = LIB_DIR / "libtimestral_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          f"-I{REPO / 'include'}", f"-I{PKG / 'csrc'}", f"-I{PKG / 'host'}"]
CUDA_FLAGS = ARCH + ["-lineinfo", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
HOST_CXX = ["-Xcompiler", "-ffp-contract=off"]
# Sources whose float arithmetic must not be contracted into fused multiply-adds.
NO_FMAD = {"rows.cu"}


def sources():
    cu = sorted((PKG / "csrc").glob("*.cu"))
    cpp = sorted((PKG / "host").glob("*.cpp"))
    return cu, cpp


def headers():
    hs = list((PKG / "csrc").glob("*.cuh")) + list((PKG / "csrc").glob("*.h")) + list((PKG / "host").glob("*.hpp"))
    hs += list((REPO / "include").glob("*.h"))
    return hs


def ccbin():
    for c in ("/usr/bin/g++",):
        if Path(c).exists():
            return ["-ccbin", c]
    return []


def compile_one(src: Path, verbose: bool, newest_header: float):
    obj = OBJ_DIR / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj, ""
    flags = (CUDA_FLAGS + (["-fmad=false"] if src.name in NO_FMAD else [])) if src.suffix == ".cu" else ["-x", "c++"] + HOST_CXX
    cmd = [NVCC] + ccbin() + COMMON + flags + ["-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(jobs: int | None = None, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    cu, cpp = sources()
    newest = max([h.stat().st_mtime for h in headers()] + [Path(__file__).stat().st_mtime])
    objs = []
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        futs = [ex.submit(compile_one, s, verbose, newest) for s in cu + cpp]
        for f in futs:
            obj, log = f.result()
            objs.append(obj)
            if log.strip() and verbose:
                print(log)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC] + ccbin() + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args()
    if a.clean and LIB_DIR.exists():
        shutil.rmtree(LIB_DIR)
    print(build(a.j, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
