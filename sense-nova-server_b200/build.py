"""Build the sm_100a C-ABI library (libsnl_b200.so) and the CPU checker library.

The CUDA library is compiled with nvcc straight from csrc/*.cu for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked into one shared object next to
this file, so it travels with the source tree. The CPU checker (oracle/oracle.cpp)
is test infrastructure and is built into oracle/_build/.

Usage: python sense-nova-server_b200/build.py [--lib] [--oracle] [--jobs N]
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
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libsnl_b200.so"
ORACLE_SRC = ROOT / "oracle" / "oracle.cpp"
ORACLE_LIB = ROOT / "oracle" / "_build" / "liboracle.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newer(out: Path, deps: list[Path]) -> bool:
    return out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps)


def build_lib(jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if _newer(obj, [src, *headers]):
            return obj
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, sources))
    if not _newer(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


def build_oracle() -> Path:
    ORACLE_LIB.parent.mkdir(parents=True, exist_ok=True)
    deps = [ORACLE_SRC, *INCLUDE.glob("*.h"), CSRC / "synth.h", CSRC / "synth_model.h"]
    if _newer(ORACLE_LIB, deps):
        return ORACLE_LIB
    cxx = os.environ.get("SNL_CXX") or shutil.which("g++") or "g++"  # $CXX may lack libgomp
    cmd = [cxx, "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=c++17",
           "-I", str(INCLUDE), "-I", str(CSRC), str(ORACLE_SRC), "-o", str(ORACLE_LIB)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return ORACLE_LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", action="store_true")
    ap.add_argument("--oracle", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    both = not (a.lib or a.oracle)
    if a.lib or both:
        print(build_lib(a.jobs, a.verbose))
    if a.oracle or both:
        print(build_oracle())


if __name__ == "__main__":
    main()
