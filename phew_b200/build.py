"""Builds the native library ``phew_b200/libphew_b200.so`` with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled by nvcc, and every ``csrc/*.cpp`` file
(host-only code) by the host C++ compiler, to an object under
``phew_b200/_build``; the objects are linked into one shared library next to
this file, so the built library travels with the source tree.  NVRTC (used at run time for emitted fused
kernels) is linked dynamically from the CUDA toolkit.

Usage: ``python -m phew_b200.build [--verbose-ptxas] [--force]``.
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
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libphew_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def nvcc_cmd() -> str:
    return str(cuda_home() / "bin" / "nvcc")


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [
        nvcc_cmd(),
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-I",
        str(INCLUDE),
        "-c",
        str(src),
        "-o",
        str(obj),
    ]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def _compile_host(src: Path) -> tuple[Path, str]:
    """Host-only C++ (no CUDA headers): the host compiler at -O3 with fused
    multiply-adds off, so every SIMD clone of a function rounds alike, and
    without errno from math functions, so sqrtf vectorises."""
    obj = BUILD / (src.stem + ".o")
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    cmd = [cxx, "-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-math-errno", "-I", str(INCLUDE),
           "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{cxx} failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def _stale(sources: list[Path]) -> bool:
    if not LIB.exists():
        return True
    lib_mtime = LIB.stat().st_mtime
    deps = sources + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > lib_mtime for p in deps)


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library; returns its path.  Raises on failure."""
    sources = sorted(CSRC.glob("*.cu"))
    host_sources = sorted(CSRC.glob("*.cpp"))
    if not sources:
        raise RuntimeError("no CUDA sources under phew_b200/csrc")
    if not force and not verbose_ptxas and not _stale(sources + host_sources):
        return LIB
    BUILD.mkdir(exist_ok=True)
    jobs = jobs or min(len(sources) + len(host_sources), os.cpu_count() or 4)
    logs = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_compile, s, verbose_ptxas) for s in sources]
        futs += [ex.submit(_compile_host, s) for s in host_sources]
        results = [f.result() for f in futs]
    objs = [o for o, _ in results]
    logs = [log for _, log in results if log.strip()]
    cuda_lib = cuda_home() / "lib64"
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc_cmd(),
        *ARCH,
        "-shared",
        "-o",
        str(tmp),
        *map(str, objs),
        "-L",
        str(cuda_lib),
        "-lnvrtc",
        "-Xlinker",
        f"-rpath,{cuda_lib}",
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    if verbose_ptxas:
        sys.stderr.write("\n".join(logs))
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
