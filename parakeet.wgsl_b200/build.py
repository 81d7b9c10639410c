"""Build libpk_b200.so in-tree for sm_100a.

    python parakeet.wgsl_b200/build.py [--verbose]

Each ``csrc/*.cu`` (device and host code) and ``csrc/*.cpp`` (host-only
code, forwarded by nvcc to the host compiler) is compiled by nvcc (``-gencode arch=compute_100a,
code=sm_100a -lineinfo -O3``) into ``_build/`` in parallel and linked into
``parakeet.wgsl_b200/libpk_b200.so`` with the CUDA runtime linked statically,
so the library carries no dependency on the caller's CUDA runtime.  nvcc
cross-compiles without a GPU.
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
BUILD = PKG.parent / "_build" / "pk_b200"
LIB = PKG / "libpk_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler() -> list[str]:
    # The image exports CXX as a wrapper; nvcc is happiest with the system g++.
    return ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []


def flags(verbose: bool = False) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I", str(PKG.parent / "include")] + _host_compiler()
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime > max(
        [src.stat().st_mtime] + [h.stat().st_mtime for h in CSRC.glob("*.h*")]
        + [(PKG.parent / "include" / "pk_b200.h").stat().st_mtime]
    ) and not verbose:
        return obj, ""
    cmd = [nvcc(), "-c", str(src), "-o", str(obj)] + flags(verbose)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), sources))
    objs = [r[0] for r in results]
    if verbose:
        for _, log in results:
            if log:
                print(log)
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), "-shared", "-o", str(LIB)] + [str(o) for o in objs] + ARCH + _host_compiler() + [
            "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(verbose=args.verbose))
    sys.exit(0)
