"""Build the sm_100a kernel library ``libb2m.so`` in-tree with nvcc.

Usage: ``python -m td_benchmark_b200.build [--verbose]``.  Sources are compiled in
parallel into ``td_benchmark_b200/_build/`` and linked into
``td_benchmark_b200/libb2m.so`` (CUDA runtime linked statically, so the library
loads without a GPU; the driver is reached through cudaGetDriverEntryPoint).
IEEE division and no fast-math: the quant kernels must be bit-exact with the
reference's fp32 rounding.
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
LIB = PKG / "libb2m.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              "-DNDEBUG"] + ARCH


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the b2m kernels need the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _compile(nvcc: str, src: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [PKG.parent / "include" / "b2m.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(nvcc, s, verbose), srcs))
    if verbose:
        for _, log in results:
            if log.strip():
                print(log, file=sys.stderr)
    objs = [str(o) for o, _ in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-lcudart_static", "-ldl", "-lrt",
           "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
