"""Builds libvkcompute.so (sm_100a) in-tree, the oracle library, and -- when
the vk-compute sources are mounted -- the reference artefacts in oracle/_ref.

    python -m vk_compute_b200._build [--force] [--no-ref]

Objects are cached under vk_compute_b200/_build/ and rebuilt when a source
or header is newer than its object.
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
OBJ = PKG / "_build"
LIB = PKG / "libvkcompute.so"
E2E_BIN = PKG / "vkc_e2e_bench"
ORACLE = ROOT / "oracle"
ORACLE_LIB = ORACLE / "liboracle.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    f"-I{INCLUDE}", f"-I{INCLUDE / 'vkshim'}", f"-I{CSRC}",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libvkcompute")


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.rglob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    sources = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = OBJ / (src.name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for cmd in jobs:
                if verbose:
                    print(" ".join(cmd))
            list(ex.map(_run, jobs))
    if force or jobs or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)])
    return LIB


def build_e2e(force: bool = False) -> Path:
    """The C end-to-end timing host (csrc/e2e_bench.c) against libvkcompute."""
    src = CSRC / "e2e_bench.c"
    if force or _stale(E2E_BIN, [src, LIB]):
        _run(["gcc", "-O2", "-Wall", f"-I{INCLUDE / 'vkshim'}", f"-I{INCLUDE}", "-o", str(E2E_BIN), str(src),
              f"-L{PKG}", "-lvkcompute", "-Wl,-rpath,$ORIGIN"])
    return E2E_BIN


def build_oracle(force: bool = False) -> Path:
    src = ORACLE / "oracle.c"
    if force or _stale(ORACLE_LIB, [src, ORACLE / "oracle.h"]):
        _run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-Wall", "-o", str(ORACLE_LIB), str(src), "-lm"])
    return ORACLE_LIB


def build_reference(force: bool = False) -> bool:
    """Compile the reference's own C sources into oracle/_ref (checker only).
    oracle/build_ref.sh locates the sources (VKC_REFERENCE, or where they are
    mounted) and exits 3 when they are absent, as on a machine that only runs
    the prebuilt files."""
    script = ORACLE / "build_ref.sh"
    env = dict(os.environ, VKC_FORCE="1" if force else "0")
    proc = subprocess.run(["bash", str(script)], capture_output=True, text=True, env=env)
    if proc.returncode == 3:
        return False
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("reference build recipe failed")
    return True


def build_all(force: bool = False, with_ref: bool = True, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_e2e(force=force)
    build_oracle(force=force)
    if with_ref:
        build_reference(force=force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-ref", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    build_all(force=args.force, with_ref=not args.no_ref, verbose=args.verbose)
    print(f"built {LIB}")


if __name__ == "__main__":
    main()
