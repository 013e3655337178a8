"""Build libabra_b200.so in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` is compiled to an object in ``abra_b200/_build/`` (in
parallel), then linked into ``abra_b200/libabra_b200.so`` with the static CUDA
runtime.  NCCL is not linked: the tensor-parallel exchange is a peer-memory
push from the MMVQ epilogue over NVLink (CUDA IPC mappings), and
torch.distributed only carries the IPC handles and barriers.

    python abra_b200/build.py [--force] [--verbose]
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
LIB = PKG / "libabra_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, sep="\n", flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    extra = list(extra or [])
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs if force or extra or _stale(BUILD / (s.stem + ".o"), [s, *hdrs])]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(lambda s: _compile(s, verbose, extra), todo))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
               *map(str, objs), "-o", str(tmp)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    lib = build(force=a.force, verbose=a.verbose or a.ptxas_verbose, extra=extra)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
