"""Build libb200q.so in-tree with nvcc for sm_100a.

    python -m cybel_b200.build [--verbose]

Compiles every ``csrc/*.cu`` to an object (in parallel, skipping objects
newer than their sources and headers) and links ``cybel_b200/_lib/libb200q.so``.
The library depends only on the CUDA runtime (no torch types cross the ABI).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
OBJ_DIR = PKG / "_build"
LIB = OUT_DIR / "libb200q.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libb200q.so")
    return cand


def _needs(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = _nvcc()
    OUT_DIR.mkdir(exist_ok=True)
    OBJ_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = []
    for src in srcs:
        obj = OBJ_DIR / (src.stem + ".o")
        if _needs(obj, src, headers) or ptxas_verbose:
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for src, r in ex.map(run, jobs):
            if r.stdout or r.stderr:
                if verbose or r.returncode or ptxas_verbose:
                    sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for: {', '.join(failed)}")
    objs = [str(OBJ_DIR / (s.stem + ".o")) for s in srcs]
    if jobs or not LIB.exists():
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
