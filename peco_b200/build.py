"""Build libpeco_b200.so for sm_100a with nvcc (in-tree, so it travels with the repo).

    python -m peco_b200.build          # incremental
    python -m peco_b200.build --force

Each ``csrc/*.cu`` compiles to an object in ``peco_b200/_build`` in parallel,
then everything links into ``peco_b200/libpeco_b200.so``.  Only the CUDA
runtime is linked; the TMA encoder is resolved through the driver entry point.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libpeco_b200.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")):
        if cand and Path(cand).exists():
            return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set NVCC or CUDA_HOME)")
    return found


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime_ns
    return any(d.stat().st_mtime_ns > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdrs = headers()
    cc = nvcc()
    jobs = []
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *hdrs, Path(__file__)]):
            cmd = [cc, *ARCH, *FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            print(f"[nvcc] {src.name}\n{r.stdout}{r.stderr}")
        if r.returncode:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
        return src.name

    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))


if __name__ == "__main__":
    main()
