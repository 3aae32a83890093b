"""Compile the sm_100a CUDA library librdna2_b200.so in-tree.

  python rdna2-gfx1030-ai-handbook_b200/build.py [--force] [-v]

Each csrc/*.cu compiles in parallel with
  nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -std=c++17
and links into rdna2_ops/lib/librdna2_b200.so with the CUDA runtime linked
statically, so the library depends only on the driver (libcuda) at run time.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "rdna2_ops" / "lib" / "librdna2_b200.so"
INCLUDE = HERE.parent / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         f"-I{INCLUDE}"]


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False):
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for src, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                failed.append(src.name)
    if failed:
        raise RuntimeError("nvcc failed for " + ", ".join(failed))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if force or jobs or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
