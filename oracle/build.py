"""Build the CPU oracle shared library (test infrastructure only).

Output: oracle/_build/libqlinear_oracle.so.  -ffp-contract=off keeps every
a*b+c in the oracle as two IEEE roundings; -march=x86-64-v3 keeps the binary
runnable on the GPU hosts, which may be a different CPU than the build host.
"""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "qlinear_oracle.c"
OUT = HERE / "_build" / "libqlinear_oracle.so"


def build(force=False):
    OUT.parent.mkdir(exist_ok=True)
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math",
           "-fopenmp", "-fPIC", "-shared", "-o", str(OUT), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
