"""Builds libtsrc.so (the C-ABI library of include/tsrc.h) in-tree for sm_100a with nvcc.

    python build.py            # from anywhere; writes tesseract-npu_b200/libtsrc.so

Flags that carry the numerics contract: -fmad=false (no FMA contraction of separately rounded
f32 operations), -ftz=false (gradual underflow; the flush rule is applied in code),
-prec-div=true / -prec-sqrt=true (IEEE division), never --use_fast_math.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libtsrc.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
    "-Xptxas", "-v",
]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    deps.append(os.path.join(HERE, "..", "include", "tsrc.h"))
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    subprocess.run([sys.executable, os.path.join(CSRC, "gen_exp_tables.py")], check=True)
    cmd = [NVCC, *FLAGS, "-o", OUT + ".tmp", *sources()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libtsrc.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
