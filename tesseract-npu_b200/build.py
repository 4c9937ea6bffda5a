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
    """Compiles every .cu to an object in parallel (each translation unit is self-contained),
    then links the shared library."""
    if not force and up_to_date():
        return OUT
    from concurrent.futures import ThreadPoolExecutor
    subprocess.run([sys.executable, os.path.join(CSRC, "gen_exp_tables.py")], check=True)
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    compile_flags = [f for f in FLAGS if f != "-shared"]

    def one(src):
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        return subprocess.run([NVCC, *compile_flags, "-c", "-o", obj, src], capture_output=True, text=True), obj

    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
        results = list(ex.map(one, sources()))
    for r, _ in results:
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed building libtsrc.so")
        if verbose:
            sys.stderr.write(r.stderr)
    r = subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", OUT + ".tmp",
                        *[o for _, o in results]], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking libtsrc.so")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
