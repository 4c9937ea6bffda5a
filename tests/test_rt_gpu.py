"""The C++ runtime front end (include/tsrc_rt.hpp: tsrc::rt::device, the counterpart of the reference's
tsr::rt::device, sw/rt/tsr_rt.h:66-288) through a compiled C++ program (tests/rt_check.cpp): upload from
each host type, read_blocks, and linear() on host activations, against the oracle bit for bit -- the
f32 weight through its load-time conversion to Q8_0, and a weight split into K parts accumulated in
order with one f32 add each (the reference's K-part rule). The header's compilation (-Wall -Werror) is
checked on any machine."""
import os
import subprocess

import numpy as np
import pytest

import ggml_types as G
import helpers as H
import tsrc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "tesseract-npu_b200")


def _compile(out_dir: str) -> str:
    exe = os.path.join(out_dir, "rt_check")
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "rt_check.cpp"), "-L", LIBDIR, "-ltsrc", f"-Wl,-rpath,{LIBDIR}", "-o", exe],
                   check=True, capture_output=True)
    return exe


def test_runtime_header_compiles(tmp_path):
    tsrc.lib()                                    # the library the program links against
    assert os.path.exists(_compile(str(tmp_path)))


RT_F32, RT_Q8_0, RT_Q4_K = 0, 3, 4


@pytest.mark.gpu
@pytest.mark.parametrize("rt_type,N,K,T,x_pad,max_part_k", [
    (RT_Q8_0, 70, 512, 3, 0, 0),           # as shipped, one K part
    (RT_F32, 40, 256, 2, 16, 0),           # f32 -> Q8_0 at upload; x rows 16 floats apart from the next
    (RT_Q4_K, 50, 1024, 2, 0, 512),        # two K parts, accumulated in order
    (RT_Q8_0, 30, 2048, 9, 0, 768),        # three K parts (768, 768, 512), the tensor-core path (T > 8)
])
def test_runtime_linear_bit_exact(tmp_path, tsro, rt_type, N, K, T, x_pad, max_part_k):
    fmt = tsrc.FMT_Q4_K if rt_type == RT_Q4_K else tsrc.FMT_Q8_0
    rng = np.random.default_rng(N + K)
    if rt_type == RT_F32:
        w_host = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        w_dev = G.rows_to_dev(G.F32, w_host.view(np.uint8), N, K)    # the load-time conversion
        wbytes = w_host.view(np.uint8)
    else:
        w_dev = H.weights(tsro, fmt, N, K, N + 1)
        wbytes = w_dev
    x = H.acts(K, T, K + 3)
    xs = K + x_pad
    x_file = np.zeros((T, xs), np.float32)
    x_file[:, :K] = x
    paths = {n: os.path.join(tmp_path, n) for n in ("w.bin", "x.bin", "y.bin", "b.bin")}
    np.ascontiguousarray(wbytes).tofile(paths["w.bin"])
    x_file.tofile(paths["x.bin"])
    exe = _compile(str(tmp_path))
    r = subprocess.run([exe, str(rt_type), str(N), str(K), str(T), str(xs), str(max_part_k), paths["w.bin"], paths["x.bin"],
                        paths["y.bin"], paths["b.bin"]], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    y = np.fromfile(paths["y.bin"], np.float32).reshape(T, N)
    blocks = np.fromfile(paths["b.bin"], np.uint8).reshape(N, -1)
    np.testing.assert_array_equal(blocks, np.asarray(w_dev).reshape(N, -1))
    # the oracle: the K parts in order, y = MUL_MAT(part 0); y = MUL_MAT(part j) + y
    kp = K if max_part_k == 0 else min(K, max_part_k)
    bs, bb = (256, 144) if fmt == tsrc.FMT_Q4_K else (32, 34)
    rows = np.asarray(w_dev).reshape(N, -1)
    want = None
    for k0 in range(0, K, kp):
        k1 = min(K, k0 + kp)
        part = np.ascontiguousarray(rows[:, k0 // bs * bb:k1 // bs * bb])
        if want is None:
            want = tsro.matvec(fmt, part, k1 - k0, np.ascontiguousarray(x[:, k0:k1]))
        else:
            want = tsro.matvec(fmt, part, k1 - k0, np.ascontiguousarray(x[:, k0:k1]), flags=tsrc.MM_ADD, add=want)
    np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32))
    assert f"k_parts {(K + kp - 1) // kp} " in r.stdout
