"""tsrc_mul_mat_noalloc: MUL_MAT for hosts that cannot let a library allocate device memory.

A host that plans every byte of device memory itself (llama.cpp's ggml allocator reserves the
compute buffers before the first graph), or that must not synchronise the device in the middle of a
decode loop, cannot call a function that may cudaMalloc a scratch buffer. This entry point keeps
its scratch in a fixed array inside the library instead. The test calls it through the C ABI twice
in a row (the second call reuses the array the first one filled) and checks that both results are
bit for bit those of tsrc_mul_mat on the same inputs, the tolerance every MUL_MAT test here uses.

The file name sorts last so that a run that stops at the first failure has run everything else.
"""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu


def _run(dev, fn, w, x, T):
    import torch
    y = torch.full((T, w.n_rows), float("nan"), device="cuda")
    fn(w, torch.from_numpy(np.ascontiguousarray(x)).cuda(), y, T=T)
    dev.sync()
    return y.cpu().numpy()


def test_noalloc_matches_mul_mat_twice(dev, tsro):
    cases = [(1, 300, 4096, 3, 61), (0, 257, 896, 9, 62)]      # the second call spans two token tiles
    for fmt, N, K, T, seed in cases:
        w = H.weights(tsro, fmt, N, K, seed)
        x = H.special_acts(K, T, seed + 1)
        wd = dev.upload(fmt, w, N, K)
        try:
            y_noalloc = _run(dev, dev.mul_mat_noalloc, wd, x, T)
            y_ref = _run(dev, dev.mul_mat, wd, x, T)
            np.testing.assert_array_equal(y_noalloc.view(np.uint32), y_ref.view(np.uint32))
            np.testing.assert_array_equal(y_noalloc.view(np.uint32), tsro.matvec(fmt, w, K, x).view(np.uint32))
        finally:
            wd.free()


def test_noalloc_rejects_bad_arguments(dev):
    import torch
    w = dev.synth(0, 64, 256, seed=3)
    try:
        x = torch.zeros(256, device="cuda")
        y = torch.zeros(64, device="cuda")
        with pytest.raises(tsrc.TsrcError):
            dev.mul_mat_noalloc(w, x, y, T=1, flags=0x80)
        with pytest.raises(tsrc.TsrcError):
            dev.mul_mat_noalloc(w, x, y, T=1, flags=tsrc.MM_ADD)          # an addend flag without an addend
    finally:
        w.free()
