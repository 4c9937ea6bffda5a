"""tsrc_mul_mat_noalloc: MUL_MAT for hosts that cannot let a library allocate device memory.

A host that plans every byte of device memory itself (llama.cpp's ggml allocator reserves the
compute buffers before the first graph), or that must not synchronise the device in the middle of a
decode loop, cannot call a function that may cudaMalloc a scratch buffer. This entry point keeps
its scratch in a fixed array inside the library instead. Each case calls it through the C ABI twice
in a row (the second call reuses the array the first one filled) and checks that both results are
bit for bit those of tsrc_mul_mat on the same inputs, and the oracle's: the tolerance every MUL_MAT
test here uses.

Cases: one token (its own QACT launch, then the matvec), several tokens in one and in two token
tiles, a large K whose shared-memory image allows fewer than 8 tokens per launch (the token-tile
shrink), an addend with row 0 for every token (add_stride 0) and with a per-token stride, SCALE
and SOFTCAP epilogues, and an activation stride longer than K.

The file name sorts last so that a run that stops at the first failure has run everything else.
"""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu

# fmt, N, K, T, seed, x_stride (0 = K), epilogue
CASES = [
    (1, 300, 4096, 1, 60, 0, None),
    (1, 300, 4096, 3, 61, 0, None),
    (0, 257, 896, 9, 62, 0, None),                 # two token tiles (8 + 1)
    (0, 64, 32768, 7, 63, 0, None),                # the image allows 5 tokens per launch: 5 + 2
    (0, 200, 896, 4, 64, 0, ("add", 0)),           # one addend row for every token
    (1, 96, 2048, 3, 65, 0, ("add", "tok")),      # an addend row per token (add_stride = N)
    (0, 130, 512, 2, 66, 0, ("scale", None)),
    (1, 70, 1024, 2, 67, 0, ("softcap", None)),
    (0, 90, 256, 3, 68, 384, None),               # x rows 384 floats apart
]


def _inputs(tsro, case):
    fmt, N, K, T, seed, xs, epi = case
    w = H.weights(tsro, fmt, N, K, seed)
    x = H.special_acts(K, T, seed + 1)
    x_pad = x
    if xs:
        x_pad = np.full((T, xs), np.nan, np.float32)
        x_pad[:, :K] = x
    kw, okw = {}, {}
    if epi is not None:
        kind, how = epi
        if kind == "add":
            rows = 1 if how == 0 else T
            add = np.random.default_rng(seed + 2).standard_normal((rows, N)).astype(np.float32)
            okw = dict(add=add, add_stride=0 if how == 0 else N)
            kw = dict(add_stride=0 if how == 0 else N)
            kw["add"] = add
        elif kind == "scale":
            okw = kw = dict(flags=tsrc.MM_SCALE, s1=0.37)
        else:
            okw = kw = dict(flags=tsrc.MM_SOFTCAP, s0=0.02, s1=30.0)
    return w, x, x_pad, kw, okw


def _run(dev, fn, wd, x_pad, T, xs, kw):
    import torch
    args = dict(kw)
    if "add" in args:
        args["add"] = torch.from_numpy(np.ascontiguousarray(args["add"])).cuda()
    y = torch.full((T, wd.n_rows), float("nan"), device="cuda")
    fn(wd, torch.from_numpy(np.ascontiguousarray(x_pad)).cuda(), y, T=T, x_stride=xs, **args)
    dev.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"fmt{c[0]}_N{c[1]}_K{c[2]}_T{c[3]}_{c[6][0] if c[6] else 'plain'}"
                         + (f"_xs{c[5]}" if c[5] else ""))
def test_noalloc_matches_mul_mat_twice(dev, tsro, case):
    fmt, N, K, T, seed, xs, _ = case
    w, x, x_pad, kw, okw = _inputs(tsro, case)
    wd = dev.upload(fmt, w, N, K)
    try:
        y_ref = _run(dev, dev.mul_mat, wd, x_pad, T, xs, kw)
        y_orc = tsro.matvec(fmt, w, K, x, **okw)
        np.testing.assert_array_equal(y_ref.view(np.uint32), y_orc.view(np.uint32))
        for _ in range(2):                         # two calls in a row share the array
            y = _run(dev, dev.mul_mat_noalloc, wd, x_pad, T, xs, kw)
            np.testing.assert_array_equal(y.view(np.uint32), y_ref.view(np.uint32))
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
        # T = 0 does nothing and checks nothing further, as tsrc_mul_mat
        dev.mul_mat_noalloc(w, x, y, T=0, flags=0x80)
        dev.mul_mat(w, x, y, T=0, flags=0x80)
    finally:
        w.free()
