"""Prefill MUL_MAT (many tokens) on the tcgen05 tensor cores, through the C ABI, against the oracle.

Q8_0 and Q4_K calls with more than eight tokens run one QACT over all tokens and one tensor-core
kernel (the exact int32 block / sub-block sums from tcgen05.mma kind::i8, the f32 row rule in
registers). The results must be the reference's bit for bit, as for the matvec kernel: same
tolerance (exact equality of the f32 bits).
"""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu


def _mul_mat(dev, wd, x, T, flags=0, add=None, s0=1.0, s1=1.0):
    import torch
    y = torch.full((T, wd.n_rows), float("nan"), device="cuda")
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    ad = None if add is None else torch.from_numpy(np.ascontiguousarray(add)).cuda()
    dev.mul_mat(wd, xd, y, T=T, flags=flags, add=ad, add_stride=None if add is None else wd.n_rows, s0=s0, s1=s1)
    dev.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("N,K,T,seed", [(300, 896, 9, 1), (1000, 4096, 64, 2), (257, 512, 33, 3), (129, 96, 100, 4),
                                        (4864, 896, 17, 5), (130, 1024, 300, 6), (64, 8192, 48, 7)])
def test_prefill_q8_0_bit_exact(dev, tsro, N, K, T, seed):
    w = H.weights(tsro, 0, N, K, seed)
    x = H.acts(K, T, seed + 100)
    wd = dev.upload(0, w, N, K)
    try:
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(0, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("N,K,T,seed", [(300, 1024, 9, 21), (1000, 4096, 64, 22), (257, 256, 33, 23), (129, 512, 100, 24),
                                        (896, 4864, 17, 25), (130, 2048, 300, 26), (64, 8192, 20, 27)])
def test_prefill_q4_k_bit_exact(dev, tsro, N, K, T, seed):
    w = H.weights(tsro, 1, N, K, seed)
    x = H.acts(K, T, seed + 100)
    wd = dev.upload(1, w, N, K)
    try:
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(1, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("fmt", [0, 1])
def test_prefill_tiny_activations(dev, tsro, fmt):
    """Blocks scaled down to 1e-20 .. 1e-37: activation scales far below 2^-79, so products and
    sums go subnormal and the reference's flush rule decides the low bits."""
    N, K, T = 160, 1024, 24
    w = H.weights(tsro, fmt, N, K, 31 + fmt)
    x = H.acts(K, T, 32 + fmt)
    rng = np.random.default_rng(33 + fmt)
    for t in range(T):
        for b in range(K // 32):
            if rng.integers(0, 3) == 0:
                x[t, 32 * b:32 * b + 32] *= np.float32(10.0 ** -rng.integers(20, 38))
    wd = dev.upload(fmt, w, N, K)
    try:
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(fmt, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("fmt", [0, 1])
def test_prefill_special_values_and_epilogues(dev, tsro, fmt):
    N, K, T = 200, 1024 if fmt else 640, 40
    w = H.weights(tsro, fmt, N, K, 11)
    x = H.special_acts(K, T, 12)
    wd = dev.upload(fmt, w, N, K)
    try:
        want = tsro.matvec(fmt, w, K, x)
        np.testing.assert_array_equal(_mul_mat(dev, wd, x, T).view(np.uint32), want.view(np.uint32))
        add = np.random.default_rng(13).standard_normal((T, N)).astype(np.float32)
        got = _mul_mat(dev, wd, x, T, add=add)
        want_add = tsro.matvec(fmt, w, K, x, flags=tsrc.MM_ADD, add=add)
        np.testing.assert_array_equal(got.view(np.uint32), want_add.view(np.uint32))
        got = _mul_mat(dev, wd, x, T, flags=tsrc.MM_SOFTCAP, s0=0.03, s1=30.0)
        want_sc = tsro.matvec(fmt, w, K, x, flags=tsrc.MM_SOFTCAP, s0=0.03, s1=30.0)
        np.testing.assert_array_equal(got.view(np.uint32), want_sc.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("fmt,N,K,T,seed", [(1, 14336, 4096, 2048, 501), (0, 4864, 896, 512, 401)],
                         ids=["cfg5_ffn_q4k_14336x4096_T2048", "cfg4_ffn_q80_4864x896_T512"])
def test_prefill_bench_shapes_bit_exact(dev, tsro, fmt, N, K, T, seed):
    """The bench's prefill workloads at their full size (the seeded weights bench.py times, every
    row and every token) against the oracle, bit for bit."""
    wd = dev.synth(fmt, N, K, seed=seed)
    try:
        w = wd.download()
        x = H.acts(K, T, seed + 1)
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(fmt, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("fmt,T", [(0, 16), (0, 32), (0, 100), (1, 16), (1, 32), (1, 100)])
def test_prefill_tile_widths_large_n(dev, tsro, fmt, T):
    """Token-tile widths of the tensor-core kernels at N = K = 4096, every row: Q4_K 16 / 32 / 64 tokens,
    Q8_0 16 / 32 (at T = 100 its launch picks 32-token tiles)."""
    N, K = 4096, 4096
    wd = dev.synth(fmt, N, K, seed=600 + T + fmt)
    try:
        w = wd.download()
        x = H.acts(K, T, 700 + T + fmt)
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(fmt, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()


@pytest.mark.parametrize("N,K,T", [(2048, 896, 1024), (896, 896, 512)])
def test_prefill_q8_0_tile_width_choice(dev, tsro, N, K, T):
    """Q8_0 shapes for which the launch picks 64-token tiles (2048 rows, 1024 tokens: a grid of many
    tiles) and 32-token tiles (896 rows: 64-token tiles would fill 56 of the SMs), every row and token
    bit for bit; the config-4 FFN shape, which picks 48, is checked above."""
    wd = dev.synth(0, N, K, seed=900 + N)
    try:
        w = wd.download()
        x = H.acts(K, T, 901 + N)
        got = _mul_mat(dev, wd, x, T)
        want = tsro.matvec(0, w, K, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        wd.free()
