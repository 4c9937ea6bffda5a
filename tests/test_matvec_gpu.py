"""MUL_MAT parity on the GPU through the C ABI: the CUDA results against the oracle, bit for bit
(y, the int32 block sums, the QACT image), on the fixture cases, on BASELINE configs 1 and 2, with
special activations, every epilogue, multi-token tiles, row shards and weights generated on the
device."""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def run_mm(dev, w, x, add=None, flags=0, s0=1.0, s1=1.0):
    import torch
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    T = x.shape[0]
    y = torch.full((T, w.n_rows), float("nan"), device="cuda")
    ad = None if add is None else torch.from_numpy(np.ascontiguousarray(add)).cuda()
    dev.mul_mat(w, xd, y, T=T, add=ad, flags=flags, s0=s0, s1=s1)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("name", list(H.MV_CASES))
def test_cases(dev, tsro, name):
    case = H.MV_CASES[name]
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
    w, x, add = H.mv_inputs(tsro, case)
    wd = dev.upload(fmt, w, N, K)
    try:
        np.testing.assert_array_equal(wd.download(), w)               # layout round trip
        y = run_mm(dev, wd, x, add=add, flags=flags & ~1, s0=s0, s1=s1)
        ye = tsro.matvec(fmt, w, K, x, add=add, flags=flags & ~1, s0=s0, s1=s1)
        np.testing.assert_array_equal(bits(y), bits(ye))
    finally:
        wd.free()


@pytest.mark.parametrize("name", list(H.MV_CASES) + list(H.MV_CONFIGS))
def test_block_sums(dev, tsro, name):
    import torch
    case = {**H.MV_CASES, **H.MV_CONFIGS}[name]
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
    w, x, _ = H.mv_inputs(tsro, case)
    wd = dev.upload(fmt, w, N, K)
    try:
        nb = K // (32 if fmt == 0 else 256)
        isum = torch.zeros((N, nb, 1 if fmt == 0 else 2), dtype=torch.int32, device="cuda")
        y = torch.zeros(N, device="cuda")
        dev.mul_mat_isums(wd, torch.from_numpy(x[0].copy()).cuda(), y, isum)
        torch.cuda.synchronize()
        q, d, bs = tsro.qact(fmt, x[:1])
        ie = tsro.block_isums(fmt, w, K, q[0], d[0], None if bs is None else bs[0]).reshape(N, nb, -1)
        np.testing.assert_array_equal(isum.cpu().numpy(), ie)
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(tsro.matvec(fmt, w, K, x[:1])[0]))
    finally:
        wd.free()


@pytest.mark.parametrize("fmt,K,T", [(0, 896, 3), (0, 4096, 1), (1, 4096, 2), (1, 256, 9)])
def test_qact(dev, tsro, fmt, K, T):
    import torch
    x = H.special_acts(K, T, 7 + K)
    xd = torch.from_numpy(x).cuda()
    q = torch.zeros((T, K), dtype=torch.int8, device="cuda")
    d = torch.zeros((T, K // (32 if fmt == 0 else 256)), device="cuda")
    bs = torch.zeros((T, K // 16), dtype=torch.int16, device="cuda") if fmt == 1 else None
    dev.qact(fmt, xd, K, T, q, d, bs)
    torch.cuda.synchronize()
    qe, de, be = tsro.qact(fmt, x)
    np.testing.assert_array_equal(q.cpu().numpy(), qe)
    np.testing.assert_array_equal(bits(d.cpu().numpy()), bits(de))
    if fmt == 1:
        np.testing.assert_array_equal(bs.cpu().numpy(), be)


@pytest.mark.parametrize("name", list(H.MV_CONFIGS))
def test_configs_synth(dev, tsro, name):
    """BASELINE configs 1 / 2 with weights generated on the device (the bench's inputs): the
    downloaded ggml blocks through the oracle give the GPU's y bit for bit."""
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = H.MV_CONFIGS[name]
    wd = dev.synth(fmt, N, K, seed=ws)
    try:
        w = wd.download()
        x = H.acts(K, 4, xs)
        y = run_mm(dev, wd, x)
        np.testing.assert_array_equal(bits(y), bits(tsro.matvec(fmt, w, K, x)))
        # sanity of the generator: the dequantized weights have the requested spread
        assert 0.01 < float(np.abs(y).mean()) < 10.0
    finally:
        wd.free()


@pytest.mark.parametrize("fmt,N,K,G", [(1, 14336, 4096, 8), (0, 4864, 896, 3), (1, 1000, 512, 7)])
def test_row_shards(dev, tsro, fmt, N, K, G):
    """Row shards (tensor parallelism): each shard's y equals the same rows of the full y, and a
    synthetic shard holds the same rows as an unsharded generation."""
    full = dev.synth(fmt, N, K, seed=77)
    try:
        x = H.acts(K, 1, 78)
        y = run_mm(dev, full, x)
        R = (N + G - 1) // G
        wfull = full.download()
        for g in range(G):
            r0, nr = g * R, min(R, N - g * R)
            if nr <= 0:
                continue
            sh = dev.synth(fmt, N, K, seed=77, row0=r0, n_rows=nr)
            try:
                np.testing.assert_array_equal(sh.download(), wfull[r0:r0 + nr])
                np.testing.assert_array_equal(bits(run_mm(dev, sh, x)[0]), bits(y[0, r0:r0 + nr]))
            finally:
                sh.free()
    finally:
        full.free()


def test_many_tokens_and_strides(dev, tsro):
    import torch
    fmt, N, K, T = 1, 300, 2048, 21
    w = H.weights(tsro, fmt, N, K, 55)
    x = H.acts(K, T, 56)
    wd = dev.upload(fmt, w, N, K)
    try:
        xs = torch.zeros((T, K + 64), device="cuda")
        xs[:, :K] = torch.from_numpy(x).cuda()
        y = torch.full((T, N + 7), -1.0, device="cuda")
        dev.mul_mat(wd, xs, y, T=T, x_stride=K + 64, y_stride=N + 7)
        torch.cuda.synchronize()
        yy = y.cpu().numpy()
        np.testing.assert_array_equal(bits(yy[:, :N]), bits(tsro.matvec(fmt, w, K, x)))
        assert (yy[:, N:] == -1.0).all()                      # nothing written past the rows
    finally:
        wd.free()


def test_argument_errors(dev, tsro):
    import torch
    w = dev.synth(0, 64, 256, seed=1)
    try:
        x = torch.zeros(256, device="cuda")
        y = torch.zeros(64, device="cuda")
        with pytest.raises(tsrc.TsrcError):
            dev.mul_mat(w, x, y, T=1, flags=tsrc.MM_ADD | tsrc.MM_SCALE, add=y)
        with pytest.raises(tsrc.TsrcError):
            dev.mul_mat(w, x, y, T=1, flags=0x80)
        with pytest.raises(tsrc.TsrcError):
            dev.synth(1, 10, 300, seed=1)
    finally:
        w.free()


@pytest.mark.parametrize("fmt,N,K,T", [(1, 300, 4096, 1), (0, 129, 4864, 3), (1, 50, 14336, 2), (0, 64, 896, 8)])
def test_mvm_prequantized(dev, tsro, fmt, N, K, T):
    """The MVM op on a QA image from tsrc_qact (the kernel's staging path) equals MUL_MAT."""
    import torch
    w = H.weights(tsro, fmt, N, K, 90 + N)
    x = H.special_acts(K, T, 91 + N)
    wd = dev.upload(fmt, w, N, K)
    try:
        xd = torch.from_numpy(x).cuda()
        q = torch.zeros((T, K), dtype=torch.int8, device="cuda")
        d = torch.zeros((T, K // (32 if fmt == 0 else 256)), device="cuda")
        bs = torch.zeros((T, K // 16), dtype=torch.int16, device="cuda") if fmt == 1 else None
        dev.qact(fmt, xd, K, T, q, d, bs)
        y = torch.zeros((T, N), device="cuda")
        dev.mvm(wd, q, d, bs, y, T=T)
        dev.sync()
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(tsro.matvec(fmt, w, K, x)))
    finally:
        wd.free()


def test_sync_reports_no_error(dev):
    dev.sync()
