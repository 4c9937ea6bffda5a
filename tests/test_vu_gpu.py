"""The decoder layer's vector kinds on the GPU, through the C ABI, against the oracle (which
tests/test_oracle_vu.py pins to the reference's own vector-unit library). Tolerance: equal f32
bit patterns."""
import numpy as np
import pytest

import helpers as H
import tsrc
from test_oracle_vu import _special

pytestmark = pytest.mark.gpu


def _cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _eq(got, want):
    np.testing.assert_array_equal(np.asarray(got, np.float32).view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


@pytest.mark.parametrize("n,rows,eps", [(896, 7, 1e-6), (4096, 3, 1e-5), (64, 2, 0.5)])
def test_rms_norm(dev, tsro, n, rows, eps):
    import torch
    rng = np.random.default_rng(n + rows)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    x[0] = _special(rng, n)
    x[1 % rows] *= np.float32(1e-20)
    w = rng.standard_normal(n).astype(np.float32)
    xd, wd = _cuda(x), _cuda(w)
    y = torch.full_like(xd, float("nan"))
    dev.rms_norm(xd, y, n, rows, w=wd, eps=eps)
    dev.sync()
    _eq(y.cpu().numpy(), tsro.rms_norm(x, w, eps))
    dev.rms_norm(xd, xd, n, rows, eps=eps)                      # in place, no weight
    dev.sync()
    _eq(xd.cpu().numpy(), tsro.rms_norm(x, None, eps))


@pytest.mark.parametrize("mode,hd,nd,base", [(0, 128, 128, 500000.0), (1, 64, 64, 1e6), (1, 128, 64, 10000.0)])
def test_rope(dev, tsro, mode, hd, nd, base):
    import torch
    rng = np.random.default_rng(hd + nd + mode)
    n_heads, T = 5, 6
    x = rng.standard_normal((T, n_heads * hd)).astype(np.float32)
    x[1, :11] = _special(rng, 11)
    pos = np.array([0, 1, 511, 2047, 8191, 131071], np.int32)
    ts = float(np.power(np.float32(base), np.float32(-2.0) / np.float32(nd), dtype=np.float32))
    want = tsro.rope(x, pos, n_heads=n_heads, head_dim=hd, n_dims=nd, mode=mode, ts=ts)
    xd, pd = _cuda(x), _cuda(pos)
    y = torch.full_like(xd, float("nan"))
    dev.rope(xd, y, pd, T, n_heads, hd, nd, mode, ts)
    dev.rope(xd, xd, pd, T, n_heads, hd, nd, mode, ts)           # in place
    dev.sync()
    _eq(y.cpu().numpy(), want)
    _eq(xd.cpu().numpy(), want)


@pytest.mark.parametrize("func", [tsrc.VOP_ADD, tsrc.VOP_MUL, tsrc.VOP_SILU, tsrc.VOP_SWIGLU])
def test_vop(dev, tsro, func):
    import torch
    rng = np.random.default_rng(func + 3)
    n, rows = 3000, 3
    a = np.concatenate([rng.standard_normal(n * rows - 600) * 8, _special(rng, 594), [-100, 100, -88, 89, 1e-20, -1e-20]])
    a = a.astype(np.float32).reshape(rows, n)
    b = _special(rng, n * rows).reshape(rows, n)
    y = torch.full((rows, n), float("nan"), device="cuda")
    dev.vop(func, _cuda(a), _cuda(b), y, n, rows)
    dev.sync()
    _eq(y.cpu().numpy(), tsro.vop(func, a, b))


@pytest.mark.parametrize("fmt,K", [(0, 896), (1, 4096), (1, 1024)])
def test_get_rows(dev, tsro, fmt, K):
    import torch
    N = 40
    w = H.weights(tsro, fmt, N, K, 60 + fmt)
    for r, d16 in ((3, 0x7BFF), (5, 0x0001), (7, 0x7E00), (9, 0x7C00)):
        w[r, 0:2] = np.frombuffer(np.uint16(d16).tobytes(), np.uint8)
    wd = dev.upload(fmt, w, N, K)
    try:
        ids = np.array([3, 0, 39, 5, 5, 7, 9, 21], np.int32)
        y = torch.full((ids.size, K), float("nan"), device="cuda")
        dev.get_rows(wd, _cuda(ids), ids.size, y)
        dev.sync()
        _eq(y.cpu().numpy(), tsro.dequant(fmt, w[ids], K))
        bad = _cuda(np.array([1, N], np.int32))
        dev.get_rows(wd, bad, 2, y)
        with pytest.raises(tsrc.TsrcError):
            dev.sync()
        dev.sync()                                               # the flag was cleared
    finally:
        wd.free()
