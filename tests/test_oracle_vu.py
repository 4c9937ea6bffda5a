"""The decoder layer's vector kinds in the oracle (oracle/tsro_vu.c) against the reference's own
vector-unit library (oracle/_ref: sw/sim/tsr_ref_vu.c, tsr_ref_math.c, tsr_ref.c compiled where they
lie): RMS_NORM + MUL, SIN / COS, ROPE (NORM and NEOX), the VOPs ADD / MUL / SILU / SWIGLU and the
dequantization of a ggml row (GET_ROWS). Tolerance: equal f32 bit patterns."""
import numpy as np
import pytest

import helpers as H


def _special(rng, n):
    """Normal values mixed with zeros, subnormals, huge values, infinities and NaNs."""
    x = rng.standard_normal(n).astype(np.float32)
    u = x.view(np.uint32)
    k = rng.integers(0, 12, n)
    u[k == 0] = 0
    u[k == 1] = rng.integers(1, 0x007FFFFF, (k == 1).sum()).astype(np.uint32) | (rng.integers(0, 2, (k == 1).sum()).astype(np.uint32) << 31)
    x[k == 2] = np.float32(3e38)
    x[k == 3] = -np.inf
    u[k == 4] = 0x7FC01234
    x[k == 5] *= np.float32(1e-30)
    return x


def _eq(a, b):
    np.testing.assert_array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("n,eps", [(896, 1e-6), (4096, 1e-5), (64, 1e-6), (100, 0.5)])
def test_rms_norm(tsro, ref, n, eps):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((4, n)).astype(np.float32) * np.float32(3)
    x[1] *= np.float32(1e-20)                  # sum of squares near the flush boundary
    x[2, :7] = np.float32(1e19)                # overflow of the squares
    w = rng.standard_normal(n).astype(np.float32)
    _eq(tsro.rms_norm(x, w, eps), ref.rms_norm(x, w, eps))
    _eq(tsro.rms_norm(x, None, eps), ref.rms_norm(x, None, eps))
    xs = _special(rng, 3 * n).reshape(3, n)
    _eq(tsro.rms_norm(xs, w, eps), ref.rms_norm(xs, w, eps))


def test_sincos(tsro, ref):
    rng = np.random.default_rng(5)
    t = np.concatenate([rng.uniform(-10, 10, 3000), rng.uniform(-1e6, 1e6, 3000), rng.standard_normal(500) * 1e-3,
                        np.float32(2.0) ** rng.integers(-130, 127, 500) * rng.choice([-1, 1], 500),
                        [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, np.pi / 2, np.pi, 3e38]]).astype(np.float32)
    s1, c1 = tsro.sincos(t)
    s2, c2 = ref.sincos(t)
    _eq(s1, s2)
    _eq(c1, c2)


@pytest.mark.parametrize("mode,hd,nd,base", [(0, 128, 128, 500000.0), (1, 64, 64, 1e6), (0, 64, 32, 10000.0), (1, 128, 64, 10000.0)])
def test_rope(tsro, ref, mode, hd, nd, base):
    rng = np.random.default_rng(hd + nd + mode)
    n_heads, T = 3, 5
    x = rng.standard_normal((T, n_heads * hd)).astype(np.float32)
    x[2, :9] = _special(rng, 9)
    pos = np.array([0, 1, 77, 2047, 131000], np.int32)
    ts = np.float32(np.power(np.float32(base), np.float32(-2.0) / np.float32(nd), dtype=np.float32))
    kw = dict(n_heads=n_heads, head_dim=hd, n_dims=nd, mode=mode, ts=ts)
    _eq(tsro.rope(x, pos, **kw), ref.rope(x, pos, **kw))
    _eq(tsro.rope(x, pos, attn_factor=0.75, **kw), ref.rope(x, pos, attn_factor=0.75, **kw))


@pytest.mark.parametrize("func", [0, 2, 6, 7])
def test_vop(tsro, ref, func):
    rng = np.random.default_rng(func)
    a = np.concatenate([rng.standard_normal(2000) * 8, _special(rng, 500), [-100, 100, -88, 89, 1e-20, -1e-20]]).astype(np.float32)
    b = _special(rng, a.size)
    _eq(tsro.vop(func, a, b), ref.vop(func, a, None if func == 6 else b))


@pytest.mark.parametrize("fmt,K", [(0, 896), (1, 1024)])
def test_dequant(tsro, ref, fmt, K):
    w = H.weights(tsro, fmt, 6, K, 40 + fmt)
    rb = w.shape[1]
    # extreme block scales: fp16 max, subnormal, NaN, Inf in d (and dmin for Q4_K)
    for r, d16 in ((1, 0x7BFF), (2, 0x0001), (3, 0x7E00), (4, 0x7C00)):
        w[r, 0:2] = np.frombuffer(np.uint16(d16).tobytes(), np.uint8)
        if fmt == 1:
            w[r, rb - 144 + 2:rb - 144 + 4] = np.frombuffer(np.uint16(d16 ^ 0x8000).tobytes(), np.uint8)
    _eq(tsro.dequant(fmt, w, K), ref.dequant(fmt, w, K))
