"""The restatement against the reference's own library on fresh random inputs (where
oracle/_ref was built): f32 rules on random bit patterns, EXPK / TANH, QACT, MUL_MAT with every
epilogue, flash attention with every mask kind and chunk order."""
import numpy as np
import pytest

import helpers as H


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_fp_rules(tsro, ref):
    rng = np.random.default_rng(5)
    a = rng.integers(0, 2 ** 32, 4000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    b = rng.integers(0, 2 ** 32, 4000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    # values near the flush boundary: products of 2^-126-ish numbers
    c = (np.float32(2.0 ** -63) * (1 + rng.random(4000, dtype=np.float32))).astype(np.float32)
    for op in ("fadd", "fsub", "fmul", "fdiv"):
        np.testing.assert_array_equal(bits(tsro.fp(op, a, b)), bits(ref.fp(op, a, b)))
        np.testing.assert_array_equal(bits(tsro.fp(op, c, -c[::-1])), bits(ref.fp(op, c, -c[::-1])))
    np.testing.assert_array_equal(bits(tsro.fp("frecip", a)), bits(ref.fp("frecip", a)))


def test_expk_tanh(tsro, ref):
    rng = np.random.default_rng(6)
    v = np.concatenate([rng.integers(0, 2 ** 32, 6000, dtype=np.uint64).astype(np.uint32).view(np.float32),
                        rng.normal(0, 40, 6000).astype(np.float32)])
    for k in range(4):
        np.testing.assert_array_equal(bits(tsro.expk(v, k)), bits(ref.expk(v, k)))
    np.testing.assert_array_equal(bits(tsro.tanh(v)), bits(ref.tanh(v)))


@pytest.mark.parametrize("fmt,K", [(0, 32), (0, 896), (1, 256), (1, 4096)])
def test_qact(tsro, ref, fmt, K):
    x = H.special_acts(K, 16, 100 + K)
    qa, da, ba = tsro.qact(fmt, x)
    qb, db, bb = ref.qact(fmt, x)
    np.testing.assert_array_equal(qa, qb)
    np.testing.assert_array_equal(bits(da), bits(db))
    if fmt == 1:
        np.testing.assert_array_equal(ba, bb)


@pytest.mark.parametrize("fmt,N,K,T,flags", [(0, 77, 4864, 2, 0), (1, 50, 14336, 1, 0), (0, 31, 2080, 3, 1),
                                             (1, 19, 768, 2, 4), (0, 23, 96, 1, 2), (1, 3, 256, 8, 0)])
def test_matvec(tsro, ref, fmt, N, K, T, flags):
    w = H.weights(tsro, fmt, N, K, 300 + N)
    x = H.special_acts(K, T, 301 + N) if flags == 0 else H.acts(K, T, 302 + N, 3.0)
    add = H.acts(N, T, 303) if flags & 1 else None
    ya = tsro.matvec(fmt, w, K, x, add=add, flags=flags & ~1, s0=0.05, s1=20.0)
    yb = ref.matvec(fmt, w, K, x, add=add, flags=flags & ~1, s0=0.05, s1=20.0)
    np.testing.assert_array_equal(bits(ya), bits(yb))


def test_matvec_random_blocks(tsro, ref):
    """Any block bytes are legal inputs: random qs / scales, fp16 scales incl. subnormal, Inf, NaN."""
    rng = np.random.default_rng(9)
    for fmt, K in ((0, 512), (1, 1024)):
        N = 40
        bpr = K // (32 if fmt == 0 else 256)
        bb = 34 if fmt == 0 else 144
        w = rng.integers(0, 256, (N, bpr * bb), dtype=np.uint8)
        d = rng.choice(np.array([0x0001, 0x03FF, 0x3C00, 0x7C00, 0x7E01, 0x1234, 0xBC00, 0x0000], np.uint16), (N, bpr))
        for b in range(bpr):
            w[:, b * bb] = d[:, b] & 0xFF
            w[:, b * bb + 1] = d[:, b] >> 8
        x = H.special_acts(K, 2, 10 + fmt)
        np.testing.assert_array_equal(bits(tsro.matvec(fmt, w, K, x)), bits(ref.matvec(fmt, w, K, x)))


@pytest.mark.parametrize("name", list(H.FA_CASES))
def test_fa_vs_ref(tsro, ref, name):
    case = list(H.FA_CASES[name])
    case[-1] += 500            # fresh inputs, not the fixture's
    q, k, v, kw = H.fa_inputs(tsro, tuple(case))
    rc1, o1 = tsro.fa(q, k, v, **kw)
    rc2, o2 = ref.fa(q, k, v, **kw)
    assert rc1 == rc2 == 0
    np.testing.assert_array_equal(bits(o1), bits(o2))
