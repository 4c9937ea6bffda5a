"""The oracle (libtsro.so, this repository's restatement) against the golden fixtures produced by
the reference's own library (tests/golden/make_golden.py). Bit-exact everywhere."""
import os

import numpy as np
import pytest

import helpers as H

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gm():
    return np.load(os.path.join(GOLD, "golden_matvec.npz"))


@pytest.fixture(scope="module")
def gf():
    return np.load(os.path.join(GOLD, "golden_fa.npz"))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", list(H.MV_CASES))
def test_matvec_cases(tsro, gm, name):
    case = H.MV_CASES[name]
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
    w, x, add = H.mv_inputs(tsro, case)
    assert str(gm[f"{name}.digest"]) == H.digest(w, x, add if add is not None else np.zeros(0))
    if f"{name}.w" in gm:
        np.testing.assert_array_equal(gm[f"{name}.w"], w)
    y = tsro.matvec(fmt, w, K, x, add=add, flags=flags & ~1, s0=s0, s1=s1)
    np.testing.assert_array_equal(bits(y), bits(gm[f"{name}.y"]))
    q, d, bs = tsro.qact(fmt, x)
    np.testing.assert_array_equal(q, gm[f"{name}.q"])
    np.testing.assert_array_equal(bits(d), bits(gm[f"{name}.d"]))
    if bs is not None:
        np.testing.assert_array_equal(bs, gm[f"{name}.bs"])
    isum = tsro.block_isums(fmt, w, K, q[0], d[0], bs[0] if bs is not None else None)
    np.testing.assert_array_equal(isum, gm[f"{name}.isum"])


@pytest.mark.parametrize("name", list(H.MV_CONFIGS))
def test_matvec_configs(tsro, gm, name):
    case = H.MV_CONFIGS[name]
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
    w, x, add = H.mv_inputs(tsro, case)
    assert str(gm[f"{name}.digest"]) == H.digest(w, x, np.zeros(0))
    y = tsro.matvec(fmt, w, K, x)
    np.testing.assert_array_equal(bits(y), bits(gm[f"{name}.y"]))
    q, d, bs = tsro.qact(fmt, x)
    isum = tsro.block_isums(fmt, w, K, q[0], d[0], bs[0] if bs is not None else None)
    assert H.digest(isum) == str(gm[f"{name}.isum_digest"])


@pytest.mark.parametrize("name", list(H.FA_CASES) + list(H.FA_CONFIGS))
def test_fa(tsro, gf, name):
    case = {**H.FA_CASES, **H.FA_CONFIGS}[name]
    q, k, v, kw = H.fa_inputs(tsro, case)
    assert str(gf[f"{name}.digest"]) == H.digest(q, k, v, kw["mask"] if kw["mask"] is not None else np.zeros(0))
    rc, out = tsro.fa(q, k, v, **kw)
    assert rc == 0
    np.testing.assert_array_equal(bits(out), bits(gf[f"{name}.out"]))


def test_math(tsro):
    g = np.load(os.path.join(GOLD, "golden_math.npz"))
    v = H.math_inputs()
    assert str(g["digest"]) == H.digest(v)
    for k in range(4):
        np.testing.assert_array_equal(bits(tsro.expk(v, k)), bits(g[f"expk{k}"]))
    np.testing.assert_array_equal(bits(tsro.tanh(v)), bits(g["tanh"]))
