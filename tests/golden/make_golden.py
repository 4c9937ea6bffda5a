"""Generates the golden fixtures of tests/golden/ by running the REFERENCE's own C library
(oracle/_ref/libtsr_refdrv.so: jwkim04/tesseract-npu sw/sim/tsr_ref.c, tsr_ref_at.c,
tsr_ref_math.c compiled where they lie, see oracle/Makefile).

    make -C oracle all ref && python tests/golden/make_golden.py

Inputs are the seeded cases of tests/helpers.py; the fixtures keep the reference's outputs and,
for the inputs, SHA-256 digests (plus the bytes themselves for the small matvec cases).
Block sums are recomputed with numpy integer arithmetic from the reference's QACT output and the
blocks (the reference API does not return them; they are exact and order-free).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]

import oracle  # noqa: E402
import helpers as H  # noqa: E402


def isums_np(fmt, w, K, q, bs):
    """Exact block sums of every row against token 0's QA (numpy int64)."""
    N = w.shape[0]
    q = q.astype(np.int64)
    if fmt == 0:
        blk = w.reshape(N, K // 32, 34)
        qw = blk[:, :, 2:].view(np.int8).astype(np.int64)
        return np.einsum("nbi,bi->nb", qw, q.reshape(K // 32, 32)).astype(np.int32)
    sb = w.reshape(N, K // 256, 144)
    sc_b = sb[:, :, 4:16].astype(np.int64)
    qs = sb[:, :, 16:].astype(np.int64).reshape(N, K // 256, 4, 32)
    nib = np.stack([qs & 15, qs >> 4], axis=3).reshape(N, K // 256, 8, 32)    # sub-block j = 2c + (high)
    S = np.einsum("nsjl,sjl->nsj", nib, q.reshape(K // 256, 8, 32))
    sc = np.zeros((N, K // 256, 8), np.int64)
    mn = np.zeros((N, K // 256, 8), np.int64)
    for j in range(8):
        if j < 4:
            sc[..., j] = sc_b[..., j] & 63
            mn[..., j] = sc_b[..., j + 4] & 63
        else:
            sc[..., j] = (sc_b[..., j + 4] & 15) | ((sc_b[..., j - 4] >> 6) << 4)
            mn[..., j] = (sc_b[..., j + 4] >> 4) | ((sc_b[..., j] >> 6) << 4)
    b16 = bs.astype(np.int64).reshape(K // 256, 8, 2).sum(axis=2)
    isum = (sc * S).sum(axis=2)
    msum = (mn * b16[None]).sum(axis=2)
    return np.stack([isum, msum], axis=2).astype(np.int32)


def main():
    oracle.build(ref=True)
    tsro, ref = oracle.Tsro(), oracle.Ref()
    out = {}
    for name, case in {**H.MV_CASES, **H.MV_CONFIGS}.items():
        fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
        w, x, add = H.mv_inputs(tsro, case)
        y = ref.matvec(fmt, w, K, x, add=add, flags=flags & ~1, s0=s0, s1=s1)
        q, d, bs = ref.qact(fmt, x)
        out[f"{name}.digest"] = np.array(H.digest(w, x, add if add is not None else np.zeros(0)))
        out[f"{name}.y"] = y
        isum = isums_np(fmt, w, K, q[0], bs[0] if bs is not None else None)
        if name in H.MV_CASES:
            out[f"{name}.isum"] = isum
        else:
            out[f"{name}.isum_digest"] = np.array(H.digest(isum))
        if name in H.MV_CASES:
            out[f"{name}.q"], out[f"{name}.d"] = q, d
            if bs is not None:
                out[f"{name}.bs"] = bs
            if N * K <= 40 * 1024:
                out[f"{name}.w"], out[f"{name}.x"] = w, x
        print(name, y.shape)
    np.savez_compressed(os.path.join(HERE, "golden_matvec.npz"), **out)

    out = {}
    for name, case in {**H.FA_CASES, **H.FA_CONFIGS}.items():
        q, k, v, kw = H.fa_inputs(tsro, case)
        rc, o = ref.fa(q, k, v, **kw)
        assert rc == 0, (name, rc)
        out[f"{name}.digest"] = np.array(H.digest(q, k, v, kw["mask"] if kw["mask"] is not None else np.zeros(0)))
        out[f"{name}.out"] = o
        print(name, o.shape)
    np.savez_compressed(os.path.join(HERE, "golden_fa.npz"), **out)

    v = H.math_inputs()
    m = {"digest": np.array(H.digest(v)), "tanh": ref.tanh(v)}
    for k in range(4):
        m[f"expk{k}"] = ref.expk(v, k)
    np.savez_compressed(os.path.join(HERE, "golden_math.npz"), **m)


if __name__ == "__main__":
    main()
