"""One-token MUL_MAT (decode: QACT fused into the matvec kernel) bit for bit against the oracle over
the shapes a decoder meets and their edges: K from one block to K_MAX, partial last tiles, row
counts that leave short last CTAs, the reference's special activations (zero blocks, subnormals,
Inf, NaN, ties; the flush-checked path) at T = 1, every epilogue, and many launches back to back
on one stream (each launch's L2 prefetch runs under the previous launch)."""
import numpy as np
import pytest

import helpers as H

pytestmark = pytest.mark.gpu

# fmt, N, K, activation kind, flags, s0, s1, seed
CASES = {
    "q4k_k4096": (1, 300, 4096, "normal", 0, 1.0, 1.0, 301),
    "q4k_partial_tile": (1, 77, 1536, "normal", 0, 1.0, 1.0, 302),
    "q4k_k6144": (1, 150, 6144, "normal", 0, 1.0, 1.0, 303),
    "q4k_k14336_ragged": (1, 61, 14336, "normal", 0, 1.0, 1.0, 304),
    "q4k_k32768": (1, 20, 32768, "normal", 0, 1.0, 1.0, 305),
    "q4k_kmax": (1, 4, 65536, "normal", 0, 1.0, 1.0, 320),
    "q80_kmax": (0, 3, 65536, "normal", 0, 1.0, 1.0, 321),
    "q4k_one_superblock": (1, 9, 256, "normal", 0, 1.0, 1.0, 306),
    "q4k_special": (1, 70, 4352, "special", 0, 1.0, 1.0, 307),
    "q4k_special_k2048": (1, 40, 2048, "special", 0, 1.0, 1.0, 308),
    "q4k_add": (1, 199, 4096, "normal", 1, 1.0, 1.0, 309),
    "q4k_scale": (1, 33, 2048, "normal", 2, 0.5, 0.125, 310),
    "q80_cfg1_shape": (0, 1000, 896, "normal", 0, 1.0, 1.0, 311),
    "q80_one_block": (0, 5, 32, "normal", 0, 1.0, 1.0, 312),
    "q80_partial_tile": (0, 64, 800, "normal", 0, 1.0, 1.0, 313),
    "q80_k4864": (0, 151, 4864, "normal", 0, 1.0, 1.0, 314),
    "q80_k14336": (0, 37, 14336, "normal", 0, 1.0, 1.0, 315),
    "q80_special": (0, 50, 1024, "special", 0, 1.0, 1.0, 316),
    "q80_special_k8192": (0, 23, 8192, "special", 0, 1.0, 1.0, 317),
    "q80_softcap": (0, 90, 512, "big", 4, 0.033, 30.0, 318),
    "q80_add": (0, 129, 4096, "normal", 1, 1.0, 1.0, 319),
}


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", list(CASES))
def test_one_token(dev, tsro, name):
    import torch
    fmt, N, K, kind, flags, s0, s1, seed = CASES[name]
    w = H.weights(tsro, fmt, N, K, seed)
    if kind == "special":
        x = H.special_acts(K, 1, seed + 1)
    elif kind == "big":
        x = H.acts(K, 1, seed + 1, scale=40.0)
    else:
        x = H.acts(K, 1, seed + 1)
    add = H.acts(N, 1, seed + 2) if flags & 1 else None
    wd = dev.upload(fmt, w, N, K)
    try:
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        y = torch.full((1, N + 64), float("nan"), device="cuda")      # guard band past the row count
        ad = None if add is None else torch.from_numpy(np.ascontiguousarray(add)).cuda()
        dev.mul_mat(wd, xd, y[:, :N], T=1, add=ad, flags=flags, s0=s0, s1=s1)
        dev.sync()
        got = y.cpu().numpy()
        ye = tsro.matvec(fmt, w, K, x, add=add, flags=flags, s0=s0, s1=s1)
        np.testing.assert_array_equal(bits(got[:, :N]), bits(ye))
        assert np.isnan(got[:, N:]).all(), "the kernel wrote past the last row"
    finally:
        wd.free()


@pytest.mark.parametrize("fmt,N,K", [(1, 14336, 4096), (0, 4864, 896), (1, 4096, 14336)])
def test_back_to_back(dev, tsro, fmt, N, K):
    """Many launches on one stream over three weight copies (programmatic dependent launch lets each
    launch start under the previous one); every output equals the single-launch result of its
    copy."""
    import torch
    ws = [dev.synth(fmt, N, K, seed=900 + c) for c in range(3)]
    try:
        x = torch.from_numpy(H.acts(K, 1, 77)).cuda()
        ref = []
        for w in ws:
            y = torch.empty((1, N), device="cuda")
            dev.mul_mat(w, x, y, T=1)
            dev.sync()
            ref.append(y.cpu().numpy().view(np.uint32).copy())
        ys = [torch.empty((1, N), device="cuda") for _ in range(30)]
        for i, y in enumerate(ys):
            dev.mul_mat(ws[i % 3], x, y, T=1)
        dev.sync()
        for i, y in enumerate(ys):
            np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), ref[i % 3])
        # and the first copy against the oracle
        ye = tsro.matvec(fmt, ws[0].download(), K, x.cpu().numpy())
        np.testing.assert_array_equal(ref[0], bits(ye))
    finally:
        for w in ws:
            w.free()
