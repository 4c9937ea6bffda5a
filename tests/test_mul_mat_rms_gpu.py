"""RMS_NORM + MUL fused into the one-token MUL_MAT (tsrc_mul_mat_rms) against the two kinds run one
after the other (tsrc_rms_norm, then tsrc_mul_mat), bit for bit: both formats, K from one block to
14336, with and without the norm weight, with an addend epilogue, and on the reference's special
activations; and the fused result against the oracle's RMS_NORM followed by its matvec."""
import numpy as np
import pytest

import helpers as H

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("fmt,N,K,kind,with_w,with_add", [
    (1, 300, 4096, "normal", True, False),
    (1, 64, 14336, "normal", True, True),
    (1, 40, 256, "normal", False, False),
    (1, 33, 2048, "special", True, False),
    (0, 500, 896, "normal", True, True),
    (0, 77, 4864, "normal", True, False),
    (0, 9, 32, "normal", True, False),
    (0, 50, 1024, "special", False, True),
])
def test_fused_equals_rms_norm_then_mul_mat(dev, tsro, fmt, N, K, kind, with_w, with_add):
    import torch
    seed = 700 + 10 * fmt + K % 97
    w = H.weights(tsro, fmt, N, K, seed)
    x = (H.special_acts(K, 1, seed + 1) if kind == "special" else H.acts(K, 1, seed + 1, scale=3.0))[0]
    nw = (1.0 + 0.25 * H.acts(K, 1, seed + 2)[0]).astype(np.float32) if with_w else None
    add = H.acts(N, 1, seed + 3)[0] if with_add else None
    wd = dev.upload(fmt, w, N, K)
    try:
        xd = torch.from_numpy(x).cuda()
        nwd = None if nw is None else torch.from_numpy(nw).cuda()
        ad = None if add is None else torch.from_numpy(add).cuda()
        inv_n = float(np.float32(1.0) / np.float32(K))
        y = torch.full((N + 32,), float("nan"), device="cuda")
        dev.mul_mat_rms(wd, xd, y[:N], norm_w=nwd, eps=1e-5, inv_n=inv_n, add=ad)
        h = torch.empty(K, device="cuda")
        dev.rms_norm(xd, h, K, 1, w=nwd, eps=1e-5, inv_n=inv_n)
        y2 = torch.empty(N, device="cuda")
        dev.mul_mat(wd, h, y2, T=1, add=ad)
        dev.sync()
        got = y.cpu().numpy()
        np.testing.assert_array_equal(bits(got[:N]), bits(y2.cpu().numpy()))
        assert np.isnan(got[N:]).all(), "the kernel wrote past the last row"
        # and against the oracle: its RMS_NORM kind, then its MUL_MAT
        he = tsro.rms_norm(x.reshape(1, K), nw, 1e-5, inv_n)
        ye = tsro.matvec(fmt, w, K, he, add=None if add is None else add.reshape(1, N), flags=1 if with_add else 0)
        np.testing.assert_array_equal(bits(got[:N]), bits(ye.reshape(-1)))
    finally:
        wd.free()
