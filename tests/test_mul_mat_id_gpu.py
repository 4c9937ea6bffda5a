"""MUL_MAT_ID (tsrc_mul_mat_id: ggml's expert-routed product, the reference's MUL_MAT_ID kind) through
the C ABI, against the oracle: for every token t and slot j the output row must equal, bit for bit,
the oracle's one-token MUL_MAT of expert ids[t][j]'s rows with that pair's activation row (the
tolerance every MUL_MAT test here uses). Both formats; one activation row per token shared by its
slots (the gate / up of a MoE block) and one per slot (its down projection); strided outputs; an
expert id outside the weight reported by tsrc_sync and its outputs left unwritten."""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu


def _run(dev, wd, n_exp, x, ids, n_used, T, x_slots, **kw):
    import torch
    Ne = wd.n_rows // n_exp
    y = torch.full((T, n_used, Ne), float("nan"), device="cuda")
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    idd = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).cuda()
    dev.mul_mat_id(wd, n_exp, xd, idd, y, n_used=n_used, T=T, x_slots=x_slots, **kw)
    dev.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("fmt,n_exp,Ne,K,n_used,T,x_slots,seed", [
    (0, 8, 96, 512, 2, 3, 1, 1),        # Q8_0, gate / up style: one x per token
    (1, 6, 64, 1024, 3, 2, 3, 2),       # Q4_K, down style: one x per slot
    (1, 4, 160, 4096, 2, 1, 1, 3),      # Q4_K, one decode token, a one-tile row (x in registers)
    (0, 5, 50, 4864, 4, 2, 4, 4),       # Q8_0, long rows (x from shared memory)
])
def test_mul_mat_id_bit_exact(dev, tsro, fmt, n_exp, Ne, K, n_used, T, x_slots, seed):
    w = H.weights(tsro, fmt, n_exp * Ne, K, seed)
    x = H.acts(K, T * x_slots, seed + 10).reshape(T, x_slots, K)
    rng = np.random.default_rng(seed + 20)
    ids = np.stack([rng.choice(n_exp, n_used, replace=False) for _ in range(T)]).astype(np.int32)
    wd = dev.upload(fmt, w, n_exp * Ne, K)
    try:
        got = _run(dev, wd, n_exp, x, ids, n_used, T, x_slots)
        row = w.reshape(n_exp * Ne, -1)
        for t in range(T):
            for j in range(n_used):
                e = int(ids[t, j])
                want = tsro.matvec(fmt, row[e * Ne:(e + 1) * Ne], K, x[t, j % x_slots][None, :])[0]
                np.testing.assert_array_equal(got[t, j].view(np.uint32), want.view(np.uint32), err_msg=f"t={t} j={j} e={e}")
    finally:
        wd.free()


def test_mul_mat_id_strides(dev, tsro):
    """Token and slot strides longer than a row, in x and y."""
    import torch
    fmt, n_exp, Ne, K, n_used, T = 0, 3, 40, 256, 2, 2
    w = H.weights(tsro, fmt, n_exp * Ne, K, 31)
    xs = H.acts(K, T, 32)
    x_pad = np.full((T, K + 64), np.nan, np.float32)
    x_pad[:, :K] = xs
    ids = np.array([[2, 0], [1, 2]], np.int32)
    wd = dev.upload(fmt, w, n_exp * Ne, K)
    try:
        y = torch.full((T, n_used, Ne + 8), float("nan"), device="cuda")
        dev.mul_mat_id(wd, n_exp, torch.from_numpy(x_pad).cuda(), torch.from_numpy(ids).cuda(), y, n_used=n_used, T=T,
                       x_slots=1, x_tok_stride=K + 64, y_slot_stride=Ne + 8, y_tok_stride=n_used * (Ne + 8))
        dev.sync()
        got = y.cpu().numpy()
        row = w.reshape(n_exp * Ne, -1)
        for t in range(T):
            for j in range(n_used):
                e = int(ids[t, j])
                want = tsro.matvec(fmt, row[e * Ne:(e + 1) * Ne], K, xs[t][None, :])[0]
                np.testing.assert_array_equal(got[t, j, :Ne].view(np.uint32), want.view(np.uint32))
                assert np.isnan(got[t, j, Ne:]).all()            # the padding is not written
    finally:
        wd.free()


def test_mul_mat_id_bad_expert_reported(dev, tsro):
    import torch
    fmt, n_exp, Ne, K = 0, 4, 32, 256
    w = H.weights(tsro, fmt, n_exp * Ne, K, 41)
    x = H.acts(K, 1, 42)
    wd = dev.upload(fmt, w, n_exp * Ne, K)
    try:
        y = torch.full((1, 2, Ne), float("nan"), device="cuda")
        ids = torch.tensor([[1, 7]], dtype=torch.int32, device="cuda")      # 7 is not an expert
        dev.mul_mat_id(wd, n_exp, torch.from_numpy(x).cuda(), ids, y, n_used=2, T=1)
        with pytest.raises(tsrc.TsrcError):
            dev.sync()
        got = y.cpu().numpy()
        want = tsro.matvec(fmt, w.reshape(n_exp * Ne, -1)[Ne:2 * Ne], K, x)[0]
        np.testing.assert_array_equal(got[0, 0].view(np.uint32), want.view(np.uint32))
        assert np.isnan(got[0, 1]).all()
        dev.sync()                                                           # the flag was cleared
        with pytest.raises(tsrc.TsrcError):
            dev.mul_mat_id(wd, 3, torch.from_numpy(x).cuda(), ids, y, n_used=2, T=1)   # 128 rows are not 3 experts
    finally:
        wd.free()
