"""FLASH_ATTN_EXT over the q8_0 KV cache on the GPU, through the C ABI, against the oracle.

The oracle (oracle/tsro_fa.c) is pinned bit for bit to the reference's own tsr_ref_fa
(tests/test_oracle_ref.py, tests/golden/golden_fa.npz), so "equal to the oracle" here means equal
to the reference. The tolerance is exact equality of the f32 bit patterns: every step of the
reference's composite (QACT, exact block sums, EXPK, block floating point P.V, channel tree,
online merge) is deterministic and the kernels keep its order where order matters.

Also covered: the KV cache's ggml q8_0 image round trip (set_tensor / get_tensor of a KV tensor)
and KVST (SET_ROWS: QACT A32 of f32 rows) against the oracle's quantizer, cell indices included.
"""
import numpy as np
import pytest

import helpers as H
import tsrc

pytestmark = pytest.mark.gpu


def _fa_gpu(dev, q, k, v, kw):
    import torch
    T, n_head, D = q.shape
    kv = dev.kv_create(kw["n_head_kv"], D, max(kw["n_kv"], 1))
    try:
        if kw["n_kv"]:
            kv.set_bytes(tsrc.KV_K, k[:kw["n_kv"]])
            kv.set_bytes(tsrc.KV_V, v[:kw["n_kv"]])
        qd = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        out = torch.full((T, n_head, D), float("nan"), device="cuda")
        dev.flash_attn(kv, qd, out, T=T, n_head=n_head, n_kv=kw["n_kv"], scale=kw["scale"], mask=kw["mask"],
                       new=kw["new"], cfg=(kw["C"], kw["t_max"], kw["pcap"], 32768))
        dev.sync()
        return out.cpu().numpy()
    finally:
        kv.free()


@pytest.mark.parametrize("name", sorted(H.FA_CASES))
def test_fa_cases_bit_exact(dev, tsro, name):
    q, k, v, kw = H.fa_inputs(tsro, H.FA_CASES[name])
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    got = _fa_gpu(dev, q, k, v, kw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_fa_cfg3_bit_exact(dev, tsro):
    """BASELINE config 3 at full size: 32 q / 8 kv heads, D 128, 8192 cells, decode."""
    q, k, v, kw = H.fa_inputs(tsro, H.FA_CONFIGS["cfg3"])
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    got = _fa_gpu(dev, q, k, v, kw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_fa_special_values(dev, tsro):
    """Queries with NaN / Inf / subnormal / huge values and KV blocks with extreme fp16 scales."""
    rng = np.random.default_rng(71)
    D, nkvh, G, T, n_kv = 64, 2, 2, 3, 200
    E = nkvh * D
    k = H.kv_rows(tsro, n_kv, E, 72)
    v = H.kv_rows(tsro, n_kv, E, 73)
    # a few cells with large / tiny / NaN V scales and huge K scales
    for cell, d16 in ((5, 0x7BFF), (17, 0x0001), (90, 0x7E00), (130, 0x7C00)):
        v[cell, 0:2] = np.frombuffer(np.uint16(d16).tobytes(), np.uint8)
    k[40, 0:2] = np.frombuffer(np.uint16(0x7BFF).tobytes(), np.uint8)
    q = rng.standard_normal((T, nkvh * G, D)).astype(np.float32)
    q[0, 0, 3] = np.inf
    q[1, 1, 7] = np.float32(1e-42)
    q[2, 2, 9] = np.nan
    q[2, 3, :] = np.float32(3e38)
    mask = H.fa_mask("causal", T, n_kv, 150, seed=74)
    kw = dict(D=D, n_head=nkvh * G, n_head_kv=nkvh, n_kv=n_kv, scale=0.125, mask=mask, C=4, t_max=4, pcap=9344,
              new=(0, 0))
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    got = _fa_gpu(dev, q, k, v, kw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("shape", ["cfg4", "cfg5", "d256"])
def test_fa_prefill_bench_shapes(dev, tsro, shape):
    """Prefill attention of the bench's models at their prompt lengths, all query rows: config 4
    (Qwen2.5-0.5B: 14 q / 2 KV heads of 64, 512 tokens) and config 5 (Llama-3-8B: 32 q / 8 KV heads
    of 128, 2048 tokens), causal from position 0, the release attention configuration; and a head
    size of 256 (4 KV heads, 300 tokens). Calls with this many work items run the 4-warp chunk CTAs."""
    D, nkvh, G, T, seed = {"cfg4": (64, 2, 7, 512, 81), "cfg5": (128, 8, 4, 2048, 85), "d256": (256, 4, 2, 300, 89)}[shape]
    E = nkvh * D
    k = H.kv_rows(tsro, T, E, seed)
    v = H.kv_rows(tsro, T, E, seed + 1)
    q = np.random.default_rng(seed + 2).standard_normal((T, nkvh * G, D)).astype(np.float32)
    mask = H.fa_mask("causal", T, T, 0, seed=seed + 3)
    kw = dict(D=D, n_head=nkvh * G, n_head_kv=nkvh, n_kv=T, scale=float(np.float32(1.0) / np.sqrt(np.float32(D))),
              mask=mask, C=4, t_max=4, pcap=9344, new=(0, T))
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    got = _fa_gpu(dev, q, k, v, kw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("C,t_max,pcap", [(1, 1, 9344), (2, 8, 4096), (8, 4, 9344), (16, 2, 16384)])
def test_fa_attention_configs(dev, tsro, C, t_max, pcap):
    """The output depends on C, T_MAX and PCAP (chunking and channel trees); the kernels follow."""
    case = (128, 2, 4, 5, 700, 650, "causal", C, t_max, pcap, 0.0883883, 1.0, 650, 655, 75)
    q, k, v, kw = H.fa_inputs(tsro, case)
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    got = _fa_gpu(dev, q, k, v, kw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_kv_bytes_round_trip(dev):
    rng = np.random.default_rng(76)
    kv = dev.kv_create(3, 64, 37)
    try:
        img = rng.integers(0, 256, (37, kv.row_bytes), dtype=np.uint8)
        kv.set_bytes(tsrc.KV_V, img)
        np.testing.assert_array_equal(kv.get_bytes(tsrc.KV_V), img)
        part = rng.integers(0, 256, (5, kv.row_bytes), dtype=np.uint8)
        kv.set_bytes(tsrc.KV_V, part, cell0=30)
        img[30:35] = part
        np.testing.assert_array_equal(kv.get_bytes(tsrc.KV_V), img)
        assert not kv.get_bytes(tsrc.KV_K).any()          # the other plane is untouched (zeroed)
    finally:
        kv.free()


def test_kv_set_rows_is_kvst(dev, tsro):
    """SET_ROWS / KVST: QACT A32 of each f32 row, stored at given cells or consecutively."""
    import torch
    rng = np.random.default_rng(77)
    D, nkvh, n_cells = 128, 2, 50
    E = D * nkvh
    rows = rng.standard_normal((12, E)).astype(np.float32)
    rows[3, 5] = np.nan
    rows[4, :32] = 0.0
    rows[5, 40] = np.float32(1e-40)
    kv = dev.kv_create(nkvh, D, n_cells)
    try:
        rd = torch.from_numpy(rows).cuda()
        kv.set_rows(tsrc.KV_K, rd[:4], cell0=10)
        cells = torch.tensor([49, 0, 7, 3, 20, 21, 22, 23], dtype=torch.int64, device="cuda")
        kv.set_rows(tsrc.KV_K, rd[4:], cells=cells)
        dev.sync()
        got = kv.get_bytes(tsrc.KV_K)
        want = tsro.quantize(0, rows)
        np.testing.assert_array_equal(got[10:14], want[:4])
        for i, c in enumerate(cells.cpu().numpy()):
            np.testing.assert_array_equal(got[c], want[4 + i])
    finally:
        kv.free()


def test_kv_set_rows_bad_cell_reports(dev):
    import torch
    kv = dev.kv_create(1, 64, 16)
    try:
        rows = torch.ones((2, 64), device="cuda")
        cells = torch.tensor([3, 16], dtype=torch.int64, device="cuda")     # 16 is outside the cache
        kv.set_rows(tsrc.KV_K, rows, cells=cells)
        with pytest.raises(tsrc.TsrcError):
            dev.sync()
        got = kv.get_bytes(tsrc.KV_K)
        assert got[3].any() and not np.delete(got, 3, axis=0).any()
        dev.sync()                                                          # the flag was cleared
    finally:
        kv.free()


def test_fa_rejects(dev):
    import torch
    kv = dev.kv_create(2, 64, 64)
    try:
        q = torch.zeros((1, 4, 64), device="cuda")
        out = torch.zeros_like(q)
        with pytest.raises(tsrc.TsrcError):        # n_kv beyond the cache
            dev.flash_attn(kv, q, out, T=1, n_head=4, n_kv=65, scale=0.125)
        with pytest.raises(tsrc.TsrcError):        # negative scale
            dev.flash_attn(kv, q, out, T=1, n_head=4, n_kv=10, scale=-1.0)
        with pytest.raises(tsrc.TsrcError):        # n_head not a multiple of n_head_kv
            dev.flash_attn(kv, q, out, T=1, n_head=3, n_kv=10, scale=0.125)
        with pytest.raises(tsrc.TsrcError):        # C = 0
            dev.flash_attn(kv, q, out, T=1, n_head=4, n_kv=10, scale=0.125, cfg=(0, 4, 9344, 0))
        with pytest.raises(tsrc.TsrcError):
            dev.kv_create(2, 96, 10)                # head_dim 96
    finally:
        kv.free()


def test_fa_kv_head_shards_plan_as_one_device(dev, tsro):
    """Tensor parallelism by KV heads, emulated with one cache per shard on one GPU: with the
    model's KV heads as plan_n_head_kv every shard chunks as the single device does (PCAP binds
    the chunk size here, and it depends on E), so the concatenated heads are the single-device
    output bit for bit; planning with the shard's own E would not be."""
    import torch
    from tsrc import parallel as P
    D, nkvh, G = 128, 8, 4
    case = (D, nkvh, G, 1, 3000, 2999, "causal", 4, 4, 2048, 0.0883883, 1.0, 2999, 3000, 81)
    q, k, v, kw = H.fa_inputs(tsro, case)
    rc, want = tsro.fa(q, k, v, **kw)
    assert rc == 0
    rb = D // 32 * 34
    for world in (2, 4):
        outs, outs_own = [], []
        for r in range(world):
            h0, hn = P.kv_head_shard(nkvh, world, r)
            kv = dev.kv_create(hn, D, kw["n_kv"])
            try:
                kv.set_bytes(tsrc.KV_K, np.ascontiguousarray(k[:, h0 * rb:(h0 + hn) * rb]))
                kv.set_bytes(tsrc.KV_V, np.ascontiguousarray(v[:, h0 * rb:(h0 + hn) * rb]))
                qd = torch.from_numpy(np.ascontiguousarray(q[:, h0 * G:(h0 + hn) * G])).cuda()
                for plan, dst in ((nkvh, outs), (0, outs_own)):
                    out = torch.full_like(qd, float("nan"))
                    dev.flash_attn(kv, qd, out, T=1, n_head=hn * G, n_kv=kw["n_kv"], scale=kw["scale"], mask=kw["mask"],
                                   new=kw["new"], cfg=(kw["C"], kw["t_max"], kw["pcap"], 32768, plan))
                    dev.sync()
                    dst.append(out.cpu().numpy())
            finally:
                kv.free()
        got = np.concatenate(outs, axis=1)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        assert not np.array_equal(np.concatenate(outs_own, axis=1).view(np.uint32), want.view(np.uint32))
