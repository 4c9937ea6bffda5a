"""Weight ingestion on the host (no GPU): the load-time conversion of ggml tensor types to the device
formats (tsrc_ggml_rows_to_dev, the counterpart of tsr_row_to_dev_blocks,
sw/ggml-tesseract/tsr-weights.h:1-30) against the numpy restatement in oracle/ggml_types.py, bit
for bit; native Q8_0 / Q4_K rows pass unchanged; other types are refused; and the GGUF reader /
writer round trip."""
import os

import numpy as np
import pytest

import tsrc
import tsrc.gguf as gguf
import ggml_types as G

CONVERTED = [G.F32, G.F16, G.BF16, G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q5_K, G.Q6_K]


def random_rows(t: int, n_rows: int, K: int, seed: int) -> np.ndarray:
    """Random rows of type t: random quant bytes with finite, varied fp16 scales."""
    rng = np.random.default_rng(seed)
    be, bb = G.BLOCK[t]
    if t == G.F32:
        x = (rng.standard_normal((n_rows, K)) * 10.0 ** rng.integers(-3, 3, (n_rows, 1))).astype(np.float32)
        x[0, :32] = 0.0                                               # an all-zero block
        x[0, 40] = 1e-40                                              # a subnormal
        return x.view(np.uint8)
    if t in (G.F16, G.BF16):
        x = rng.standard_normal((n_rows, K)).astype(np.float32)
        return (x.astype(np.float16) if t == G.F16 else (x.view(np.uint32) >> 16).astype(np.uint16)).view(np.uint8)
    b = rng.integers(0, 256, (n_rows, K // be, bb), dtype=np.uint8)

    def put_h(col, scale):
        v = (rng.random((n_rows, K // be)) * scale + scale / 64).astype(np.float16)
        b[:, :, col:col + 2] = v.view(np.uint8).reshape(n_rows, K // be, 2)

    if t in (G.Q4_0, G.Q5_0):
        put_h(0, 0.05)
    elif t in (G.Q4_1, G.Q5_1, G.Q5_K):
        put_h(0, 0.05)
        put_h(2, 0.02)
    elif t == G.Q6_K:
        put_h(208, 0.01)
    return b.reshape(n_rows, -1)


@pytest.mark.parametrize("t", CONVERTED)
def test_conversion_matches_restatement(t):
    n_rows, K = 5, 512
    rows = random_rows(t, n_rows, K, 100 + t)
    got = tsrc.ggml_rows_to_dev(t, rows, n_rows, K)
    want = G.rows_to_dev(t, rows, n_rows, K)
    assert got.shape == (n_rows, K // 32 * 34)
    np.testing.assert_array_equal(got.reshape(-1), want.reshape(-1))


def test_conversion_many_rows_threads():
    """A tensor large enough to be split over host threads converts as row by row."""
    n_rows, K = 600, 2048
    rows = random_rows(G.Q6_K, n_rows, K, 7)
    got = tsrc.ggml_rows_to_dev(G.Q6_K, rows, n_rows, K)
    for r in (0, 1, 299, 599):
        np.testing.assert_array_equal(got[r], G.rows_to_dev(G.Q6_K, rows[r:r + 1], 1, K)[0])


@pytest.mark.parametrize("t,fmt", [(G.Q8_0, tsrc.FMT_Q8_0), (G.Q4_K, tsrc.FMT_Q4_K)])
def test_native_types_pass_unchanged(t, fmt):
    rng = np.random.default_rng(5)
    rows = rng.integers(0, 256, (3, tsrc.ggml_row_bytes(fmt, 512)), dtype=np.uint8)
    np.testing.assert_array_equal(tsrc.ggml_rows_to_dev(t, rows, 3, 512), rows)
    assert tsrc.ggml_type_info(t)[2] == fmt


def test_q8_0_round_trip_through_f32_is_exact():
    """Q8_0 blocks whose largest |q| is 127 (what QACT-style quantization gives) survive
    dequantization to f32 and re-quantization exactly."""
    rng = np.random.default_rng(9)
    q = rng.integers(-127, 128, (4, 16, 32)).astype(np.int8)
    q[:, :, 5] = 127
    d = (rng.random((4, 16)) * 0.05 + 0.001).astype(np.float16)
    blocks = np.concatenate([d.view(np.uint8).reshape(4, 16, 2), q.view(np.uint8)], axis=2).reshape(4, -1)
    f = np.stack([(q[r].astype(np.float32) * d[r].astype(np.float32)[:, None]).reshape(-1) for r in range(4)])
    np.testing.assert_array_equal(tsrc.ggml_rows_to_dev(G.F32, f.view(np.uint8), 4, 512), blocks)


@pytest.mark.parametrize("t", [9, 10, 11, 15, 16, 99])
def test_unloadable_types_refused(t):
    with pytest.raises(tsrc.TsrcError):
        tsrc.ggml_type_info(t)
    with pytest.raises(tsrc.TsrcError):
        tsrc.ggml_rows_to_dev(t, np.zeros(64, np.uint8), 1, 256)


def test_bad_row_length_refused():
    with pytest.raises(tsrc.TsrcError):
        tsrc.ggml_rows_to_dev(G.Q4_K, np.zeros(144, np.uint8), 1, 128)       # K not a whole superblock


def test_gguf_write_read_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    a = rng.integers(0, 256, (3, 34 * 8), dtype=np.uint8)                # 3 rows of K = 256, Q8_0
    b = rng.standard_normal(256).astype(np.float32)
    c = rng.integers(0, 256, (2, 144), dtype=np.uint8)                   # 2 rows of K = 256, Q4_K
    kv = {"general.architecture": (gguf.T_STR, "llama"), "llama.block_count": (gguf.T_U32, 2),
          "llama.rope.freq_base": (gguf.T_F32, 10000.0), "x.flag": (gguf.T_BOOL, True),
          "x.list": (gguf.T_ARR, (gguf.T_I32, [1, -2, 3])), "x.big": (gguf.T_U64, 1 << 40)}
    path = os.path.join(tmp_path, "t.gguf")
    gguf.write_gguf(path, kv, [("a", G.Q8_0, (256, 3), a), ("b", G.F32, (256,), b), ("c", G.Q4_K, (256, 2), c)], align=64)
    r = gguf.GGUFReader(path)
    assert r.version == 3
    assert r.kv["general.architecture"] == "llama" and r.kv["llama.block_count"] == 2
    assert r.kv["x.flag"] is True and r.kv["x.list"] == [1, -2, 3] and r.kv["x.big"] == 1 << 40
    assert r.kv["general.alignment"] == 64
    np.testing.assert_array_equal(np.asarray(r.tensors["a"].data).reshape(3, -1), a)
    np.testing.assert_array_equal(np.asarray(r.tensors["b"].data).view(np.float32), b)
    np.testing.assert_array_equal(np.asarray(r.tensors["c"].data).reshape(2, -1), c)
    assert r.tensors["a"].n_rows == 3 and r.tensors["a"].row_len == 256


def test_gguf_rejects_other_files(tmp_path):
    path = os.path.join(tmp_path, "x.bin")
    with open(path, "wb") as f:
        f.write(b"NOPE" + b"\0" * 60)
    with pytest.raises(tsrc.TsrcError):
        gguf.GGUFReader(path)
