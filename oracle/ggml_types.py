"""Test infrastructure (the checker, never the product): a numpy restatement of the load-time
conversion of ggml tensor types to Q8_0 blocks.

The reference keeps Q8_0 and Q4_K weights as shipped and converts every other type at load with
ggml's to_float of the type followed by quantize_row_q8_0_ref
(sw/ggml-tesseract/tsr-weights.h:1-30, tsr_row_to_dev_blocks). ggml itself is not in
/root/reference (the submodule is empty), so these functions restate ggml's published block
formats and its reference quantizer: dequantize_row_q4_0 / q4_1 / q5_0 / q5_1 / q5_K / q6_K, fp16
and bf16 widening, and quantize_row_q8_0_ref (amax = MAX(amax, |x|) with MAX(a, b) = a > b ? a : b,
d = amax / 127, id = d ? 1 / d : 0, fp16(d) to nearest even, q = roundf(x * id) half away from
zero). Every f32 product and sum is one numpy float32 operation (separately rounded, as ggml's
scalar C code compiled without contraction). Parity unpinned against ggml's own binaries (not
available here); the library's host conversion (tsrc_ggml_rows_to_dev) is tested against this.
"""
import numpy as np

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 3, 6, 7, 8, 12, 13, 14, 30
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
         Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


def _h(b: np.ndarray) -> np.ndarray:
    """little-endian fp16 fields (uint8 [..., 2]) -> float32"""
    return np.ascontiguousarray(b).view(np.float16)[..., 0].astype(np.float32)


def _scale_min_k4(sc: np.ndarray, j: int):
    """ggml's 6-bit scale / min j of the 12 scale bytes (sc: uint8 [nb, 12])."""
    sc = sc.astype(np.int32)
    if j < 4:
        return sc[:, j] & 63, sc[:, j + 4] & 63
    return (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4), (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)


def to_float(t: int, row: np.ndarray, K: int) -> np.ndarray:
    """ggml's to_float of one row (uint8 bytes) of K values of type t."""
    row = np.asarray(row, np.uint8)
    f = np.float32
    if t == F32:
        return row.view(np.float32).copy()
    if t == F16:
        return row.view(np.float16).astype(np.float32)
    if t == BF16:
        return (row.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    be, bb = BLOCK[t]
    b = row.reshape(K // be, bb)
    if t in (Q4_0, Q4_1):
        d = _h(b[:, 0:2])[:, None]
        qs = b[:, 4:20] if t == Q4_1 else b[:, 2:18]
        lo, hi = (qs & 0x0F).astype(np.int32), (qs >> 4).astype(np.int32)
        if t == Q4_0:
            y = np.concatenate([(lo - 8).astype(f) * d, (hi - 8).astype(f) * d], axis=1)
        else:
            m = _h(b[:, 2:4])[:, None]
            y = np.concatenate([lo.astype(f) * d + m, hi.astype(f) * d + m], axis=1)
        return y.reshape(-1).astype(f)
    if t in (Q5_0, Q5_1):
        d = _h(b[:, 0:2])[:, None]
        o = 4 if t == Q5_1 else 2
        qh = np.ascontiguousarray(b[:, o:o + 4]).view(np.uint32)[:, 0].astype(np.int64)[:, None]
        qs = b[:, o + 4:o + 20].astype(np.int32)
        j = np.arange(16)[None, :]
        xh0 = ((qh >> j) << 4) & 0x10
        xh1 = (qh >> (j + 12)) & 0x10
        x0, x1 = (qs & 0x0F) | xh0, (qs >> 4) | xh1
        if t == Q5_0:
            y = np.concatenate([(x0 - 16).astype(f) * d, (x1 - 16).astype(f) * d], axis=1)
        else:
            m = _h(b[:, 2:4])[:, None]
            y = np.concatenate([x0.astype(f) * d + m, x1.astype(f) * d + m], axis=1)
        return y.reshape(-1).astype(f)
    if t == Q5_K:
        d, mn = _h(b[:, 0:2]), _h(b[:, 2:4])
        sc, qh, ql = b[:, 4:16], b[:, 16:48].astype(np.int32), b[:, 48:176].astype(np.int32)
        out = []
        for c in range(4):
            s1, m1 = _scale_min_k4(sc, 2 * c)
            s2, m2 = _scale_min_k4(sc, 2 * c + 1)
            d1, mm1 = (d * s1.astype(f))[:, None], (mn * m1.astype(f))[:, None]
            d2, mm2 = (d * s2.astype(f))[:, None], (mn * m2.astype(f))[:, None]
            q = ql[:, 32 * c:32 * c + 32]
            u1, u2 = 1 << (2 * c), 2 << (2 * c)
            out.append(d1 * ((q & 0xF) + np.where(qh & u1, 16, 0)).astype(f) - mm1)
            out.append(d2 * ((q >> 4) + np.where(qh & u2, 16, 0)).astype(f) - mm2)
        return np.concatenate(out, axis=1).reshape(-1).astype(f)
    if t == Q6_K:
        ql, qh = b[:, 0:128].astype(np.int32), b[:, 128:192].astype(np.int32)
        sc = b[:, 192:208].view(np.int8).astype(f)
        d = _h(b[:, 208:210])[:, None]
        y = np.empty((b.shape[0], 256), f)
        for n in range(2):
            L, H, S = ql[:, 64 * n:64 * n + 64], qh[:, 32 * n:32 * n + 32], sc[:, 8 * n:8 * n + 8]
            is_ = np.arange(32) // 16
            q1 = ((L[:, :32] & 0xF) | (((H >> 0) & 3) << 4)) - 32
            q2 = ((L[:, 32:] & 0xF) | (((H >> 2) & 3) << 4)) - 32
            q3 = ((L[:, :32] >> 4) | (((H >> 4) & 3) << 4)) - 32
            q4 = ((L[:, 32:] >> 4) | (((H >> 6) & 3) << 4)) - 32
            base = 128 * n
            y[:, base:base + 32] = d * S[:, is_ + 0] * q1.astype(f)
            y[:, base + 32:base + 64] = d * S[:, is_ + 2] * q2.astype(f)
            y[:, base + 64:base + 96] = d * S[:, is_ + 4] * q3.astype(f)
            y[:, base + 96:base + 128] = d * S[:, is_ + 6] * q4.astype(f)
        return y.reshape(-1)
    raise ValueError(f"ggml type {t} has no to_float here")


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """quantize_row_q8_0_ref of one row of float32 values -> uint8 [K / 32 * 34]."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.zeros(x.shape[0], np.float32)
    for j in range(32):
        a = np.abs(x[:, j])
        amax = np.where(amax > a, amax, a)
    with np.errstate(divide="ignore", invalid="ignore"):
        d = amax / np.float32(127)
        idv = np.where(d != 0, np.float32(1) / d, np.float32(0)).astype(np.float32)
        v = x * idv[:, None]
        r = np.trunc(v)
        r = r + np.where(np.abs(v - r) >= np.float32(0.5), np.sign(v), np.float32(0)).astype(np.float32)
    q = np.where(np.isfinite(r) & (r >= -2147483648.0) & (r < 2147483648.0), r, -2147483648.0).astype(np.int64)
    out = np.empty((x.shape[0], 34), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = (q & 0xFF).astype(np.uint8)
    return out.reshape(-1)


def rows_to_dev(t: int, rows: np.ndarray, n_rows: int, K: int) -> np.ndarray:
    """Rows of type t -> device-format ggml rows (native Q8_0 / Q4_K copied, others to Q8_0)."""
    be, bb = BLOCK[t]
    rows = np.asarray(rows, np.uint8).reshape(n_rows, K // be * bb)
    if t in (Q8_0, Q4_K):
        return rows.copy()
    return np.stack([quantize_q8_0(to_float(t, r, K)) for r in rows])
