"""Seeded synthetic inputs shared by the tests and the golden-fixture generator.

Inputs are numpy PCG64 normal draws (BASELINE's distributions: weights N(0, 0.02), activations,
K, V and Q N(0, 1)) quantized with the oracle's encoders. The quantized bytes are pinned by
SHA-256 digests stored in the fixtures, so a test knows it regenerated the same inputs.
"""
import hashlib

import numpy as np

NEG = np.float16(-np.inf)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def weights(tsro, fmt, N, K, seed, sigma=0.02):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(sigma)).astype(np.float32)
    return tsro.quantize(fmt, W)


def acts(K, T, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((T, K), dtype=np.float32) * np.float32(scale)).astype(np.float32)


def special_acts(K, T, seed):
    """Activations with the reference's special cases (sw/sim/tests/test_sim_mvm.c:25-41): zero
    blocks, subnormals, ties for the max, Inf, NaN, all-subnormal blocks."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K), dtype=np.float32)
    u = x.view(np.uint32)
    for t in range(T):
        for b in range(K // 32):
            s = slice(32 * b, 32 * b + 32)
            c = rng.integers(0, 12)
            if c == 0:
                x[t, s] = 0
            elif c == 1:
                u[t, 32 * b + rng.integers(0, 32)] = 0x00012345 | (int(rng.integers(0, 2)) << 31)
            elif c == 2:
                m = x[t, 32 * b]
                x[t, 32 * b + 5] = -m
                x[t, 32 * b + 9] = m
            elif c == 3:
                x[t, 32 * b + rng.integers(0, 32)] = np.inf
            elif c == 4:
                u[t, 32 * b + rng.integers(0, 32)] = 0x7FC01234
            elif c == 5:
                u[t, s] = 0x100 * np.arange(1, 33, dtype=np.uint32)
    return x


def kv_rows(tsro, n_cells, E, seed):
    rng = np.random.default_rng(seed)
    return tsro.quantize(0, rng.standard_normal((n_cells, E), dtype=np.float32))


def fa_mask(kind, T, n_kv, pos0, nswa=64, seed=0):
    """F16 KQ masks: causal, sliding window, finite values, holes, a wrapped ring (two runs),
    an empty row, or all visible."""
    rng = np.random.default_rng(seed)
    m = np.full((T, n_kv), NEG, np.float16)
    for q in range(T):
        p = pos0 + q
        if kind == "causal":
            m[q, :min(p + 1, n_kv)] = 0
        elif kind == "swa":
            m[q, max(0, p - nswa + 1):min(p + 1, n_kv)] = 0
        elif kind == "finite":
            n = min(p + 1, n_kv)
            m[q, :n] = rng.normal(0, 2, n).astype(np.float16)
        elif kind == "holes":
            m[q, :min(p + 1, n_kv)] = 0
            m[q, 3:9] = NEG
            m[q, 40:41] = NEG
            m[q, 60:70] = NEG
        elif kind == "ring":
            m[q, :] = 0
            m[q, (p % n_kv):((p % n_kv) + n_kv // 3)] = NEG
        elif kind == "empty":
            if q == 1:
                m[q, :] = NEG
            else:
                m[q, :min(p + 1, n_kv)] = 0
        elif kind == "none":
            m[q, :] = 0
    return m


# ---- shared case tables (golden fixtures and parity tests) ----------------------------------
# matvec: name -> (fmt, N, K, T, w_seed, x_seed, x_kind, flags, s0, s1)
MV_CASES = {
    "q80_small": (0, 40, 896, 3, 11, 12, "normal", 0, 1.0, 1.0),
    "q4k_small": (1, 24, 4352, 2, 13, 14, "normal", 0, 1.0, 1.0),
    "q80_special": (0, 32, 1024, 4, 15, 16, "special", 0, 1.0, 1.0),
    "q4k_special": (1, 18, 2048, 3, 17, 18, "special", 0, 1.0, 1.0),
    "q80_add": (0, 33, 2048, 2, 19, 20, "normal", 1, 1.0, 1.0),
    "q4k_add": (1, 17, 1536, 1, 21, 22, "normal", 1, 1.0, 1.0),
    "q80_softcap": (0, 30, 512, 2, 23, 24, "big", 4, 0.033, 30.0),
    "q4k_scale": (1, 20, 1024, 2, 25, 26, "normal", 2, 0.5, 0.125),
    "q80_long": (0, 9, 14336, 1, 27, 28, "normal", 0, 1.0, 1.0),
    "q4k_long": (1, 7, 14336, 5, 29, 30, "normal", 0, 1.0, 1.0),
}
# BASELINE configs 1 and 2 (outputs only in the fixture; inputs regenerated and digest-checked)
MV_CONFIGS = {
    "cfg1": (0, 4864, 896, 1, 101, 102, "normal", 0, 1.0, 1.0),
    "cfg2": (1, 14336, 4096, 1, 201, 202, "normal", 0, 1.0, 1.0),
}


def mv_inputs(tsro, case):
    fmt, N, K, T, ws, xs, xk, flags, s0, s1 = case
    w = weights(tsro, fmt, N, K, ws)
    if xk == "special":
        x = special_acts(K, T, xs)
    elif xk == "big":
        x = acts(K, T, xs, scale=40.0)
    else:
        x = acts(K, T, xs)
    add = acts(N, T, xs + 1000) if flags & 1 else None
    return w, x, add


# FA: name -> (D, n_head_kv, G, T, n_kv, pos0, mask, C, t_max, pcap, scale, qmul, new_lo, new_hi, seed)
FA_CASES = {
    "decode_d64_g7": (64, 2, 7, 1, 256, 199, "causal", 4, 8, 9344, 0.125, 1.0, 0, 0, 31),
    "prefill_d128": (128, 2, 5, 5, 160, 120, "causal", 3, 8, 9344, 0.0883883, 1.5, 0, 0, 32),
    "prefill_swa_d256": (256, 2, 2, 7, 200, 150, "swa", 4, 8, 9344, 1.0, 0.25, 0, 0, 33),
    "prefill_c1": (64, 1, 1, 13, 300, 250, "causal", 1, 8, 9344, 0.125, 2.0, 0, 0, 34),
    "decode_ring": (128, 1, 4, 1, 256, 300, "ring", 4, 8, 9344, 0.0883883, 1.0, 0, 0, 35),
    "decode_g16_d512": (512, 1, 16, 1, 128, 100, "causal", 4, 8, 9344, 1.0, 0.05, 0, 0, 36),
    "prefill_finite": (128, 1, 2, 6, 100, 90, "finite", 2, 8, 9344, 0.0883883, 1.0, 0, 0, 37),
    "prefill_holes": (64, 2, 3, 4, 120, 100, "holes", 4, 8, 9344, 0.125, 1.0, 0, 0, 38),
    "empty_row": (64, 1, 2, 3, 64, 40, "empty", 4, 1, 9344, 0.125, 1.0, 0, 0, 39),
    "small_pcap": (128, 2, 3, 1, 512, 511, "causal", 4, 8, 512, 0.0883883, 3.0, 0, 0, 40),
    "decode_gqa_2chunk": (128, 8, 4, 1, 2048, 2047, "none", 4, 4, 9344, 0.0883883, 1.0, 0, 0, 41),
    "decode_new_mid": (128, 2, 4, 1, 1500, 1499, "causal", 4, 4, 9344, 0.0883883, 1.0, 700, 701, 42),
    "prefill_t9": (64, 2, 7, 9, 700, 600, "causal", 4, 4, 9344, 0.125, 1.0, 600, 609, 43),
    "qwen_decode": (64, 2, 7, 1, 640, 639, "causal", 4, 4, 9344, 0.125, 1.0, 639, 640, 44),
}
# 32 q / 8 kv heads, D 128, n_kv 8192, decode, all cells visible
FA_CONFIGS = {
    "cfg3": (128, 8, 4, 1, 8192, 8191, "none", 4, 4, 9344, float(np.float32(1.0 / np.sqrt(128.0))), 1.0, 0, 0, 301),
}


def fa_inputs(tsro, case):
    D, nkvh, G, T, n_kv, pos0, mk, C, tmax, pcap, scale, qmul, nlo, nhi, seed = case
    E = nkvh * D
    k = kv_rows(tsro, n_kv, E, seed)
    v = kv_rows(tsro, n_kv, E, seed + 1000)
    rng = np.random.default_rng(seed + 2000)
    q = (rng.standard_normal((T, nkvh * G, D), dtype=np.float32) * np.float32(qmul)).astype(np.float32)
    mask = None if mk == "none" else fa_mask(mk, T, n_kv, pos0, seed=seed + 3000)
    kw = dict(D=D, n_head=nkvh * G, n_head_kv=nkvh, n_kv=n_kv, scale=float(np.float32(scale)), mask=mask, C=C,
              t_max=tmax, pcap=pcap, new=(nlo, nhi))
    return q, k, v, kw


def math_inputs():
    """EXPK / TANH inputs: random bit patterns plus the ranges attention and softcap use."""
    rng = np.random.default_rng(51)
    bits = rng.integers(0, 2 ** 32, 8192, dtype=np.uint64).astype(np.uint32).view(np.float32)
    return np.concatenate([bits, rng.normal(0, 30, 4096).astype(np.float32),
                           -np.abs(rng.normal(0, 8, 4096)).astype(np.float32)])
