"""ctypes view of the parity oracle (TEST INFRASTRUCTURE ONLY).

Two libraries live under ``oracle/``:

* ``libtsro.so`` -- this repository's C restatement of the reference numerics (``tsro.c``,
  ``tsro_fa.c``); it is built from committed sources on any machine (``make -C oracle``).
* ``_ref/libtsr_refdrv.so`` -- the reference's own ``sw/sim`` C library compiled where it lies,
  plus ``ref_driver.c`` (``make -C oracle ref``). It exists only where the reference tree was
  present when it was built; it travels with the working tree as a built file.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this
module; the product never does.
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TSRO_PATH = os.path.join(HERE, "libtsro.so")
REF_PATH = os.path.join(HERE, "_ref", "libtsr_refdrv.so")

FMT_Q8_0, FMT_Q4_K = 0, 1
MM_ADD, MM_SCALE, MM_SOFTCAP = 1, 2, 4

_p = ct.c_void_p
_u32, _i32, _f32, _sz = ct.c_uint32, ct.c_int32, ct.c_float, ct.c_size_t


def _ptr(a):
    return a.ctypes.data_as(_p) if a is not None else None


def build(ref: bool = True) -> None:
    """Builds libtsro.so (always) and, where the reference tree is present, the reference driver."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    root = os.environ.get("REF_ROOT")
    if ref and root and os.path.isdir(os.path.join(root, "sw", "sim")):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


class FaParams(ct.Structure):
    _fields_ = [("C", _u32), ("t_max", _u32), ("pcap", _u32), ("T", _u32), ("D", _u32), ("n_head", _u32),
                ("n_head_kv", _u32), ("n_kv", _u32), ("scale", _f32), ("new_lo", _u32), ("new_hi", _u32)]


class Tsro:
    """The restatement (libtsro.so)."""

    def __init__(self, path: str = TSRO_PATH):
        if not os.path.exists(path):
            build(ref=False)
        L = self.lib = ct.CDLL(path)
        for n in ("tsro_fadd", "tsro_fsub", "tsro_fmul", "tsro_fdiv"):
            getattr(L, n).restype = _f32
            getattr(L, n).argtypes = [_f32, _f32]
        L.tsro_frecip.restype = _f32
        L.tsro_frecip.argtypes = [_f32]
        L.tsro_expk.restype = _f32
        L.tsro_expk.argtypes = [_f32, ct.c_uint]
        L.tsro_tanh.restype = _f32
        L.tsro_tanh.argtypes = [_f32]
        L.tsro_f32_to_fp16.restype = ct.c_uint16
        L.tsro_f32_to_fp16.argtypes = [_f32]
        L.tsro_qact_a32.argtypes = [_p, _u32, _p, _p]
        L.tsro_qact_a256.argtypes = [_p, _u32, _p, _p, _p]
        L.tsro_dot_q8_0.restype = _f32
        L.tsro_dot_q8_0.argtypes = [_p, _u32, _p, _p, _p]
        L.tsro_dot_q4_K.restype = _f32
        L.tsro_dot_q4_K.argtypes = [_p, _u32, _p, _p, _p, _p]
        L.tsro_matvec.restype = ct.c_int
        L.tsro_matvec.argtypes = [_u32, _p, _u32, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p, ct.c_int]
        L.tsro_fa.restype = ct.c_int
        L.tsro_fa.argtypes = [ct.POINTER(FaParams), _p, _p, _p, _p, _sz, _p]
        L.tsro_fa_qk_isums.argtypes = [ct.POINTER(FaParams), _p, _p, _p]
        L.tsro_quantize_q8_0.argtypes = [_p, _u32, _p]
        L.tsro_quantize_q4_K.argtypes = [_p, _u32, _p]
        L.tsro_rms_norm.argtypes = [_p, _p, _p, _u32, _u32, _f32, _f32]
        L.tsro_sincos.argtypes = [_f32, _p, _p]
        L.tsro_rope.argtypes = [_p, _p, _p, _u32, _u32, _u32, _u32, _u32, _f32, _f32]
        L.tsro_vop.argtypes = [_u32, _p, _p, _p, _sz]
        L.tsro_dequant_row.argtypes = [_u32, _p, _u32, _p]

    # -- scalar rules, vectorised by a Python loop (small inputs only) --
    def fp(self, op: str, a, b=None):
        a = np.asarray(a, np.float32).ravel()
        f = getattr(self.lib, "tsro_" + op)
        if op == "frecip":
            return np.array([f(float(x)) for x in a], np.float32)
        b = np.asarray(b, np.float32).ravel()
        return np.array([f(float(x), float(y)) for x, y in zip(a, b)], np.float32)

    def expk(self, v, kappa=0):
        v = np.asarray(v, np.float32).ravel()
        return np.array([self.lib.tsro_expk(float(x), kappa) for x in v], np.float32)

    def tanh(self, v):
        v = np.asarray(v, np.float32).ravel()
        return np.array([self.lib.tsro_tanh(float(x)) for x in v], np.float32)

    def qact(self, fmt: int, x):
        """x [T, K] f32 -> (q [T, K] int8, d [T, K/bs] f32, bs [T, K/16] int16 or None)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T, K = x.shape
        q = np.zeros((T, K), np.int8)
        if fmt == FMT_Q8_0:
            d = np.zeros((T, K // 32), np.float32)
            for t in range(T):
                self.lib.tsro_qact_a32(_ptr(x[t]), K, _ptr(q[t]), _ptr(d[t]))
            return q, d, None
        d = np.zeros((T, K // 256), np.float32)
        bs = np.zeros((T, K // 16), np.int16)
        for t in range(T):
            self.lib.tsro_qact_a256(_ptr(x[t]), K, _ptr(q[t]), _ptr(d[t]), _ptr(bs[t]))
        return q, d, bs

    def block_isums(self, fmt: int, w, K: int, q, d, bs=None):
        """Exact int32 block sums of every row against one QA vector: Q8_0 [N, K/32];
        Q4_K [N, K/256, 2] ({sum sc*S, sum m*BS})."""
        w = np.ascontiguousarray(w, np.uint8)
        N = w.shape[0]
        q = np.ascontiguousarray(q, np.int8)
        d = np.ascontiguousarray(d, np.float32)
        if fmt == FMT_Q8_0:
            out = np.zeros((N, K // 32), np.int32)
            for n in range(N):
                self.lib.tsro_dot_q8_0(_ptr(w[n]), K, _ptr(q), _ptr(d), _ptr(out[n]))
            return out
        bs = np.ascontiguousarray(bs, np.int16)
        out = np.zeros((N, K // 256, 2), np.int32)
        for n in range(N):
            self.lib.tsro_dot_q4_K(_ptr(w[n]), K, _ptr(q), _ptr(d), _ptr(bs), _ptr(out[n]))
        return out

    def matvec(self, fmt: int, w, K: int, x, add=None, add_stride=None, flags: int = 0, s0: float = 1.0,
               s1: float = 1.0, threads: int | None = None):
        """w: [N, row_bytes] ggml blocks; x: [T, K] f32 -> y [T, N] f32."""
        w = np.ascontiguousarray(w, np.uint8)
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        N, T = w.shape[0], x.shape[0]
        y = np.zeros((T, N), np.float32)
        if add is not None:
            add = np.ascontiguousarray(add, np.float32)
            flags |= MM_ADD
            if add_stride is None:
                add_stride = N if add.ndim == 2 and add.shape[0] > 1 else 0
        rc = self.lib.tsro_matvec(fmt, _ptr(w), N, K, _ptr(x), T, _ptr(add), add_stride or 0, flags, s0, s1,
                                  _ptr(y), threads or os.cpu_count() or 1)
        if rc != 0:
            raise ValueError("tsro_matvec refused the arguments")
        return y

    def fa(self, q, k_rows, v_rows, *, D, n_head, n_head_kv, n_kv, scale, mask=None, C=4, t_max=4, pcap=9344,
           new=(0, 0)):
        """q [T, n_head, D] f32; k_rows / v_rows [kv_size, E/32*34] uint8; mask f16 [T, >= n_kv] or None."""
        q = np.ascontiguousarray(q, np.float32)
        T = q.shape[0]
        p = FaParams(C, t_max, pcap, T, D, n_head, n_head_kv, n_kv, scale, new[0], new[1])
        out = np.zeros((T, n_head, D), np.float32)
        mk = None if mask is None else np.ascontiguousarray(mask, np.float16).view(np.uint16)
        rc = self.lib.tsro_fa(ct.byref(p), _ptr(q), _ptr(np.ascontiguousarray(k_rows)),
                              _ptr(np.ascontiguousarray(v_rows)), _ptr(mk), 0 if mk is None else mk.shape[1],
                              _ptr(out))
        return rc, out

    def fa_qk_isums(self, q, k_rows, *, D, n_head, n_head_kv, n_kv):
        q = np.ascontiguousarray(q, np.float32)
        p = FaParams(4, 4, 9344, 1, D, n_head, n_head_kv, n_kv, 1.0, 0, 0)
        out = np.zeros((n_head, n_kv, D // 32), np.int32)
        self.lib.tsro_fa_qk_isums(ct.byref(p), _ptr(q), _ptr(np.ascontiguousarray(k_rows)), _ptr(out))
        return out

    def quantize(self, fmt: int, x):
        """f32 rows [N, K] -> ggml blocks [N, row_bytes] uint8."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        N, K = x.shape
        rb = K // 32 * 34 if fmt == FMT_Q8_0 else K // 256 * 144
        out = np.zeros((N, rb), np.uint8)
        f = self.lib.tsro_quantize_q8_0 if fmt == FMT_Q8_0 else self.lib.tsro_quantize_q4_K
        for n in range(N):
            f(_ptr(x[n]), K, _ptr(out[n]))
        return out


    # -- decoder-layer vector kinds (tsro_vu.c) --
    def rms_norm(self, x, w=None, eps=1e-5, inv_n=None):
        """RMS_NORM + MUL of rows of x [rows, n] (w [n] or None); inv_n defaults to f32(1/n)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        rows, n = x.shape
        inv_n = np.float32(1.0) / np.float32(n) if inv_n is None else inv_n
        y = np.empty_like(x)
        w = None if w is None else np.ascontiguousarray(w, np.float32)
        self.lib.tsro_rms_norm(_ptr(x), _ptr(y), _ptr(w), n, rows, float(np.float32(eps)), float(np.float32(inv_n)))
        return y

    def sincos(self, t):
        t = np.ascontiguousarray(t, np.float32).ravel()
        s, c = np.empty_like(t), np.empty_like(t)
        sv, cv = ct.c_float(), ct.c_float()
        for i, v in enumerate(t):
            self.lib.tsro_sincos(float(v), ct.byref(sv), ct.byref(cv))
            s[i], c[i] = sv.value, cv.value
        return s, c

    def rope(self, x, pos, *, n_heads, head_dim, n_dims, mode, ts, attn_factor=1.0):
        """x [T, n_heads * head_dim] f32, pos [T] int32 -> rotated copy."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        pos = np.ascontiguousarray(pos, np.int32)
        y = np.empty_like(x)
        self.lib.tsro_rope(_ptr(x), _ptr(y), _ptr(pos), x.shape[0], n_heads, head_dim, n_dims, mode, float(np.float32(ts)),
                           float(np.float32(attn_factor)))
        return y

    def vop(self, func: int, a, b=None):
        a = np.ascontiguousarray(a, np.float32)
        b = a if b is None else np.ascontiguousarray(b, np.float32)
        y = np.empty_like(a)
        self.lib.tsro_vop(func, _ptr(a), _ptr(b), _ptr(y), a.size)
        return y

    def dequant(self, fmt: int, w, K: int):
        """ggml rows [N, row bytes] -> f32 [N, K]."""
        w = np.ascontiguousarray(np.atleast_2d(w), np.uint8)
        y = np.empty((w.shape[0], K), np.float32)
        for r in range(w.shape[0]):
            self.lib.tsro_dequant_row(fmt, _ptr(w[r]), K, _ptr(y[r]))
        return y


class RopeCfg(ct.Structure):
    """tsr_ref_rope_cfg (sw/sim/include/tsr_ref_vu.h:111-123)."""
    _fields_ = [(n, _u32) for n in ("mode", "ff", "fs", "atab", "m", "ts", "freq_scale", "head_dim", "n_dims", "n_heads", "T")]


def _bits(v) -> int:
    return int(np.float32(v).view(np.uint32))


class Ref:
    """The reference's own library (oracle/_ref/libtsr_refdrv.so), when it was built."""

    @staticmethod
    def available(path: str = REF_PATH) -> bool:
        return os.path.exists(path)

    def __init__(self, path: str = REF_PATH):
        L = self.lib = ct.CDLL(path)
        L.refdrv_expk_n.argtypes = [_p, _sz, ct.c_uint, _p]
        L.refdrv_tanh_n.argtypes = [_p, _sz, _p]
        L.refdrv_fp_n.argtypes = [ct.c_int, _p, _p, _sz, _p]
        L.refdrv_f32_to_fp16_n.argtypes = [_p, _sz, _p]
        L.refdrv_qact.argtypes = [_u32, _p, _u32, _p, _p, _p]
        L.refdrv_row_bytes.restype = _sz
        L.refdrv_row_bytes.argtypes = [_u32, _u32]
        L.refdrv_repack.argtypes = [_u32, _p, _u32, _u32, _p]
        L.refdrv_matvec_repacked.restype = ct.c_int
        L.refdrv_matvec_repacked.argtypes = [_u32, _p, _u32, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p, ct.c_int]
        L.refdrv_fa_prepare.restype = _p
        L.refdrv_fa_prepare.argtypes = [_u32] * 9 + [_f32, _p, _p, _p, _sz, _u32, _u32]
        L.refdrv_fa_run.restype = ct.c_int
        L.refdrv_fa_run.argtypes = [_p, _p, _p]
        L.refdrv_fa_free.argtypes = [_p]
        L.tsr_ref_red_row.restype = _u32
        L.tsr_ref_red_row.argtypes = [_u32, _u32, _p, _u32, _u32, _u32]
        L.tsr_ref_vop.argtypes = [_u32, _u32, _u32, _u32, _p, _u32, _p, _u32, _p, _u32, _p]
        L.tsr_m_sincos.argtypes = [_f32, _p, _p]
        L.tsr_ref_rope.argtypes = [ct.POINTER(RopeCfg), _p, _u32, _p, _u32, _p, _p]
        L.tsr_dequant_row.argtypes = [_u32, _p, _u32, _p]

    def expk(self, v, kappa=0):
        v = np.ascontiguousarray(v, np.float32).ravel()
        out = np.empty_like(v)
        self.lib.refdrv_expk_n(_ptr(v), v.size, kappa, _ptr(out))
        return out

    def tanh(self, v):
        v = np.ascontiguousarray(v, np.float32).ravel()
        out = np.empty_like(v)
        self.lib.refdrv_tanh_n(_ptr(v), v.size, _ptr(out))
        return out

    def fp(self, op: str, a, b=None):
        ops = {"fadd": 0, "fsub": 1, "fmul": 2, "fdiv": 3, "frecip": 4}
        a = np.ascontiguousarray(a, np.float32).ravel()
        b = a if b is None else np.ascontiguousarray(b, np.float32).ravel()
        out = np.empty_like(a)
        self.lib.refdrv_fp_n(ops[op], _ptr(a), _ptr(b), a.size, _ptr(out))
        return out

    def f32_to_fp16(self, a):
        a = np.ascontiguousarray(a, np.float32).ravel()
        out = np.empty(a.size, np.uint16)
        self.lib.refdrv_f32_to_fp16_n(_ptr(a), a.size, _ptr(out))
        return out

    def qact(self, fmt: int, x):
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T, K = x.shape
        bsz = 32 if fmt == FMT_Q8_0 else 256
        q = np.zeros((T, K), np.int8)
        d = np.zeros((T, K // bsz), np.float32)
        bs = np.zeros((T, K // 16), np.int16) if fmt == FMT_Q4_K else None
        for t in range(T):
            self.lib.refdrv_qact(fmt, _ptr(x[t]), K, _ptr(q[t]), _ptr(d[t]), _ptr(bs[t]) if bs is not None else None)
        return q, d, bs

    def repack(self, fmt: int, w, K: int):
        w = np.ascontiguousarray(w, np.uint8)
        rb = self.lib.refdrv_row_bytes(fmt, K)
        out = np.zeros((w.shape[0], rb), np.uint8)
        self.lib.refdrv_repack(fmt, _ptr(w), w.shape[0], K, _ptr(out))
        return out

    def matvec_repacked(self, fmt: int, rows, K: int, x, add=None, add_stride=None, flags: int = 0, s0=1.0, s1=1.0,
                        threads: int | None = None, out=None):
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        N, T = rows.shape[0], x.shape[0]
        y = out if out is not None else np.zeros((T, N), np.float32)
        if add is not None:
            add = np.ascontiguousarray(add, np.float32)
            flags |= MM_ADD
            if add_stride is None:
                add_stride = N if add.ndim == 2 and add.shape[0] > 1 else 0
        rc = self.lib.refdrv_matvec_repacked(fmt, _ptr(rows), N, K, _ptr(x), T, _ptr(add), add_stride or 0, flags,
                                             s0, s1, _ptr(y), threads or os.cpu_count() or 1)
        if rc != 0:
            raise RuntimeError("refdrv_matvec_repacked failed")
        return y

    def matvec(self, fmt: int, w, K: int, x, **kw):
        return self.matvec_repacked(fmt, self.repack(fmt, w, K), K, x, **kw)

    def fa_prepare(self, k_rows, v_rows, *, T, D, n_head, n_head_kv, n_kv, scale, mask=None, C=4, t_max=4,
                   pcap=9344, new=(0, 0)):
        k_rows = np.ascontiguousarray(k_rows, np.uint8)
        v_rows = np.ascontiguousarray(v_rows, np.uint8)
        mk = None if mask is None else np.ascontiguousarray(mask, np.float16).view(np.uint16)
        h = self.lib.refdrv_fa_prepare(C, t_max, pcap, T, D, n_head, n_head_kv, n_kv, k_rows.shape[0], scale,
                                       _ptr(k_rows), _ptr(v_rows), _ptr(mk), 0 if mk is None else mk.shape[1],
                                       new[0], new[1])
        return h

    def fa_run(self, h, q):
        q = np.ascontiguousarray(q, np.float32)
        out = np.zeros_like(q)
        rc = self.lib.refdrv_fa_run(h, _ptr(q), _ptr(out))
        return rc, out

    def fa_free(self, h):
        self.lib.refdrv_fa_free(h)

    def fa(self, q, k_rows, v_rows, **kw):
        q = np.ascontiguousarray(q, np.float32)
        h = self.fa_prepare(k_rows, v_rows, T=q.shape[0], **kw)
        try:
            return self.fa_run(h, q)
        finally:
            self.fa_free(h)

    # -- the reference's vector unit (tsr_ref_vu.c, tsr_ref_math.c, tsr_ref.c) --
    def rms_norm(self, x, w=None, eps=1e-5, inv_n=None):
        """RED.SUMSQ post RMS per row, then VOP.MULCB (MULC without w), as rmsnorm_ref_rows does."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        rows, n = x.shape
        inv_n = np.float32(1.0) / np.float32(n) if inv_n is None else inv_n
        L = -(-n // 16) * 16
        y = np.zeros((rows, n), np.float32)
        wp = None if w is None else np.ascontiguousarray(np.pad(np.asarray(w, np.float32), (0, L - n)), np.float32)
        for r in range(rows):
            xr = np.ascontiguousarray(np.pad(x[r], (0, L - n)), np.float32)
            s = self.lib.tsr_ref_red_row(1, 2, _ptr(xr), n, _bits(inv_n), _bits(eps))
            c = np.array([s], np.uint32)
            out = np.zeros(L, np.float32)
            if wp is None:
                self.lib.tsr_ref_vop(4, 1, 1, n, _ptr(out), 0, _ptr(xr), 0, None, 0, _ptr(c))
            else:
                self.lib.tsr_ref_vop(12, 1, 1, n, _ptr(out), 0, _ptr(xr), 0, _ptr(wp), 0, _ptr(c))
            y[r] = out[:n]
        return y

    def sincos(self, t):
        t = np.ascontiguousarray(t, np.float32).ravel()
        s, c = np.empty_like(t), np.empty_like(t)
        sv, cv = ct.c_float(), ct.c_float()
        for i, v in enumerate(t):
            self.lib.tsr_m_sincos(float(v), ct.byref(sv), ct.byref(cv))
            s[i], c[i] = sv.value, cv.value
        return s, c

    def rope(self, x, pos, *, n_heads, head_dim, n_dims, mode, ts, attn_factor=1.0):
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = x.shape[0]
        cfg = RopeCfg(mode, 0, 0, 0, _bits(attn_factor), _bits(ts), 0, head_dim, n_dims, n_heads, T)
        y = np.zeros_like(x)
        pos = np.ascontiguousarray(np.asarray(pos, np.int32).view(np.uint32))
        self.lib.tsr_ref_rope(ct.byref(cfg), _ptr(y), 0, _ptr(x), 0, _ptr(pos), None)
        return y

    def vop(self, func: int, a, b=None):
        a = np.ascontiguousarray(a, np.float32).ravel()
        n = a.size
        L = -(-n // 16) * 16
        ap = np.ascontiguousarray(np.pad(a, (0, L - n)), np.float32)
        bp = None if b is None else np.ascontiguousarray(np.pad(np.asarray(b, np.float32).ravel(), (0, L - n)), np.float32)
        out = np.zeros(L, np.float32)
        self.lib.tsr_ref_vop(func, 0, 1, n, _ptr(out), 0, _ptr(ap), 0, _ptr(bp), 0, None)
        return out[:n]

    def dequant(self, fmt: int, w, K: int):
        w = np.ascontiguousarray(np.atleast_2d(w), np.uint8)
        rows = self.repack(fmt, w, K)
        y = np.empty((w.shape[0], K), np.float32)
        for r in range(w.shape[0]):
            self.lib.tsr_dequant_row(fmt, _ptr(rows[r]), K, _ptr(y[r]))
        return y


class OracleModel:
    """CPU composition of the decoder graph (llama / qwen2 layers) over the oracle's kinds, in the
    order tsrc_model_forward runs them: GET_ROWS, RMS_NORM + MUL, MUL_MAT of the stacked q | k | v rows
    (+ bias), ROPE, KVST into ggml q8_0 cache rows, FA, MUL_MAT + residual, RMS_NORM + MUL, the stacked
    gate | up rows, SWIGLU, down + residual, output norm and head of the last token. A layer dict holds
    wqkv, wo, wgu, wd (ggml rows), attn_norm, ffn_norm and optionally bqkv. Test and baseline
    infrastructure only."""

    def __init__(self, tsro: "Tsro", cfg: dict, layers: list, emb, head, out_norm, ts: float, kq_scale: float,
                 threads: int | None = None):
        self.o, self.c, self.layers = tsro, cfg, layers
        self.emb, self.head, self.out_norm = emb, head, out_norm
        self.ts, self.kq_scale, self.threads = ts, kq_scale, threads
        E = cfg["n_head_kv"] * cfg["head_dim"]
        self.kc = [np.zeros((cfg["n_ctx"], E // 32 * 34), np.uint8) for _ in layers]
        self.vc = [np.zeros((cfg["n_ctx"], E // 32 * 34), np.uint8) for _ in layers]

    def embed(self, ids):
        """GET_ROWS of the token embedding: [T, n_embd] f32."""
        ids = np.asarray(ids, np.int64)
        return self.o.dequant(self.c["fmt"], self.emb[ids], self.c["n_embd"])

    def layer(self, li: int, x, pos0: int):
        """Decoder layer li over the T rows of x at positions pos0 .. pos0 + T - 1 (causal); writes
        the layer's cache cells and returns the layer's output rows."""
        o, c = self.o, self.c
        T = x.shape[0]
        E, D, nh, nkv, F, fmt = c["n_embd"], c["head_dim"], c["n_head"], c["n_head_kv"], c["n_ff"], c["fmt"]
        Hq, Hkv, n_kv = nh * D, nkv * D, pos0 + T
        inv_n = np.float32(1.0) / np.float32(E)
        pos = np.arange(pos0, pos0 + T, dtype=np.int32)
        mask = None
        if T > 1:
            mask = np.full((T, n_kv), -np.inf, np.float16)
            for t in range(T):
                mask[t, :pos0 + t + 1] = 0
        th = self.threads
        rope = dict(head_dim=D, n_dims=D, mode=c["rope_mode"], ts=self.ts)
        L = self.layers[li]
        h = o.rms_norm(x, L["attn_norm"], c["rms_eps"], inv_n)
        b = L.get("bqkv")
        qkv = o.matvec(fmt, L["wqkv"], E, h, add=None if b is None else b[None, :], add_stride=0, threads=th)
        q = o.rope(np.ascontiguousarray(qkv[:, :Hq]), pos, n_heads=nh, **rope)
        k = o.rope(np.ascontiguousarray(qkv[:, Hq:Hq + Hkv]), pos, n_heads=nkv, **rope)
        v = np.ascontiguousarray(qkv[:, Hq + Hkv:])
        self.kc[li][pos0:n_kv] = o.quantize(FMT_Q8_0, k)
        self.vc[li][pos0:n_kv] = o.quantize(FMT_Q8_0, v)
        rc, att = o.fa(q.reshape(T, nh, D), self.kc[li], self.vc[li], D=D, n_head=nh, n_head_kv=nkv, n_kv=n_kv,
                       scale=self.kq_scale, mask=mask, new=(pos0, n_kv))
        if rc != 0:
            raise RuntimeError(f"FA returned {rc}")
        x = o.matvec(fmt, L["wo"], Hq, att.reshape(T, Hq), add=x, add_stride=E, threads=th)
        h = o.rms_norm(x, L["ffn_norm"], c["rms_eps"], inv_n)
        gu = o.matvec(fmt, L["wgu"], E, h, threads=th)
        s = o.vop(7, np.ascontiguousarray(gu[:, :F]), np.ascontiguousarray(gu[:, F:]))
        return o.matvec(fmt, L["wd"], F, s, add=x, add_stride=E, threads=th)

    def logits(self, x):
        """Output RMS_NORM + MUL and the head of the last row of x."""
        c = self.c
        h = self.o.rms_norm(x[-1:], self.out_norm, c["rms_eps"], np.float32(1.0) / np.float32(c["n_embd"]))
        return self.o.matvec(c["fmt"], self.head, c["n_embd"], h, threads=self.threads)[0]

    def forward(self, ids, pos0: int):
        x = self.embed(ids)
        for li in range(len(self.layers)):
            x = self.layer(li, x, pos0)
        return self.logits(x)


class RefOps:
    """The reference library's kinds in the shape OracleModel calls them: MUL_MAT, FA, RMS_NORM,
    ROPE, VOP and GET_ROWS run the reference's own functions (weights are repacked to its row
    layout once, as its weight upload does); the KV rows are quantized by the restatement's Q8_0
    quantizer, which the tests pin to the reference's QACT A32 bit for bit. Baseline timing only."""

    def __init__(self, ref: "Ref", tsro: "Tsro"):
        self.ref, self.tsro = ref, tsro
        self._rows = {}

    def matvec(self, fmt: int, w, K: int, x, **kw):
        key = (id(w), fmt, K)
        if key not in self._rows:
            self._rows[key] = (w, self.ref.repack(fmt, w, K))
        return self.ref.matvec_repacked(fmt, self._rows[key][1], K, x, **kw)

    def quantize(self, fmt: int, x):
        return self.tsro.quantize(fmt, x)

    def __getattr__(self, name):
        return getattr(self.ref, name)
