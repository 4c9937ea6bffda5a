"""Host-side binding of libtsrc.so (include/tsrc.h), the B200 hot path of the Tesseract stack.

The classes mirror the ggml-tesseract backend's view of the path (jwkim04/tesseract-npu
sw/ggml-tesseract/ggml-tesseract.cpp): a ``Device`` opened once per process and GPU
(tsr_dev_open_locked, :463), ``Weight`` tensors uploaded into device memory in the device's own
layout (the WEIGHTS buffer's set_tensor / get_tensor, :1905 / :1947), ``mul_mat`` with the MUL_MAT
semantics (tsr_lower_mul_mat, :2790-2928, with the ADD / SCALE / softcap epilogues), and
``mul_mat_unsupported`` for the supports_op refusals (:4199-4299).

Device buffers are passed as torch CUDA tensors (or raw addresses); torch is only the allocator
and stream provider here. There is no CPU path: if the library cannot be loaded, or no sm_100
device is present, every call raises ``TsrcError``.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libtsrc.so")
INCLUDE = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include", "tsrc.h")

FMT_Q8_0, FMT_Q4_K = 0, 1
QA_A32, QA_A256 = 0, 1
MM_ADD, MM_SCALE, MM_SOFTCAP = 0x1, 0x2, 0x4
ROPE_NORM, ROPE_NEOX = 0, 1
VOP_ADD, VOP_MUL, VOP_SILU, VOP_SWIGLU = 0, 2, 6, 7
E_ARG, E_SHAPE, E_CUDA, E_NOMEM, E_NODEV, E_DEVICE = -1, -2, -3, -4, -5, -6

BLOCK = {FMT_Q8_0: 32, FMT_Q4_K: 256}
BLOCK_BYTES = {FMT_Q8_0: 34, FMT_Q4_K: 144}


class TsrcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tsrc error {code}: {msg}")
        self.code = code


_p, _u32, _u64, _f32, _i = ct.c_void_p, ct.c_uint32, ct.c_uint64, ct.c_float, ct.c_int
_lib = None

# argtypes of every exported function (kept in the order of include/tsrc.h)
_SIGS = {
    "tsrc_last_error": (ct.c_char_p, []),
    "tsrc_version": (ct.c_char_p, []),
    "tsrc_open": (_i, [_i, ct.POINTER(_p)]),
    "tsrc_close": (_i, [_p]),
    "tsrc_sync": (_i, [_p, _p]),
    "tsrc_weight_upload": (_i, [_p, _u32, _p, _u32, _u32, _u32, _u32, ct.POINTER(_p)]),
    "tsrc_weight_upload_device": (_i, [_p, _u32, _p, _u32, _u32, _u32, _u32, _p, ct.POINTER(_p)]),
    "tsrc_weight_synth": (_i, [_p, _u32, _u32, _u32, _u32, _u32, _u64, _f32, _p, ct.POINTER(_p)]),
    "tsrc_ggml_type_info": (_i, [_u32, ct.POINTER(_u32), ct.POINTER(_u32), ct.POINTER(_u32)]),
    "tsrc_ggml_rows_to_dev": (_i, [_u32, _p, _u32, _u32, _p]),
    "tsrc_weight_upload_ggml": (_i, [_p, _u32, _p, _u32, _u32, _u32, _u32, ct.POINTER(_p)]),
    "tsrc_weight_download": (_i, [_p, _p]),
    "tsrc_weight_info": (_i, [_p] + [ct.POINTER(_u32)] * 5 + [ct.POINTER(_u64)]),
    "tsrc_weight_free": (_i, [_p]),
    "tsrc_mul_mat": (_i, [_p, _p, _p, _u32, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p]),
    "tsrc_rms_norm": (_i, [_p, _p, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p]),
    "tsrc_mul_mat_rms": (_i, [_p, _p, _p, _p, _f32, _f32, _p, _p, _u32, _f32, _f32, _p]),
    "tsrc_model_create": (_i, [_p, _p, _u64, ct.POINTER(_p)]),
    "tsrc_model_create_tp": (_i, [_p, _p, _u64, _p, ct.POINTER(_p)]),
    "tsrc_model_free": (_i, [_p]),
    "tsrc_model_kv": (_i, [_p, _u32, ct.POINTER(_p)]),
    "tsrc_model_forward": (_i, [_p, _p, _u32, _u32, _p, _p]),
    "tsrc_model_decode": (_i, [_p, _p, _u32, _p, _p]),
    "tsrc_model_weight": (_i, [_p, _u32, _u32, ct.POINTER(_p)]),
    "tsrc_model_set_weight": (_i, [_p, _u32, _u32, _u32, _p, _u32, _u32]),
    "tsrc_model_set_f32": (_i, [_p, _u32, _u32, _p, _u32]),
    "tsrc_model_params": (_i, [_p, ct.POINTER(_f32), ct.POINTER(_f32)]),
    "tsrc_model_f32_value": (_f32, [_u64, _u32, _u32, _u32]),
    "tsrc_rope": (_i, [_p, _p, _u32, _p, _u32, _p, _u32, _u32, _u32, _u32, _u32, _f32, _f32, _p]),
    "tsrc_vop": (_i, [_p, _u32, _p, _u32, _p, _u32, _p, _u32, _u32, _u32, _p]),
    "tsrc_get_rows": (_i, [_p, _p, _p, _u32, _p, _u32, _p]),
    "tsrc_dev_alloc": (_i, [_p, ct.c_size_t, ct.POINTER(_p)]),
    "tsrc_dev_free": (_i, [_p, _p]),
    "tsrc_copy": (_i, [_p, _p, _p, ct.c_size_t, _u32, _p]),
    "tsrc_mul_mat_id": (_i, [_p, _p, _u32, _p, _u32, _u32, _u32, _p, _u32, _u32, _u32, _p, _u32, _u32, _p]),
    "tsrc_mul_mat_noalloc": (_i, [_p, _p, _p, _u32, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p]),
    "tsrc_mvm": (_i, [_p, _p, _p, _p, _p, _u32, _p, _u32, _p, _u32, _u32, _f32, _f32, _p]),
    "tsrc_mul_mat_unsupported": (ct.c_char_p, [_u32, _u64, _u64, _u64]),
    "tsrc_qact": (_i, [_p, _u32, _p, _u32, _u32, _u32, _p, _p, _p, _p]),
    "tsrc_mul_mat_isums": (_i, [_p, _p, _p, _p, _p, _p]),
    "tsrc_team_connect_local": (_i, [_p, _p]),
    "tsrc_team_create": (_i, [_p, _u32, _u32, _u32, _p, ct.POINTER(_p)]),
    "tsrc_team_connect": (_i, [_p, _p]),
    "tsrc_team_free": (_i, [_p]),
    "tsrc_mul_mat_allgather": (_i, [_p, _p, _p, _p, _p, _p]),
    "tsrc_kv_create": (_i, [_p, _u32, _u32, _u32, ct.POINTER(_p)]),
    "tsrc_kv_free": (_i, [_p]),
    "tsrc_kv_set_rows": (_i, [_p, _p, _u32, _p, _u32, _u32, _p, _u32, _p]),
    "tsrc_kv_set_bytes": (_i, [_p, _u32, _p, _u32, _u32]),
    "tsrc_kv_get_bytes": (_i, [_p, _u32, _p, _u32, _u32]),
    "tsrc_flash_attn": (_i, [_p, _p, _p, _u32, _u32, _u32, _p, _u32, _f32, _u32, _u32, _p, _p, _p]),
}


class FaCfg(ct.Structure):
    """tsrc_fa_cfg: the attention configuration (channels C, T_MAX, PCAP, K_MAX) and the model's KV
    heads when a cache holds a shard of them (0: the cache's own)."""
    _fields_ = [("C", _u32), ("t_max", _u32), ("pcap", _u32), ("k_max", _u32), ("plan_n_head_kv", _u32)]


class ModelCfg(ct.Structure):
    """tsrc_model_cfg: the shape of a random-init decoder (llama / qwen2 graph)."""
    _fields_ = [(n, _u32) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab", "fmt",
                                   "rope_mode")] + [("rope_base", _f32), ("rms_eps", _f32)] + \
               [(n, _u32) for n in ("qkv_bias", "tied_head", "n_ctx")] + [("fa", FaCfg)]


MODEL_GLOBAL = 0xFFFFFFFF
KV_K, KV_V = 0, 1
TEAM_HANDLE_BYTES = 64
Q8_0_BLOCK_BYTES = 34


def declared_symbols() -> list[str]:
    """Function names include/tsrc.h declares (parsed from the header)."""
    import re
    with open(INCLUDE) as f:
        return re.findall(r"^TSRC_API [^(]*?\b(tsrc_\w+)\(", f.read(), flags=re.M)


def lib() -> ct.CDLL:
    """Loads libtsrc.so (building it first if it is missing and nvcc is present)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        import importlib.util
        spec = importlib.util.spec_from_file_location("tsrc_build", os.path.join(os.path.dirname(HERE), "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    L = ct.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != 0:
        raise TsrcError(rc, lib().tsrc_last_error().decode())


def _addr(t) -> int | None:
    """Device address of a torch tensor (or an int address, or None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream or None
        except Exception:
            return None
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


def ggml_row_bytes(fmt: int, K: int) -> int:
    return K // BLOCK[fmt] * BLOCK_BYTES[fmt]


# ggml_type values (ggml.h) of the tensor types the loader knows
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q8_0 = 0, 1, 2, 3, 6, 7, 8
GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 12, 13, 14, 30


def ggml_type_info(ggml_type: int) -> tuple[int, int, int]:
    """(block elements, block bytes, device format) of a loadable ggml type; TsrcError otherwise."""
    be, bb, fmt = _u32(), _u32(), _u32()
    _check(lib().tsrc_ggml_type_info(ggml_type, ct.byref(be), ct.byref(bb), ct.byref(fmt)))
    return be.value, bb.value, fmt.value


def ggml_rows_to_dev(ggml_type: int, rows, n_rows: int, K: int):
    """Host-only load-time conversion: rows of a ggml type -> numpy uint8 [n_rows, row bytes] of the
    device format's ggml blocks (Q8_0 unless the type is Q4_K)."""
    import numpy as np
    be, bb, fmt = ggml_type_info(ggml_type)
    a = np.ascontiguousarray(rows).view(np.uint8).reshape(-1)
    if a.size != n_rows * (K // be) * bb:
        raise TsrcError(E_ARG, f"ggml_rows_to_dev: {a.size} bytes for {n_rows} rows of K={K}")
    out = np.empty((n_rows, ggml_row_bytes(fmt, K)), np.uint8)
    _check(lib().tsrc_ggml_rows_to_dev(ggml_type, a.ctypes.data, n_rows, K, out.ctypes.data))
    return out


def mul_mat_unsupported(fmt: int, N: int, K: int, T: int = 1) -> str | None:
    r = lib().tsrc_mul_mat_unsupported(fmt, N, K, T)
    return None if r is None else r.decode()


class Device:
    """One opened GPU (the backend device "Tesseract0" of the reference, now a B200)."""

    def __init__(self, index: int = 0):
        h = _p()
        _check(lib().tsrc_open(index, ct.byref(h)))
        self.handle = h
        self.index = index

    def close(self) -> None:
        if self.handle:
            _check(lib().tsrc_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def sync(self, stream=None) -> None:
        """Waits for queued work and raises if a kernel reported an error."""
        _check(lib().tsrc_sync(self.handle, _stream(stream)))

    # ---- weights ----
    def upload(self, fmt: int, ggml_rows, N: int, K: int, row0: int = 0, n_rows: int | None = None) -> "Weight":
        """ggml rows (numpy uint8 [n_rows, row_bytes], host) -> a device weight shard."""
        import numpy as np
        n_rows = N - row0 if n_rows is None else n_rows
        a = np.ascontiguousarray(ggml_rows, dtype=np.uint8)
        if a.size != n_rows * ggml_row_bytes(fmt, K):
            raise TsrcError(E_ARG, f"upload: {a.size} bytes for {n_rows} rows of K={K}")
        h = _p()
        _check(lib().tsrc_weight_upload(self.handle, fmt, a.ctypes.data, N, K, row0, n_rows, ct.byref(h)))
        return Weight(self, h)

    def upload_ggml(self, ggml_type: int, rows, N: int, K: int, row0: int = 0, n_rows: int | None = None) -> "Weight":
        """Rows of any loadable ggml type (host) -> a device weight shard (non-native types are
        converted to Q8_0 on the host first)."""
        import numpy as np
        n_rows = N - row0 if n_rows is None else n_rows
        be, bb, _ = ggml_type_info(ggml_type)
        a = np.ascontiguousarray(rows).view(np.uint8).reshape(-1)
        if a.size != n_rows * (K // be) * bb:
            raise TsrcError(E_ARG, f"upload_ggml: {a.size} bytes for {n_rows} rows of K={K}")
        h = _p()
        _check(lib().tsrc_weight_upload_ggml(self.handle, ggml_type, a.ctypes.data, N, K, row0, n_rows, ct.byref(h)))
        return Weight(self, h)

    def upload_device(self, fmt: int, rows_dev, N: int, K: int, row0: int = 0, n_rows: int | None = None,
                      stream=None) -> "Weight":
        n_rows = N - row0 if n_rows is None else n_rows
        h = _p()
        _check(lib().tsrc_weight_upload_device(self.handle, fmt, _addr(rows_dev), N, K, row0, n_rows,
                                               _stream(stream), ct.byref(h)))
        return Weight(self, h)

    def synth(self, fmt: int, N: int, K: int, seed: int, sigma: float = 0.02, row0: int = 0,
              n_rows: int | None = None, stream=None) -> "Weight":
        n_rows = N - row0 if n_rows is None else n_rows
        h = _p()
        _check(lib().tsrc_weight_synth(self.handle, fmt, N, K, row0, n_rows, seed, sigma, _stream(stream),
                                       ct.byref(h)))
        return Weight(self, h)

    # ---- MUL_MAT ----
    # ---- the decoder layer's vector kinds ----
    def rms_norm(self, x, y, n: int, rows: int, w=None, eps: float = 1e-5, inv_n: float | None = None,
                 x_stride: int = 0, y_stride: int = 0, stream=None) -> None:
        inv_n = float(np.float32(1.0) / np.float32(n)) if inv_n is None else inv_n
        _check(lib().tsrc_rms_norm(self.handle, _addr(x), x_stride, _addr(y), y_stride, _addr(w), n, rows, eps, inv_n,
                                   _stream(stream)))

    def mul_mat_rms(self, w: "Weight", x, y, norm_w=None, eps: float = 1e-5, inv_n: float | None = None, add=None,
                    flags: int = 0, s0: float = 1.0, s1: float = 1.0, stream=None) -> None:
        """y = MUL_MAT(w, RMS_NORM(x) * norm_w) for one token in one launch (bit for bit rms_norm then
        mul_mat)."""
        inv_n = float(np.float32(1.0) / np.float32(w.K)) if inv_n is None else inv_n
        if add is not None:
            flags |= MM_ADD
        _check(lib().tsrc_mul_mat_rms(self.handle, w.handle, _addr(x), _addr(norm_w), eps, inv_n, _addr(y), _addr(add),
                                      flags, s0, s1, _stream(stream)))

    def rope(self, x, y, pos, T: int, n_heads: int, head_dim: int, n_dims: int, mode: int, ts: float,
             attn_factor: float = 1.0, x_stride: int = 0, y_stride: int = 0, stream=None) -> None:
        _check(lib().tsrc_rope(self.handle, _addr(x), x_stride, _addr(y), y_stride, _addr(pos), T, n_heads, head_dim,
                               n_dims, mode, ts, attn_factor, _stream(stream)))

    def vop(self, func: int, a, b, y, n: int, rows: int = 1, a_stride: int = 0, b_stride: int = 0, y_stride: int = 0,
            stream=None) -> None:
        _check(lib().tsrc_vop(self.handle, func, _addr(a), a_stride, _addr(b), b_stride, _addr(y), y_stride, n, rows,
                              _stream(stream)))

    def get_rows(self, w: "Weight", ids, T: int, y, y_stride: int = 0, stream=None) -> None:
        _check(lib().tsrc_get_rows(self.handle, w.handle, _addr(ids), T, _addr(y), y_stride, _stream(stream)))

    def mul_mat(self, w: "Weight", x, y, T: int | None = None, add=None, add_stride: int | None = None,
                flags: int = 0, s0: float = 1.0, s1: float = 1.0, x_stride: int = 0, y_stride: int = 0,
                stream=None) -> None:
        """y[t, n] = epilogue(W row n . QACT(x[t])) (torch CUDA tensors or addresses)."""
        if T is None:
            T = 1 if len(x.shape) == 1 else x.shape[0]
        if add is not None:
            flags |= MM_ADD
            if add_stride is None:
                add_stride = 0 if (len(add.shape) == 1 or add.shape[0] == 1) else w.n_rows
        _check(lib().tsrc_mul_mat(self.handle, w.handle, _addr(x), T, x_stride, _addr(y), y_stride, _addr(add),
                                  add_stride or 0, flags, s0, s1, _stream(stream)))

    def mul_mat_id(self, w: "Weight", n_exp: int, x, ids, y, n_used: int, T: int, x_slots: int = 1, x_slot_stride: int = 0,
                   x_tok_stride: int = 0, ids_stride: int = 0, y_slot_stride: int = 0, y_tok_stride: int = 0,
                   stream=None) -> None:
        """MUL_MAT_ID: y[t][j] = MUL_MAT of expert ids[t][j] (rows of the stacked weight) with x[t][j mod x_slots]."""
        _check(lib().tsrc_mul_mat_id(self.handle, w.handle, n_exp, _addr(x), x_slots, x_slot_stride, x_tok_stride, _addr(ids),
                                     ids_stride, n_used, T, _addr(y), y_slot_stride, y_tok_stride, _stream(stream)))

    def mul_mat_noalloc(self, w: "Weight", x, y, T: int | None = None, add=None, add_stride: int | None = None,
                        flags: int = 0, s0: float = 1.0, s1: float = 1.0, x_stride: int = 0, y_stride: int = 0,
                        stream=None) -> None:
        """mul_mat without any device allocation by the library (its scratch is a fixed array in the
        library's device image); for hosts that plan all device memory themselves."""
        if T is None:
            T = 1 if len(x.shape) == 1 else x.shape[0]
        if add is not None:
            flags |= MM_ADD
            if add_stride is None:
                add_stride = 0 if (len(add.shape) == 1 or add.shape[0] == 1) else w.n_rows
        _check(lib().tsrc_mul_mat_noalloc(self.handle, w.handle, _addr(x), T, x_stride, _addr(y), y_stride, _addr(add),
                                          add_stride or 0, flags, s0, s1, _stream(stream)))

    def mvm(self, w: "Weight", q, d, bs, y, T: int = 1, add=None, add_stride: int = 0, flags: int = 0,
            s0: float = 1.0, s1: float = 1.0, y_stride: int = 0, stream=None) -> None:
        """The MVM op alone on a QA image from qact()."""
        if add is not None:
            flags |= MM_ADD
        _check(lib().tsrc_mvm(self.handle, w.handle, _addr(q), _addr(d), _addr(bs), T, _addr(y), y_stride, _addr(add),
                              add_stride, flags, s0, s1, _stream(stream)))

    def mul_mat_isums(self, w: "Weight", x, y, isum, stream=None) -> None:
        _check(lib().tsrc_mul_mat_isums(self.handle, w.handle, _addr(x), _addr(y), _addr(isum), _stream(stream)))

    def qact(self, kind: int, x, K: int, T: int, q, d, bs=None, x_stride: int = 0, stream=None) -> None:
        _check(lib().tsrc_qact(self.handle, kind, _addr(x), K, T, x_stride, _addr(q), _addr(d), _addr(bs),
                               _stream(stream)))

    # ---- tensor parallelism: MUL_MAT with the all-gather fused in ----
    def team_create(self, rank: int, world: int, n_max: int) -> "Team":
        """This rank's side of a team of `world` GPUs; exchange `team.handle` (bytes) with the other
        ranks and call team.connect(all handles in rank order)."""
        h = _p()
        buf = ct.create_string_buffer(TEAM_HANDLE_BYTES)
        _check(lib().tsrc_team_create(self.handle, rank, world, n_max, buf, ct.byref(h)))
        return Team(self, h, rank, world, bytes(buf.raw))

    def mul_mat_allgather(self, team: "Team", w: "Weight", x, y, stream=None) -> None:
        """y (all N rows, device) = this rank's row shard of W . QACT(x) gathered from every rank."""
        _check(lib().tsrc_mul_mat_allgather(self.handle, team.handle, w.handle, _addr(x), _addr(y), _stream(stream)))

    # ---- KV cache and FLASH_ATTN_EXT ----
    def kv_create(self, n_head_kv: int, head_dim: int, n_cells: int) -> "KvCache":
        h = _p()
        _check(lib().tsrc_kv_create(self.handle, n_head_kv, head_dim, n_cells, ct.byref(h)))
        return KvCache(self, h, n_head_kv, head_dim, n_cells)

    def flash_attn(self, kv: "KvCache", q, out, T: int, n_head: int, n_kv: int, scale: float, mask=None,
                   new=(0, 0), cfg=None, stream=None) -> None:
        """out[t][h] = the reference's composite FA of q[t][h] over cells [0, n_kv) of kv.
        q / out: device f32 [T][n_head][head_dim]; mask: host numpy f16 [T][stride] or None;
        cfg: (C, t_max, pcap, k_max[, plan_n_head_kv]) or None for the release values."""
        import numpy as np
        mptr, mstride, keep = None, 0, None
        if mask is not None:
            keep = np.ascontiguousarray(mask, dtype=np.float16)
            mptr, mstride = keep.ctypes.data, keep.shape[-1]
        c = None if cfg is None else FaCfg(*(tuple(cfg) + (0,) * (5 - len(cfg))))
        _check(lib().tsrc_flash_attn(self.handle, kv.handle, _addr(q), T, n_head, n_kv, mptr, mstride, scale,
                                     new[0], new[1], None if c is None else ct.byref(c), _addr(out),
                                     _stream(stream)))


class Weight:
    """A weight shard resident in device memory."""

    def __init__(self, dev: Device, handle):
        self.dev, self.handle = dev, handle
        f, n, k, r0, nr = (_u32() for _ in range(5))
        b = _u64()
        _check(lib().tsrc_weight_info(handle, ct.byref(f), ct.byref(n), ct.byref(k), ct.byref(r0), ct.byref(nr),
                                      ct.byref(b)))
        self.fmt, self.N, self.K, self.row0, self.n_rows = f.value, n.value, k.value, r0.value, nr.value
        self.device_bytes = b.value

    @property
    def ggml_bytes(self) -> int:
        return self.n_rows * ggml_row_bytes(self.fmt, self.K)

    def download(self):
        """The shard's ggml rows as numpy uint8 [n_rows, row_bytes]."""
        import numpy as np
        out = np.zeros((self.n_rows, ggml_row_bytes(self.fmt, self.K)), np.uint8)
        _check(lib().tsrc_weight_download(self.handle, out.ctypes.data))
        return out

    def free(self) -> None:
        if self.handle and self.dev.handle:
            _check(lib().tsrc_weight_free(self.handle))
        self.handle = None


class Model:
    """A random-init decoder on the device (tsrc_model_*)."""

    def __init__(self, dev: Device, cfg: ModelCfg, seed: int, team: "Team | None" = None):
        """team: a connected team -> this rank's tensor-parallel share (tsrc_model_create_tp)."""
        h = _p()
        self.dev, self.cfg, self.seed, self.team = dev, cfg, seed, team
        if team is None:
            _check(lib().tsrc_model_create(dev.handle, ct.byref(cfg), seed, ct.byref(h)))
        else:
            _check(lib().tsrc_model_create_tp(dev.handle, ct.byref(cfg), seed, team.handle, ct.byref(h)))
        self.handle = h
        ts, ks = _f32(), _f32()
        _check(lib().tsrc_model_params(h, ct.byref(ts), ct.byref(ks)))
        self.ts, self.kq_scale = ts.value, ks.value

    def forward(self, ids, T: int, pos0: int, logits, stream=None) -> None:
        _check(lib().tsrc_model_forward(self.handle, _addr(ids), T, pos0, _addr(logits), _stream(stream)))

    def decode(self, ids, pos0: int, logits, stream=None) -> None:
        """One token through the captured decode graph (keep ids / logits at fixed addresses)."""
        _check(lib().tsrc_model_decode(self.handle, _addr(ids), pos0, _addr(logits), _stream(stream)))

    def weight(self, layer: int, which: int) -> "Weight":
        h = _p()
        _check(lib().tsrc_model_weight(self.handle, layer, which, ct.byref(h)))
        w = Weight(self.dev, h)
        w.free = lambda: None                       # owned by the model
        return w

    def set_weight(self, layer: int, which: int, ggml_type: int, rows, N: int, K: int) -> None:
        """Replaces a weight with host rows of a loadable ggml type (tsrc_model_set_weight)."""
        import numpy as np
        a = np.ascontiguousarray(rows).view(np.uint8).reshape(-1)
        be, bb, _ = ggml_type_info(ggml_type)
        if a.size != N * (K // be) * bb:
            raise TsrcError(E_ARG, f"set_weight: {a.size} bytes for {N} rows of K={K}")
        _check(lib().tsrc_model_set_weight(self.handle, layer, which, ggml_type, a.ctypes.data, N, K))

    def set_f32(self, layer: int, which: int, values) -> None:
        """Replaces an f32 vector (norms, q | k | v bias) from host values (tsrc_model_set_f32)."""
        a = np.ascontiguousarray(values, dtype=np.float32)
        _check(lib().tsrc_model_set_f32(self.handle, layer, which, a.ctypes.data, a.size))

    def kv(self, layer: int) -> "KvCache":
        """Layer `layer`'s cache (owned by the model; a rank's holds its KV heads)."""
        h = _p()
        _check(lib().tsrc_model_kv(self.handle, layer, ct.byref(h)))
        world = 1 if self.team is None else self.team.world
        kv = KvCache(self.dev, h, self.cfg.n_head_kv // world, self.cfg.head_dim, self.cfg.n_ctx)
        kv.free = lambda: None                      # owned by the model
        return kv

    def f32_vector(self, layer: int, which: int, n: int):
        f = lib().tsrc_model_f32_value
        return np.array([f(self.seed, layer, which, i) for i in range(n)], np.float32)

    def free(self) -> None:
        if self.handle and self.dev.handle:
            _check(lib().tsrc_model_free(self.handle))
        self.handle = None


class KvCache:
    """One layer's q8_0 K and V cache resident in device memory."""

    def __init__(self, dev: Device, handle, n_head_kv: int, head_dim: int, n_cells: int):
        self.dev, self.handle = dev, handle
        self.n_head_kv, self.head_dim, self.n_cells = n_head_kv, head_dim, n_cells
        self.E = n_head_kv * head_dim

    @property
    def row_bytes(self) -> int:
        return self.E // 32 * Q8_0_BLOCK_BYTES

    def set_bytes(self, which: int, ggml_rows, cell0: int = 0) -> None:
        """ggml q8_0 rows (numpy uint8 [n, row_bytes]) -> cells [cell0, cell0 + n)."""
        import numpy as np
        a = np.ascontiguousarray(ggml_rows, dtype=np.uint8).reshape(-1, self.row_bytes)
        _check(lib().tsrc_kv_set_bytes(self.handle, which, a.ctypes.data, cell0, a.shape[0]))

    def get_bytes(self, which: int, cell0: int = 0, n: int | None = None):
        import numpy as np
        n = self.n_cells - cell0 if n is None else n
        out = np.zeros((n, self.row_bytes), np.uint8)
        _check(lib().tsrc_kv_get_bytes(self.handle, which, out.ctypes.data, cell0, n))
        return out

    def set_rows(self, which: int, rows, n: int | None = None, cells=None, cell0: int = 0, row_stride: int = 0,
                 stream=None) -> None:
        """KVST of f32 device rows [n][E] (SET_ROWS): at cells (device int64) or cell0 + i."""
        n = rows.shape[0] if n is None else n
        _check(lib().tsrc_kv_set_rows(self.dev.handle, self.handle, which, _addr(rows), n, row_stride,
                                      _addr(cells), cell0, _stream(stream)))

    def free(self) -> None:
        if self.handle and self.dev.handle:
            _check(lib().tsrc_kv_free(self.handle))
        self.handle = None


class Team:
    """One rank's side of a tensor-parallel team (CUDA IPC buffers of every rank)."""

    def __init__(self, dev: Device, handle, rank: int, world: int, ipc_handle: bytes):
        self.dev, self.handle, self.rank, self.world, self.ipc_handle = dev, handle, rank, world, ipc_handle

    def connect(self, handles: bytes) -> None:
        """handles: world x TEAM_HANDLE_BYTES bytes, rank order."""
        buf = ct.create_string_buffer(bytes(handles), len(handles))
        _check(lib().tsrc_team_connect(self.handle, buf))

    def connect_local(self, members: list) -> None:
        """Test hook: members = the teams of ranks 0..world-1 in this process (this one included)."""
        arr = (_p * len(members))(*[m.handle.value for m in members])
        _check(lib().tsrc_team_connect_local(self.handle, arr))

    def free(self) -> None:
        if self.handle and self.dev.handle:
            _check(lib().tsrc_team_free(self.handle))
        self.handle = None
