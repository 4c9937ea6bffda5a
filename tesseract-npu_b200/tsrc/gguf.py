"""GGUF files: read, write, and load a llama / qwen2 model into a tsrc Model.

The reference runs models that llama.cpp loads from GGUF: llama.cpp parses the file and hands every
weight to the backend's set_tensor as ggml rows, where Q8_0 and Q4_K rows keep their blocks and any
other type is converted to Q8_0 (sw/ggml-tesseract/tsr-weights.h:1-30). Here `GGUFReader` parses the
file (GGUF v2 / v3: header, key-value metadata, tensor infos, aligned data section, memory-mapped),
and `load_model` maps llama.cpp's tensor names onto a `tsrc.Model`: the q, k, v rows are stacked and
the gate and up rows given gate-then-up (the model interleaves them), every matrix converted to its
device format on the host (`tsrc.ggml_rows_to_dev`), the norms and biases copied as f32.
`write_gguf` writes a file of the same format (used by the tests to build small models).
"""
from __future__ import annotations

import struct

import numpy as np

from . import (GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q8_0, MODEL_GLOBAL, ROPE_NEOX, ROPE_NORM, Device, FaCfg,
               Model, ModelCfg, TsrcError, E_ARG, E_SHAPE, ggml_rows_to_dev, ggml_type_info)

GGUF_MAGIC = b"GGUF"
# metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


class GGUFTensor:
    """One tensor of a GGUF file: name, ggml type, dims (ne[0] first: the row length), raw bytes."""

    def __init__(self, name: str, ggml_type: int, dims: tuple, data):
        self.name, self.type, self.dims, self.data = name, ggml_type, tuple(int(d) for d in dims), data

    @property
    def n_rows(self) -> int:
        n = 1
        for d in self.dims[1:]:
            n *= d
        return n

    @property
    def row_len(self) -> int:
        return self.dims[0]


class GGUFReader:
    """Parses a GGUF file; `kv` holds the metadata, `tensors` maps names to GGUFTensor (data are
    read-only views of the memory-mapped file)."""

    def __init__(self, path: str):
        self.path = path
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        buf = memoryview(self._mm)
        self._o = 0

        def take(n):
            b = buf[self._o:self._o + n]
            if len(b) != n:
                raise TsrcError(E_ARG, f"{path}: truncated GGUF file")
            self._o += n
            return bytes(b)

        def scalar(fmt):
            return struct.unpack(fmt, take(struct.calcsize(fmt)))[0]

        def string():
            n = scalar("<Q")
            return take(n).decode("utf-8")

        def value(t):
            if t in _SCALAR:
                return scalar(_SCALAR[t])
            if t == T_STR:
                return string()
            if t == T_ARR:
                et, n = scalar("<I"), scalar("<Q")
                return [value(et) for _ in range(n)]
            raise TsrcError(E_ARG, f"{path}: unknown GGUF value type {t}")

        if take(4) != GGUF_MAGIC:
            raise TsrcError(E_ARG, f"{path}: not a GGUF file")
        self.version = scalar("<I")
        if self.version not in (2, 3):
            raise TsrcError(E_ARG, f"{path}: GGUF version {self.version} (2 or 3 supported)")
        n_tensors, n_kv = scalar("<Q"), scalar("<Q")
        self.kv = {}
        for _ in range(n_kv):
            k = string()
            self.kv[k] = value(scalar("<I"))
        infos = []
        for _ in range(n_tensors):
            name = string()
            nd = scalar("<I")
            dims = tuple(scalar("<Q") for _ in range(nd))
            t, off = scalar("<I"), scalar("<Q")
            infos.append((name, dims, t, off))
        align = int(self.kv.get("general.alignment", 32))
        data0 = (self._o + align - 1) // align * align
        self.tensors = {}
        for name, dims, t, off in infos:
            be, bb = _block(t)
            nbytes = int(np.prod(dims, dtype=np.int64)) // be * bb
            self.tensors[name] = GGUFTensor(name, t, dims, self._mm[data0 + off:data0 + off + nbytes])


def _block(ggml_type: int) -> tuple[int, int]:
    be, bb, _ = ggml_type_info(ggml_type)
    return be, bb


def write_gguf(path: str, kv: dict, tensors: list, align: int = 32) -> None:
    """Writes a GGUF v3 file. kv: {key: (value_type, value)} (T_ARR values as (T_ARR, (elem_type,
    list))). tensors: [(name, ggml_type, dims, bytes-like)] with dims ne[0] first."""
    out = bytearray()

    def string(s):
        b = s.encode("utf-8")
        out.extend(struct.pack("<Q", len(b)))
        out.extend(b)

    def value(t, v):
        if t in _SCALAR:
            out.extend(struct.pack(_SCALAR[t], v))
        elif t == T_STR:
            string(v)
        elif t == T_ARR:
            et, items = v
            out.extend(struct.pack("<IQ", et, len(items)))
            for x in items:
                value(et, x)
        else:
            raise TsrcError(E_ARG, f"unknown GGUF value type {t}")

    kv = dict(kv)
    kv.setdefault("general.alignment", (T_U32, align))
    out.extend(GGUF_MAGIC)
    out.extend(struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for k, (t, v) in kv.items():
        string(k)
        out.extend(struct.pack("<I", t))
        value(t, v)
    offs, o = [], 0
    for name, t, dims, data in tensors:
        offs.append(o)
        o = (o + len(memoryview(data).cast("B")) + align - 1) // align * align
    for (name, t, dims, data), off in zip(tensors, offs):
        string(name)
        out.extend(struct.pack("<I", len(dims)))
        for d in dims:
            out.extend(struct.pack("<Q", d))
        out.extend(struct.pack("<IQ", t, off))
    out.extend(b"\0" * ((-len(out)) % align))
    data0 = len(out)
    for (name, t, dims, data), off in zip(tensors, offs):
        out.extend(b"\0" * (data0 + off - len(out)))
        out.extend(memoryview(data).cast("B"))
    with open(path, "wb") as f:
        f.write(out)


def _dev_rows(t: GGUFTensor) -> tuple[np.ndarray, int]:
    """A matrix tensor's rows in its device format: (uint8 [rows, row bytes], ggml type of the rows)."""
    _, _, fmt = ggml_type_info(t.type)
    rows = ggml_rows_to_dev(t.type, np.asarray(t.data), t.n_rows, t.row_len)
    return rows, (GGML_Q4_K if fmt == 1 else GGML_Q8_0)


def _stack(parts: list[GGUFTensor], what: str) -> tuple[np.ndarray, int]:
    """Rows of several matrices stacked in order, in one device format."""
    conv = [_dev_rows(t) for t in parts]
    types = {ty for _, ty in conv}
    if len(types) != 1:
        raise TsrcError(E_SHAPE, f"{what}: the stacked matrices load as different device formats "
                                 f"({', '.join(f'{t.name}: type {t.type}' for t in parts)})")
    return np.concatenate([r for r, _ in conv]), types.pop()


def _f32(t: GGUFTensor) -> np.ndarray:
    a = np.asarray(t.data)
    if t.type == GGML_F32:
        return a.view(np.float32).copy()
    if t.type == GGML_F16:
        return a.view(np.float16).astype(np.float32)
    if t.type == GGML_BF16:
        return (a.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    raise TsrcError(E_SHAPE, f"{t.name}: a vector of ggml type {t.type} (F32 / F16 / BF16 expected)")


def model_cfg(r: GGUFReader, n_ctx: int, fa: FaCfg | None = None) -> ModelCfg:
    """The tsrc model configuration of a llama / qwen2 GGUF file."""
    arch = r.kv.get("general.architecture")
    if arch not in ("llama", "qwen2"):
        raise TsrcError(E_SHAPE, f"{r.path}: architecture {arch!r} (llama or qwen2 supported)")
    kv, T = r.kv, r.tensors
    n_head = int(kv[f"{arch}.attention.head_count"])
    n_embd = int(kv[f"{arch}.embedding_length"])
    q = T["blk.0.attn_q.weight"]
    _, _, fmt = ggml_type_info(q.type)
    return ModelCfg(
        n_layer=int(kv[f"{arch}.block_count"]), n_embd=n_embd, n_ff=int(kv[f"{arch}.feed_forward_length"]),
        n_head=n_head, n_head_kv=int(kv.get(f"{arch}.attention.head_count_kv", n_head)),
        head_dim=int(kv.get(f"{arch}.attention.key_length", n_embd // n_head)),
        n_vocab=T["token_embd.weight"].n_rows, fmt=fmt, rope_mode=ROPE_NEOX if arch == "qwen2" else ROPE_NORM,
        rope_base=float(kv.get(f"{arch}.rope.freq_base", 10000.0)),
        rms_eps=float(kv.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)),
        qkv_bias=int("blk.0.attn_q.bias" in T), tied_head=int("output.weight" not in T), n_ctx=n_ctx,
        fa=fa if fa is not None else FaCfg())


def load_model(dev: Device, path: str, n_ctx: int, fa: FaCfg | None = None) -> Model:
    """Builds a Model from a llama / qwen2 GGUF file (llama.cpp's tensor names). The model is created
    with the file's shapes and every weight and vector is then replaced by the file's."""
    r = GGUFReader(path)
    cfg = model_cfg(r, n_ctx, fa)
    T = r.tensors
    m = Model(dev, cfg, seed=0)
    try:
        def put(layer, which, rows_type, N, K):
            rows, ty = rows_type
            m.set_weight(layer, which, ty, rows, N, K)

        E = cfg.n_embd
        emb = T["token_embd.weight"]
        put(MODEL_GLOBAL, 0, _dev_rows(emb), emb.n_rows, E)
        if not cfg.tied_head:
            put(MODEL_GLOBAL, 1, _dev_rows(T["output.weight"]), cfg.n_vocab, E)
        Hq, Hkv = cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
        for l in range(cfg.n_layer):
            b = f"blk.{l}."
            put(l, 0, _stack([T[b + "attn_q.weight"], T[b + "attn_k.weight"], T[b + "attn_v.weight"]], b + "q|k|v"),
                Hq + 2 * Hkv, E)
            put(l, 1, _dev_rows(T[b + "attn_output.weight"]), E, Hq)
            put(l, 2, _stack([T[b + "ffn_gate.weight"], T[b + "ffn_up.weight"]], b + "gate|up"), 2 * cfg.n_ff, E)
            put(l, 3, _dev_rows(T[b + "ffn_down.weight"]), E, cfg.n_ff)
            m.set_f32(l, 0, _f32(T[b + "attn_norm.weight"]))
            m.set_f32(l, 1, _f32(T[b + "ffn_norm.weight"]))
            if cfg.qkv_bias:
                m.set_f32(l, 2, np.concatenate([_f32(T[b + n]) for n in ("attn_q.bias", "attn_k.bias", "attn_v.bias")]))
        m.set_f32(cfg.n_layer, 5, _f32(T["output_norm.weight"]))
    except Exception:
        m.free()
        raise
    return m
