"""A model loaded from a GGUF file (tsrc.gguf.load_model: llama.cpp's tensor names, the q / k / v and
gate / up stacks, norms and biases through tsrc_model_set_weight / tsrc_model_set_f32) runs exactly
as the model the file was written from: a small random-init model is written out tensor by tensor
as llama.cpp names them, loaded back into a second model, and both run the same prompt and decode
token; the logits must be equal bit for bit. In the Q8_0 model the v projection is written as F32
(the dequantized blocks), so its rows take the load-time conversion to Q8_0 on the way in, which
gives back the same blocks. A Q4_K stack with an F32 member (a different device format) is
refused."""
import os

import numpy as np
import pytest

import ggml_types as G
import tsrc
import tsrc.gguf as gguf

pytestmark = pytest.mark.gpu

SHAPES = {
    "qwen_q8": dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, n_vocab=320, fmt=0,
                    rope_mode=tsrc.ROPE_NEOX, rope_base=1e6, rms_eps=1e-6, qkv_bias=1, tied_head=1, n_ctx=64),
    "llama_q4k": dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=300, fmt=1,
                      rope_mode=tsrc.ROPE_NORM, rope_base=500000.0, rms_eps=1e-5, qkv_bias=0, tied_head=0, n_ctx=64),
}


def q8_0_to_f32(rows: np.ndarray) -> np.ndarray:
    b = rows.reshape(rows.shape[0], -1, 34)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.float16)[..., 0].astype(np.float32)
    q = b[:, :, 2:].view(np.int8).astype(np.float32)
    return (q * d[:, :, None]).reshape(rows.shape[0], -1).astype(np.float32)


def write_model(m, s, path, v_as_f32=False):
    E, D, F = s["n_embd"], s["head_dim"], s["n_ff"]
    Hq, Hkv = s["n_head"] * D, s["n_head_kv"] * D
    ty = G.Q8_0 if s["fmt"] == tsrc.FMT_Q8_0 else G.Q4_K
    arch = "qwen2" if s["rope_mode"] == tsrc.ROPE_NEOX else "llama"
    kv = {"general.architecture": (gguf.T_STR, arch), f"{arch}.block_count": (gguf.T_U32, s["n_layer"]),
          f"{arch}.embedding_length": (gguf.T_U32, E), f"{arch}.feed_forward_length": (gguf.T_U32, F),
          f"{arch}.attention.head_count": (gguf.T_U32, s["n_head"]),
          f"{arch}.attention.head_count_kv": (gguf.T_U32, s["n_head_kv"]),
          f"{arch}.attention.key_length": (gguf.T_U32, D), f"{arch}.rope.freq_base": (gguf.T_F32, s["rope_base"]),
          f"{arch}.attention.layer_norm_rms_epsilon": (gguf.T_F32, s["rms_eps"])}
    T = [("token_embd.weight", ty, (E, s["n_vocab"]), m.weight(tsrc.MODEL_GLOBAL, 0).download())]
    if not s["tied_head"]:
        T.append(("output.weight", ty, (E, s["n_vocab"]), m.weight(tsrc.MODEL_GLOBAL, 1).download()))
    T.append(("output_norm.weight", G.F32, (E,), m.f32_vector(s["n_layer"], 5, E)))
    for l in range(s["n_layer"]):
        b = f"blk.{l}."
        qkv = m.weight(l, 0).download()
        v = qkv[Hq + Hkv:]
        T += [(b + "attn_q.weight", ty, (E, Hq), qkv[:Hq]), (b + "attn_k.weight", ty, (E, Hkv), qkv[Hq:Hq + Hkv]),
              (b + "attn_v.weight", G.F32, (E, Hkv), q8_0_to_f32(v)) if v_as_f32 else (b + "attn_v.weight", ty, (E, Hkv), v)]
        T.append((b + "attn_output.weight", ty, (Hq, E), m.weight(l, 1).download()))
        gu = m.weight(l, 2).download()                  # the model's rows interleave (gate_j, up_j)
        T += [(b + "ffn_gate.weight", ty, (E, F), np.ascontiguousarray(gu[0::2])),
              (b + "ffn_up.weight", ty, (E, F), np.ascontiguousarray(gu[1::2]))]
        T.append((b + "ffn_down.weight", ty, (F, E), m.weight(l, 3).download()))
        T += [(b + "attn_norm.weight", G.F32, (E,), m.f32_vector(l, 0, E)),
              (b + "ffn_norm.weight", G.F32, (E,), m.f32_vector(l, 1, E))]
        if s["qkv_bias"]:
            bias = m.f32_vector(l, 2, Hq + 2 * Hkv)
            T += [(b + "attn_q.bias", G.F32, (Hq,), bias[:Hq]), (b + "attn_k.bias", G.F32, (Hkv,), bias[Hq:Hq + Hkv]),
                  (b + "attn_v.bias", G.F32, (Hkv,), bias[Hq + Hkv:])]
    gguf.write_gguf(path, kv, [(n, t, d, np.ascontiguousarray(a)) for n, t, d, a in T])


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_gguf_model_matches_source_model(dev, tmp_path, name):
    import torch
    s = SHAPES[name]
    a = tsrc.Model(dev, tsrc.ModelCfg(**s), seed=11)
    b = None
    try:
        path = os.path.join(tmp_path, f"{name}.gguf")
        write_model(a, s, path, v_as_f32=s["fmt"] == tsrc.FMT_Q8_0)
        b = gguf.load_model(dev, path, n_ctx=s["n_ctx"])
        for k in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab", "rope_mode", "qkv_bias",
                  "tied_head"):
            assert getattr(b.cfg, k) == s[k], k
        prompt = np.random.default_rng(4).integers(0, s["n_vocab"], 12).astype(np.int32)
        ids = torch.from_numpy(prompt).cuda()
        la = torch.full((s["n_vocab"],), float("nan"), device="cuda")
        lb = torch.full((s["n_vocab"],), float("nan"), device="cuda")
        a.forward(ids, prompt.size, 0, la)
        b.forward(ids, prompt.size, 0, lb)
        dev.sync()
        np.testing.assert_array_equal(la.cpu().numpy().view(np.uint32), lb.cpu().numpy().view(np.uint32))
        one = torch.tensor([int(torch.argmax(la))], dtype=torch.int32, device="cuda")
        a.decode(one, prompt.size, la)
        b.decode(one, prompt.size, lb)
        dev.sync()
        np.testing.assert_array_equal(la.cpu().numpy().view(np.uint32), lb.cpu().numpy().view(np.uint32))
    finally:
        a.free()
        if b is not None:
            b.free()


def test_gguf_mixed_device_formats_in_a_stack_refused(dev, tmp_path):
    s = SHAPES["llama_q4k"]
    a = tsrc.Model(dev, tsrc.ModelCfg(**s), seed=12)
    try:
        path = os.path.join(tmp_path, "mixed.gguf")
        # attn_v as F32 loads as Q8_0 while q and k are Q4_K: the fused q | k | v weight cannot hold both
        qkv = a.weight(0, 0).download()
        write_model(a, s, path)
        r = gguf.GGUFReader(path)
        Hq, Hkv = s["n_head"] * s["head_dim"], s["n_head_kv"] * s["head_dim"]
        v = np.zeros((Hkv, s["n_embd"]), np.float32)
        T = [(n, t.type, t.dims, np.asarray(t.data)) for n, t in r.tensors.items()]
        T = [(n, G.F32, d, v) if n == "blk.0.attn_v.weight" else (n, ty, d, x) for n, ty, d, x in T]
        kv = {k: (gguf.T_STR, v_) if isinstance(v_, str) else ((gguf.T_F32, v_) if isinstance(v_, float) else (gguf.T_U32, v_))
              for k, v_ in r.kv.items()}
        del r
        path2 = os.path.join(tmp_path, "mixed2.gguf")
        gguf.write_gguf(path2, kv, T)
        assert qkv.shape[0] == Hq + 2 * Hkv
        with pytest.raises(tsrc.TsrcError):
            gguf.load_model(dev, path2, n_ctx=s["n_ctx"])
    finally:
        a.free()
