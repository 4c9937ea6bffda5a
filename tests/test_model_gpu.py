"""End-to-end decoder (tsrc_model_forward) against the oracle's composition of the same graph
(oracle.OracleModel over the kinds pinned to the reference): a prompt through the prefill path (more
than eight tokens: the tensor-core MUL_MAT and FA query tiles), then decode steps through the
matvec path, eagerly and through the captured decode graph (whose FA plans are rewritten per
token). Small random-init models of both architectures; tolerance: equal f32 bit patterns of the
logits."""
import numpy as np
import pytest

import tsrc

pytestmark = pytest.mark.gpu

SHAPES = {
    # qwen2-like: NEOX rope, q/k/v biases, tied head, Q8_0
    "qwen_q8": dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, n_vocab=320, fmt=0,
                    rope_mode=tsrc.ROPE_NEOX, rope_base=1e6, rms_eps=1e-6, qkv_bias=1, tied_head=1, n_ctx=64),
    # llama-like: NORM rope, untied head, Q4_K
    "llama_q4k": dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=300, fmt=1,
                      rope_mode=tsrc.ROPE_NORM, rope_base=500000.0, rms_eps=1e-5, qkv_bias=0, tied_head=0, n_ctx=64),
}


def oracle_of(tsro, m, shape):
    import oracle
    L = []
    for l in range(shape["n_layer"]):
        w = {n: m.weight(l, i).download() for i, n in enumerate(("wqkv", "wo", "wgu", "wd"))}
        w["wgu"] = np.concatenate([w["wgu"][0::2], w["wgu"][1::2]])      # the model interleaves (gate_j, up_j)
        E, Hq, Hkv = shape["n_embd"], shape["n_head"] * shape["head_dim"], shape["n_head_kv"] * shape["head_dim"]
        w["attn_norm"] = m.f32_vector(l, 0, E)
        w["ffn_norm"] = m.f32_vector(l, 1, E)
        if shape["qkv_bias"]:
            w["bqkv"] = m.f32_vector(l, 2, Hq + 2 * Hkv)
        L.append(w)
    emb = m.weight(tsrc.MODEL_GLOBAL, 0).download()
    head = m.weight(tsrc.MODEL_GLOBAL, 1).download()
    out_norm = m.f32_vector(shape["n_layer"], 5, shape["n_embd"])
    return oracle.OracleModel(tsro, shape, L, emb, head, out_norm, m.ts, m.kq_scale)


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_model_prefill_then_decode_bit_exact(dev, tsro, name):
    import torch
    shape = SHAPES[name]
    cfg = tsrc.ModelCfg(**{k: v for k, v in shape.items()})
    m = tsrc.Model(dev, cfg, seed=7)
    try:
        ref = oracle_of(tsro, m, shape)
        rng = np.random.default_rng(3)
        prompt = rng.integers(0, shape["n_vocab"], 12).astype(np.int32)
        logits = torch.full((shape["n_vocab"],), float("nan"), device="cuda")
        ids = torch.from_numpy(prompt).cuda()
        m.forward(ids, prompt.size, 0, logits)
        dev.sync()
        want = ref.forward(prompt, 0)
        np.testing.assert_array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
        pos = prompt.size
        tok = int(np.argmax(want))
        one = torch.zeros(1, dtype=torch.int32, device="cuda")
        for step in range(5):                                # greedy decode: eagerly, then through the graph
            one.fill_(tok)
            if step == 0:
                m.forward(one, 1, pos, logits)
            else:
                m.decode(one, pos, logits)                   # step 1 captures, later steps patch the graph
            dev.sync()
            want = ref.forward(np.array([tok], np.int32), pos)
            np.testing.assert_array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
            tok, pos = int(np.argmax(want)), pos + 1
    finally:
        m.free()
