"""Tensor-parallel decode and prefill (tsrc_model_create_tp) against the single-GPU model, bit for
bit. Decode: both get the same KV cache cells (seeded rows through KVST; a rank's cache holds its KV
heads' columns), then decode tokens eagerly and through the captured decode graph. Prefill: two
prompt chunks (12 tokens at position 0, then 9 at position 12: the tensor-core MUL_MATs of the
rank's rows and the gathers of token rows, several team steps per gather since the team's n_max
holds only one or two rows) and then decode tokens. On one GPU a team of one runs every step of the
tensor-parallel path (shards, the tagged-word gathers, the fused gathers of o, down and the head);
on two GPUs (skipped when the box has one) two processes, one per GPU, each hold half the heads and
rows."""
import os
import socket

import numpy as np
import pytest

import tsrc

pytestmark = pytest.mark.gpu

SHAPES = {
    "llama_q4k": dict(n_layer=2, n_embd=512, n_ff=1024, n_head=8, n_head_kv=4, head_dim=64, n_vocab=1000, fmt=1,
                      rope_mode=tsrc.ROPE_NORM, rope_base=500000.0, rms_eps=1e-5, qkv_bias=0, tied_head=0, n_ctx=96),
    "qwen_q8": dict(n_layer=2, n_embd=256, n_ff=768, n_head=4, n_head_kv=2, head_dim=64, n_vocab=500, fmt=0,
                    rope_mode=tsrc.ROPE_NEOX, rope_base=1e6, rms_eps=1e-6, qkv_bias=1, tied_head=1, n_ctx=96),
}
PROMPT = 70          # cells filled before decoding


def fill_caches(torch, model, shape, rank, world):
    """Cells [0, PROMPT) of every layer: seeded full-width K / V rows, this rank's KV heads' columns."""
    E = shape["n_head_kv"] * shape["head_dim"]
    w = E // world
    for l in range(shape["n_layer"]):
        g = torch.Generator(device="cuda").manual_seed(1000 + l)
        kv = model.kv(l)
        for which in (tsrc.KV_K, tsrc.KV_V):
            rows = torch.randn((PROMPT, E), device="cuda", generator=g) * 2.0
            kv.set_rows(which, rows[:, rank * w:(rank + 1) * w].contiguous())


def decode_run(torch, dev, model, shape, steps=4):
    """Greedy decode from position PROMPT (the first token eagerly, the rest through the graph);
    returns the logits of every step."""
    out = []
    logits = torch.full((shape["n_vocab"],), float("nan"), device="cuda")
    one = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok, pos = 7, PROMPT
    for step in range(steps):
        one.fill_(tok)
        if step == 0:
            model.forward(one, 1, pos, logits)
        else:
            model.decode(one, pos, logits)
        dev.sync()
        v = logits.cpu().numpy().copy()
        out.append(v)
        tok, pos = int(np.argmax(v)), pos + 1
    return out


def prefill_run(torch, dev, model, shape, steps=2):
    """Two prompt chunks through tsrc_model_forward, then greedy decode; the logits of each call."""
    out = []
    logits = torch.full((shape["n_vocab"],), float("nan"), device="cuda")
    ids = torch.from_numpy(np.random.default_rng(5).integers(0, shape["n_vocab"], 21).astype(np.int32)).cuda()
    for t0, T in ((0, 12), (12, 9)):
        model.forward(ids[t0:t0 + T], T, t0, logits)
        dev.sync()
        out.append(logits.cpu().numpy().copy())
    one = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = 21
    for _ in range(steps):
        one.fill_(int(np.argmax(out[-1])))
        model.decode(one, pos, logits)
        dev.sync()
        out.append(logits.cpu().numpy().copy())
        pos += 1
    return out


def n_max_of(shape):
    return max(shape["n_vocab"], shape["n_ff"], shape["n_head"] * shape["head_dim"], shape["n_embd"])


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_team_of_one_equals_single_gpu(dev, name):
    import torch
    shape = SHAPES[name]
    cfg = tsrc.ModelCfg(**shape)
    single = tsrc.Model(dev, cfg, seed=11)
    team = dev.team_create(0, 1, n_max_of(shape))
    tp = None
    try:
        team.connect_local([team])
        tp = tsrc.Model(dev, cfg, seed=11, team=team)
        fill_caches(torch, single, shape, 0, 1)
        fill_caches(torch, tp, shape, 0, 1)
        want = decode_run(torch, dev, single, shape)
        got = decode_run(torch, dev, tp, shape)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    finally:
        if tp is not None:
            tp.free()
        single.free()
        team.free()


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_team_of_one_prefill_equals_single_gpu(dev, name):
    import torch
    shape = SHAPES[name]
    cfg = tsrc.ModelCfg(**shape)
    single = tsrc.Model(dev, cfg, seed=13)
    team = dev.team_create(0, 1, n_max_of(shape))
    tp = None
    try:
        team.connect_local([team])
        tp = tsrc.Model(dev, cfg, seed=13, team=team)
        want = prefill_run(torch, dev, single, shape)
        got = prefill_run(torch, dev, tp, shape)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    finally:
        if tp is not None:
            tp.free()
        single.free()
        team.free()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir, name, mode):
    import sys
    import datetime
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "tesseract-npu_b200"))
    import torch
    import torch.distributed as dist
    import tsrc as T
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    dev = T.Device(rank)
    ok = True
    try:
        shape = SHAPES[name]
        cfg = T.ModelCfg(**shape)
        team = dev.team_create(rank, world, n_max_of(shape))
        hs = [None] * world
        dist.all_gather_object(hs, team.ipc_handle)
        team.connect(b"".join(hs))
        tp = T.Model(dev, cfg, seed=11, team=team)
        single = T.Model(dev, cfg, seed=11)
        if mode == "prefill":
            got = prefill_run(torch, dev, tp, shape)
            want = prefill_run(torch, dev, single, shape)
        else:
            fill_caches(torch, tp, shape, rank, world)
            got = decode_run(torch, dev, tp, shape)
            fill_caches(torch, single, shape, 0, 1)
            want = decode_run(torch, dev, single, shape)
        ok = all(np.array_equal(a.view(np.uint32), b.view(np.uint32)) for a, b in zip(got, want))
        dist.barrier()
        single.free()
        tp.free()
        team.free()
        dist.barrier()
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write("ok" if ok else "mismatch")
        dev.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["decode", "prefill"])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_two_gpus_equal_single_gpu(tmp_path, name, mode):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), name, mode), nprocs=2, start_method="spawn", join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", f"rank {r}"
