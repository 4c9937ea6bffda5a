"""Bench of the B200 hot path: decode MUL_MAT (QACT + Q4_K / Q8_0 matvec) through the C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg2|cfg1]

Metric: matvec HBM GB/s. The N = 1 workload is BASELINE config 2 (Q4_K
14336 x 4096, one token); config 1 (Q8_0 4864 x 896) with --config cfg1. A step is one MUL_MAT of
one token over one weight matrix: QACT of the f32 activation, then the matvec; on N > 1 GPUs each
rank holds a contiguous row shard (the reference's symmetric row split) and the step ends with the
all-gather of y fused into the matvec kernel (P2P stores of tagged words over NVLink; an NCCL
all_gather with --collective nccl). Algorithmic bytes per step: N*(K/256)*144 (or N*(K/32)*34) + 4K + 4N.

  value      K steps with x resident in HBM, inputs larger than L2 (each step reads the next of a
             ring of distinct weight copies, >= 4x L2 per GPU); CUDA graph replay on one GPU.
  roofline   the matvec kernel alone (tsrc_mvm), CUDA events on its stream, same weight ring.
  e2e        tsrc_mul_mat with the activation copied in from pinned host memory and y read back
             to pinned host memory every step.
  cpu_baseline  the reference's own CPU path (tsr_qact + tsr_dot_row, oracle/_ref) on the host's
             cores for ~10 s, rank 0 at N = 1 only.
--impl reference times that CPU path alone (rank 0; other ranks exit) on a bounded row sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tesseract-npu_b200"))

CONFIGS = {
    # name: (fmt, N, K, weight seed, x seed, description)
    "cfg2": (1, 14336, 4096, 201, 202, "BASELINE config 2: Q4_K matvec 14336x4096, one token (decode)"),
    "cfg1": (0, 4864, 896, 101, 102, "BASELINE config 1: Q8_0 matvec 4864x896, one token (decode)"),
    "cfg3": (None, None, None, 301, 303, "BASELINE config 3: flash-attention decode over a q8_0 KV cache, "
             "32 q / 8 kv heads, head_dim 128, 8192 cells, one token"),
}
CONFIGS["cfg4"] = (None, None, None, 41, 42, "BASELINE config 4: Qwen2.5-0.5B architecture (random-init, Q8_0), decode")
CONFIGS["cfg5"] = (None, None, None, 51, 52, "BASELINE config 5: Llama-3-8B architecture (random-init, Q4_K), decode")
METRIC = "Q8_0/Q4_K matvec HBM GB/s"
FA = dict(D=128, n_head_kv=8, G=4, n_kv=8192)


def capture(torch, body, sync):
    """A CUDA graph of body() (NCCL collectives included), replayed once; None if capture fails
    (the loops then run eagerly)."""
    try:
        sync()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        g.replay()
        sync()
        return g
    except Exception as e:  # noqa: BLE001
        print(f"bench: CUDA graph capture failed ({e}); timing eager launches", file=sys.stderr)
        sync()
        return None


E2E_BUFFERS = 4        # device input / output buffers the end-to-end pipeline rotates through


def pipelined(torch, n, copy_in, compute, copy_out, s_in, s_out):
    """Issues n end-to-end steps with later steps' copies in (stream s_in) and earlier steps' copies
    out (stream s_out) under step i's compute on the current stream; the device buffers rotate
    (b = i % E2E_BUFFERS), so a copy waits only for the step E2E_BUFFERS back that used its buffer,
    and every step still copies its own input in and its own result out."""
    comp = torch.cuda.current_stream()
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    k_done, out_done = {}, {}
    nb = E2E_BUFFERS
    for i in range(n):
        b = i % nb
        ev_in = torch.cuda.Event()
        with torch.cuda.stream(s_in):
            if i >= nb:
                s_in.wait_event(k_done[i - nb])             # the step that last computed from buffer b
            copy_in(b)
            ev_in.record(s_in)
        comp.wait_event(ev_in)
        if i >= nb:
            comp.wait_event(out_done[i - nb])               # that step's result left buffer b
        compute(i, b)
        k_done[i] = torch.cuda.Event()
        k_done[i].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(k_done[i])
            copy_out(b)
            out_done[i] = torch.cuda.Event()
            out_done[i].record(s_out)
    comp.wait_stream(s_in)
    comp.wait_stream(s_out)


# prefill MUL_MAT on the tensor cores (many tokens): BASELINE configs 5 and 4 FFN shapes
PREFILL = [
    (1, 14336, 4096, 2048, 501, "cfg5 FFN gate/up: Q4_K 14336x4096, 2048-token prefill"),
    (0, 4864, 896, 512, 401, "cfg4 FFN gate/up: Q8_0 4864x896, 512-token prefill"),
]


def prefill_measure(dev, tsrc, torch, reps=10, warmup=3):
    """tsrc_mul_mat over T tokens (QACT of every token + the tcgen05 kernel), inputs resident in
    HBM; int8 ops = 2 N K T. Compute-bound, so L2 residency of the weights does not matter."""
    peak = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak = 2.0 * float(json.load(f)["bf16_tflops"])     # int8 dense = 2x bf16 dense on this tensor pipe
    res = []
    for fmt, N, K, T, seed, desc in PREFILL:
        w = dev.synth(fmt, N, K, seed=seed)
        g = torch.Generator(device="cuda")
        g.manual_seed(seed + 1)
        x = torch.randn(T, K, device="cuda", generator=g)
        y = torch.empty(T, N, device="cuda")
        for _ in range(warmup):
            dev.mul_mat(w, x, y, T=T)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            dev.mul_mat(w, x, y, T=T)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        tops = 2.0 * N * K * T / (us * 1e-6) / 1e12
        res.append({"workload": desc, "us_per_call": round(us, 1), "TOPS": round(tops, 1),
                    "frac_of_int8_peak": round(tops / peak, 4) if peak else None,
                    "int8_peak_TOPS": round(peak, 1) if peak else None})
        w.free()
    return {"metric": "prefill MUL_MAT int8 TOPS (tcgen05 kind::i8, bit-exact f32 block scaling)", "runs": res,
            "peak_kind": "2x measured bf16 dense (MEASURED_PEAKS.json)" if peak else None,
            "note": "the reference's per-32-value f32 scale-and-accumulate runs on the CUDA cores (tensor-pipe "
                    "activity: the committed ncu summary of the prefill kernels)"}


# end-to-end random-init models (BASELINE configs 4 and 5): decode tokens/s
MODELS = {
    "cfg4": dict(desc="BASELINE config 4: Qwen2.5-0.5B architecture, random-init, all Q8_0, 512-token prefill then decode",
                 shape=dict(n_layer=24, n_embd=896, n_ff=4864, n_head=14, n_head_kv=2, head_dim=64, n_vocab=151936, fmt=0,
                            rope_mode=1, rope_base=1e6, rms_eps=1e-6, qkv_bias=1, tied_head=1),
                 prompt=512, decode=128, seed=41),
    "cfg5": dict(desc="BASELINE config 5: Llama-3-8B architecture, random-init, all Q4_K, 2048-token prefill then decode",
                 shape=dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256, fmt=1,
                            rope_mode=0, rope_base=500000.0, rms_eps=1e-5, qkv_bias=0, tied_head=0),
                 prompt=2048, decode=256, seed=51),
}


def model_row_bytes(fmt, N, K):
    return N * (K // 32 * 34 if fmt == 0 else K // 256 * 144)


def model_algo_bytes(s, n_kv):
    """Bytes one decode token must read: every layer's seven matrices, the K / V cells it attends
    (q8_0, 34 B per 32 values), the head, and the token's embedding row."""
    fmt, E, D, F = s["fmt"], s["n_embd"], s["head_dim"], s["n_ff"]
    Hq, Hkv = s["n_head"] * D, s["n_head_kv"] * D
    layer = (model_row_bytes(fmt, Hq, E) + 2 * model_row_bytes(fmt, Hkv, E) + model_row_bytes(fmt, E, Hq)
             + 2 * model_row_bytes(fmt, F, E) + model_row_bytes(fmt, E, F))
    kv = 2 * n_kv * (Hkv // 32) * 34
    return s["n_layer"] * (layer + kv) + model_row_bytes(fmt, s["n_vocab"], E) + model_row_bytes(fmt, 1, E)


def model_measure(dev, tsrc, torch, name, steps, warmup, e2e_steps=32):
    """Prefill of the config's prompt, then `warmup` + `steps` timed decode tokens (CUDA events on
    the stream, inputs resident) and `e2e_steps` decode tokens with the token id copied in from
    pinned host memory and the logits read back every step. Returns a dict and the model (for the
    CPU sample's weights); the caller frees the model."""
    spec = MODELS[name]
    prompt = spec["prompt"]
    n_ctx = prompt + warmup + steps + e2e_steps
    s = dict(spec["shape"], n_ctx=n_ctx)
    model = tsrc.Model(dev, tsrc.ModelCfg(**s), seed=spec["seed"])
    g = torch.Generator(device="cuda")
    g.manual_seed(spec["seed"])
    ids = torch.randint(0, s["n_vocab"], (n_ctx,), dtype=torch.int32, device="cuda", generator=g)
    logits = torch.empty(s["n_vocab"], device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    model.forward(ids, prompt, 0, logits)                      # warm-up prefill (first launches), then timed
    torch.cuda.synchronize()
    e0.record()
    model.forward(ids, prompt, 0, logits)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    pos = prompt
    one = torch.empty(1, dtype=torch.int32, device="cuda")     # the graph's token buffer
    for _ in range(warmup):
        one.copy_(ids[pos:pos + 1])
        model.decode(one, pos, logits)
        pos += 1
    torch.cuda.synchronize()
    kv0 = pos
    e0.record()
    for _ in range(steps):
        one.copy_(ids[pos:pos + 1])
        model.decode(one, pos, logits)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    host_ids = ids[pos:pos + e2e_steps].cpu().pin_memory()
    host_logits = torch.empty(s["n_vocab"], pin_memory=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(e2e_steps):
        one.copy_(host_ids[i:i + 1], non_blocking=True)
        model.decode(one, pos, logits)
        host_logits.copy_(logits, non_blocking=True)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    algo = model_algo_bytes(s, kv0 + steps // 2)
    # state, GET_ROWS; per layer 4 MUL_MATs (q / k / v and gate / up with RMS_NORM fused in, gate / up
    # with SWIGLU as its epilogue), ROPE + KVST, FA chunk + merge; then the head (RMS_NORM fused in)
    launches = 3 + 7 * s["n_layer"]
    return dict(shape=s, prefill_ms=prefill_ms, ms=ms, e2e_ms=e2e_ms, algo_bytes=algo, launches=launches,
                n_kv=(kv0, pos)), model


def model_measure_tp(dev, tsrc, torch, dist, name, steps, warmup, rank, world, e2e_steps=32):
    """The config split over `world` GPUs (tsrc_model_create_tp over a team): the prompt's prefill
    through tsrc_model_forward (timed: a warm-up pass, then the measured one), then `warmup` +
    `steps` timed decode tokens and `e2e_steps` with the token id in from pinned host memory and the
    logits out. Device times are the maximum over the ranks. The team's staging holds 64 rows of
    the widest exchanged vector, so a prompt's gathers take few team steps."""
    spec = MODELS[name]
    prompt = spec["prompt"]
    n_ctx = prompt + warmup + steps + e2e_steps
    s = dict(spec["shape"], n_ctx=n_ctx)
    n_max = 64 * max(s["n_vocab"], s["n_ff"], s["n_head"] * s["head_dim"], s["n_embd"])
    team = dev.team_create(rank, world, n_max)
    hs = [None] * world
    dist.all_gather_object(hs, team.ipc_handle)
    team.connect(b"".join(hs))
    model = tsrc.Model(dev, tsrc.ModelCfg(**s), seed=spec["seed"], team=team)
    g = torch.Generator(device="cuda")
    g.manual_seed(spec["seed"])
    ids = torch.randint(0, s["n_vocab"], (n_ctx,), dtype=torch.int32, device="cuda", generator=g)
    logits = torch.empty(s["n_vocab"], device="cuda")
    one = torch.empty(1, dtype=torch.int32, device="cuda")

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    model.forward(ids, prompt, 0, logits)                      # warm-up prefill (first launches), then timed
    barrier()
    e0.record()
    model.forward(ids, prompt, 0, logits)
    e1.record()
    barrier()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1))
    pos = prompt
    for _ in range(warmup):
        one.copy_(ids[pos:pos + 1])
        model.decode(one, pos, logits)
        pos += 1
    barrier()
    kv0 = pos
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        one.copy_(ids[pos:pos + 1])
        model.decode(one, pos, logits)
        pos += 1
    e1.record()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    host_ids = ids[pos:pos + e2e_steps].cpu().pin_memory()
    host_logits = torch.empty(s["n_vocab"], pin_memory=True)
    barrier()
    e0.record()
    for i in range(e2e_steps):
        one.copy_(host_ids[i:i + 1], non_blocking=True)
        model.decode(one, pos, logits)
        host_logits.copy_(logits, non_blocking=True)
        pos += 1
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    # state, GET_ROWS; per layer q / k / v (RMS_NORM fused), ROPE + KVST, FA chunk + merge, the
    # attention gather, o (+ gather), gate / up (RMS_NORM, SWIGLU and the gather fused), down
    # (+ gather); then the head (RMS_NORM and the gather fused)
    launches = 3 + 8 * s["n_layer"]
    return dict(shape=s, prefill_ms=prefill_ms, ms=ms, e2e_ms=e2e_ms, algo_bytes=model_algo_bytes(s, kv0 + steps // 2),
                launches=launches, n_kv=(kv0, pos)), model, team


def cpu_reference_model(name, threads, model=None):
    """One decode token of the config on the host cores: one decoder layer at the config's KV length
    (synthetic q8_0 cache rows) and the output norm + head, each timed directly (a second run of
    each, after a first that faults the pages in), the layer time times the layer count plus the
    head. The kinds are the reference's own functions (oracle/_ref: MUL_MAT, FA, RMS_NORM, ROPE, VOP,
    GET_ROWS) when that library was built, else the restatement. Weights: the device model's rows
    when given, else quantized on the host from seeded normals. Returns (tokens/s, kind, sample)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    tsro = oracle.Tsro()
    kind = "reference" if oracle.Ref.available() else "port"
    ops = oracle.RefOps(oracle.Ref(), tsro) if kind == "reference" else tsro
    spec = MODELS[name]
    prompt = spec["prompt"]
    s = dict(spec["shape"], n_ctx=prompt + 1)
    fmt, E, D, F, V = s["fmt"], s["n_embd"], s["head_dim"], s["n_ff"], s["n_vocab"]
    Hq, Hkv = s["n_head"] * D, s["n_head_kv"] * D
    rng = np.random.default_rng(spec["seed"])
    names = ("wqkv", "wo", "wgu", "wd")
    shapes = ((Hq + 2 * Hkv, E), (E, Hq), (2 * F, E), (E, F))
    if model is not None:
        L = {n: model.weight(0, i).download() for i, n in enumerate(names)}
        L["wgu"] = np.concatenate([L["wgu"][0::2], L["wgu"][1::2]])     # the model interleaves (gate_j, up_j)
        head = model.weight(0xFFFFFFFF, 1).download()
        emb = model.weight(0xFFFFFFFF, 0).download()[:16]
        src = "the device model's layer-0 and head rows"
    else:
        L = {n: tsro.quantize(fmt, (rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02))) for n, sh in zip(names, shapes)}
        head = tsro.quantize(fmt, rng.standard_normal((V, E), dtype=np.float32) * np.float32(0.02))
        emb = head[:16]
        src = "host-quantized seeded N(0, 0.02) rows"
    L["attn_norm"] = np.ones(E, np.float32)
    L["ffn_norm"] = np.ones(E, np.float32)
    if s["qkv_bias"]:
        L["bqkv"] = np.zeros(Hq + 2 * Hkv, np.float32)
    ts = float(np.power(np.float32(s["rope_base"]), np.float32(-2.0) / np.float32(D), dtype=np.float32))
    om = oracle.OracleModel(ops, dict(s, n_layer=1), [L], emb, head, np.ones(E, np.float32), ts,
                            float(np.float32(1.0) / np.sqrt(np.float32(D))), threads=threads)
    kv = tsro.quantize(0, rng.standard_normal((prompt, Hkv), dtype=np.float32))
    om.kc[0][:prompt] = kv
    om.vc[0][:prompt] = kv[::-1]
    x = om.embed(np.array([3], np.int32))
    t_layer = t_head = None
    for _ in range(2):                      # the second run of each piece is the one reported
        t0 = time.perf_counter()
        y = om.layer(0, x, prompt)
        t_layer = time.perf_counter() - t0
        t0 = time.perf_counter()
        om.logits(y)
        t_head = time.perf_counter() - t0
    t_tok = s["n_layer"] * t_layer + t_head
    what = ("the reference's own kinds (oracle/_ref)" if kind == "reference"
            else "the restatement of the reference's kinds (oracle/_ref not built)")
    sample = (f"one decode token at KV length {prompt}: one layer timed directly ({t_layer * 1e3:.1f} ms) x "
              f"{s['n_layer']} layers + output norm and head ({t_head * 1e3:.1f} ms); {src}; {what}, {threads} host "
              f"threads for the MUL_MATs")
    return 1.0 / t_tok, kind, sample


def fa_algo_bytes(n_head_kv, D, G, n_kv):
    """K and V q8_0 bytes of the visible cells + f32 q in + f32 out (per call)."""
    E = n_head_kv * D
    return 2 * n_kv * (E // 32) * 34 + 2 * 4 * n_head_kv * G * D


def fa_measure(dev, tsrc, torch, steps, warmup, world=1, rank=0, dist=None):
    """FA decode (config 3) on this rank's KV heads (8 / world of them): a ring of caches larger
    than 4x L2, each step one tsrc_flash_attn (plus the all-gather of out on N > 1 GPUs).
    Returns (device ms for `steps` steps, e2e ms for min(steps, 2000) steps, info)."""
    import numpy as np
    D, H, G, n_kv = FA["D"], FA["n_head_kv"], FA["G"], FA["n_kv"]
    h_loc = H // world
    E = h_loc * D
    local = torch.cuda.current_device()
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    cache_bytes = 2 * n_kv * (E // 32) * 34
    n_ring = max(2, math.ceil(4 * l2 / cache_bytes))
    gen = torch.Generator(device="cuda").manual_seed(301 + rank)
    kvs = []
    for _ in range(n_ring):
        kv = dev.kv_create(h_loc, D, n_kv)
        for which in (0, 1):
            kv.set_rows(which, torch.randn((n_kv, E), device="cuda", generator=gen))
        kvs.append(kv)
    torch.cuda.synchronize()
    q = torch.randn((1, h_loc * G, D), device="cuda", generator=torch.Generator(device="cuda").manual_seed(303 + rank))
    out = torch.empty_like(q)
    out_all = torch.empty((world, h_loc * G, D), device="cuda")
    scale = float(np.float32(1.0 / np.sqrt(D)))

    cfg = (4, 4, 9344, 32768, H)          # release configuration; shards plan with the model's 8 KV heads

    def step(i):
        dev.flash_attn(kvs[i % n_ring], q, out, T=1, n_head=h_loc * G, n_kv=n_kv, scale=scale, new=(n_kv - 1, n_kv),
                       cfg=cfg)
        if world > 1:
            dist.all_gather_into_tensor(out_all, out)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    def sync_all():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    graph = capture(torch, lambda: [step(i) for i in range(n_ring)], sync_all)

    def loop(n):
        if graph is not None:
            reps, rem = divmod(n, n_ring)
            for _ in range(reps):
                graph.replay()
            for i in range(rem):
                step(i)
        else:
            for i in range(n):
                step(i)

    q_host = q.cpu().pin_memory()
    o_host = torch.empty((world, h_loc * G, D)).pin_memory()
    n_e2e = min(steps, 2000)

    # end to end, pipelined over steps as for the matvec (q and out rotate over E2E_BUFFERS buffers)
    qb = [q] + [torch.empty_like(q) for _ in range(E2E_BUFFERS - 1)]
    ob = [out] + [torch.empty_like(out) for _ in range(E2E_BUFFERS - 1)]
    oab = [out_all] + [torch.empty_like(out_all) for _ in range(E2E_BUFFERS - 1)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def fa_step(i, b):
        dev.flash_attn(kvs[i % n_ring], qb[b], ob[b], T=1, n_head=h_loc * G, n_kv=n_kv, scale=scale,
                       new=(n_kv - 1, n_kv), cfg=cfg)
        if world > 1:
            dist.all_gather_into_tensor(oab[b], ob[b])

    def e2e_steps(n):
        pipelined(torch, n, lambda b: qb[b].copy_(q_host, non_blocking=True), fa_step,
                  lambda b: o_host.copy_(oab[b] if world > 1 else ob[b].view(1, h_loc * G, D), non_blocking=True),
                  s_in, s_out)

    egraph = capture(torch, lambda: e2e_steps(n_ring), sync_all)

    def e2e(n):
        if egraph is not None:
            reps, rem = divmod(n, n_ring)
            for _ in range(reps):
                egraph.replay()
            if rem:
                e2e_steps(rem)
        else:
            e2e_steps(n)

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn(n)
        e1.record()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms = timed(loop, steps)
    ms_e2e = timed(e2e, n_e2e)
    used_graph = graph is not None
    e2e_graph = egraph is not None
    del graph, egraph
    for kv in kvs:
        kv.free()
    info = {"ring": n_ring, "ring_mb_per_gpu": round(n_ring * cache_bytes / 1e6, 1), "heads_kv_per_gpu": h_loc,
            "h2d_bytes_per_step": 4 * h_loc * G * D, "d2h_bytes_per_step": 4 * world * h_loc * G * D, "e2e_steps": n_e2e,
            "cuda_graph": used_graph, "e2e_cuda_graph": e2e_graph}
    return ms, ms_e2e, info


def row_bytes(fmt, K):
    return K // 256 * 144 if fmt == 1 else K // 32 * 34


def algo_bytes(fmt, N, K):
    return N * row_bytes(fmt, K) + 4 * K + 4 * N


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples (SM clock, max, throttle reasons) while the timed loops run."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index):
        self.proc = None
        self.dev_index = dev_index

    def __enter__(self):
        import torch
        uuid = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.dev_index).uuid)
        except Exception:
            pass
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if uuid:
            cmd[1:1] = ["-i", uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                rows.append((float(f[0]), float(f[1]), f[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def cpu_reference_matvec(fmt, N, K, x, seconds, threads):
    """The reference's CPU path (oracle/_ref, else the oracle port) on rows of config-like weights.
    Returns (GB/s, kind, sample description)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle
    import helpers as H
    tsro = oracle.Tsro()
    rows = min(N, 2048)                       # weight rows generated on the host; cycled to N
    w = H.weights(tsro, fmt, rows, K, 999)
    if oracle.Ref.available():
        ref = oracle.Ref()
        packed = ref.repack(fmt, w, K)
        tile = np.ascontiguousarray(np.tile(packed, (math.ceil(N / rows), 1))[:N])
        y = np.zeros((1, N), np.float32)
        run = lambda: ref.matvec_repacked(fmt, tile, K, x, threads=threads, out=y)  # noqa: E731
        kind = "reference"
    else:
        tile = np.ascontiguousarray(np.tile(w, (math.ceil(N / rows), 1))[:N])
        run = lambda: tsro.matvec(fmt, tile, K, x, threads=threads)  # noqa: E731
        kind = "port"
    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * algo_bytes(fmt, N, K) / el / 1e9
    return gbs, kind, f"{n} full {N}x{K} matvecs in {el:.1f} s ({threads} threads)", el / n


def cpu_reference_fa(seconds, threads, calls=None):
    """The reference's tsr_ref_fa (oracle/_ref) -- else the restatement -- on config 3, one full call
    per worker thread at a time, for about `seconds` (or exactly `calls` calls per thread).
    Returns (GB/s of algorithmic bytes, kind, sample text, seconds per call)."""
    import threading
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle
    import helpers as H
    tsro = oracle.Tsro()
    q, k, v, kw = H.fa_inputs(tsro, H.FA_CONFIGS["cfg3"])
    kw = dict(kw, new=(kw["n_kv"] - 1, kw["n_kv"]))
    kind = "reference" if oracle.Ref.available() else "port"
    if kind == "reference":
        ref = oracle.Ref()
        hs = [ref.fa_prepare(k, v, T=1, **kw) for _ in range(threads)]
        run = lambda i: ref.fa_run(hs[i], q)  # noqa: E731
    else:
        run = lambda i: tsro.fa(q, k, v, **kw)  # noqa: E731
    t0 = time.perf_counter()
    run(0)
    per = time.perf_counter() - t0
    n_each = calls if calls is not None else max(1, int(seconds / per / 1.0))
    done = [0] * threads

    def worker(i):
        for _ in range(n_each):
            run(i)
            done[i] += 1

    t0 = time.perf_counter()
    ths = [threading.Thread(target=worker, args=(i,)) for i in range(threads)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    el = time.perf_counter() - t0
    if kind == "reference":
        for h in hs:
            ref.fa_free(h)
    n = sum(done)
    gbs = n * fa_algo_bytes(FA["n_head_kv"], FA["D"], FA["G"], FA["n_kv"]) / el / 1e9
    return gbs, kind, f"{n} full config-3 FA calls in {el:.1f} s ({threads} threads, one call per thread at a time)", el / max(1, n_each)


def run_fa(args):
    """--config cfg3: FA decode over the q8_0 KV cache; KV heads sharded over the ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import tsrc
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    if FA["n_head_kv"] % world:
        raise SystemExit(f"cfg3 shards 8 KV heads: --gpus must divide 8, not {world}")
    dev = tsrc.Device(local)
    steps = args.steps if args.steps != 50000 else 5000
    with Clocks(local) as clk:
        ms, ms_e2e, info = fa_measure(dev, tsrc, torch, steps, args.warmup, world, rank, dist)
    total = fa_algo_bytes(FA["n_head_kv"], FA["D"], FA["G"], FA["n_kv"])
    shard = fa_algo_bytes(FA["n_head_kv"] // world, FA["D"], FA["G"], FA["n_kv"])
    us = ms * 1e3 / steps
    peak, peak_kind = peaks()
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        threads = len(os.sched_getaffinity(0))
        gbs, kind, sample, _ = cpu_reference_fa(args.cpu_seconds, threads)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}
    traffic = None
    prof = os.path.join(ROOT, "profiles", "traffic_cfg3.json")
    if os.path.exists(prof):
        with open(prof) as f:
            t = json.load(f).get("dram_bytes_per_launch")
        traffic = None if t is None else int(t // world)        # measured on one GPU (8 KV heads)
    line = {
        "metric": "FA decode HBM GB/s (q8_0 KV cache)", "value": round(steps * total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms / steps, 6),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) K, V through KVST, N(0,1) q)",
        "config": {"workload": CONFIGS["cfg3"][5], "parallelism": f"kv-head split x{world}" if world > 1 else "single",
                   "l2": f"inputs larger than L2: ring of {info['ring']} caches, {info['ring_mb_per_gpu']} MB per GPU",
                   "cuda_graph": info["cuda_graph"], "collective": "NCCL all_gather of out" if world > 1 else None},
        "roofline": {"bound": "hbm", "achieved": round(shard / (us * 1e-6) / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(shard / (us * 1e-6) / 1e9 / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": "fa_chunk_kernel<128> + fa_merge_kernel<4> (one step)", "us_per_launch": round(us, 3),
                     "algorithmic_bytes_per_launch": shard},
        "e2e": {"value": round(info["e2e_steps"] * total / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": info["h2d_bytes_per_step"], "d2h_bytes_per_step": info["d2h_bytes_per_step"],
                "ms_per_step": round(ms_e2e / info["e2e_steps"], 6), "cuda_graph": info["e2e_cuda_graph"],
                "pipelined": f"later steps' copies in and earlier steps' copies out overlap step i's FA (two copy streams, {E2E_BUFFERS} rotating device buffers)"},
        "gpu_launches": 2 * steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_model(args):
    """--config cfg4 / cfg5: end-to-end decode tokens/s of the random-init model on one GPU."""
    import torch
    import tsrc
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    spec = MODELS[args.config]
    if world > 1:
        return run_model_tp(args, spec, world, rank)
    args.warmup = min(args.warmup, 8)                      # decode tokens before timing (>= 3)
    steps = max(1, min(args.steps, spec["decode"] - args.warmup))
    torch.cuda.set_device(0)
    dev = tsrc.Device(0)
    with Clocks(0) as clk:
        r, model = model_measure(dev, tsrc, torch, args.config, steps, args.warmup)
    clocks = clk.summary()
    cpu = None
    if args.cpu_seconds > 0:
        threads = len(os.sched_getaffinity(0))
        tps, kind, sample = cpu_reference_model(args.config, threads, model)
        cpu = {"value": round(tps, 4), "unit": "tokens/s", "cores": threads, "kind": kind, "sample": sample}
    model.free()
    dev.close()
    peak, peak_kind = peaks()
    s = r["shape"]
    achieved = r["algo_bytes"] / (r["ms"] * 1e-3) / 1e9
    line = {
        "metric": "decode tokens/s", "value": round(1e3 / r["ms"], 2), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(r["ms"], 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (random-init weights quantized on device, random token ids)",
        "config": {"workload": spec["desc"], "prompt_tokens": spec["prompt"], "kv_cells_during_timing": list(r["n_kv"]),
                   "l2": "inputs larger than L2 (every decode token reads all weights: "
                         f"{r['algo_bytes'] / 1e6:.0f} MB)", "cuda_graph": "one graph launch per token (tsrc_model_decode)",
                   "prefill_ms": round(r["prefill_ms"], 2),
                   "prefill_tokens_per_s": round(spec["prompt"] / (r["prefill_ms"] * 1e-3), 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None, "peak_kind": peak_kind, "kernel": "whole decode step (all kernels)",
                     "algorithmic_bytes_per_step": r["algo_bytes"]},
        "e2e": {"value": round(1e3 / r["e2e_ms"], 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * s["n_vocab"], "ms_per_step": round(r["e2e_ms"], 4)},
        "gpu_launches": r["launches"] * steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_model_tp(args, spec, world, rank):
    """--config cfg4 / cfg5 on N > 1 GPUs: decode tokens/s of the model split over the GPUs."""
    import datetime
    import torch
    import torch.distributed as dist
    import tsrc
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    s = spec["shape"]
    if s["n_head_kv"] % world:
        if rank == 0:
            print(json.dumps({"metric": "decode tokens/s", "impl": "ours", "n_gpus": world,
                              "unavailable": f"{s['n_head_kv']} KV heads do not split over {world} GPUs"}), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return 0
    args.warmup = min(args.warmup, 8)
    steps = max(1, min(args.steps, spec["decode"] - args.warmup))
    dev = tsrc.Device(local)
    with Clocks(local) as clk:
        r, model, team = model_measure_tp(dev, tsrc, torch, dist, args.config, steps, args.warmup, rank, world)
    clocks = clk.summary()
    dist.barrier()
    model.free()
    team.free()
    peak, peak_kind = peaks()
    achieved = r["algo_bytes"] / (r["ms"] * 1e-3) / 1e9
    line = {
        "metric": "decode tokens/s", "value": round(1e3 / r["ms"], 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(r["ms"], 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (random-init weights quantized on device, random token ids)",
        "config": {"workload": spec["desc"], "parallelism": f"tensor-parallel x{world} (heads, rows)",
                   "kv_cells_during_timing": list(r["n_kv"]), "prompt_tokens": spec["prompt"],
                   "prefill_ms": round(r["prefill_ms"], 2),
                   "prefill_tokens_per_s": round(spec["prompt"] / (r["prefill_ms"] * 1e-3), 1),
                   "collective": "tagged-word gathers over NVLink (attention output, SWIGLU row; fused into o, down, head)",
                   "l2": f"inputs larger than L2 (a token reads {r['algo_bytes'] / 1e6:.0f} MB over all GPUs)", "cuda_graph": True},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak * world, "unit": "GB/s",
                     "frac": round(achieved / (peak * world), 4), "traffic": None, "peak_kind": peak_kind + " x GPUs",
                     "kernel": "whole decode step (all kernels, all GPUs)", "algorithmic_bytes_per_step": r["algo_bytes"]},
        "e2e": {"value": round(1e3 / r["e2e_ms"], 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * r["shape"]["n_vocab"], "ms_per_step": round(r["e2e_ms"], 4)},
        "gpu_launches": r["launches"] * steps,
        "clocks": clocks,
        "cpu_baseline": None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dev.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_reference(args, cfg):
    """--impl reference: the reference's own CPU implementation of the path, rank 0 only."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.config in MODELS:
        threads = len(os.sched_getaffinity(0))
        tps, kind, sample = cpu_reference_model(args.config, threads)
        line = {
            "impl": "reference", "metric": "decode tokens/s", "value": round(tps, 4), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 0, "ms_per_step": round(1e3 / tps, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded weights quantized on the host)",
            "config": {"workload": MODELS[args.config]["desc"], "host_threads": threads},
            "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    if args.config == "cfg3":
        threads = len(os.sched_getaffinity(0))
        n_each = max(1, min(args.steps, 3))
        gbs, kind, sample, per = cpu_reference_fa(0, threads, calls=n_each)
        line = {
            "impl": "reference", "metric": "FA decode HBM GB/s (q8_0 KV cache)", "value": round(gbs, 4), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": 0, "ms_per_step": round(per * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded N(0,1) K, V, q)", "config": {"workload": CONFIGS["cfg3"][5], "host_threads": threads},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    fmt, N, K, ws, xs, desc = cfg
    threads = len(os.sched_getaffinity(0))
    x = np.random.default_rng(xs).standard_normal((1, K), dtype=np.float32)
    # calibrate one full matvec, then size each step's row sample so the run ends in ~2 minutes
    _, kind, _, t_full = cpu_reference_matvec(fmt, N, K, x, 0.5, threads)
    steps_total = args.steps + args.warmup
    budget = 120.0 / max(1, steps_total)
    S = int(min(N, max(16 * threads, N * budget / t_full)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle
    import helpers as H
    tsro = oracle.Tsro()
    w = H.weights(tsro, fmt, min(S, 2048), K, 999)
    w = np.ascontiguousarray(np.tile(w, (math.ceil(S / w.shape[0]), 1))[:S])
    if kind == "reference":
        ref = oracle.Ref()
        rows = ref.repack(fmt, w, K)
        y = np.zeros((1, S), np.float32)
        step = lambda: ref.matvec_repacked(fmt, rows, K, x, threads=threads, out=y)  # noqa: E731
    else:
        step = lambda: tsro.matvec(fmt, w, K, x, threads=threads)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    bytes_step = algo_bytes(fmt, S, K)
    v = args.steps * bytes_step / el / 1e9
    sample = f"rows [0, {S}) of {N} per step ({threads} host threads)"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activation)",
        "config": {"workload": desc, "row_sample": S, "host_threads": threads},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg2", choices=list(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-fa", action="store_true", help="skip the config-3 FA summary in the default line")
    ap.add_argument("--no-prefill", action="store_true", help="skip the tensor-core prefill summary in the default line")
    ap.add_argument("--no-model", action="store_true", help="skip the config 4 / 5 decode summaries in the default line")
    ap.add_argument("--collective", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1 matvec: all-gather fused into the kernel (P2P stores) or an NCCL all_gather")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.config == "cfg3":
        return run_fa(args)
    if args.config in MODELS:
        return run_model(args)

    import numpy as np
    import torch
    import torch.distributed as dist
    import tsrc

    fmt, N, K, ws, xs, desc = cfg
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = tsrc.Device(local)
    stream = torch.cuda.current_stream()

    # row shard of this rank (symmetric split R = ceil(N / world), sw/sim/tsr_ref.c:335-357)
    from tsrc import parallel
    R = (N + world - 1) // world
    row0, n_rows = parallel.row_shard(N, world, rank)
    shard_bytes = n_rows * row_bytes(fmt, K)
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    n_copies = max(2, math.ceil(4 * l2 / max(1, shard_bytes)))
    weights = [dev.synth(fmt, N, K, seed=ws + 1000 * c, row0=row0, n_rows=n_rows) for c in range(n_copies)]
    torch.cuda.synchronize()

    x = torch.from_numpy(np.random.default_rng(xs).standard_normal(K, dtype=np.float32)).cuda()
    y_loc = torch.zeros(n_rows, device="cuda")
    y_full = torch.zeros(R * world, device="cuda")
    team = None
    if world > 1 and args.collective == "p2p":
        # MUL_MAT with the all-gather fused in: rows stored into every rank's buffer over NVLink
        team = dev.team_create(rank, world, N)
        hs = [None] * world
        dist.all_gather_object(hs, team.ipc_handle)
        team.connect(b"".join(hs))

    def step(i):
        if team is not None:
            dev.mul_mat_allgather(team, weights[i % n_copies], x, y_full)
            return
        dev.mul_mat(weights[i % n_copies], x, y_loc, T=1)
        if world > 1:
            dist.all_gather_into_tensor(y_full, torch.nn.functional.pad(y_loc, (0, R - n_rows)))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, n):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn(n)
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # one CUDA graph of the ring of steps (on N > 1 GPUs the NCCL all-gathers are captured too)
    use_graph = not args.no_graph
    graph = None
    if use_graph:
        graph = capture(torch, lambda: [step(i) for i in range(n_copies)], barrier)
        use_graph = graph is not None

    # K steps = whole replays of the ring graph plus one replay of a graph of the remaining steps
    # (so no step of the timed region is an eager launch)
    rem_graph = None
    if graph is not None and args.steps % n_copies:
        rem_graph = capture(torch, lambda: [step(i) for i in range(args.steps % n_copies)], barrier)

    def value_loop(n):
        if graph is not None:
            reps, rem = divmod(n, n_copies)
            for _ in range(reps):
                graph.replay()
            if rem and rem_graph is not None and rem == args.steps % n_copies:
                rem_graph.replay()
            else:
                for i in range(rem):
                    step(i)
        else:
            for i in range(n):
                step(i)

    # kernel-only loop: the MUL_MAT kernel alone (QACT fused in it for one token) over the ring of
    # copies, replayed from a CUDA graph; on N > 1 GPUs this excludes the all-gather
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph):
        for i in range(n_copies):
            dev.mul_mat(weights[i], x, y_loc, T=1)
    kgraph.replay()
    torch.cuda.synchronize()
    n_kernel = max(n_copies, (min(args.steps, 20000) // n_copies) * n_copies)

    def kernel_loop(n):
        for _ in range(n // n_copies):
            kgraph.replay()

    # e2e: pinned host activation in, y out, through the public MUL_MAT call
    x_host = torch.from_numpy(np.random.default_rng(xs).standard_normal(K, dtype=np.float32)).pin_memory()
    y_host = torch.zeros(R * world if world > 1 else n_rows).pin_memory()
    n_e2e = min(args.steps, 20000)

    def e2e_step(i):
        x.copy_(x_host, non_blocking=True)
        step(i)
        y_host.copy_(y_full if world > 1 else y_loc, non_blocking=True)

    # (1) serial: copy in, MUL_MAT, copy out, one after the other on one stream
    egraph = capture(torch, lambda: [e2e_step(i) for i in range(n_copies)], barrier) if use_graph else None
    egraph_rem = (capture(torch, lambda: [e2e_step(i) for i in range(n_e2e % n_copies)], barrier)
                  if egraph is not None and n_e2e % n_copies else None)

    def e2e_serial(n):
        if egraph is not None:
            reps, rem = divmod(n, n_copies)
            for _ in range(reps):
                egraph.replay()
            if rem and egraph_rem is not None and rem == n_e2e % n_copies:
                egraph_rem.replay()
            else:
                for i in range(rem):
                    e2e_step(i)
        else:
            for i in range(n):
                e2e_step(i)

    # (2) pipelined over steps: step i's activation comes in on one copy stream while earlier steps
    # compute, and its result goes out on another while later steps compute (the device buffers
    # rotate over E2E_BUFFERS); every step still copies its own input in and its own result out
    xb = [x] + [torch.empty_like(x) for _ in range(E2E_BUFFERS - 1)]
    yb_loc = [y_loc] + [torch.empty_like(y_loc) for _ in range(E2E_BUFFERS - 1)]
    yb_full = [y_full] + [torch.empty_like(y_full) for _ in range(E2E_BUFFERS - 1)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def mm_step(i, b):
        if team is not None:
            dev.mul_mat_allgather(team, weights[i % n_copies], xb[b], yb_full[b])
            return
        dev.mul_mat(weights[i % n_copies], xb[b], yb_loc[b], T=1)
        if world > 1:
            dist.all_gather_into_tensor(yb_full[b], torch.nn.functional.pad(yb_loc[b], (0, R - n_rows)))

    def e2e_steps(n):
        pipelined(torch, n, lambda b: xb[b].copy_(x_host, non_blocking=True), mm_step,
                  lambda b: y_host.copy_(yb_full[b] if world > 1 else yb_loc[b], non_blocking=True), s_in, s_out)

    pgraph = capture(torch, lambda: e2e_steps(n_copies), barrier) if use_graph else None
    pgraph_rem = (capture(torch, lambda: e2e_steps(n_e2e % n_copies), barrier)
                  if pgraph is not None and n_e2e % n_copies else None)

    def e2e_loop(n):
        if pgraph is not None:
            reps, rem = divmod(n, n_copies)
            for _ in range(reps):
                pgraph.replay()
            if rem and pgraph_rem is not None and rem == n_e2e % n_copies:
                pgraph_rem.replay()
            elif rem:
                e2e_steps(rem)
        else:
            e2e_steps(n)

    kernel_loop(n_copies)
    e2e_loop(10)
    e2e_serial(10)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ms_value = timed(value_loop, args.steps)
        ms_kernel = timed(kernel_loop, n_kernel)
        ms_e2e = timed(e2e_loop, n_e2e)
        ms_e2e_serial = timed(e2e_serial, n_e2e)
    clocks = clk.summary()

    total_bytes = algo_bytes(fmt, N, K)
    shard_algo = n_rows * row_bytes(fmt, K) + 4 * K + 4 * n_rows
    value = args.steps * total_bytes / (ms_value * 1e-3) / 1e9
    e2e = n_e2e * total_bytes / (ms_e2e * 1e-3) / 1e9
    kern_us = ms_kernel * 1e3 / n_kernel
    achieved = shard_algo / (kern_us * 1e-6) / 1e9
    peak, peak_kind = peaks()

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        xn = x.cpu().numpy().reshape(1, K)
        threads = len(os.sched_getaffinity(0))
        gbs, kind, sample, _ = cpu_reference_matvec(fmt, N, K, xn, args.cpu_seconds, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}

    also = {}
    if world == 1 and not args.no_fa:
        ms_fa, ms_fa_e2e, info = fa_measure(dev, tsrc, torch, 2000, 20)
        fa_b = fa_algo_bytes(FA["n_head_kv"], FA["D"], FA["G"], FA["n_kv"])
        fa_us = ms_fa * 1e3 / 2000
        also["fa_cfg3"] = {"metric": "FA decode HBM GB/s (q8_0 KV cache)", "workload": CONFIGS["cfg3"][5],
                           "value": round(fa_b / (fa_us * 1e-6) / 1e9, 1), "unit": "GB/s", "us_per_step": round(fa_us, 3),
                           "frac": round(fa_b / (fa_us * 1e-6) / 1e9 / peak, 4),
                           "e2e_us_per_step": round(ms_fa_e2e * 1e3 / info["e2e_steps"], 3),
                           "l2": f"ring of {info['ring']} caches ({info['ring_mb_per_gpu']} MB)", "cuda_graph": True,
                           "full_line": "python bench.py --config cfg3"}

    if world == 1 and not args.no_prefill:
        also["prefill"] = prefill_measure(dev, tsrc, torch)
    if world == 1 and not args.no_model:
        for name in ("cfg5", "cfg4"):
            try:
                r, model = model_measure(dev, tsrc, torch, name, 64, 3, e2e_steps=16)
                entry = {"metric": "decode tokens/s", "workload": MODELS[name]["desc"], "value": round(1e3 / r["ms"], 2),
                         "unit": "tokens/s", "ms_per_token": round(r["ms"], 4), "steps": 64,
                         "e2e_tokens_per_s": round(1e3 / r["e2e_ms"], 2),
                         "prefill_tokens_per_s": round(MODELS[name]["prompt"] / (r["prefill_ms"] * 1e-3), 1),
                         "hbm_frac": round(r["algo_bytes"] / (r["ms"] * 1e-3) / 1e9 / peaks()[0], 4),
                         "full_line": f"python bench.py --config {name}"}
                if rank == 0 and args.cpu_seconds > 0:
                    tps, kind, sample = cpu_reference_model(name, len(os.sched_getaffinity(0)), model)
                    entry["cpu_baseline"] = {"value": round(tps, 4), "unit": "tokens/s", "kind": kind, "sample": sample}
                model.free()
            except Exception as e:  # noqa: BLE001
                entry = {"error": str(e)[:300]}
            also[f"decode_{name}"] = entry

    traffic = None
    prof = os.path.join(ROOT, "profiles", f"traffic_{args.config}.json")
    if os.path.exists(prof):
        with open(prof) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_value / args.steps, 6), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) activation)",
        "config": {"workload": desc, "rows_per_gpu": n_rows, "parallelism": f"row-split tp{world}" if world > 1 else "single",
                   "l2": f"inputs larger than L2: ring of {n_copies} weight copies, {n_copies * shard_bytes / 1e6:.0f} MB per GPU",
                   "cuda_graph": use_graph,
                   "collective": None if world == 1 else ("all-gather fused in the matvec kernel (P2P stores over NVLink)"
                                                           if team is not None else "NCCL all_gather of y")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, copied from the "
                                        "committed profile summary (not measured in this run)") if traffic else None,
                     "peak_kind": peak_kind,
                     "kernel": "dec_kernel (one-token MUL_MAT: QACT fused, weights staged in shared memory by TMA bulk copies)",
                     "us_per_launch": round(kern_us, 3),
                     "algorithmic_bytes_per_launch": shard_algo},
        "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * K,
                "d2h_bytes_per_step": 4 * (R * world if world > 1 else n_rows),
                "ms_per_step": round(ms_e2e / n_e2e, 6), "cuda_graph": pgraph is not None,
                "pipelined": f"later steps' copies in and earlier steps' copies out overlap step i's MUL_MAT (two copy streams, {E2E_BUFFERS} rotating device buffers)",
                "serial_value": round(n_e2e * total_bytes / (ms_e2e_serial * 1e-3) / 1e9, 2),
                "serial_ms_per_step": round(ms_e2e_serial / n_e2e, 6)},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if also:
        line["also"] = also
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph, kgraph, egraph, pgraph, rem_graph, egraph_rem, pgraph_rem
    if world > 1:
        dist.barrier()
    if team is not None:
        team.free()
    for w in weights:
        w.free()
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
