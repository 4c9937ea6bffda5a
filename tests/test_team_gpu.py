"""The fused MUL_MAT + all-gather of a tensor-parallel team.

On one GPU: the team's flag protocol gives up a wait that nothing answers (rank 1 of a two-rank
team never runs) within its bound and reports it through tsrc_sync, with no fault and the context
usable afterwards. On two GPUs (skipped when the box has one): two processes, one per GPU, each
holding a row shard, gather the whole vector on both ranks over several steps (both halves of the
double buffer), bit for bit the single-GPU MUL_MAT.
"""
import os
import socket

import numpy as np
import pytest

import tsrc

pytestmark = pytest.mark.gpu


def test_team_wait_that_nobody_answers_is_reported(dev):
    import torch
    from tsrc import parallel as P
    N, K = 1000, 896
    t0 = dev.team_create(0, 2, N)
    t1 = dev.team_create(1, 2, N)
    try:
        t0.connect_local([t0, t1])
        r0, n = P.row_shard(N, 2, 0)
        w = dev.synth(tsrc.FMT_Q8_0, N, K, seed=5, row0=r0, n_rows=n)
        try:
            x = torch.randn(K, device="cuda")
            y = torch.zeros(N, device="cuda")
            dev.mul_mat_allgather(t0, w, x, y)
            with pytest.raises(tsrc.TsrcError) as ei:
                dev.sync()
            assert ei.value.code == tsrc.E_DEVICE
            dev.sync()                      # the error was read and cleared; the context still works
            y2 = torch.zeros(n, device="cuda")
            dev.mul_mat(w, x, y2, T=1)
            dev.sync()
            assert torch.equal(y[:n], y2)   # this rank's own rows arrived before the wait
        finally:
            w.free()
    finally:
        t0.free()
        t1.free()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import sys
    import datetime
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "tesseract-npu_b200"))
    import torch
    import torch.distributed as dist
    import tsrc as T
    from tsrc import parallel as P
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    dev = T.Device(rank)
    ok = True
    try:
        for fmt, N, K in ((T.FMT_Q4_K, 14336, 4096), (T.FMT_Q8_0, 4864, 896)):
            team = dev.team_create(rank, world, N)
            hs = [None] * world
            dist.all_gather_object(hs, team.ipc_handle)
            team.connect(b"".join(hs))
            r0, n = P.row_shard(N, world, rank)
            w = dev.synth(fmt, N, K, seed=11, row0=r0, n_rows=n)
            full = dev.synth(fmt, N, K, seed=11)
            g = torch.Generator(device="cuda").manual_seed(12)
            for step in range(5):
                x = torch.randn(K, device="cuda", generator=g)
                y = torch.full((N,), float("nan"), device="cuda")
                dev.mul_mat_allgather(team, w, x, y)
                ref = torch.zeros(N, device="cuda")
                dev.mul_mat(full, x, ref, T=1)
                dev.sync()
                ok = ok and torch.equal(y.view(torch.int32), ref.view(torch.int32))
            dist.barrier()
            w.free()
            full.free()
            team.free()
            dist.barrier()
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write("ok" if ok else "mismatch")
        dev.close()
        dist.destroy_process_group()


def test_two_gpus_gather_the_single_gpu_result(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok"
