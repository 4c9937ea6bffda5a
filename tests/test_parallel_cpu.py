"""Host logic of the multi-GPU path on CPU: row / KV-head shards and the gathers, run as two gloo
ranks (spawned processes) that each compute their shard with the oracle. The gathered result must
be the single-device result bit for bit, as the GPU ranks' results are (every output row is one
full dot product on one rank; a KV-head shard plans its chunks with the model's E)."""
import os
import socket

import numpy as np
import pytest

import helpers as H
from tsrc import parallel as P


def test_row_shards_cover_every_row_once():
    for N in (1, 7, 896, 4864, 14336, 14337):
        for world in (1, 2, 3, 4, 8):
            seen = []
            R = (N + world - 1) // world
            for r in range(world):
                r0, n = P.row_shard(N, world, r)
                assert n <= R
                seen.extend(range(r0, r0 + n))
            assert seen == list(range(N)), (N, world)


def test_kv_head_shards():
    assert [P.kv_head_shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 2), (4, 2), (6, 2)]
    with pytest.raises(ValueError):
        P.kv_head_shard(8, 3, 0)
    with pytest.raises(ValueError):
        P.row_shard(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, what):
    import sys
    import datetime
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "tesseract-npu_b200"))
    import torch
    import torch.distributed as dist
    import oracle
    import helpers as Hh
    from tsrc import parallel as Pp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    tsro = oracle.Tsro()
    try:
        if what == "matvec":
            for fmt, N, K, T in ((0, 301, 896, 2), (1, 257, 1024, 1)):
                w = Hh.weights(tsro, fmt, N, K, 91 + fmt)
                x = Hh.acts(K, T, 92 + fmt)
                r0, n = Pp.row_shard(N, world, rank)
                y = tsro.matvec(fmt, w[r0:r0 + n], K, x) if n else np.zeros((T, 0), np.float32)
                full = Pp.all_gather_rows(torch.from_numpy(np.ascontiguousarray(y)), N, world).numpy()
                if rank == 0:
                    np.save(os.path.join(out_dir, f"mv_{fmt}.npy"), full)
        else:
            # decode over 4 KV heads split in two; n_kv small enough that the chunk size comes from
            # n, not from PCAP (the oracle plans with the E of the heads it is given)
            D, nkvh, G, n_kv = 64, 4, 2, 300
            case = (D, nkvh, G, 1, n_kv, n_kv - 1, "causal", 4, 4, 9344, 0.125, 1.0, 0, 0, 93)
            q, k, v, kw = Hh.fa_inputs(tsro, case)
            h0, hn = Pp.kv_head_shard(nkvh, world, rank)
            rb = D // 32 * 34
            ks = np.ascontiguousarray(k[:, h0 * rb:(h0 + hn) * rb])
            vs = np.ascontiguousarray(v[:, h0 * rb:(h0 + hn) * rb])
            qs = np.ascontiguousarray(q[:, h0 * G:(h0 + hn) * G])
            kws = dict(kw, n_head=hn * G, n_head_kv=hn)
            rc, o = tsro.fa(qs, ks, vs, **kws)
            assert rc == 0
            full = Pp.all_gather_heads(torch.from_numpy(o), world).numpy()
            if rank == 0:
                np.save(os.path.join(out_dir, "fa.npy"), full)
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("what", ["matvec", "fa"])
def test_two_gloo_ranks_gather_the_single_device_result(tmp_path, tsro, what):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), what), nprocs=world, start_method="spawn",
                       join=True)
    if what == "matvec":
        for fmt, N, K, T in ((0, 301, 896, 2), (1, 257, 1024, 1)):
            w = H.weights(tsro, fmt, N, K, 91 + fmt)
            x = H.acts(K, T, 92 + fmt)
            np.testing.assert_array_equal(np.load(tmp_path / f"mv_{fmt}.npy").view(np.uint32),
                                          tsro.matvec(fmt, w, K, x).view(np.uint32))
    else:
        case = (64, 4, 2, 1, 300, 299, "causal", 4, 4, 9344, 0.125, 1.0, 0, 0, 93)
        q, k, v, kw = H.fa_inputs(tsro, case)
        rc, want = tsro.fa(q, k, v, **kw)
        assert rc == 0
        np.testing.assert_array_equal(np.load(tmp_path / "fa.npy").view(np.uint32), want.view(np.uint32))
