"""Tensor parallelism of the path over the GPUs of one box: which rows / KV heads a rank owns and
how the ranks' outputs are put back together.

The reference spreads a weight over its memory channels with a symmetric row split, R = ceil(N / C)
rows per channel (jwkim04/tesseract-npu sw/sim/tsr_ref.c:335-357); the same rule spreads MUL_MAT
rows over GPUs here. Every output row is one full-K dot product on one GPU, so a gathered result
is the single-GPU result bit for bit. Flash attention splits by KV heads (each rank owns
n_head_kv / world heads and their G query heads); a rank plans its chunks with the model's E
(``plan_n_head_kv`` of ``tsrc_fa_cfg``), so its rows are the single-device rows bit for bit.

The gathers use ``torch.distributed.all_gather`` and run on NCCL (GPU tensors) or gloo (CPU
tensors, as in the tests).
"""
from __future__ import annotations


def row_shard(N: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, n_rows) of rank's contiguous row block: R = ceil(N / world) rows per rank, the last
    ranks possibly shorter or empty."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    R = (N + world - 1) // world
    row0 = min(N, rank * R)
    return row0, max(0, min(R, N - row0))


def kv_head_shard(n_head_kv: int, world: int, rank: int) -> tuple[int, int]:
    """(first KV head, KV heads) of rank; the heads split evenly (world must divide n_head_kv)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if n_head_kv % world:
        raise ValueError(f"{n_head_kv} KV heads do not split over {world} ranks")
    h = n_head_kv // world
    return rank * h, h


def all_gather_rows(y_local, N: int, world: int, group=None):
    """y_local [..., n_rows] of every rank -> [..., N] in row order (ranks padded to R rows for the
    collective, the padding dropped)."""
    import torch
    import torch.distributed as dist
    R = (N + world - 1) // world
    pad = R - y_local.shape[-1]
    y = torch.nn.functional.pad(y_local, (0, pad)) if pad else y_local.contiguous()
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y, group=group)
    return torch.cat(parts, dim=-1)[..., :N]


def all_gather_heads(out_local, world: int, group=None):
    """out_local [T, heads of this rank, D] of every rank -> [T, all heads, D] in head order."""
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(out_local) for _ in range(world)]
    dist.all_gather(parts, out_local.contiguous(), group=group)
    return torch.cat(parts, dim=1)
