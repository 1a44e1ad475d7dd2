"""Multi-GPU decode: one process per GPU, torch.distributed over NCCL.

Two regimes (the reference is single-GPU; these are B200-native additions):
  * sequence / kv-head sharding: independent decode per rank, no collective
    (`shard_sequences` balances sequences by token count);
  * sequence parallel for one long context (>= 128K tokens): the KV sequence
    is split in page-aligned contiguous ranges (`split_tokens`), each rank
    decodes its range to a partial softmax state (m, l, acc), the states are
    all-gathered (16.6 KB per rank at 32 heads x 128) and merged locally with
    the log-sum-exp kernel (`seq_parallel_decode`).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

BLOCK = 16


def split_tokens(S: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous token range [a, b) of rank `rank`: pages are dealt out evenly,
    boundaries fall on 16-token pages, the last rank also takes the tail."""
    n_pages = S // BLOCK
    a = (n_pages * rank // world) * BLOCK
    b = (n_pages * (rank + 1) // world) * BLOCK if rank + 1 < world else S
    return a, b


def shard_sequences(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of sequence indices to ranks, balancing
    the total tokens (= packed bytes) per rank."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        out[r].append(i)
        loads[r] += lengths[i]
    for o in out:
        o.sort()
    return out


def merge_partials_torch(m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor) -> torch.Tensor:
    """Reference math of the merge (m in log2 units) for host-side checks:
    m/l [R, rows], acc [R, rows, D] -> fp32 [rows, D]."""
    M = m.max(dim=0).values
    Mr = torch.where(torch.isinf(M), torch.zeros_like(M), M)
    w = torch.exp2(m - Mr)
    return (acc * w[..., None]).sum(0) / (l * w).sum(0)[..., None]


def seq_parallel_decode(q: torch.Tensor, stacked_shard: dict, n_qh: int, sm_scale: Optional[float] = None,
                        group=None, fmt: str = "int4") -> torch.Tensor:
    """Decode q [B, n_qh, D] over this rank's KV shard, all-gather the partial
    states over `group` (NCCL) and merge them; every rank returns the bf16
    output [B, n_qh, D]."""
    import torch.distributed as dist

    from .decode import decode_packed, lse_merge
    world = dist.get_world_size(group)
    m, l, acc = decode_packed(q, stacked_shard, n_qh, sm_scale, fmt=fmt,
                              g_k=stacked_shard.get("g_k", 1.0), g_v=stacked_shard.get("g_v", 1.0), partial=True)
    rows, D = acc.shape
    packed = torch.cat([m[:, None], l[:, None], acc], dim=1)           # [rows, D + 2]
    gathered = torch.empty((world,) + tuple(packed.shape), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    out = lse_merge(gathered[:, :, 0].contiguous(), gathered[:, :, 1].contiguous(),
                    gathered[:, :, 2:].contiguous())
    return out.reshape(q.shape)
