"""Host-side multi-rank logic on CPU (gloo, world size 2): page-aligned sequence
splitting, sequence sharding, and the all-gather + log-sum-exp merge of partial
decode states, with per-rank partials computed by the CPU oracle."""
import math
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from int4_kivi.distributed import merge_partials_torch, plan_shards, shard_heads, shard_sequences, split_tokens


def test_split_tokens_page_aligned():
    for S in (1, 15, 16, 17, 1000, 262144, 262150):
        for W in (1, 2, 4, 8):
            rs = [split_tokens(S, W, r) for r in range(W)]
            assert rs[0][0] == 0 and rs[-1][1] == S
            for (a, b), (c, d) in zip(rs, rs[1:]):
                assert b == c and b % 16 == 0
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 16 + S % 16


def test_shard_sequences_balanced():
    rng = np.random.default_rng(0)
    lengths = rng.integers(1024, 32768, size=256).tolist()
    for W in (2, 4, 8):
        sh = shard_sequences(lengths, W)
        assert sorted(sum(sh, [])) == list(range(256))
        loads = [sum(lengths[i] for i in s) for s in sh]
        assert max(loads) / min(loads) < 1.01


def _partial_oracle(q, k, v, sm):
    """(m in log2 units, l, acc) of one KV range, double precision."""
    s = (q.double() @ k.double().T) * sm * (1 / math.log(2))          # [rows, T]
    m = s.max(dim=1).values
    p = torch.exp2(s - m[:, None])
    return m.float(), p.sum(1).float(), (p @ v.double()).float()


def _worker(rank, world, port, q, k, v, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, b = split_tokens(k.shape[0], world, rank)
    m, l, acc = _partial_oracle(q, k[a:b], v[a:b], 1 / math.sqrt(q.shape[1]))
    packed = torch.cat([m[:, None], l[:, None], acc], 1)
    gathered = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(gathered, packed)
    g = torch.stack(gathered)
    out = merge_partials_torch(g[:, :, 0], g[:, :, 1], g[:, :, 2:])
    ret[rank] = out
    dist.destroy_process_group()


def test_gloo_sequence_parallel_merge():
    torch.manual_seed(0)
    T, D, rows = 1000, 64, 4
    q, k, v = torch.randn(rows, D), torch.randn(T, D) * 2, torch.randn(T, D)
    mgr = mp.Manager()
    ret = mgr.dict()
    port = 29500 + os.getpid() % 1000
    mp.spawn(_worker, args=(2, port, q, k, v, ret), nprocs=2, join=True)
    ref = torch.softmax((q.double() @ k.double().T) / math.sqrt(D), -1) @ v.double()
    for r in range(2):
        assert (ret[r].double() - ref).abs().max().item() < 1e-5


def test_shard_heads_cover_all_heads():
    for Hkv in (1, 4, 8, 16):
        for W in (1, 2, 4, 8, 16):
            rs = [shard_heads(Hkv, W, r) for r in range(W)]
            assert rs[0][0] == 0 and rs[-1][1] == Hkv
            assert all(b == c for (_, b), (c, _) in zip(rs, rs[1:]))
            assert max(b - a for a, b in rs) - min(b - a for a, b in rs) <= 1
    with pytest.raises(ValueError):
        shard_heads(8, 2, 2)


def test_plan_shards_uses_every_rank():
    """Batches smaller than the world split kv heads so every rank has work;
    every (sequence, head) is decoded exactly once."""
    rng = np.random.default_rng(1)
    for B in (1, 2, 3, 4, 8, 64):
        lens = rng.integers(1024, 32769, size=B).tolist()
        for W in (1, 2, 4, 8):
            plan = plan_shards(lens, 8, W)
            cover = sorted((b, h) for units in plan for (b, h0, h1) in units for h in range(h0, h1))
            assert cover == [(b, h) for b in range(B) for h in range(8)]
            if B * 8 >= W:
                assert all(plan), (B, W, plan)


def _heads_worker(rank, world, port, q, k, v, ret):
    """Attention of this rank's kv-head range only (no collective on the data
    path); the host gathers the pieces only to check them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    Hkv, G = k.shape[0], q.shape[0] // k.shape[0]
    h0, h1 = shard_heads(Hkv, world, rank)
    outs = []
    for h in range(h0, h1):
        for j in range(G):
            s = (q[h * G + j].double() @ k[h].double().T) / math.sqrt(q.shape[1])
            outs.append(torch.softmax(s, -1) @ v[h].double())
    ret[rank] = (h0, h1, torch.stack(outs))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_kv_head_sharding():
    torch.manual_seed(1)
    Hkv, G, T, D = 8, 4, 300, 64
    q, k, v = torch.randn(Hkv * G, D), torch.randn(Hkv, T, D), torch.randn(Hkv, T, D)
    ret = mp.Manager().dict()
    mp.spawn(_heads_worker, args=(2, 29400 + os.getpid() % 90, q, k, v, ret), nprocs=2, join=True)
    assert [ret[r][:2] for r in range(2)] == [(0, 4), (4, 8)]
    out = torch.cat([ret[r][2] for r in range(2)])
    ref = torch.stack([torch.softmax((q[i].double() @ k[i // G].double().T) / math.sqrt(D), -1) @ v[i // G].double()
                       for i in range(Hkv * G)])
    assert (out - ref).abs().max().item() < 1e-12
