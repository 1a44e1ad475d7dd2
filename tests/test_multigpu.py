"""Sequence-parallel decode across 2 GPUs against the CPU oracle.

Each rank stores and decodes its page-aligned KV range to a partial state
(m, l, acc); the states are merged by an NCCL all-gather plus local merge, by
reading the peers' memory over NVLink (PeerMerge), or inside the decode's
combine kernel over NVLink (SeqParallelExchange).  Checked with the decode bar
of conftest.py against the oracle's attention over the whole sequence:
  * fp32 state: the ranks' partial states, all-gathered and merged in fp32;
  * bf16 output of the merge under test, on every rank, every step;
and every rank's output must be bit-identical to every other rank's (all of
them merge the same states in the same order).  Skipped with fewer than 2
GPUs.  NVLS is off; the peer buffers are plain point-to-point mappings.
Also: KV-head-group sharding (each rank its own kv heads and their q heads,
no collective) against the oracle."""
import math
import os

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from conftest import check_decode_bf16, check_decode_fp32, gen_kv

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, k, v, q, ret, how="nccl"):
    import torch.distributed as dist
    from int4_kivi import store_kivi
    from int4_kivi.decode import decode_packed
    from int4_kivi.distributed import (PeerMerge, SeqParallelExchange, merge_partials_torch, seq_parallel_decode,
                                       split_tokens)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    a, b = split_tokens(k.shape[1], world, rank)
    c = store_kivi(k[:, a:b].contiguous().to(dev), v[:, a:b].contiguous().to(dev))
    st = dict(k_packed=c.k_packed, k_scale=c.k_scale, k_hot=c.k_hot, v_packed=c.v_packed, v_scale=c.v_scale,
              H=c.H, S=c.S, D=c.D, B=1)
    qd = q.to(dev)
    # fp32 state: this rank's partial, all ranks' partials gathered and merged in fp32
    m, l, acc = decode_packed(qd, st, q.shape[1], partial=True)
    parts = [torch.empty_like(t)[None].repeat(world, *([1] * t.dim())) for t in (m, l, acc)]
    for t, g in zip((m, l, acc), parts):
        dist.all_gather_into_tensor(g, t.contiguous())
    ret[f"fp32_{rank}"] = merge_partials_torch(*parts).cpu()
    outs = []
    if how != "nccl":
        pm = (PeerMerge if how == "peer" else SeqParallelExchange)(q.shape[1], q.shape[2], dev)
        for _ in range(3):                       # reuse both buffer slots
            outs.append(seq_parallel_decode(qd, st, q.shape[1], merger=pm).clone())
        from int4_kivi import _native as N
        assert N.device_status(dev) == 0
        with pytest.raises(ValueError):                 # shape the buffer was not made for
            seq_parallel_decode(q[:, :8].to(dev), st, 8, merger=pm)
        pm.close()
        pm.close()                                      # idempotent
        with pytest.raises(ValueError):
            seq_parallel_decode(qd, st, q.shape[1], merger=pm)
    else:
        outs.append(seq_parallel_decode(qd, st, q.shape[1]))
    ret[f"out_{rank}"] = torch.stack([o.cpu() for o in outs])
    dist.barrier()
    dist.destroy_process_group()


def _oracle(k, v, q):
    kd, vd = oracle.dequant_int4(oracle.store_int4(k, v))
    return oracle.decode_attention(q.float(), kd[None], vd[None], 1.0 / math.sqrt(k.shape[-1]))


@pytest.mark.parametrize("how", ["nccl", "peer", "fused"])
def test_seq_parallel_two_gpus(how):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    k, v, q = gen_kv(8, 5000, 128, seed=77, Hq=32)
    q = q[None, :, 0]
    ret = mp.Manager().dict()
    port = 29600 + os.getpid() % 300 + ["nccl", "peer", "fused"].index(how) * 7
    mp.spawn(_rank, args=(2, port, k, v, q, ret, how), nprocs=2, join=True)
    want = _oracle(k, v, q)                                          # [1, 32, 128]
    for r in range(2):
        check_decode_fp32(ret[f"fp32_{r}"].reshape(want.shape), want, f"rank {r} fp32 state")
        for i, o in enumerate(ret[f"out_{r}"]):
            check_decode_bf16(o, want, f"rank {r} step {i} ({how})")
            assert torch.equal(o, ret["out_0"][0]), (r, i)


def _heads_rank(rank, world, port, k, v, q, ret):
    import torch.distributed as dist
    from int4_kivi import store_kivi
    from int4_kivi.decode import decode_packed, stack_caches
    from int4_kivi.distributed import shard_heads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    B, Hkv = k.shape[0], k.shape[1]
    G = q.shape[1] // Hkv
    h0, h1 = shard_heads(Hkv, world, rank)
    st = stack_caches([store_kivi(k[b, h0:h1].to(dev), v[b, h0:h1].to(dev)) for b in range(B)])
    out = decode_packed(q[:, h0 * G:h1 * G].contiguous().to(dev), st, (h1 - h0) * G)
    ret[rank] = (h0, h1, out.cpu())
    dist.barrier()
    dist.destroy_process_group()


def test_kv_head_sharding_two_gpus():
    """Each rank holds kv heads [h0, h1) of every sequence and decodes their
    q heads; no collective.  The concatenated outputs meet the decode bar."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    k, v, q = gen_kv(8, 3000, 128, seed=78, Hq=32, B=2)
    q = q[:, :, 0]
    ret = mp.Manager().dict()
    mp.spawn(_heads_rank, args=(2, 29950 + os.getpid() % 40, k, v, q, ret), nprocs=2, join=True)
    out = torch.cat([ret[r][2] for r in range(2)], dim=1)
    assert [ret[r][:2] for r in range(2)] == [(0, 4), (4, 8)]
    want = [_oracle(k[b], v[b], q[b:b + 1])[0] for b in range(2)]
    check_decode_bf16(out, torch.stack([torch.from_numpy(w) for w in want]), "head-sharded")
