"""Sequence-parallel decode across 2 GPUs: each rank decodes its page-aligned
KV range to a partial (m, l, acc), and the states are merged through an NCCL
all-gather, by reading the peers' memory over NVLink (PeerMerge), or inside
the decode's combine kernel over NVLink (SeqParallelExchange); the result must
match the single-GPU decode of the whole sequence.  Skipped when
fewer than 2 GPUs are visible.  NVLS is off and the peer buffers are plain
point-to-point mappings."""
import os

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gen_kv

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, k, v, q, ret, how="nccl"):
    import torch.distributed as dist
    from int4_kivi import store_kivi
    from int4_kivi.distributed import PeerMerge, SeqParallelExchange, seq_parallel_decode, split_tokens
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    a, b = split_tokens(k.shape[1], world, rank)
    c = store_kivi(k[:, a:b].contiguous().to(dev), v[:, a:b].contiguous().to(dev))
    st = dict(k_packed=c.k_packed, k_scale=c.k_scale, k_hot=c.k_hot, v_packed=c.v_packed, v_scale=c.v_scale,
              H=c.H, S=c.S, D=c.D, B=1)
    if how != "nccl":
        pm = (PeerMerge if how == "peer" else SeqParallelExchange)(q.shape[1], q.shape[2], dev)
        for _ in range(3):                       # reuse both buffer slots
            out = seq_parallel_decode(q.to(dev), st, q.shape[1], merger=pm)
        from int4_kivi import _native as N
        assert N.device_status(dev) == 0
        out = out.clone()
        with pytest.raises(ValueError):                 # shape the buffer was not made for
            seq_parallel_decode(q[:, :8].to(dev), st, 8, merger=pm)
        pm.close()
        pm.close()                                      # idempotent
        with pytest.raises(ValueError):
            seq_parallel_decode(q.to(dev), st, q.shape[1], merger=pm)
    else:
        out = seq_parallel_decode(q.to(dev), st, q.shape[1])
    ret[rank] = out.cpu()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("how", ["nccl", "peer", "fused"])
def test_seq_parallel_two_gpus(how):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from int4_kivi import store_kivi
    from int4_kivi.decode import decode_packed
    k, v, q = gen_kv(8, 5000, 128, seed=77, Hq=32)
    q = q[None, :, 0]
    ret = mp.Manager().dict()
    port = 29600 + os.getpid() % 300 + ["nccl", "peer", "fused"].index(how) * 7
    mp.spawn(_rank, args=(2, port, k, v, q, ret, how), nprocs=2, join=True)
    c = store_kivi(k.cuda(), v.cuda())
    st = dict(k_packed=c.k_packed, k_scale=c.k_scale, k_hot=c.k_hot, v_packed=c.v_packed, v_scale=c.v_scale,
              H=8, S=5000, D=128, B=1)
    want = decode_packed(q.cuda(), st, 32).cpu().float()
    for r in range(2):
        got = ret[r].float()
        assert bool(((got - want).abs() <= 2e-3 + want.abs() * 2.0 ** -7).all())
