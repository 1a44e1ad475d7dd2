"""Multi-GPU decode: one process per GPU, torch.distributed over NCCL.

Two regimes (the reference is single-GPU; these are B200-native additions):
  * sequence / kv-head sharding: independent decode per rank, no collective
    (`shard_sequences` balances sequences by token count, `shard_heads` deals
    out kv-head groups, `plan_shards` combines the two for small batches);
  * sequence parallel for one long context (>= 128K tokens): the KV sequence
    is split in page-aligned contiguous ranges (`split_tokens`), each rank
    decodes its range to a partial softmax state (m, l, acc), and the states
    (16.6 KB per rank at 32 heads x 128) are merged with log-sum-exp on every
    rank (`seq_parallel_decode`): either read directly from the peers' memory
    over NVLink (`PeerMerge`: CUDA IPC buffers + kivi_peer_publish /
    kivi_peer_merge) or all-gathered with NCCL and merged locally.
"""
from __future__ import annotations

import ctypes
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


def shard_heads(Hkv: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous kv-head range [h0, h1) of `rank` when the kv heads of every
    sequence are dealt out over `world` ranks (KV-head-group sharding).  Each
    rank decodes its kv heads and the GQA query heads that read them
    (q heads [h0*G, h1*G)), which needs no communication for the attention op:
    the reference's GQA kernel is one program per (sequence, kv head, split),
    int4_kivi/decode.py:466-472, so kv heads are independent.  With more
    ranks than heads the surplus ranks get an empty range."""
    if Hkv <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad shard request Hkv={Hkv} world={world} rank={rank}")
    return Hkv * rank // world, Hkv * (rank + 1) // world


def plan_shards(lengths: Sequence[int], Hkv: int, world: int) -> list[list[tuple[int, int, int]]]:
    """Units of decode work per rank as (sequence, h0, h1) triples, sharding by
    sequence and, when there are fewer sequences than ranks, by kv-head group
    too: every sequence's kv heads are split into f equal groups, f the
    smallest power of two (dividing Hkv) with len(lengths) * f >= world, and
    the (sequence, group) units are assigned longest-first to the least
    loaded rank (load = tokens x heads = packed bytes).  No unit needs data
    from another rank."""
    B = len(lengths)
    f = 1
    while B * f < world and f * 2 <= Hkv and Hkv % (f * 2) == 0:
        f *= 2
    hg = Hkv // f
    units = [(b, j * hg, (j + 1) * hg) for b in range(B) for j in range(f)]
    units.sort(key=lambda u: (-lengths[u[0]], u[0], u[1]))
    loads = [0] * world
    out: list[list[tuple[int, int, int]]] = [[] for _ in range(world)]
    for u in units:
        r = min(range(world), key=lambda j: (loads[j], j))
        out[r].append(u)
        loads[r] += lengths[u[0]] * (u[2] - u[1])
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


class _PeerBuffers:
    """One exchange buffer per rank, allocated by the library (cudaMalloc,
    zeroed) and mapped into every other rank with CUDA IPC handles that are
    all-gathered over the host: plain point-to-point peer mappings.
    `peers` is the device array of all ranks' buffer addresses."""

    def __init__(self, nbytes: int, device, group=None, timeout_s: float = 2.0):
        import torch.distributed as dist
        from . import _native as N
        self.N = N
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device("cuda", N.device_index(device))
        if nbytes <= 0:
            raise ValueError(f"unsupported exchange shape for world={self.world}")
        L = N.lib()
        with torch.cuda.device(self.device):
            self.own = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            self.opened = []
            failure = None
            try:
                N.check(L.kivi_peer_alloc(nbytes, ctypes.byref(self.own), handle), "kivi_peer_alloc")
            except Exception as ex:      # still take part in the gathers below
                failure = ex
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle) if failure is None else None, group=self.group)
            ptrs = []
            try:
                if failure is not None or any(h is None for h in handles):
                    raise failure or RuntimeError("a peer could not allocate its exchange buffer")
                for j, hj in enumerate(handles):
                    if j == self.rank:
                        ptrs.append(self.own.value)
                        continue
                    pj = ctypes.c_void_p()
                    N.check(L.kivi_peer_open((ctypes.c_char * 64).from_buffer_copy(hj), ctypes.byref(pj)),
                            "kivi_peer_open")
                    self.opened.append(pj)
                    ptrs.append(pj.value)
            except Exception as ex:      # reported to every rank below
                failure = ex
            # Every rank learns whether every open succeeded, so all of them
            # release their buffers and raise together; no rank is left
            # waiting in a later barrier for one that gave up.  Nothing has
            # read any exchange buffer yet: kernels run only after __init__.
            oks = [None] * self.world
            dist.all_gather_object(oks, failure is None, group=self.group)
            if not all(oks):
                self._release()
                if failure is not None:
                    raise failure
                raise RuntimeError(f"kivi_peer_open failed on rank(s) {[j for j, o in enumerate(oks) if not o]}")
        self.closed = False
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        dist.barrier(group=self.group)

    def _release(self) -> None:
        L = self.N.lib()
        with torch.cuda.device(self.device):
            for pj in self.opened:
                L.kivi_peer_close(pj)
            self.opened = []
            if self.own:
                L.kivi_peer_free(self.own)
                self.own = ctypes.c_void_p()

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier, so
        no peer still reads it).  Collective; a second call does nothing."""
        import torch.distributed as dist
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._release()
        self.closed = True


class PeerMerge(_PeerBuffers):
    """Merge of per-rank partial decode states (m, l, acc) through NVLink
    peer memory: kivi_peer_publish + kivi_peer_merge, two stream-ordered,
    graph-capturable launches after the partial decode."""

    def __init__(self, rows: int, D: int, device, group=None, timeout_s: float = 2.0):
        import torch.distributed as dist
        from . import _native as N
        world = dist.get_world_size(group or dist.group.WORLD)
        super().__init__(N.lib().kivi_peer_buffer_bytes(rows, D, world), device, group, timeout_s)
        self.rows, self.D = rows, D
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.out = torch.empty(rows, D, dtype=torch.bfloat16, device=self.device)

    def __call__(self, m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor) -> torch.Tensor:
        N, L = self.N, self.N.lib()
        if self.closed:
            raise ValueError("PeerMerge is closed")
        for name, t, shape in (("m", m, (self.rows,)), ("l", l, (self.rows,)), ("acc", acc, (self.rows, self.D))):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"{name} must be contiguous fp32 {list(shape)} on {self.device}, "
                                 f"got {t.dtype} {list(t.shape)} on {t.device}")
        stream = N.stream_of(acc)
        N.check(L.kivi_peer_publish(N.ptr(m), N.ptr(l), N.ptr(acc), self.rows, self.D, self.own,
                                    N.ptr(self.peers), self.world, self.rank, N.ptr(self.epoch), stream),
                "kivi_peer_publish")
        N.check(L.kivi_peer_merge(N.ptr(self.peers), self.world, self.rows, self.D, N.ptr(self.epoch),
                                  self.own, N.ptr(self.out), N.ptr(N.err_flag(acc.device)), self.timeout_ns,
                                  stream),
                "kivi_peer_merge")
        return self.out


class SeqParallelExchange(_PeerBuffers):
    """State of the fused sequence-parallel decode (kivi_decode_seqpar): the
    decode's own combine kernel publishes each output row's rank-local state
    and merges all ranks' states of that row from their memory, so a step is
    the split-K kernel plus one combine launch on every rank."""

    def __init__(self, rows: int, D: int, device, group=None, timeout_s: float = 2.0):
        import torch.distributed as dist
        from . import _native as N
        world = dist.get_world_size(group or dist.group.WORLD)
        super().__init__(N.lib().kivi_seqpar_buffer_bytes(rows, D, world), device, group, timeout_s)
        self.rows, self.D = rows, D
        self.row_epoch = torch.zeros(rows, dtype=torch.int32, device=self.device)


def seq_parallel_decode(q: torch.Tensor, stacked_shard: dict, n_qh: int, sm_scale: Optional[float] = None,
                        group=None, fmt: str = "int4", merger=None) -> torch.Tensor:
    """Decode q [B, n_qh, D] over this rank's KV shard and merge the partial
    states of all ranks; every rank returns the bf16 output [B, n_qh, D].
    `merger`: a SeqParallelExchange (merge fused into the decode's combine
    kernel over NVLink peer memory), a PeerMerge (partial decode, then
    publish + merge over peer memory), or None (NCCL all-gather over `group`
    and a local merge)."""
    import torch.distributed as dist

    from .decode import decode_packed, lse_merge
    if isinstance(merger, SeqParallelExchange):
        return decode_packed(q, stacked_shard, n_qh, sm_scale, fmt=fmt, g_k=stacked_shard.get("g_k", 1.0),
                             g_v=stacked_shard.get("g_v", 1.0), exchange=merger)
    m, l, acc = decode_packed(q, stacked_shard, n_qh, sm_scale, fmt=fmt,
                              g_k=stacked_shard.get("g_k", 1.0), g_v=stacked_shard.get("g_v", 1.0), partial=True)
    if merger is not None:
        return merger(m, l, acc).reshape(q.shape)
    world = dist.get_world_size(group)
    rows, D = acc.shape
    packed = torch.cat([m[:, None], l[:, None], acc], dim=1)           # [rows, D + 2]
    gathered = torch.empty((world,) + tuple(packed.shape), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    out = lse_merge(gathered[:, :, 0].contiguous(), gathered[:, :, 1].contiguous(),
                    gathered[:, :, 2:].contiguous())
    return out.reshape(q.shape)
