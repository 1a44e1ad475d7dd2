"""Paged 4-bit KV cache (vLLM block layout): store, gather-dequant, fused decode.

Drop-in for the fork modules the reference calls
(``vllm/v1/attention/ops/triton_int4_kivi.py`` and ``triton_nvfp4_kivi.py``;
call sites: scripts/validate_paged_decode.py:21-25,59,72,91,
scripts/validate_store_equiv.py:22-25,50-51, scripts/validate_nvfp4_kivi.py:67-75,136-150,
scripts/bench_paged_decode.py:97-100, scripts/diag_kernel_perchannel.py:18-21,69-75).
Same names, argument order and meaning; every kernel comes from
libkivi_sm100.so (``kivi_paged_*``), there is no CPU path.

Cache: ``kv_cache`` uint8 ``[num_blocks, 2, 16, H, D/2 + D/16]``; dim 1 is K/V;
a row holds D/2 packed code bytes then D/16 e4m3 scale bytes.  V and the K
rows of a sequence's partial last block are quantised per token (16-channel
blocks); K of a full block is quantised per channel over its 16 tokens, the
block's 16 x D/16 scale bytes read as D per-channel scales (WRITEUP.md:82-95).
Whether a block is per channel follows from geometry only: block b of a
sequence of length L is full iff (b + 1) * 16 <= L.

Store semantics: a call that writes the last slot of a block (with the
block's earlier slots either at the consecutive indices before it, as vLLM
lays out a request's tokens, or already in the cache) quantises that block's
K per channel; the cache rows it did not receive are dequantised first.  Every
other token's K is stored per token.  Negative slots are padding and skipped.
"""
from __future__ import annotations

import math

import torch

from . import _native as N

BLOCK = 16
QMAX = 7
PAGE = 16


def int4_kivi_kv_cache_full_dim(head_size: int) -> int:
    """Row bytes per (slot, head): D/2 code bytes + D/16 scale bytes."""
    return head_size // 2 + head_size // 16


nvfp4_kivi_kv_cache_full_dim = int4_kivi_kv_cache_full_dim


def _same_device(*ts) -> None:
    devs = {t.device for t in ts if t is not None}
    if len(devs) > 1:
        raise ValueError(f"tensors are on different devices: {sorted(map(str, devs))}")


def _check_cache(kv_cache: torch.Tensor, head_size: int) -> int:
    if kv_cache.dtype != torch.uint8 or kv_cache.dim() != 5 or kv_cache.shape[1] != 2 or kv_cache.shape[2] != PAGE:
        raise ValueError("kv_cache must be uint8 [num_blocks, 2, 16, H, D/2 + D/16]")
    if kv_cache.shape[4] != int4_kivi_kv_cache_full_dim(head_size):
        raise ValueError(f"kv_cache last dim {kv_cache.shape[4]} != D/2 + D/16 for D={head_size}")
    if not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be contiguous")
    return kv_cache.shape[3]


def _store(fmt: str, key, value, kv_cache, slot_mapping, head_size, calib):
    N.require_cuda(key, value, kv_cache, slot_mapping)
    _same_device(key, value, kv_cache, slot_mapping)
    if calib not in N.CALIB:
        raise ValueError(f"unknown calib {calib!r} (expected one of {sorted(N.CALIB)})")
    H = _check_cache(kv_cache, head_size)
    if key.dim() != 3 or key.shape != value.shape or key.shape[1] != H or key.shape[2] != head_size:
        raise ValueError("key/value must be [num_tokens, num_kv_heads, head_size]")
    if key.dtype != value.dtype or key.dtype not in N.DTYPE:
        raise ValueError("key/value must share a bf16/fp16/fp32 dtype")
    n = key.shape[0]
    slots = slot_mapping.reshape(-1)[:n]
    if slots.dtype != torch.int64:
        slots = slots.to(torch.int64)
    slots = slots.contiguous()
    if slots.numel() < n:
        raise ValueError("slot_mapping shorter than the number of tokens")
    L = N.lib()
    N.check(L.kivi_paged_store(N.ptr(key), N.ptr(value), N.DTYPE[key.dtype],
                               key.stride(0), key.stride(1), key.stride(2),
                               value.stride(0), value.stride(1), value.stride(2),
                               n, H, head_size, N.FMT[fmt], N.CALIB[calib], N.ptr(slots), N.ptr(kv_cache),
                               kv_cache.shape[0], N.ptr(N.err_flag(key.device)), N.stream_of(key)),
            f"{fmt}_kivi_store")


def _gather(fmt, kv_cache, block_table, seq_lens, head_size, num_kv_heads, max_seq):
    N.require_cuda(kv_cache, block_table, seq_lens)
    _same_device(kv_cache, block_table, seq_lens)
    H = _check_cache(kv_cache, head_size)
    if H != num_kv_heads:
        raise ValueError(f"num_kv_heads {num_kv_heads} != cache heads {H}")
    bt = block_table.to(torch.int32).contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    B = bt.shape[0]
    k = torch.empty(B, H, max_seq, head_size, dtype=torch.bfloat16, device=kv_cache.device)
    v = torch.empty_like(k)
    L = N.lib()
    N.check(L.kivi_paged_gather_dequant(N.ptr(kv_cache), kv_cache.shape[0], N.ptr(bt), bt.shape[1], N.ptr(sl), B,
                                        H, head_size, N.FMT[fmt], max_seq, N.ptr(k), N.ptr(v),
                                        N.ptr(N.err_flag(kv_cache.device)), N.stream_of(kv_cache)),
            f"{fmt}_kivi_gather_dequant")
    return k, v


def _decode(fmt, q, kv_cache, block_table, seq_lens, sm_scale, out=None):
    N.require_cuda(q, kv_cache, block_table, seq_lens)
    _same_device(q, kv_cache, block_table, seq_lens, out)
    if q.dim() != 3 or q.dtype != torch.bfloat16 or q.stride(2) != 1:
        raise ValueError("q must be bf16 [B, num_q_heads, head_size] with a contiguous last dim")
    B, Hq, D = q.shape
    H = _check_cache(kv_cache, D)
    if Hq % H:
        raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {H}")
    bt = block_table if (block_table.dtype == torch.int32 and block_table.is_contiguous()) \
        else block_table.to(torch.int32).contiguous()
    sl = seq_lens if (seq_lens.dtype == torch.int32 and seq_lens.is_contiguous()) \
        else seq_lens.to(torch.int32).contiguous()
    if bt.dim() != 2 or bt.shape[0] != B or sl.numel() != B:
        raise ValueError("block_table must be [B, max_blocks] and seq_lens [B]")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=q.device)
    if out.shape != (B, Hq, D) or out.dtype not in (torch.bfloat16, torch.float32) or not out.is_contiguous():
        raise ValueError(f"out must be contiguous bf16 or fp32 [{B}, {Hq}, {D}]")
    L = N.lib()
    need = L.kivi_paged_decode_workspace_floats(B, Hq, H, bt.shape[1], D)
    work = N.workspace(q.device, need, kind="paged")
    entry = L.kivi_paged_decode if out.dtype == torch.bfloat16 else L.kivi_paged_decode_f32
    N.check(entry(N.ptr(q), q.stride(0), q.stride(1), N.ptr(kv_cache), kv_cache.shape[0], N.ptr(bt),
                                bt.shape[1], N.ptr(sl), B, Hq, H, D, N.FMT[fmt], float(sm_scale), N.ptr(out),
                                N.ptr(work), work.numel(), N.ptr(N.err_flag(q.device)), N.stream_of(q)),
            f"{fmt}_kivi_paged_decode")
    return out


# ---- INT4 (fork module triton_int4_kivi) ----
def int4_kivi_store(key, value, kv_cache, slot_mapping, head_size, calib: str = "mse"):
    """Quantise key/value [num_tokens, H, D] into kv_cache at slot_mapping."""
    _store("int4", key, value, kv_cache, slot_mapping, head_size, calib)


def int4_kivi_gather_dequant(kv_cache, block_table, seq_lens, head_size, num_kv_heads, max_seq):
    """Dense bf16 (k, v) [B, H, max_seq, D]; positions at or past seq_len are 0."""
    return _gather("int4", kv_cache, block_table, seq_lens, head_size, num_kv_heads, max_seq)


def int4_kivi_paged_decode(q, kv_cache, block_table, seq_lens, sm_scale=None, out=None):
    """One decode token per sequence: q bf16 [B, Hq, D] -> bf16 [B, Hq, D]
    (or, given an fp32 `out`, the normalised output before the bf16 cast)."""
    return _decode("int4", q, kv_cache, block_table, seq_lens, sm_scale, out)


# ---- NVFP4 (fork module triton_nvfp4_kivi) ----
def nvfp4_kivi_store(key, value, kv_cache, slot_mapping, head_size, calib: str = "mse"):
    _store("nvfp4", key, value, kv_cache, slot_mapping, head_size, calib)


def nvfp4_kivi_gather_dequant(kv_cache, block_table, seq_lens, head_size, num_kv_heads, max_seq):
    return _gather("nvfp4", kv_cache, block_table, seq_lens, head_size, num_kv_heads, max_seq)


def nvfp4_kivi_paged_decode(q, kv_cache, block_table, seq_lens, sm_scale=None, out=None):
    return _decode("nvfp4", q, kv_cache, block_table, seq_lens, sm_scale, out)
