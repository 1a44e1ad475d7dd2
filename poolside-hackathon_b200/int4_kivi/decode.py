"""Fused INT4-KIVI flash-decode attention (the reference's int4_kivi/decode.py
API, decode.py:177-533), running on libkivi_sm100's split-K decode kernels.

Single-query decode attention that reads the packed cache directly and
dequantises K and V in registers, with a log-sum-exp merge of the splits and
the bf16 hot-page tail folded into the merge.  The `split` / `block_n`
arguments of the reference are accepted for API compatibility; the B200
kernel sizes its own persistent grid from the SM count.

Public (unchanged signatures):
  kivi_decode_attention(q [Hq,1,D], cache, sm_scale=None, block_n=64) -> [Hq,1,D]
  kivi_decode_attention_batched(q [B,Hq,D], stacked, n_qh, sm_scale=None, split=8, block_n=64)
  kivi_decode_attention_gqa(q [B,Hq,D], stacked, n_qh, sm_scale=None, split=16, block_n=64)
  stack_caches([KIVICache, ...]) -> dict
and, beyond the reference (which decodes one token per call):
  kivi_decode_attention_multiquery(q [B,Tq,Hq,D], stacked, n_qh, sm_scale=None, q_pos=None)
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor

from . import _native as N
from .cache import BLOCK, PACK, KIVICache, alloc_packed, cache_geometry


def _stacked_geometry(st: dict) -> tuple[int, int, dict]:
    """(page stride, token stride, tensors) for a stacked dict, re-laid out into
    aligned buffers if needed (slow path for externally built dicts)."""
    try:
        nps, ss = cache_geometry((st["k_packed"], st["k_scale"], st["v_packed"], st["v_scale"]))
        return nps, ss, st
    except ValueError:
        BH, D, NP, _ = st["k_packed"].shape
        S = st["v_packed"].shape[1]
        kp, ks, vp, vs = alloc_packed(BH, S, D, st["k_packed"].device, st["k_scale"].dtype,
                                      v_pack=st["v_packed"].shape[3])
        kp[:, :, :NP].copy_(st["k_packed"]); ks[:, :, :NP].copy_(st["k_scale"])
        vp[:, :S].copy_(st["v_packed"]); vs[:, :S].copy_(st["v_scale"])
        out = dict(st, k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP], v_packed=vp[:, :S], v_scale=vs[:, :S])
        return kp.shape[2], vp.shape[1], out


def decode_packed(q: Tensor, st: dict, n_qh: int, sm_scale: Optional[float] = None,
                  fmt: Optional[str] = None, g_k: Optional[float] = None, g_v: Optional[float] = None,
                  out: Optional[Tensor] = None, partial: bool = False, v_hot: Optional[Tensor] = None,
                  exchange=None, check: bool = False):
    """Core entry: q [B, n_qh, D] bf16 over a stacked packed cache (B*H heads).

    Returns bf16 [B, n_qh, D], or with partial=True the merged per-row state
    (m [B*n_qh] in log2 units, l [B*n_qh], acc [B*n_qh, D]) for a cross-GPU
    log-sum-exp merge.  With v_hot (bf16 [B*H, S % 16, D]) the tail tokens'
    V is taken unquantised like their K (caches that keep the partial page in
    bf16); v_packed then only has to cover the paged tokens, and the packed
    tensors may be None when there is no full page yet.

    check=True synchronises after the launch and raises KiviError(status=5)
    if a bounded device wait ran out (the sync-free alternative for per-step
    callers is int4_kivi._native.poll_errors)."""
    res = _decode_packed(q, st, n_qh, sm_scale, fmt, g_k, g_v, out, partial, v_hot, exchange)
    if check:
        N.raise_device_status(q.device, "decode")
    return res


def _decode_packed(q, st, n_qh, sm_scale, fmt, g_k, g_v, out, partial, v_hot, exchange):
    B, H, S, D = st["B"], st["H"], st["S"], st["D"]
    fmt = st.get("fmt", "int4") if fmt is None else fmt
    g_k = st.get("g_k", 1.0) if g_k is None else g_k
    g_v = st.get("g_v", 1.0) if g_v is None else g_v
    N.require_cuda(q, st["v_packed"])
    assert q.shape == (B, n_qh, D), f"q must be [B={B}, n_qh={n_qh}, D={D}]"
    assert n_qh % H == 0, "n_q_heads must be a multiple of n_kv_heads"
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    q = q.to(torch.bfloat16)
    if q.stride(2) != 1:
        q = q.contiguous()
    if st["k_packed"] is None:                 # no full page yet (tail-only, v_hot path)
        assert v_hot is not None and S < 16, "packed tensors are required once a page is full"
        nps, ss = 1, 16
    else:
        nps, ss, st = _stacked_geometry(st)
    khot = st["k_hot"]
    if khot.shape[1] and not khot.is_contiguous():      # rows are addressed as (bh * hot_stride + j) * D
        khot = khot.contiguous()
    hot_stride = khot.shape[1]
    dev = q.device
    need = N.lib().kivi_decode_workspace_floats(B, n_qh, H, S, D)
    work = N.workspace(dev, need)
    err = N.err_flag(dev)
    L = N.lib()
    if partial:
        m = torch.empty(B * n_qh, dtype=torch.float32, device=dev)
        l = torch.empty(B * n_qh, dtype=torch.float32, device=dev)
        acc = torch.empty(B * n_qh, D, dtype=torch.float32, device=dev)
        rc = L.kivi_decode_partial(
            N.ptr(q), q.stride(0), q.stride(1), N.ptr(st["k_packed"]), N.ptr(st["k_scale"]), nps,
            N.ptr(khot) if hot_stride else None, hot_stride, N.ptr(st["v_packed"]), N.ptr(st["v_scale"]), ss,
            B, n_qh, H, S, D, N.FMT[fmt], sm_scale, g_k, g_v, N.ptr(m), N.ptr(l), N.ptr(acc),
            N.ptr(work), work.numel(), N.ptr(err), N.stream_of(q))
        N.check(rc, "kivi_decode_partial")
        return m, l, acc
    if out is None:
        out = torch.empty((B, n_qh, D), dtype=torch.bfloat16, device=dev)
    if exchange is not None:
        if partial or v_hot is not None or st.get("seq_lens") is not None:
            raise ValueError("exchange takes equal-length, fully packed caches and returns the merged output")
        x = exchange
        if x.closed or (x.rows, x.D) != (B * n_qh, D) or x.device != dev:
            raise ValueError(f"exchange buffer is for rows={x.rows}, D={x.D} on {x.device} "
                             f"(closed={x.closed}); this call needs rows={B * n_qh}, D={D} on {dev}")
        rc = L.kivi_decode_seqpar(
            N.ptr(q), q.stride(0), q.stride(1), N.ptr(st["k_packed"]), N.ptr(st["k_scale"]), nps,
            N.ptr(khot) if hot_stride else None, hot_stride, N.ptr(st["v_packed"]), N.ptr(st["v_scale"]), ss,
            B, n_qh, H, S, D, N.FMT[fmt], sm_scale, g_k, g_v, x.own, N.ptr(x.peers), x.world, x.rank,
            N.ptr(x.row_epoch), x.timeout_ns, N.ptr(out), N.ptr(work), work.numel(), N.ptr(err), N.stream_of(q))
        N.check(rc, "kivi_decode_seqpar")
        return out
    if v_hot is not None and hot_stride:
        assert not partial and st.get("seq_lens") is None, "v_hot is for plain (non-partial, uniform) decode"
        vh = v_hot.to(torch.bfloat16)
        if vh.shape != khot.shape or not vh.is_contiguous():
            vh = vh.contiguous()
        assert vh.shape == khot.shape, "v_hot must match k_hot [B*H, S % 16, D]"
        pk = lambda name: N.ptr(st[name]) if st[name] is not None else None
        rc = L.kivi_decode_bf16_tail(
            N.ptr(q), q.stride(0), q.stride(1), pk("k_packed"), pk("k_scale"), nps, N.ptr(khot), N.ptr(vh),
            hot_stride, pk("v_packed"), pk("v_scale"), ss, B, n_qh, H, S, D, N.FMT[fmt], sm_scale, g_k, g_v,
            N.ptr(out), N.ptr(work), work.numel(), N.ptr(err), N.stream_of(q))
        N.check(rc, "kivi_decode_bf16_tail")
        return out
    if st.get("seq_lens") is not None:
        sl = st["seq_lens"]
        assert sl.is_cuda and sl.dtype == torch.int32 and sl.numel() == B
        rc = L.kivi_decode_varlen(
            N.ptr(q), q.stride(0), q.stride(1), N.ptr(st["k_packed"]), N.ptr(st["k_scale"]), nps,
            N.ptr(khot), hot_stride, N.ptr(st["v_packed"]), N.ptr(st["v_scale"]), ss, N.ptr(sl),
            B, n_qh, H, S, D, N.FMT[fmt], sm_scale, g_k, g_v, N.ptr(out), N.ptr(work), work.numel(),
            N.ptr(err), N.stream_of(q))
        N.check(rc, "kivi_decode_varlen")
        return out
    rc = L.kivi_decode(
        N.ptr(q), q.stride(0), q.stride(1), N.ptr(st["k_packed"]), N.ptr(st["k_scale"]), nps,
        N.ptr(khot) if hot_stride else None, hot_stride, N.ptr(st["v_packed"]), N.ptr(st["v_scale"]), ss,
        B, n_qh, H, S, D, N.FMT[fmt], sm_scale, g_k, g_v, N.ptr(out), N.ptr(work), work.numel(),
        N.ptr(err), N.stream_of(q))
    N.check(rc, "kivi_decode")
    return out


def kivi_decode_attention_multiquery(q: Tensor, stacked: dict, n_qh: int, sm_scale: Optional[float] = None,
                                     q_pos: Optional[int] = None, v_hot: Optional[Tensor] = None) -> Tensor:
    """Decode Tq query tokens per sequence at once (a speculative-decoding
    verify step, or a small prefill chunk): q [B, Tq, n_qh, D] bf16 over a
    stacked cache that already holds the queries' own K/V; query j sits at
    position q_pos + j (default S - Tq, the last Tq tokens) and attends
    tokens 0 .. q_pos + j.  Returns bf16 [B, Tq, n_qh, D].  With v_hot
    (bf16 [B*H, S % 16, D]) the partial page's V is taken unquantised like
    its K, and the packed tensors may be None while no page is full.

    The reference decodes one token per call (decode.py:439-477).  Here the
    (query, head) pairs of each kv head share one pass over its pages; the
    queries go in chunks of at most 8 // group per launch so each launch stays
    on the tensor-core fast path."""
    B, H, S, D = stacked["B"], stacked["H"], stacked["S"], stacked["D"]
    fmt = stacked.get("fmt", "int4")
    assert q.dim() == 4 and q.shape[0] == B and q.shape[2] == n_qh and q.shape[3] == D, \
        f"q must be [B={B}, Tq, n_qh={n_qh}, D={D}]"
    assert n_qh % H == 0, "n_q_heads must be a multiple of n_kv_heads"
    assert stacked.get("seq_lens") is None, "multi-query decode takes equal-length caches"
    N.require_cuda(q, stacked["v_packed"])
    Tq = q.shape[1]
    q_pos = S - Tq if q_pos is None else q_pos
    if q_pos < 0 or q_pos + Tq > S:
        raise ValueError(f"queries at {q_pos}..{q_pos + Tq - 1} are outside the {S}-token cache")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    q = q.to(torch.bfloat16)
    if q.stride(3) != 1:
        q = q.contiguous()
    if stacked["k_packed"] is None:            # no full page yet (tail-only, v_hot path)
        assert v_hot is not None and S < 16, "packed tensors are required once a page is full"
        nps, ss, st = 1, 16, stacked
    else:
        nps, ss, st = _stacked_geometry(stacked)
    khot = st["k_hot"]
    if khot.shape[1] and not khot.is_contiguous():      # rows are addressed as (bh * hot_stride + j) * D
        khot = khot.contiguous()
    vh = None
    if v_hot is not None and khot.shape[1]:
        vh = v_hot.to(torch.bfloat16).contiguous()
        assert vh.shape == khot.shape, "v_hot must match k_hot [B*H, S % 16, D]"
    pk = lambda name: N.ptr(st[name]) if st[name] is not None else None
    G = n_qh // H
    chunk = max(1, 8 // G)
    L = N.lib()
    outs = []
    for j0 in range(0, Tq, chunk):
        qc = q[:, j0:j0 + chunk]
        tc = qc.shape[1]
        work = N.workspace(q.device, L.kivi_decode_workspace_floats(B, tc * n_qh, H, S, D))
        oc = torch.empty((B, tc, n_qh, D), dtype=torch.bfloat16, device=q.device)
        N.check(L.kivi_decode_multiquery(
            N.ptr(qc), qc.stride(0), qc.stride(1), qc.stride(2), pk("k_packed"), pk("k_scale"), nps,
            N.ptr(khot) if khot.shape[1] else None, N.ptr(vh), khot.shape[1], pk("v_packed"), pk("v_scale"), ss,
            B, tc, q_pos + j0, n_qh, H, S, D, N.FMT[fmt], sm_scale, stacked.get("g_k", 1.0), stacked.get("g_v", 1.0),
            N.ptr(oc), N.ptr(work), work.numel(), N.ptr(N.err_flag(q.device)), N.stream_of(q)),
            "kivi_decode_multiquery")
        outs.append(oc)
    return outs[0] if len(outs) == 1 else torch.cat(outs, dim=1)


def _single(cache) -> dict:
    return dict(k_packed=cache.k_packed, k_scale=cache.k_scale, k_hot=cache.k_hot,
                v_packed=cache.v_packed, v_scale=cache.v_scale, H=cache.H, S=cache.S, D=cache.D,
                NP=cache.k_packed.shape[2], ND=cache.v_packed.shape[2], B=1)


def kivi_decode_attention(q: Tensor, cache: KIVICache, sm_scale: float | None = None,
                          block_n: int = 64) -> Tensor:
    """Fused decode attention over a packed INT4-KIVI cache.

    q: bf16 [n_q_heads, 1, D]; cache: KIVICache of one sequence.
    Returns bf16 [n_q_heads, 1, D]."""
    assert q.is_cuda and cache.k_packed.is_cuda
    n_qh, D = q.shape[0], cache.D
    assert q.shape[-1] == D
    assert n_qh % cache.H == 0, "n_q_heads must be a multiple of n_kv_heads"
    out = decode_packed(q.reshape(1, n_qh, D), _single(cache), n_qh, sm_scale,
                        fmt=cache.fmt, g_k=getattr(cache, "g_k", 1.0), g_v=getattr(cache, "g_v", 1.0))
    return out.reshape(n_qh, 1, D)


def kivi_decode_attention_batched(q: Tensor, stacked: dict, n_qh: int, sm_scale: float | None = None,
                                  split: int = 8, block_n: int = 64) -> Tensor:
    """Split-K batched fused decode. q [B, n_qh, D] bf16, stacked from stack_caches."""
    return decode_packed(q.reshape(stacked["B"], n_qh, stacked["D"]), stacked, n_qh, sm_scale,
                         fmt=stacked.get("fmt", "int4"), g_k=stacked.get("g_k", 1.0), g_v=stacked.get("g_v", 1.0))


def kivi_decode_attention_gqa(q: Tensor, stacked: dict, n_qh: int, sm_scale: float | None = None,
                              split: int = 16, block_n: int = 64) -> Tensor:
    """GQA-grouped split-K fused decode (fast path). q [B, n_qh, D] bf16."""
    return kivi_decode_attention_batched(q, stacked, n_qh, sm_scale, split, block_n)


def stack_caches(caches: list) -> dict:
    """Stack per-sequence caches into batched packed tensors (B*H front dim).

    Same keys and shapes as the reference (decode.py:480-491); the storage is
    16-aligned so the TMA fast path applies.  All caches must share S."""
    c0 = caches[0]
    H, S, D = c0.H, c0.S, c0.D
    assert all(c.H == H and c.D == D for c in caches), "stack_caches needs equal H and D"
    if any(c.S != S for c in caches):
        return _stack_varlen(caches)
    B = len(caches)
    NP = c0.k_packed.shape[2]
    kp, ks, vp, vs = alloc_packed(B * H, S, D, c0.k_packed.device, c0.k_scale.dtype, v_pack=c0.v_packed.shape[3])
    for b, c in enumerate(caches):
        kp[b * H:(b + 1) * H, :, :NP].copy_(c.k_packed)
        ks[b * H:(b + 1) * H, :, :NP].copy_(c.k_scale)
        vp[b * H:(b + 1) * H, :S].copy_(c.v_packed)
        vs[b * H:(b + 1) * H, :S].copy_(c.v_scale)
    d = dict(k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP],
             k_hot=torch.cat([c.k_hot for c in caches], dim=0),
             v_packed=vp[:, :S], v_scale=vs[:, :S],
             H=H, S=S, D=D, NP=NP, ND=D // BLOCK, B=B)
    if getattr(c0, "fmt", "int4") != "int4":
        d.update(fmt=c0.fmt, g_k=c0.g_k, g_v=c0.g_v)
    return d


def _stack_varlen(caches: list) -> dict:
    """Unequal lengths (an extension over the reference, which requires one S):
    the stacked buffers are sized for the longest sequence, each sequence's
    bf16 tail sits in k_hot[:, :S_b % 16], and `seq_lens` (int32, device)
    tells the decode kernel how many tokens each batch entry attends."""
    c0 = caches[0]
    H, D = c0.H, c0.D
    B = len(caches)
    S = max(c.S for c in caches)
    NP = S // BLOCK
    dev = c0.k_packed.device
    kp, ks, vp, vs = alloc_packed(B * H, S, D, dev, c0.k_scale.dtype, v_pack=c0.v_packed.shape[3])
    khot = torch.zeros(B * H, BLOCK, D, dtype=torch.bfloat16, device=dev)
    for b, c in enumerate(caches):
        npb = c.k_packed.shape[2]
        kp[b * H:(b + 1) * H, :, :npb].copy_(c.k_packed)
        ks[b * H:(b + 1) * H, :, :npb].copy_(c.k_scale)
        vp[b * H:(b + 1) * H, :c.S].copy_(c.v_packed)
        vs[b * H:(b + 1) * H, :c.S].copy_(c.v_scale)
        if c.k_hot.shape[1]:
            khot[b * H:(b + 1) * H, :c.k_hot.shape[1]].copy_(c.k_hot)
    d = dict(k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP], k_hot=khot, v_packed=vp[:, :S], v_scale=vs[:, :S],
             H=H, S=S, D=D, NP=NP, ND=D // BLOCK, B=B,
             seq_lens=torch.tensor([c.S for c in caches], dtype=torch.int32, device=dev))
    if getattr(c0, "fmt", "int4") != "int4":
        d.update(fmt=c0.fmt, g_k=c0.g_k, g_v=c0.g_v)
    return d


def lse_merge(m: Tensor, l: Tensor, acc: Tensor) -> Tensor:
    """Merge R partial states m/l [R, rows], acc [R, rows, D] -> bf16 [rows, D]
    (the reference's _combine_kernel semantics, decode.py:320-340)."""
    R, rows = m.shape
    D = acc.shape[-1]
    m, l, acc = m.float().contiguous(), l.float().contiguous(), acc.float().contiguous()
    out = torch.empty(rows, D, dtype=torch.bfloat16, device=m.device)
    N.check(N.lib().kivi_lse_merge(N.ptr(m), N.ptr(l), N.ptr(acc), R, rows, D, N.ptr(out), N.stream_of(m)),
            "kivi_lse_merge")
    return out
