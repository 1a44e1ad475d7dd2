"""Host-side INT4-KIVI cache: the reference's `KIVICache`, `store_kivi` and
`dequant_kivi` (int4_kivi/cache.py:48-201), running on libkivi_sm100.

Scheme (unchanged from the reference):
    K = int4, per-channel over each 16-token page, fp16 scale per (head, channel, page);
        the trailing S % 16 tokens stay bf16 (the hot page, `k_hot`);
    V = int4, per-token over 16-channel blocks, fp16 scale per (head, token, block).
Codes are two's-complement nibbles, element 2j in the low nibble of byte j.

B200 layout detail: the packed tensors are views into buffers whose page /
token strides are rounded up to a multiple of 16 (capacity), so TMA can stage
them and new tokens can be appended in place.  Shapes, dtypes and values of
every field are exactly the reference's.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
from torch import Tensor

from . import _native as N

BLOCK = 16
QMAX = 7
N_ALPHAS = 32
PACK = BLOCK // 2
ALIGN = 16          # page / token capacity granularity


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclasses.dataclass
class KIVICache:
    """Packed INT4-KIVI K/V cache for one layer's [H, S, D] tensors."""

    k_packed: Tensor          # uint8 [H, D, NP, PACK]
    k_scale: Tensor           # fp16  [H, D, NP]
    k_hot: Tensor             # bf16  [H, S - n_full, D]
    v_packed: Tensor          # uint8 [H, S, ND, PACK]
    v_scale: Tensor           # fp16  [H, S, ND]
    H: int
    S: int
    D: int
    fmt: str = dataclasses.field(default="int4", repr=False, compare=False)

    @property
    def n_full(self) -> int:
        return (self.S // BLOCK) * BLOCK

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.k_packed, self.k_scale, self.k_hot, self.v_packed, self.v_scale))

    def bf16_nbytes(self) -> int:
        return 2 * (self.H * self.S * self.D) * 2

    def compression_ratio_vs_bf16(self) -> float:
        return self.bf16_nbytes() / max(self.nbytes, 1)


# --------------------------------------------------------------------------- #
# capacity-backed allocation
# --------------------------------------------------------------------------- #
def alloc_packed(H: int, S: int, D: int, device, scale_dtype, s_cap: Optional[int] = None, v_pack: int = PACK):
    """Zeroed capacity buffers (k_packed, k_scale, v_packed, v_scale) for up to
    s_cap tokens; page and token strides are multiples of 16.  v_pack is the
    last dim of v_packed: 8 bytes per V block, or 12 per block pair (the INT3
    V of the mixed cache, [H, S, D/32, 12])."""
    s_cap = _round_up(max(s_cap or S, S, 1), ALIGN * BLOCK)
    np_cap = s_cap // BLOCK
    ND = D // BLOCK
    kp = torch.zeros((H, D, np_cap, PACK), dtype=torch.uint8, device=device)
    ks = torch.zeros((H, D, np_cap), dtype=scale_dtype, device=device)
    vp = torch.zeros((H, s_cap, ND if v_pack == PACK else ND // 2, v_pack), dtype=torch.uint8, device=device)
    vs = torch.zeros((H, s_cap, ND), dtype=scale_dtype, device=device)
    return kp, ks, vp, vs


def cache_geometry(c) -> tuple[int, int]:
    """(k page stride, v token stride) of a cache's packed views; raises if the
    tensors are not views with the (page, token)-strided layout the kernels use.
    `c` is a cache object or a (k_packed, k_scale, v_packed, v_scale) tuple."""
    kp, ks, vp, vs = c if isinstance(c, tuple) else (c.k_packed, c.k_scale, c.v_packed, c.v_scale)
    np_stride = kp.stride(1) // PACK if kp.dim() == 4 else 0
    VP = vp.shape[3] if vp.dim() == 4 else PACK           # bytes per V block (pair)
    s_stride = vp.stride(0) // (vp.shape[2] * VP) if vp.dim() == 4 and vp.shape[2] else 0
    ok = (kp.dim() == 4 and kp.stride(3) == 1 and kp.stride(2) == PACK and kp.stride(1) == np_stride * PACK
          and kp.stride(0) == kp.shape[1] * np_stride * PACK
          and ks.dim() == 3 and ks.stride(2) == 1 and ks.stride(1) == np_stride and ks.stride(0) == ks.shape[1] * np_stride
          and vp.dim() == 4 and vp.stride(3) == 1 and vp.stride(2) == VP and vp.stride(1) == vp.shape[2] * VP
          and vp.stride(0) == s_stride * vp.shape[2] * VP
          and vs.dim() == 3 and vs.stride(2) == 1 and vs.stride(1) == vs.shape[2] and vs.stride(0) == s_stride * vs.shape[2])
    if not ok:
        raise ValueError("packed cache tensors do not have the page/token-strided layout")
    return max(np_stride, 1), max(s_stride, 1)


def relayout(c):
    """Copy a cache whose packed tensors are arbitrary (e.g. user-built or
    torch.cat'ed with odd page counts) into 16-aligned capacity buffers."""
    H, S, D = c.k_packed.shape[0], c.S, c.D
    kp, ks, vp, vs = alloc_packed(H, S, D, c.k_packed.device, c.k_scale.dtype, v_pack=c.v_packed.shape[3])
    NP = c.k_packed.shape[2]
    kp[:, :, :NP].copy_(c.k_packed); ks[:, :, :NP].copy_(c.k_scale)
    vp[:, :S].copy_(c.v_packed); vs[:, :S].copy_(c.v_scale)
    return kp[:, :, :NP], ks[:, :, :NP], vp[:, :S], vs[:, :S]


# --------------------------------------------------------------------------- #
# store / quantize
# --------------------------------------------------------------------------- #
def store_into(k: Optional[Tensor], v: Optional[Tensor], fmt: str, k_calib: str, v_calib: str,
               kp, ks, vp, vs, kpage0: int, vtok0: int, g_k: float = 1.0, g_v: float = 1.0,
               n_alphas: int = N_ALPHAS) -> None:
    """One store launch: whole 16-token K pages of k [H, S_k, D] to page kpage0
    and every token of v [H, S_v, D] to token vtok0 of the capacity buffers."""
    if k_calib not in N.CALIB or v_calib not in N.CALIB:
        raise ValueError(f"unknown calib {k_calib!r}/{v_calib!r}")
    ref = k if k is not None else v
    H, _, D = ref.shape
    S_k = k.shape[1] if k is not None else 0
    S_v = v.shape[1] if v is not None else 0
    if S_k // BLOCK == 0 and S_v == 0:
        return
    dt = N.DTYPE.get(ref.dtype)
    if dt not in (0, 1) or (k is not None and v is not None and k.dtype != v.dtype):
        raise ValueError("k/v must both be bf16 or fp16")
    al = N.alphas(ref.device, n_alphas)
    ksd = k.stride() if k is not None else (0, 0, 0)
    vsd = v.stride() if v is not None else (0, 0, 0)
    st = N.lib().kivi_store(
        N.ptr(k), N.ptr(v), dt, *ksd, *vsd, H, S_k, S_v, D, N.FMT[fmt], N.CALIB[k_calib],
        N.CALIB[v_calib], N.ptr(al), n_alphas, g_k, g_v, N.ptr(kp), N.ptr(ks), kpage0, kp.shape[2],
        N.ptr(vp), N.ptr(vs), vtok0, vp.shape[1], N.stream_of(ref))
    N.check(st, "kivi_store")


def store_kivi(k: Tensor, v: Tensor, k_calib: str = "mse", v_calib: str = "mse",
               capacity: Optional[int] = None) -> KIVICache:
    """Quantize K (per-channel) and V (per-token) into a KIVICache.

    k, v: bf16 [H, S, D] on CUDA (D a multiple of 16).  calib in {"absmax", "mse"}.
    `capacity` (tokens) reserves room for in-place `append_kivi`.
    """
    assert k.shape == v.shape, "k and v must share shape [H, S, D]"
    assert k.is_cuda and v.is_cuda, "inputs must be on CUDA"
    H, S, D = k.shape
    assert D % BLOCK == 0, "head_dim must be a multiple of 16"
    k = k.to(torch.bfloat16)
    v = v.to(torch.bfloat16)
    n_full = (S // BLOCK) * BLOCK
    NP = n_full // BLOCK
    kp, ks, vp, vs = alloc_packed(H, S, D, k.device, torch.float16, capacity)
    store_into(k, v, "int4", k_calib, v_calib, kp, ks, vp, vs, 0, 0)
    k_hot = k[:, n_full:].contiguous()
    return KIVICache(k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP], k_hot=k_hot,
                     v_packed=vp[:, :S], v_scale=vs[:, :S], H=H, S=S, D=D)


def full_views(c):
    """Capacity views (k_packed, k_scale, v_packed, v_scale) behind a cache."""
    np_stride, s_stride = cache_geometry(c)
    H, D = c.H, c.D
    ND = D // BLOCK
    kp = c.k_packed.as_strided((H, D, np_stride, PACK), c.k_packed.stride())
    ks = c.k_scale.as_strided((H, D, np_stride), c.k_scale.stride())
    vp = c.v_packed.as_strided((H, s_stride) + tuple(c.v_packed.shape[2:]), c.v_packed.stride())
    vs = c.v_scale.as_strided((H, s_stride, ND), c.v_scale.stride())
    return kp, ks, vp, vs


def append_kivi(cache, k_new: Tensor, v_new: Tensor, k_calib: str = "mse", v_calib: str = "mse"):
    """Append n new tokens [H, n, D] to a cache in place (the decode-step store).

    V is quantised for every new token; the K pages that the hot tail plus the
    new tokens complete are quantised per channel (one launch for both); the
    remainder becomes the new bf16 hot tail.  Capacity grows by copy when full.
    Works for INT4 (`KIVICache`) and NVFP4 (`NVFP4KIVICache`) caches.
    """
    H, n, D = k_new.shape
    assert (H, D) == (cache.H, cache.D) and v_new.shape == k_new.shape
    if n == 0:
        return cache
    S0, S1 = cache.S, cache.S + n
    try:
        kp, ks, vp, vs = full_views(cache)
        fits = vp.shape[1] >= S1 and kp.shape[2] >= S1 // BLOCK
    except ValueError:
        fits = False
    if not fits:
        kp, ks, vp, vs = alloc_packed(H, S1, D, k_new.device, cache.k_scale.dtype, s_cap=2 * S1,
                                      v_pack=cache.v_packed.shape[3])
        NP0 = cache.k_packed.shape[2]
        kp[:, :, :NP0].copy_(cache.k_packed); ks[:, :, :NP0].copy_(cache.k_scale)
        vp[:, :S0].copy_(cache.v_packed); vs[:, :S0].copy_(cache.v_scale)
    k_new = k_new.to(torch.bfloat16)
    v_new = v_new.to(torch.bfloat16)
    comb = torch.cat([cache.k_hot.to(torch.bfloat16), k_new], dim=1) if cache.k_hot.shape[1] else k_new
    nf = (comb.shape[1] // BLOCK) * BLOCK
    store_into(comb[:, :nf] if nf else None, v_new, cache.fmt, k_calib, v_calib, kp, ks, vp, vs,
               S0 // BLOCK, S0, getattr(cache, "g_k", 1.0), getattr(cache, "g_v", 1.0))
    cache.k_hot = comb[:, nf:].contiguous()
    cache.S = S1
    NP1 = S1 // BLOCK
    cache.k_packed, cache.k_scale = kp[:, :, :NP1], ks[:, :, :NP1]
    cache.v_packed, cache.v_scale = vp[:, :S1], vs[:, :S1]
    return cache


# --------------------------------------------------------------------------- #
# dequant
# --------------------------------------------------------------------------- #
def dequant_packed(cache) -> tuple[Tensor, Tensor]:
    """bf16 [H, S, D] K and V from any (INT4 / NVFP4) KIVI cache."""
    H, S, D = cache.H, cache.S, cache.D
    dev = cache.v_packed.device
    N.require_cuda(cache.v_packed)
    try:
        kp, ks, vp, vs = cache.k_packed, cache.k_scale, cache.v_packed, cache.v_scale
        np_stride, s_stride = cache_geometry(cache)
    except ValueError:
        kp, ks, vp, vs = relayout(cache)
        np_stride, s_stride = cache_geometry((kp, ks, vp, vs))
    kout = torch.empty((H, S, D), dtype=torch.bfloat16, device=dev)
    vout = torch.empty((H, S, D), dtype=torch.bfloat16, device=dev)
    st = N.lib().kivi_dequant(N.ptr(kp), N.ptr(ks), np_stride, N.ptr(vp), N.ptr(vs), s_stride, H, S, D,
                              N.FMT[cache.fmt], getattr(cache, "g_k", 1.0), getattr(cache, "g_v", 1.0),
                              N.ptr(kout), N.ptr(vout), kout.stride(0), kout.stride(1), kout.stride(2),
                              N.stream_of(kout))
    N.check(st, "kivi_dequant")
    n_full = (S // BLOCK) * BLOCK
    if n_full < S:
        kout[:, n_full:] = cache.k_hot.to(torch.bfloat16)
    return kout, vout


def dequant_kivi(cache: KIVICache) -> tuple[Tensor, Tensor]:
    """Dequantize a KIVICache back to (k_bf16, v_bf16), both [H, S, D]."""
    return dequant_packed(cache)
