"""Mixed-precision KIVI cache: K INT4 per channel, V INT3 per token.

The reference names a 3-bit-V / 4-bit-K cache as its next step past the
uniform 4-bit floor (WRITEUP.md:336-339) and defines the INT3 grid in
kv_quant.py:215-217 (`int3`: round half to even, clamp to [-3, 3], scale =
absmax / 3 or the MSE clip search over the same 32-point alpha grid,
kv_quant.py:247-266).  It ships no packed INT3 store or decode, so the cache
layout below is this library's own:

    K exactly as KIVICache (INT4 codes, fp16 scale per channel and 16-token
      page, the S % 16 tail kept bf16 in k_hot);
    V codes against the fp32 block scale, the scale stored as fp16 (as every
      KIVI scale); a code c in [-3, 3] is kept as its low two bits L = c & 3
      and a sign bit s (c = L - 4s), blocks in pairs (2k, 2k + 1) of 12 bytes,
      three little-endian 32-bit words A_2k, A_2k+1, S_k:
        A_b: L of element i < 8 at bits 4i..4i+1, of element 8+i at 4i+2..4i+3;
        S_k: s of element i < 8 of block 2k+o at bit 4i+2o, of 8+i at 4i+1+2o;
        v_packed u8 [H, S, D/32, 12],  v_scale f16 [H, S, D/16]
      (D a multiple of 32).  `(A & 0x33333333) | (S-bits on bit 2)` is the
      block's INT4-style nibble word, so the decode kernel turns a staged tile
      into nibbles with a few logic operations per block.

Per token and kv-head the cache holds 64 + 16 + 48 + 16 = 144 bytes (160 for
INT4 KIVI, 512 for bf16).  The fused decode is libkivi_sm100's tensor-core
decode kernel: each warp turns its TMA-staged INT3 rows into 3-bit nibbles in
shared memory, then runs the INT4 PV path on them.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
from torch import Tensor

from .cache import BLOCK, KIVICache, alloc_packed, dequant_packed, store_into

PACK3 = 12          # bytes per packed pair of INT3 V blocks
QMAX3 = 3


@dataclasses.dataclass
class Int3VKIVICache(KIVICache):
    """KIVICache with INT3 V blocks (v_packed [H, S, D/32, 12])."""
    g_k: float = 1.0
    g_v: float = 1.0

    def __post_init__(self):
        self.fmt = "int4k_int3v"


def store_kivi_int3v(k: Tensor, v: Tensor, k_calib: str = "mse", v_calib: str = "mse",
                     capacity: Optional[int] = None) -> Int3VKIVICache:
    """Quantise bf16 k/v [H, S, D] (CUDA): K INT4 per channel, V INT3 per token.
    `capacity` (tokens) reserves room for in-place `append_kivi`."""
    assert k.shape == v.shape, "k and v must share shape [H, S, D]"
    assert k.is_cuda and v.is_cuda, "inputs must be on CUDA"
    H, S, D = k.shape
    assert D % (2 * BLOCK) == 0, "head_dim must be a multiple of 32 (INT3 V blocks go in pairs)"
    k = k.to(torch.bfloat16)
    v = v.to(torch.bfloat16)
    n_full = (S // BLOCK) * BLOCK
    NP = n_full // BLOCK
    kp, ks, vp, vs = alloc_packed(H, S, D, k.device, torch.float16, capacity, v_pack=PACK3)
    store_into(k, v, "int4k_int3v", k_calib, v_calib, kp, ks, vp, vs, 0, 0)
    return Int3VKIVICache(k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP], k_hot=k[:, n_full:].contiguous(),
                          v_packed=vp[:, :S], v_scale=vs[:, :S], H=H, S=S, D=D)


def dequant_kivi_int3v(cache: Int3VKIVICache) -> tuple[Tensor, Tensor]:
    """bf16 [H, S, D] K and V (K tail verbatim bf16)."""
    return dequant_packed(cache)
