"""NVFP4-KIVI cache: e2m1 codes with fp8-e4m3 block scales in the KIVI geometry.

The reference ships this variant only inside its vLLM fork
(`nvfp4_kivi_store` / `_gather_dequant` / `_paged_decode`, called from
scripts/validate_nvfp4_kivi.py:44-77,136-150); that source is not part of the
repository, so the semantics here follow what the repository does contain:
  * grid and rounding: kv_quant.py:207-229 (`nvfp4`: e2m1 levels
    {0,.5,1,1.5,2,3,4,6}, bucketize with ties toward the smaller magnitude);
  * block scale stored as e4m3 and rounded inside the MSE clip search
    (scripts/diag_kernel_perchannel.py:30-48, WRITEUP.md:97-107), with the
    32-point alpha grid of kv_quant;
  * optional per-tensor fp32 scales g_k / g_v (WRITEUP.md:104-107 folds them
    to 1.0 by default): byte = e4m3(s / g), value = e2m1 * fp32(byte) * g.
Per token and kv-head the cache holds 64 + 8 + 64 + 8 = 144 bytes.

Layout mirrors KIVICache with 1-byte scales:
    k_packed u8 [H, D, NP, 8] (e2m1 nibble = sign << 3 | level index),
    k_scale  u8 [H, D, NP], k_hot bf16 [H, S % 16, D],
    v_packed u8 [H, S, D/16, 8], v_scale u8 [H, S, D/16].
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
from torch import Tensor

from .cache import BLOCK, KIVICache, alloc_packed, dequant_packed, store_into


@dataclasses.dataclass
class NVFP4KIVICache(KIVICache):
    g_k: float = 1.0
    g_v: float = 1.0

    def __post_init__(self):
        self.fmt = "nvfp4"


def store_nvfp4_kivi(k: Tensor, v: Tensor, k_calib: str = "mse", v_calib: str = "mse",
                     g_k: float = 1.0, g_v: float = 1.0, capacity: Optional[int] = None) -> NVFP4KIVICache:
    """Quantise bf16 k/v [H, S, D] (CUDA) into an NVFP4KIVICache."""
    assert k.shape == v.shape and k.is_cuda and v.is_cuda
    H, S, D = k.shape
    assert D % BLOCK == 0, "head_dim must be a multiple of 16"
    k = k.to(torch.bfloat16)
    v = v.to(torch.bfloat16)
    n_full = (S // BLOCK) * BLOCK
    NP = n_full // BLOCK
    kp, ks, vp, vs = alloc_packed(H, S, D, k.device, torch.uint8, capacity)
    store_into(k, v, "nvfp4", k_calib, v_calib, kp, ks, vp, vs, 0, 0, g_k, g_v)
    return NVFP4KIVICache(k_packed=kp[:, :, :NP], k_scale=ks[:, :, :NP], k_hot=k[:, n_full:].contiguous(),
                          v_packed=vp[:, :S], v_scale=vs[:, :S], H=H, S=S, D=D, g_k=g_k, g_v=g_v)


def dequant_nvfp4_kivi(cache: NVFP4KIVICache) -> tuple[Tensor, Tensor]:
    """bf16 [H, S, D] (K tail verbatim bf16)."""
    return dequant_packed(cache)
