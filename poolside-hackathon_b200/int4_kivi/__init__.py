"""int4_kivi: INT4-KIVI (and NVFP4-KIVI, INT4-K / INT3-V) KV-cache path on B200 (sm_100a).

Drop-in for the reference package of the same name (int4_kivi/__init__.py:14-25):
    store_kivi(k, v, k_calib="mse", v_calib="mse") -> KIVICache
    dequant_kivi(cache) -> (k_bf16, v_bf16)
    KIVICache  (.nbytes, .compression_ratio_vs_bf16())
    BLOCK, QMAX, N_ALPHAS, PACK
Kernels come from libkivi_sm100.so (hand-written CUDA, C ABI); there is no
Triton and no CPU fallback.
"""

from .cache import KIVICache, store_kivi, dequant_kivi, append_kivi, BLOCK, QMAX, N_ALPHAS, PACK
from .nvfp4 import NVFP4KIVICache, store_nvfp4_kivi, dequant_nvfp4_kivi
from .mixed import Int3VKIVICache, store_kivi_int3v, dequant_kivi_int3v

__all__ = [
    "KIVICache",
    "store_kivi",
    "dequant_kivi",
    "append_kivi",
    "NVFP4KIVICache",
    "store_nvfp4_kivi",
    "dequant_nvfp4_kivi",
    "Int3VKIVICache",
    "store_kivi_int3v",
    "dequant_kivi_int3v",
    "BLOCK",
    "QMAX",
    "N_ALPHAS",
    "PACK",
]
