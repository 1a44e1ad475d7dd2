"""CPU oracle for the 4-bit KV-cache path -- TEST INFRASTRUCTURE ONLY.

This package is the checker: a C restatement (``kivi_oracle.c``) of the
reference's quantiser, packer, dequantiser and decode attention, wrapped with
ctypes/numpy.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm may import it; the product library
(``poolside-hackathon_b200/``) never does.

Reference behaviour restated (paths inside a1exxd0/poolside-hackathon):
  * kv_quant.py:16-42, 206-266, 299-321  -- calibration, grids, roundtrip
  * int4_kivi/triton_kernels.py:21-24, 109-131, 137-286 -- packing, store,
    dequant geometry; int4_kivi/cache.py:48-201 -- KIVICache layout
  * scripts/validate_int4_kivi_decode.py:37-84 -- fp32-exact decode reference
  * kv_quant.py:215-217 `int3` grid with the KIVI V geometry -- the V half
    of the mixed INT4-K / INT3-V cache (WRITEUP.md:336-339 names it; the
    reference has no packed INT3 layout, the 3-bit packing is this library's)
  * scripts/diag_kernel_perchannel.py:30-48, WRITEUP.md:97-107 -- e4m3 block
    scales rounded inside the MSE search (NVFP4 variant)
  * WRITEUP.md:82-95,117-124, scripts/validate_paged_decode.py:32-64,
    scripts/validate_store_equiv.py:34-65 -- the paged vLLM cache layout
    (store, gather-dequant; decode is gather + decode_attention)

Pinned against the reference by tests/golden/*.npz (made by
tests/golden/make_golden.py, which runs the reference's own Python on CPU).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_kivi.so")
_lib = None

FMT = {"int4": 0, "int3": 1, "nvfp4": 2}
CALIB = {"absmax": 0, "mse": 1}
LAYOUT = {"headdim": 0, "channel": 1}
BLOCK = 16
PACK = 8


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off, OpenMP)."""
    src = os.path.join(_HERE, "kivi_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "-B" if force else "liboracle_kivi.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "kivi_oracle.c")
        if not os.path.exists(_LIB_PATH) or (os.path.exists(src) and
                                             os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I, F, Lg = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_long
        L.orc_calibrate.argtypes = [P, Lg, I, I, P, I, P]
        L.orc_roundtrip.argtypes = [P, P, I, I, I, I, I, I, P, I]
        L.orc_store_int4.argtypes = [P, P, I, I, I, I, I, P, I, P, P, P, P]
        L.orc_dequant_int4.argtypes = [P, P, P, P, I, I, I, P, P]
        L.orc_store_nvfp4.argtypes = [P, P, I, I, I, I, I, P, I, F, F, P, P, P, P]
        L.orc_store_v3.argtypes = [P, I, I, I, I, P, I, P, P]
        L.orc_dequant_v3.argtypes = [P, P, I, I, I, P]
        L.orc_dequant_nvfp4.argtypes = [P, P, P, P, I, I, I, F, F, P, P]
        L.orc_decode_attention.argtypes = [P, P, P, P, I, I, I, I, I, F, P]
        L.orc_f32_to_f16.argtypes = [F]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_e4m3.argtypes = [F]
        L.orc_f32_to_e4m3.restype = ctypes.c_uint8
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_to_f32.restype = F
        L.orc_num_threads.restype = I
        L.orc_set_num_threads.argtypes = [I]
        L.orc_paged_calib.argtypes = [P, I, I]
        L.orc_paged_calib.restype = ctypes.c_uint8
        L.orc_paged_store.argtypes = [P, P, I, I, I, I, I, P, P, Lg]
        L.orc_paged_store.restype = I
        L.orc_paged_gather.argtypes = [P, Lg, P, Lg, P, I, I, I, I, I, P, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(x) -> np.ndarray:
    """Accept numpy arrays or torch tensors (any float dtype); widen to fp32."""
    if hasattr(x, "detach"):
        x = x.detach().cpu().float().numpy()
    return np.ascontiguousarray(x, dtype=np.float32)


def alphas(n_alphas: int = 32) -> np.ndarray:
    """The clip-ratio grid exactly as torch.linspace(0.5, 1.0, n) on CPU builds it
    (kv_quant.py:259-260; linspace is evaluated from both ends, so a plain
    start + i*step formula differs in a few entries)."""
    n = n_alphas
    # torch's CPU kernel: fp32 step, then start + step*i (or end - step*(n-1-i)
    # for the upper half) with a single rounding of the product-sum.
    step = np.float64(np.float32((np.float32(1.0) - np.float32(0.5)) / np.float32(max(n - 1, 1))))
    out = np.empty(n, np.float32)
    half = n // 2
    for i in range(n):
        if i < half:
            out[i] = np.float32(0.5 + step * i)
        else:
            out[i] = np.float32(1.0 - step * (n - 1 - i))
    return out


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    """OpenMP threads of the oracle's loops (e.g. all host cores under a
    launcher that exported OMP_NUM_THREADS=1)."""
    lib().orc_set_num_threads(int(n))


def calibrate(blocks, fmt: str, calib: str, n_alphas: int = 32) -> np.ndarray:
    """kv_quant._calibrate over blocks [..., 16] -> scales [..., 1] (fp32)."""
    xb = _f32(blocks)
    n = xb.size // BLOCK
    out = np.empty(n, np.float32)
    al = alphas(n_alphas)
    lib().orc_calibrate(_p(xb), n, FMT[fmt], CALIB[calib], _p(al), n_alphas, _p(out))
    return out.reshape(*xb.shape[:-1], 1)


def roundtrip_f32(x, fmt: str, layout: str, calib: str, n_alphas: int = 32) -> np.ndarray:
    """kv_quant.roundtrip on [H, S, D], returned in fp32 before the dtype cast."""
    xf = _f32(x)
    H, S, D = xf.shape
    y = np.empty_like(xf)
    al = alphas(n_alphas)
    lib().orc_roundtrip(_p(xf), _p(y), H, S, D, FMT[fmt], LAYOUT[layout], CALIB[calib],
                        _p(al), n_alphas)
    return y


def store_int4(k, v, k_calib: str = "mse", v_calib: str = "mse", n_alphas: int = 32) -> dict:
    """int4_kivi.store_kivi restated: returns numpy arrays in the KIVICache layout
    (k_packed u8 [H,D,NP,8], k_scale f16 [H,D,NP], k_hot f32 [H,S%16,D],
    v_packed u8 [H,S,ND,8], v_scale f16 [H,S,ND])."""
    kf, vf = _f32(k), _f32(v)
    H, S, D = kf.shape
    NP, ND = S // BLOCK, D // BLOCK
    kp = np.zeros((H, D, NP, PACK), np.uint8)
    ks = np.zeros((H, D, NP), np.uint16)
    vp = np.zeros((H, S, ND, PACK), np.uint8)
    vs = np.zeros((H, S, ND), np.uint16)
    al = alphas(n_alphas)
    lib().orc_store_int4(_p(kf), _p(vf), H, S, D, CALIB[k_calib], CALIB[v_calib], _p(al),
                         n_alphas, _p(kp), _p(ks), _p(vp), _p(vs))
    return dict(k_packed=kp, k_scale=ks.view(np.float16), k_hot=kf[:, NP * BLOCK:].copy(),
                v_packed=vp, v_scale=vs.view(np.float16), H=H, S=S, D=D)


def dequant_int4(c: dict) -> tuple[np.ndarray, np.ndarray]:
    """dequant_kivi restated in fp32: K tokens < NP*16 from codes, tail from k_hot."""
    H, S, D = c["H"], c["S"], c["D"]
    k = np.zeros((H, S, D), np.float32)
    v = np.zeros((H, S, D), np.float32)
    kp = np.ascontiguousarray(c["k_packed"]); ks = np.ascontiguousarray(c["k_scale"]).view(np.uint16)
    vp = np.ascontiguousarray(c["v_packed"]); vs = np.ascontiguousarray(c["v_scale"]).view(np.uint16)
    lib().orc_dequant_int4(_p(kp), _p(ks), _p(vp), _p(vs), H, S, D, _p(k), _p(v))
    n_full = (S // BLOCK) * BLOCK
    if n_full < S:
        k[:, n_full:] = _f32(c["k_hot"])
    return k, v


def store_int3v(k, v, k_calib: str = "mse", v_calib: str = "mse", n_alphas: int = 32) -> dict:
    """The mixed-precision cache (K INT4 as store_int4, V INT3 per token on the
    kv_quant `int3` grid): v_packed u8 [H,S,D/32,12] (block pairs: words A_2k,
    A_2k+1 with the low two bits of each code, S_k with the sign bits; see
    kivi_oracle.c), v_scale f16 [H,S,D/16]."""
    c = store_int4(k, v, k_calib, "absmax", n_alphas)
    vf = _f32(v)
    H, S, D = vf.shape
    vp = np.zeros((H, S, D // (2 * BLOCK), 12), np.uint8)
    vs = np.zeros((H, S, D // BLOCK), np.uint16)
    lib().orc_store_v3(_p(vf), H, S, D, CALIB[v_calib], _p(alphas(n_alphas)), n_alphas, _p(vp), _p(vs))
    c.update(v_packed=vp, v_scale=vs.view(np.float16))
    return c


def unpack_int3(packed: np.ndarray) -> np.ndarray:
    """[..., D/32, 12] INT3 block pairs -> int8 codes [..., D/16, 16]."""
    w = np.ascontiguousarray(packed).view("<u4")                     # [..., D/32, 3]
    out = []
    for o in range(2):
        A, S = w[..., o].astype(np.int64), w[..., 2].astype(np.int64)
        codes = []
        for i in range(BLOCK):
            sha = 4 * i if i < 8 else 4 * (i - 8) + 2
            shs = (4 * i if i < 8 else 4 * (i - 8) + 1) + 2 * o
            codes.append(((A >> sha) & 3) - 4 * ((S >> shs) & 1))
        out.append(np.stack(codes, axis=-1))
    res = np.stack(out, axis=-2)                                     # [..., D/32, 2, 16]
    return res.reshape(res.shape[:-3] + (-1, BLOCK)).astype(np.int8)


def dequant_int3v(c: dict) -> tuple[np.ndarray, np.ndarray]:
    """fp32 K (as dequant_int4) and V (code * fp32(fp16 scale)) [H, S, D]."""
    H, S, D = c["H"], c["S"], c["D"]
    k = np.zeros((H, S, D), np.float32)
    v = np.zeros((H, S, D), np.float32)
    kp = np.ascontiguousarray(c["k_packed"]); ks = np.ascontiguousarray(c["k_scale"]).view(np.uint16)
    dummy_p = np.zeros((H, S, D // BLOCK, PACK), np.uint8)
    dummy_s = np.zeros((H, S, D // BLOCK), np.uint16)
    lib().orc_dequant_int4(_p(kp), _p(ks), _p(dummy_p), _p(dummy_s), H, S, D, _p(k), _p(v))
    vp = np.ascontiguousarray(c["v_packed"]); vs = np.ascontiguousarray(c["v_scale"]).view(np.uint16)
    lib().orc_dequant_v3(_p(vp), _p(vs), H, S, D, _p(v))
    n_full = (S // BLOCK) * BLOCK
    if n_full < S:
        k[:, n_full:] = _f32(c["k_hot"])
    return k, v


def store_nvfp4(k, v, k_calib: str = "mse", v_calib: str = "mse", g_k: float = 1.0,
                g_v: float = 1.0, n_alphas: int = 32) -> dict:
    """NVFP4-KIVI store: e2m1 nibbles + e4m3 block scales, KIVI geometry."""
    kf, vf = _f32(k), _f32(v)
    H, S, D = kf.shape
    NP, ND = S // BLOCK, D // BLOCK
    kp = np.zeros((H, D, NP, PACK), np.uint8)
    ks = np.zeros((H, D, NP), np.uint8)
    vp = np.zeros((H, S, ND, PACK), np.uint8)
    vs = np.zeros((H, S, ND), np.uint8)
    al = alphas(n_alphas)
    lib().orc_store_nvfp4(_p(kf), _p(vf), H, S, D, CALIB[k_calib], CALIB[v_calib], _p(al),
                          n_alphas, g_k, g_v, _p(kp), _p(ks), _p(vp), _p(vs))
    return dict(k_packed=kp, k_scale=ks, k_hot=kf[:, NP * BLOCK:].copy(), v_packed=vp,
                v_scale=vs, H=H, S=S, D=D, g_k=g_k, g_v=g_v)


def dequant_nvfp4(c: dict) -> tuple[np.ndarray, np.ndarray]:
    H, S, D = c["H"], c["S"], c["D"]
    k = np.zeros((H, S, D), np.float32)
    v = np.zeros((H, S, D), np.float32)
    kp = np.ascontiguousarray(c["k_packed"]); ks = np.ascontiguousarray(c["k_scale"])
    vp = np.ascontiguousarray(c["v_packed"]); vs = np.ascontiguousarray(c["v_scale"])
    lib().orc_dequant_nvfp4(_p(kp), _p(ks), _p(vp), _p(vs), H, S, D, float(c["g_k"]),
                            float(c["g_v"]), _p(k), _p(v))
    n_full = (S // BLOCK) * BLOCK
    if n_full < S:
        k[:, n_full:] = _f32(c["k_hot"])
    return k, v


def decode_attention(q, k, v, sm_scale: float, seq_lens=None) -> np.ndarray:
    """Decode attention in double: q [B,Hq,D], k/v [B,Hkv,S,D] -> [B,Hq,D] fp32."""
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    B, Hq, D = qf.shape
    _, Hkv, S, _ = kf.shape
    out = np.zeros((B, Hq, D), np.float32)
    sl = None
    if seq_lens is not None:
        sl = np.ascontiguousarray(np.asarray(seq_lens, dtype=np.int32))
    lib().orc_decode_attention(_p(qf), _p(kf), _p(vf), _p(sl) if sl is not None else None,
                               B, Hq, Hkv, S, D, sm_scale, _p(out))
    return out


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """[..., 8] u8 -> [..., 16] int codes (element 2j low nibble of byte j)."""
    p = packed.astype(np.int16)
    lo, hi = p & 0xF, (p >> 4) & 0xF
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack([lo, hi], -1).reshape(*packed.shape[:-1], -1)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """[..., 8] u8 -> [..., 16] raw nibbles 0..15."""
    p = packed.astype(np.int16)
    return np.stack([p & 0xF, (p >> 4) & 0xF], -1).reshape(*packed.shape[:-1], -1)


def lse_merge(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """int4_kivi/decode.py:320-340 `_combine_kernel` restated: partial (m, l,
    unnormalised acc) over the last split axis -> normalised output."""
    M = m.max(axis=-1, keepdims=True)
    w = np.exp((m - M).astype(np.float64))
    L = (l * w).sum(-1)
    acc = (o * w[..., None]).sum(-2)
    return (acc / L[..., None]).astype(np.float32)


# ----------------------------------------------------------------------------
# Paged (vLLM-style) cache: kv[num_blocks, 2, 16, H, D/2 + D/16] uint8
# ----------------------------------------------------------------------------
def paged_full_dim(D: int) -> int:
    return D // 2 + D // 16


def paged_calib(blocks, fmt: str = "int4", calib: str = "mse") -> np.ndarray:
    """e4m3 scale bytes of blocks [..., 16] (scripts/diag_kernel_perchannel.py:30-48)."""
    xb = _f32(blocks)
    flat = xb.reshape(-1, BLOCK)
    out = np.empty(flat.shape[0], np.uint8)
    L = lib()
    for i in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[i])
        out[i] = L.orc_paged_calib(_p(row), FMT[fmt], CALIB[calib])
    return out.reshape(xb.shape[:-1])


def paged_store(k, v, slot_mapping, kv: np.ndarray, fmt: str = "int4", calib: str = "mse") -> int:
    """Quantise k, v [N, H, D] into the uint8 cache `kv` (modified in place)."""
    kf, vf = _f32(k), _f32(v)
    N, H, D = kf.shape
    sl = np.ascontiguousarray(np.asarray(slot_mapping, dtype=np.int64))
    assert kv.dtype == np.uint8 and kv.flags.c_contiguous and kv.shape[1:] == (2, BLOCK, H, paged_full_dim(D))
    return lib().orc_paged_store(_p(kf), _p(vf), N, H, D, FMT[fmt], CALIB[calib], _p(sl), _p(kv), kv.shape[0])


def paged_gather(kv: np.ndarray, block_table, seq_lens, H: int, D: int, fmt: str, max_seq: int):
    """Dequantised fp32 k, v [B, H, max_seq, D] (zeros past each sequence's length)."""
    bt = np.ascontiguousarray(np.asarray(block_table, dtype=np.int32))
    sl = np.ascontiguousarray(np.asarray(seq_lens, dtype=np.int32))
    B = bt.shape[0]
    k = np.empty((B, H, max_seq, D), np.float32)
    v = np.empty((B, H, max_seq, D), np.float32)
    kvc = np.ascontiguousarray(kv)
    lib().orc_paged_gather(_p(kvc), kvc.shape[0], _p(bt), bt.shape[1], _p(sl), B, H, D, FMT[fmt], max_seq,
                           _p(k), _p(v))
    return k, v


def paged_decode(q, kv: np.ndarray, block_table, seq_lens, sm_scale: float, fmt: str = "int4") -> np.ndarray:
    """Paged decode attention in double: gather-dequant then softmax(q.k) v per sequence."""
    qf = _f32(q)
    B, Hq, D = qf.shape
    H = kv.shape[3]
    sl = np.asarray(seq_lens, dtype=np.int32)
    ms = max(int(sl.max()) if sl.size else 0, 1)
    k, v = paged_gather(kv, block_table, sl, H, D, fmt, ms)
    return decode_attention(qf, k, v, sm_scale, seq_lens=sl)


# ----------------------- legacy page-level API -----------------------
def page_quantize(x, calib: str = "mse", n_alphas: int = 32) -> tuple[np.ndarray, np.ndarray]:
    """kv_quant.quantize_page for one tensor x [H, T, D] (kv_quant.py:37-38,
    71-84): per-token 16-channel blocks, fp32 scale from the calibration,
    codes = clamp(rint(x / s), -7, 7) with an fp32 division, scales stored
    as fp16.  Returns (int8 codes [H, T, D], fp16 scales [H, T, D/16])."""
    xf = _f32(x)
    H, T, D = xf.shape
    xb = xf.reshape(H, T, D // BLOCK, BLOCK)
    s = calibrate(xb, "int4", calib, n_alphas)                   # [H, T, ND, 1] fp32
    codes = np.clip(np.rint(xb / s), -7, 7).astype(np.int8).reshape(H, T, D)
    return codes, s[..., 0].astype(np.float16)


def page_dequant(codes: np.ndarray, scale16: np.ndarray):
    """QuantizedPage.dequantize (kv_quant.py:62-67): fp16(code * fp16 scale),
    then bf16; returned as a torch bf16 tensor [H, T, D]."""
    import torch
    H, T, D = codes.shape
    sf = np.repeat(scale16.astype(np.float16), BLOCK, axis=-1).reshape(H, T, D)
    prod = codes.astype(np.float16) * sf                          # rounded once to fp16
    return torch.from_numpy(prod.astype(np.float32)).to(torch.bfloat16)


def page_error(x, page_size: int = 16, n_alphas: int = 32) -> tuple[float, float]:
    """kv_quant.measure_page_error (kv_quant.py:170-191): mean over complete
    pages of each page's mean squared error, absmax and MSE calibration."""
    xf = _f32(x)
    H, S, D = xf.shape
    P = S // page_size
    res = []
    for calib in ("absmax", "mse"):
        errs = []
        for i in range(P):
            pg = xf[:, i * page_size:(i + 1) * page_size]
            d = pg - roundtrip_f32(pg, "int4", "headdim", calib, n_alphas)
            errs.append(float(np.mean(d.astype(np.float64) ** 2)))
        res.append(sum(errs) / max(len(errs), 1))
    return res[0], res[1]
