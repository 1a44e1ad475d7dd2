"""kv_quant on B200: the reference's quantisation primitives (kv_quant.py) with
calibration and roundtrip running on libkivi_sm100.

Same names, signatures and results as the reference module (kv_quant.py:1-321):
`roundtrip`, `_calibrate`, `_to_blocks`, `_FORMATS`, `_q_int4/_q_int3/_q_e2m1`,
`rmse_cell`, `sweep_tensor`, `SWEEP_CELLS`, `_absmax_scale`,
`_mse_optimal_scale`, `quantize_block`, `dequantize_block`, `quantize_page`,
`QuantizedPage`, `QuantizedKVLayer`, `QuantizedKVCache`, `measure_page_error`.

Calibration (`_calibrate`, `_absmax_scale`, `_mse_optimal_scale`) and
`roundtrip` run as CUDA kernels and are bit-identical to the reference on CPU.
CPU tensors are accepted: they are copied to the current CUDA device, processed
there and copied back (the host<->device path); without a CUDA device these
functions raise instead of falling back to a CPU implementation.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
from torch import Tensor

from int4_kivi import _native as N

BLOCK = 16
PAGE = 16
QMAX = 7


def _device_of(x: Tensor) -> torch.device:
    if x.is_cuda:
        return x.device
    if not torch.cuda.is_available():
        raise RuntimeError("kv_quant (B200 build) needs a CUDA device; there is no CPU fallback")
    return torch.device("cuda", torch.cuda.current_device())


# ----------------------------- grids (elementwise) -----------------------------
_E2M1_LEVELS = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
_E2M1_BOUNDS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])


def _q_int4(y: Tensor) -> Tensor:
    return y.round().clamp(-7.0, 7.0)


def _q_int3(y: Tensor) -> Tensor:
    return y.round().clamp(-3.0, 3.0)


def _q_e2m1(y: Tensor) -> Tensor:
    levels = _E2M1_LEVELS.to(y.device, y.dtype)
    bounds = _E2M1_BOUNDS.to(y.device, y.dtype)
    idx = torch.bucketize(y.abs(), bounds, right=False)
    return torch.sign(y) * levels[idx]


_FORMATS = {"int4": (7.0, _q_int4), "int3": (3.0, _q_int3), "nvfp4": (6.0, _q_e2m1)}
_QFN_FMT = {_q_int4: "int4", _q_int3: "int3", _q_e2m1: "nvfp4"}


def _fmt_of(qmax: float, qfn) -> str:
    fmt = _QFN_FMT.get(qfn)
    if fmt is None or _FORMATS[fmt][0] != float(qmax):
        raise ValueError("calibration grid must be one of kv_quant._FORMATS")
    return fmt


def _to_blocks(x: Tensor, layout: str) -> Tensor:
    """x [H, S, D] -> blocks [..., BLOCK] ('headdim' | 'channel', S % 16 == 0)."""
    H, S, D = x.shape
    if layout == "headdim":
        return x.reshape(H, S, D // BLOCK, BLOCK)
    if layout == "channel":
        return x.transpose(1, 2).contiguous().reshape(H, D, S // BLOCK, BLOCK)
    raise ValueError(f"unknown layout {layout!r}")


def _calibrate(xb: Tensor, qmax: float, qfn, calib: str, n_alphas: int = 32) -> Tensor:
    """Per-block fp32 scale for blocks xb [..., BLOCK] -> [..., 1] (CUDA kernel)."""
    if calib not in N.CALIB:
        raise ValueError(f"unknown calib {calib!r}")
    fmt = _fmt_of(qmax, qfn)
    dev = _device_of(xb)
    blocks = xb.detach().to(dev, torch.float32).contiguous()
    n = blocks.numel() // BLOCK
    out = torch.empty(n, dtype=torch.float32, device=dev)
    al = N.alphas(dev, n_alphas)
    N.check(N.lib().kivi_calibrate(N.ptr(blocks), n, N.FMT[fmt], N.CALIB[calib], N.ptr(al), n_alphas,
                                   N.ptr(out), N.stream_of(out)), "kivi_calibrate")
    return out.reshape(*xb.shape[:-1], 1).to(xb.device)


def _absmax_scale(x: Tensor) -> Tensor:
    return _calibrate(x, 7.0, _q_int4, "absmax").to(x.dtype)


def _mse_optimal_scale(x: Tensor, n_alphas: int = 32) -> Tensor:
    return _calibrate(x, 7.0, _q_int4, "mse", n_alphas).to(x.dtype)


def quantize_block(x: Tensor, scale: Tensor) -> Tensor:
    return (x / scale).round().clamp(-QMAX, QMAX).to(torch.int8)


def dequantize_block(q: Tensor, scale: Tensor) -> Tensor:
    return q.to(scale.dtype) * scale


def roundtrip(x: Tensor, fmt: str, layout: str, calib: str, n_alphas: int = 32) -> Tensor:
    """Quantize+dequantize x [H, S, D]; same shape and dtype out (kv_quant.py:299-321).
    'channel' returns the trailing S % 16 tokens unquantized."""
    if fmt not in N.FMT:
        raise KeyError(fmt)
    if layout not in N.LAYOUT:
        raise ValueError(f"unknown layout {layout!r}")
    if calib not in N.CALIB:
        raise ValueError(f"unknown calib {calib!r}")
    H, S, D = x.shape
    if layout == "channel" and S < BLOCK:
        return x
    dev = _device_of(x)
    xd = x.detach().to(dev).contiguous()
    if xd.dtype not in N.DTYPE:
        xd = xd.float()
    y = torch.empty_like(xd)
    al = N.alphas(dev, n_alphas)
    N.check(N.lib().kivi_roundtrip(N.ptr(xd), N.ptr(y), N.DTYPE[xd.dtype], H, S, D, N.FMT[fmt],
                                   N.LAYOUT[layout], N.CALIB[calib], N.ptr(al), n_alphas, N.stream_of(y)),
            "kivi_roundtrip")
    return y.to(device=x.device, dtype=x.dtype)


def rmse_cell(x: Tensor, fmt: str, layout: str, calib: str, n_alphas: int = 32) -> float:
    """Reconstruction RMSE for one (format, layout, calib) cell. x: [H, S, D]."""
    S = x.shape[1]
    if layout == "channel":
        x = x[:, : (S // BLOCK) * BLOCK]
    xf = x.float()
    xhat = roundtrip(xf, fmt, layout, calib, n_alphas)
    return ((xf - xhat) ** 2).mean().sqrt().item()


SWEEP_CELLS = [
    (fmt, layout, calib)
    for fmt in ("nvfp4", "int4")
    for layout in ("headdim", "channel")
    for calib in ("absmax", "mse")
]
SWEEP_BASELINE = ("nvfp4", "headdim", "absmax")


def sweep_tensor(x: Tensor, n_alphas: int = 32) -> dict:
    S = x.shape[1]
    x = x[:, : (S // BLOCK) * BLOCK]
    return {cell: rmse_cell(x, *cell, n_alphas=n_alphas) for cell in SWEEP_CELLS}


# ------------------------- legacy page-level cache API -------------------------
# The reference's first cache design (kv_quant.py:37-169): per-token 16-channel
# blocks for both K and V, int8 codes, fp16 scales, pages of `page_size`
# tokens plus an unquantised hot tail.  Here every quantisation is one
# kivi_store launch (its per-token path, the same blocks and calibration) and
# every dequantisation one kivi_page_dequant launch; a layer keeps its pages in
# two capacity-backed device buffers instead of a list of per-page tensors.


def _store_tokens(x: Tensor, use_mse: bool, n_alphas: int, packed: Tensor, scale: Tensor, tok0: int) -> None:
    """Quantise rows x [R, T, D] (per token, 16-channel blocks) into packed
    [R, cap, D/16, 8] / scale fp16 [R, cap, D/16] at token tok0."""
    R, T, D = x.shape
    if T == 0:
        return
    if x.dtype not in N.DTYPE:
        x = x.float()
    calib = N.CALIB["mse" if use_mse else "absmax"]
    al = N.alphas(x.device, n_alphas)
    sv = x.stride()
    N.check(N.lib().kivi_store(None, N.ptr(x), N.DTYPE[x.dtype], 0, 0, 0, sv[0], sv[1], sv[2], R, 0, T, D,
                               N.FMT["int4"], calib, calib, N.ptr(al), n_alphas, 1.0, 1.0, None, None, 0, 0,
                               N.ptr(packed), N.ptr(scale), tok0, packed.shape[1], N.stream_of(x)),
            "kivi_store")


def _page_dequant(packed: Tensor, scale: Tensor, tokens: int, values: bool = True, codes: bool = False):
    """bf16 values and/or int8 codes [R, tokens, D] of the first `tokens`
    tokens of packed [R, cap, D/16, 8] / scale [R, cap, D/16]."""
    R, cap, ND, _ = packed.shape
    D = ND * BLOCK
    out = torch.empty(R, tokens, D, dtype=torch.bfloat16, device=packed.device) if values else None
    cod = torch.empty(R, tokens, D, dtype=torch.int8, device=packed.device) if codes else None
    N.check(N.lib().kivi_page_dequant(N.ptr(packed), N.ptr(scale), R, tokens, cap, D, N.ptr(out), N.ptr(cod),
                                      N.stream_of(packed)), "kivi_page_dequant")
    return out, cod


def _pack_codes(c: Tensor) -> Tensor:
    """int8 codes [..., D] -> packed nibbles [..., D/16, 8] (element 2j low)."""
    u = c.to(torch.uint8) & 0xF
    return (u[..., 0::2] | (u[..., 1::2] << 4)).reshape(*c.shape[:-1], c.shape[-1] // BLOCK, BLOCK // 2)


@dataclasses.dataclass
class QuantizedPage:
    """One quantised page (kv_quant.py:45-68): int8 codes [H, T, D] and fp16
    scales [H, T, D/16] for K and V, and the page's first token position."""
    k_int4: Tensor
    v_int4: Tensor
    k_scale: Tensor
    v_scale: Tensor
    start_pos: int

    def dequantize(self) -> tuple[Tensor, Tensor]:
        """bf16 K, V [H, T, D]: bf16(fp16(code * scale)), one kernel launch."""
        H, T, D = self.k_int4.shape
        dev = _device_of(self.k_int4)
        codes = torch.cat([self.k_int4, self.v_int4]).to(dev)
        packed = _pack_codes(codes).contiguous()
        sc = torch.cat([self.k_scale, self.v_scale]).to(dev, torch.float16).contiguous()
        out, _ = _page_dequant(packed, sc, T)
        out = out.to(self.k_int4.device)
        return out[:H], out[H:]

    def mem_bytes(self) -> int:
        """Bytes at 4-bit codes plus fp16 scales, K and V."""
        codes = self.k_int4.numel() // 2
        scales = self.k_scale.numel() * 2
        return 2 * (codes + scales)

    def bf16_bytes(self) -> int:
        """Bytes of the same K and V in bf16."""
        return 2 * 2 * self.k_int4.numel()


def quantize_page(k: Tensor, v: Tensor, start_pos: int, use_mse: bool = True, n_alphas: int = 32) -> QuantizedPage:
    """Quantise one page k, v [n_heads, page_tokens, head_dim] (kv_quant.py:71-84):
    per-token 16-channel blocks, absmax or MSE scale, codes from the fp32 scale,
    scales stored as fp16.  K and V go through one store launch."""
    H, T, D = k.shape
    dev = _device_of(k)
    x = torch.cat([k, v]).to(dev)
    packed = torch.empty(2 * H, T, D // BLOCK, BLOCK // 2, dtype=torch.uint8, device=dev)
    scale = torch.empty(2 * H, T, D // BLOCK, dtype=torch.float16, device=dev)
    _store_tokens(x, use_mse, n_alphas, packed, scale, 0)
    _, codes = _page_dequant(packed, scale, T, values=False, codes=True)
    codes, scale = codes.to(k.device), scale.to(k.device)
    return QuantizedPage(codes[:H], codes[H:], scale[:H], scale[H:], start_pos)


class QuantizedKVLayer:
    """Pages of one layer (kv_quant.py:87-131).  Complete pages are quantised
    straight into capacity-backed device buffers [2, H, cap, D/16, 8] (K rows
    0..H-1, V rows H..2H-1), one store launch per append; the tokens of the
    unfinished page stay in `hot_k` / `hot_v` as given."""

    def __init__(self, page_size: int = PAGE, use_mse: bool = True, n_alphas: int = 32) -> None:
        self.page_size = page_size
        self.use_mse = use_mse
        self.n_alphas = n_alphas
        self.n_pages = 0
        self._packed: Optional[Tensor] = None
        self._scale: Optional[Tensor] = None
        self.hot_k: Optional[Tensor] = None
        self.hot_v: Optional[Tensor] = None

    def _reserve(self, H: int, tokens: int, D: int, device) -> None:
        cap = self._packed.shape[1] if self._packed is not None else 0
        if tokens <= cap:
            return
        new_cap = max(tokens, 2 * cap, 4 * self.page_size)
        packed = torch.empty(2 * H, new_cap, D // BLOCK, BLOCK // 2, dtype=torch.uint8, device=device)
        scale = torch.empty(2 * H, new_cap, D // BLOCK, dtype=torch.float16, device=device)
        if cap:
            packed[:, :cap].copy_(self._packed)
            scale[:, :cap].copy_(self._scale)
        self._packed, self._scale = packed, scale

    def append(self, k: Tensor, v: Tensor) -> None:
        """k, v: [n_kv_heads, new_tokens, head_dim]."""
        self.hot_k = k if self.hot_k is None else torch.cat([self.hot_k, k], dim=1)
        self.hot_v = v if self.hot_v is None else torch.cat([self.hot_v, v], dim=1)
        n_new = self.hot_k.shape[1] // self.page_size * self.page_size
        if n_new == 0:
            return
        H, _, D = self.hot_k.shape
        dev = _device_of(self.hot_k)
        t0 = self.n_pages * self.page_size
        self._reserve(H, t0 + n_new, D, dev)
        x = torch.cat([self.hot_k[:, :n_new], self.hot_v[:, :n_new]]).to(dev)
        _store_tokens(x, self.use_mse, self.n_alphas, self._packed, self._scale, t0)
        self.n_pages += n_new // self.page_size
        self.hot_k = self.hot_k[:, n_new:]
        self.hot_v = self.hot_v[:, n_new:]

    @property
    def pages(self) -> list[QuantizedPage]:
        """The stored pages as QuantizedPage records (materialised on access)."""
        if not self.n_pages:
            return []
        H = self._packed.shape[0] // 2
        _, codes = _page_dequant(self._packed, self._scale, self.n_pages * self.page_size, values=False,
                                 codes=True)
        P = self.page_size
        return [QuantizedPage(codes[:H, i * P:(i + 1) * P], codes[H:, i * P:(i + 1) * P],
                              self._scale[:H, i * P:(i + 1) * P], self._scale[H:, i * P:(i + 1) * P], i * P)
                for i in range(self.n_pages)]

    def get_kv(self) -> tuple[Tensor, Tensor]:
        """bf16 K, V [n_kv_heads, seq_len, head_dim]: dequantised pages, then the hot tail."""
        if not self.n_pages:
            if self.hot_k is None:
                raise ValueError("Cache is empty")
            return self.hot_k.bfloat16(), self.hot_v.bfloat16()
        H = self._packed.shape[0] // 2
        out, _ = _page_dequant(self._packed, self._scale, self.n_pages * self.page_size)
        k, v = out[:H], out[H:]
        if self.hot_k is not None and self.hot_k.shape[1]:
            k = torch.cat([k, self.hot_k.to(k.device, torch.bfloat16)], dim=1)
            v = torch.cat([v, self.hot_v.to(v.device, torch.bfloat16)], dim=1)
        return k, v

    def seq_len(self) -> int:
        return self.n_pages * self.page_size + (self.hot_k.shape[1] if self.hot_k is not None else 0)

    def _page_elems(self) -> int:
        return self._packed.shape[0] // 2 * self.n_pages * self.page_size * self._packed.shape[2] * BLOCK \
            if self.n_pages else 0

    def mem_bytes(self) -> int:
        """4-bit codes + fp16 scales of the pages (K and V) plus the hot tail at 2 B per element."""
        e = self._page_elems()
        hot = 2 * 2 * self.hot_k.numel() if self.hot_k is not None else 0
        return 2 * (e // 2 + (e // BLOCK) * 2) + hot

    def bf16_bytes(self) -> int:
        """The same tokens (pages and hot tail, K and V) at bf16."""
        hot = self.hot_k.numel() if self.hot_k is not None else 0
        return 2 * 2 * (self._page_elems() + hot)


class QuantizedKVCache:
    """Per-layer paged cache with the reference's `update` / `get_kv` contract
    (kv_quant.py:134-167; batch 1, k/v [1, n_kv_heads, new_tokens, head_dim])."""

    def __init__(self, page_size: int = PAGE, use_mse: bool = True, n_alphas: int = 32) -> None:
        self.page_size = page_size
        self.use_mse = use_mse
        self.n_alphas = n_alphas
        self.layers: list[QuantizedKVLayer] = []

    def _ensure(self, layer_idx: int) -> None:
        self.layers.extend(QuantizedKVLayer(self.page_size, self.use_mse, self.n_alphas)
                           for _ in range(layer_idx + 1 - len(self.layers)))

    def update(self, layer_idx: int, k: Tensor, v: Tensor) -> None:
        self._ensure(layer_idx)
        self.layers[layer_idx].append(k.squeeze(0), v.squeeze(0))

    def get_kv(self, layer_idx: int) -> tuple[Tensor, Tensor]:
        """bf16 [1, n_kv_heads, seq_len, head_dim] K and V of one layer."""
        k, v = self.layers[layer_idx].get_kv()
        return k[None], v[None]

    def mem_bytes(self) -> int:
        return sum(layer.mem_bytes() for layer in self.layers)

    def bf16_bytes(self) -> int:
        return sum(layer.bf16_bytes() for layer in self.layers)

    def compression_ratio(self) -> float:
        return self.bf16_bytes() / max(self.mem_bytes(), 1)


def measure_page_error(k: Tensor, page_size: int = PAGE, n_alphas: int = 32) -> dict:
    """Absmax vs MSE-optimal reconstruction error over complete pages
    (kv_quant.py:170-191): the mean over pages of each page's mean squared
    error, with fp32 scales.  Each calibration is one kivi_roundtrip launch
    (per-token 16-channel blocks) over all complete pages at once."""
    H, S, D = k.shape
    P = S // page_size
    if P == 0:
        return {"absmax_mse": 0.0, "optimal_mse": 0.0, "reduction_pct": 0.0}
    x = k[:, :P * page_size].float()
    res = {}
    for calib in ("absmax", "mse"):
        d = (x - roundtrip(x, "int4", "headdim", calib, n_alphas)).pow(2)
        per_page = d.reshape(H, P, page_size * D).transpose(0, 1).reshape(P, -1).mean(dim=1)
        res[calib] = float(per_page.double().mean().item())
    a, o = res["absmax"], res["mse"]
    return {"absmax_mse": a, "optimal_mse": o, "reduction_pct": 100.0 * (a - o) / max(a, 1e-12)}
