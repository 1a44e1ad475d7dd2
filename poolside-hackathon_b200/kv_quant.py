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
@dataclasses.dataclass
class QuantizedPage:
    k_int4: Tensor
    v_int4: Tensor
    k_scale: Tensor
    v_scale: Tensor
    start_pos: int

    def dequantize(self) -> tuple[Tensor, Tensor]:
        def _deq(q: Tensor, scale: Tensor) -> Tensor:
            sf = scale.unsqueeze(-1).expand(*scale.shape, BLOCK).reshape(*q.shape)
            return dequantize_block(q, sf).to(torch.bfloat16)
        return _deq(self.k_int4, self.k_scale), _deq(self.v_int4, self.v_scale)

    def mem_bytes(self) -> int:
        return 2 * (self.k_int4.numel() // 2 + self.k_scale.numel() * 2)

    def bf16_bytes(self) -> int:
        return self.k_int4.numel() * 2 * 2


def quantize_page(k: Tensor, v: Tensor, start_pos: int, use_mse: bool = True, n_alphas: int = 32) -> QuantizedPage:
    """One page k, v [n_heads, page_tokens, head_dim] (kv_quant.py:72-84)."""
    n_heads, page_tokens, head_dim = k.shape
    kf = k.float().reshape(n_heads, page_tokens, head_dim // BLOCK, BLOCK)
    vf = v.float().reshape(n_heads, page_tokens, head_dim // BLOCK, BLOCK)
    calib = "mse" if use_mse else "absmax"
    ks = _calibrate(kf, 7.0, _q_int4, calib, n_alphas)
    vs = _calibrate(vf, 7.0, _q_int4, calib, n_alphas)
    k_q = quantize_block(kf, ks).reshape(n_heads, page_tokens, head_dim)
    v_q = quantize_block(vf, vs).reshape(n_heads, page_tokens, head_dim)
    return QuantizedPage(k_q, v_q, ks.squeeze(-1).to(torch.float16), vs.squeeze(-1).to(torch.float16), start_pos)


class QuantizedKVLayer:
    def __init__(self, page_size: int = PAGE, use_mse: bool = True, n_alphas: int = 32) -> None:
        self.page_size = page_size
        self.use_mse = use_mse
        self.n_alphas = n_alphas
        self.pages: list[QuantizedPage] = []
        self.hot_k: Optional[Tensor] = None
        self.hot_v: Optional[Tensor] = None

    def append(self, k: Tensor, v: Tensor) -> None:
        self.hot_k = torch.cat([self.hot_k, k], dim=1) if self.hot_k is not None else k
        self.hot_v = torch.cat([self.hot_v, v], dim=1) if self.hot_v is not None else v
        while self.hot_k.shape[1] >= self.page_size:
            start = len(self.pages) * self.page_size
            self.pages.append(quantize_page(self.hot_k[:, :self.page_size], self.hot_v[:, :self.page_size],
                                            start, self.use_mse, self.n_alphas))
            self.hot_k = self.hot_k[:, self.page_size:]
            self.hot_v = self.hot_v[:, self.page_size:]

    def get_kv(self) -> tuple[Tensor, Tensor]:
        if not self.pages:
            if self.hot_k is None:
                raise ValueError("Cache is empty")
            return self.hot_k.bfloat16(), self.hot_v.bfloat16()
        parts_k, parts_v = zip(*(p.dequantize() for p in self.pages))
        k = torch.cat(list(parts_k), dim=1)
        v = torch.cat(list(parts_v), dim=1)
        if self.hot_k is not None and self.hot_k.shape[1] > 0:
            k = torch.cat([k, self.hot_k.bfloat16()], dim=1)
            v = torch.cat([v, self.hot_v.bfloat16()], dim=1)
        return k, v

    def seq_len(self) -> int:
        hot = self.hot_k.shape[1] if self.hot_k is not None else 0
        return len(self.pages) * self.page_size + hot

    def mem_bytes(self) -> int:
        hot_cost = self.hot_k.numel() * 2 * 2 if self.hot_k is not None else 0
        return sum(p.mem_bytes() for p in self.pages) + hot_cost


class QuantizedKVCache:
    """Per-layer paged cache with the reference's `update`/`get_kv` contract."""

    def __init__(self, page_size: int = PAGE, use_mse: bool = True, n_alphas: int = 32) -> None:
        self.page_size = page_size
        self.use_mse = use_mse
        self.n_alphas = n_alphas
        self.layers: list[QuantizedKVLayer] = []

    def _ensure(self, layer_idx: int) -> None:
        while len(self.layers) <= layer_idx:
            self.layers.append(QuantizedKVLayer(self.page_size, self.use_mse, self.n_alphas))

    def update(self, layer_idx: int, k: Tensor, v: Tensor) -> None:
        self._ensure(layer_idx)
        self.layers[layer_idx].append(k.squeeze(0), v.squeeze(0))

    def get_kv(self, layer_idx: int) -> tuple[Tensor, Tensor]:
        k, v = self.layers[layer_idx].get_kv()
        return k.unsqueeze(0), v.unsqueeze(0)

    def mem_bytes(self) -> int:
        return sum(l.mem_bytes() for l in self.layers)

    def bf16_bytes(self) -> int:
        total = 0
        for layer in self.layers:
            total += sum(p.bf16_bytes() for p in layer.pages)
            if layer.hot_k is not None:
                total += layer.hot_k.numel() * 2 * 2
        return total

    def compression_ratio(self) -> float:
        return self.bf16_bytes() / max(self.mem_bytes(), 1)


def measure_page_error(k: Tensor, page_size: int = PAGE, n_alphas: int = 32) -> dict:
    """Absmax vs MSE-optimal reconstruction error over complete pages (kv_quant.py:147-169)."""
    n_heads, seq_len, head_dim = k.shape
    abs_errs, opt_errs = [], []
    for i in range(seq_len // page_size):
        page = k[:, i * page_size:(i + 1) * page_size].float()
        pg = page.reshape(n_heads, page_size, head_dim // BLOCK, BLOCK)
        for calib, errs in (("absmax", abs_errs), ("mse", opt_errs)):
            s = _calibrate(pg, 7.0, _q_int4, calib, n_alphas)
            errs.append(((pg - dequantize_block(quantize_block(pg, s), s)) ** 2).mean().item())
    absmax_mse = float(sum(abs_errs) / max(len(abs_errs), 1))
    optimal_mse = float(sum(opt_errs) / max(len(opt_errs), 1))
    return {"absmax_mse": absmax_mse, "optimal_mse": optimal_mse,
            "reduction_pct": 100.0 * (absmax_mse - optimal_mse) / max(absmax_mse, 1e-12)}
