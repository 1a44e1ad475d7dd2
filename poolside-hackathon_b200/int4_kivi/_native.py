"""ctypes binding of libkivi_sm100.so (the C ABI in include/kivi_sm100.h).

PyTorch is used only for device memory and the current CUDA stream; every
kernel comes from the library.  There is no CPU or Triton fallback: if the
library cannot be loaded, or the tensors are not on a CUDA device, the call
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KIVI_LIB_PATH") or os.path.join(os.path.dirname(_HERE), "libkivi_sm100.so")

FMT = {"int4": 0, "int3": 1, "nvfp4": 2, "int4k_int3v": 3}
CALIB = {"absmax": 0, "mse": 1}
LAYOUT = {"headdim": 0, "channel": 1}
DTYPE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_lib = None
_lock = threading.Lock()


class KiviError(RuntimeError):
    """A nonzero status returned by libkivi_sm100 (or raised by a kernel
    through the device error flag); `status` is the kivi_status code."""

    def __init__(self, msg: str, status: int = 0):
        super().__init__(msg)
        self.status = status


KIVI_ERR_TIMEOUT = 5


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python poolside-hackathon_b200/build.py` "
                    "(this package has no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            P, I, F, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
            L.kivi_status_string.restype = ctypes.c_char_p
            L.kivi_status_string.argtypes = [I]
            L.kivi_version.restype = I
            L.kivi_last_cuda_error.restype = I
            L.kivi_store.argtypes = [P, P, I, I64, I64, I64, I64, I64, I64, I, I, I, I, I, I, I, P, I, F, F,
                                     P, P, I, I, P, P, I, I, P]
            L.kivi_dequant.argtypes = [P, P, I, P, P, I, I, I, I, I, F, F, P, P, I64, I64, I64, P]
            L.kivi_roundtrip.argtypes = [P, P, I, I, I, I, I, I, I, P, I, P]
            L.kivi_calibrate.argtypes = [P, I64, I, I, P, I, P, P]
            L.kivi_page_dequant.argtypes = [P, P, I, I, I, I, P, P, P]
            L.kivi_decode_workspace_floats.restype = I64
            L.kivi_decode_workspace_floats.argtypes = [I, I, I, I, I]
            L.kivi_decode.argtypes = [P, I64, I64, P, P, I, P, I, P, P, I, I, I, I, I, I, I, F, F, F,
                                      P, P, I64, P, P]
            L.kivi_decode_partial.argtypes = [P, I64, I64, P, P, I, P, I, P, P, I, I, I, I, I, I, I, F, F,
                                              F, P, P, P, P, I64, P, P]
            L.kivi_lse_merge.argtypes = [P, P, P, I, I, I, P, P]
            L.kivi_decode_varlen.argtypes = [P, I64, I64, P, P, I, P, I, P, P, I, P, I, I, I, I, I, I, F, F,
                                             F, P, P, I64, P, P]
            L.kivi_decode_multiquery.argtypes = [P, I64, I64, I64, P, P, I, P, P, I, P, P, I, I, I, I, I, I, I,
                                                 I, I, F, F, F, P, P, I64, P, P]
            L.kivi_decode_bf16_tail.argtypes = [P, I64, I64, P, P, I, P, P, I, P, P, I, I, I, I, I, I, I, F, F, F,
                                                P, P, I64, P, P]
            L.kivi_seqpar_buffer_bytes.restype = I64
            L.kivi_seqpar_buffer_bytes.argtypes = [I, I, I]
            L.kivi_decode_seqpar.argtypes = [P, I64, I64, P, P, I, P, I, P, P, I, I, I, I, I, I, I, F, F, F,
                                             P, P, I, I, P, ctypes.c_longlong, P, P, I64, P, P]
            L.kivi_peer_buffer_bytes.restype = I64
            L.kivi_peer_buffer_bytes.argtypes = [I, I, I]
            L.kivi_peer_alloc.argtypes = [I64, ctypes.POINTER(P), P]
            L.kivi_peer_open.argtypes = [P, ctypes.POINTER(P)]
            L.kivi_peer_close.argtypes = [P]
            L.kivi_peer_free.argtypes = [P]
            L.kivi_peer_publish.argtypes = [P, P, P, I, I, P, P, I, I, P, P]
            L.kivi_peer_merge.argtypes = [P, I, I, I, P, P, P, P, ctypes.c_longlong, P]
            L.kivi_paged_full_dim.restype = I
            L.kivi_paged_full_dim.argtypes = [I]
            L.kivi_paged_store.argtypes = [P, P, I, I64, I64, I64, I64, I64, I64, I, I, I, I, I, P, P, I64, P, P]
            L.kivi_paged_gather_dequant.argtypes = [P, I64, P, I64, P, I, I, I, I, I, P, P, P, P]
            L.kivi_paged_decode_workspace_floats.restype = I64
            L.kivi_paged_decode_workspace_floats.argtypes = [I, I, I, I64, I]
            L.kivi_paged_decode.argtypes = [P, I64, I64, P, I64, P, I64, P, I, I, I, I, I, F, P, P, I64, P, P]
            L.kivi_paged_decode_f32.argtypes = [P, I64, I64, P, I64, P, I64, P, I, I, I, I, I, F, P, P, I64, P, P]
            _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.kivi_status_string(status).decode()
        extra = f" (cudaError {L.kivi_last_cuda_error()})" if status == 4 else ""
        raise KiviError(f"{what}: {msg}{extra}", status)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("int4_kivi kernels run on CUDA tensors only (no CPU fallback)")


# -------- per-device cached helpers (alpha grid, error flag, workspace) --------
_alpha_cache: dict = {}
_err_cache: dict = {}
_work_cache: dict = {}


def device_index(device) -> int:
    """CUDA ordinal of `device` ("cuda", "cuda:1", torch.device or int); a
    bare "cuda" means the current device, so every spelling of one GPU
    shares one error flag and one workspace."""
    d = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    if d.type != "cuda":
        raise ValueError(f"not a CUDA device: {d}")
    return d.index if d.index is not None else torch.cuda.current_device()


def alphas(device, n_alphas: int) -> torch.Tensor:
    """linspace(0.5, 1.0, n) built on the CPU (bit-identical to kv_quant's grid),
    copied once per device."""
    key = (device_index(device), n_alphas)
    a = _alpha_cache.get(key)
    if a is None:
        a = torch.linspace(0.5, 1.0, n_alphas, dtype=torch.float32).to(device)
        _alpha_cache[key] = a
    return a


def err_flag(device) -> torch.Tensor:
    key = device_index(device)
    e = _err_cache.get(key)
    if e is None:
        e = torch.zeros(1, dtype=torch.int32, device=device)
        _err_cache[key] = e
    return e


def device_status(device) -> int:
    """Read (and clear) the device-side timeout flag; synchronises."""
    e = err_flag(device)
    v = int(e.item())
    if v:
        e.zero_()
    return v


def raise_device_status(device, what: str = "kernel") -> None:
    """Synchronise the current stream and raise KiviError if a kernel set the
    device error flag (a bounded wait that ran out); the flag is cleared."""
    torch.cuda.current_stream(device).synchronize()
    v = device_status(device)
    if v:
        raise KiviError(f"{what}: {lib().kivi_status_string(v).decode()}", v)


_poll: dict = {}


def poll_errors(device) -> None:
    """Sync-free error check for per-step callers: copies the device error
    flag into pinned host memory behind the work already queued on the
    current stream, and raises KiviError for a flag whose copy (from an
    earlier poll) has completed; a raised flag is cleared.  An error is thus
    reported at most one poll after the step whose kernel set it has
    finished, without ever blocking the host."""
    if torch.cuda.is_current_stream_capturing():
        return
    key = device_index(device)
    e = err_flag(device)
    st = _poll.get(key)
    if st is None:
        st = {"host": torch.zeros(1, dtype=torch.int32).pin_memory(), "event": None}
        _poll[key] = st
    ev = st["event"]
    if ev is not None and ev.query():
        v = int(st["host"][0])
        if v:
            st["host"][0] = 0
            st["event"] = None
            e.zero_()
            raise KiviError(f"device error flag: {lib().kivi_status_string(v).decode()}", v)
    if ev is None or ev.query():
        st["host"].copy_(e, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        st["event"] = ev


def workspace(device, n_floats: int, kind: str = "decode") -> torch.Tensor:
    """Grow-only scratch buffer for decode partials, one per (device, stream,
    kind: the contiguous and the paged decode keep separate ones)."""
    key = (device_index(device), torch.cuda.current_stream(device).cuda_stream, kind)
    w = _work_cache.get(key)
    if w is None or w.numel() < n_floats:
        w = torch.zeros(max(n_floats, 1), dtype=torch.float32, device=device)
        _work_cache[key] = w
    return w
