"""kivi_decode_noalloc: the allocation-free decode entry point.

Callers that cannot allocate device memory while decoding (an engine that
owns all device memory through its own pool, an FFI host with no CUDA
allocator) call this variant; it keeps the split-K
partials in a fixed library-owned device array instead of a workspace.
This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.  It passes alone in a fresh process
and after the rest of the suite.
"""
import ctypes
import math

import pytest
import torch

from conftest import gen_kv

pytestmark = pytest.mark.gpu

P, I, F, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
NOALLOC_FLOATS = 1 << 21          # KIVI_NOALLOC_SCRATCH_FLOATS in include/kivi_sm100.h
KIVI_ERR_SCRATCH = 6


def _lib():
    from int4_kivi import _native
    L = _native.lib()
    L.kivi_decode_noalloc.argtypes = [P, I64, I64, P, P, I, P, I, P, P, I, I, I, I, I, I, I, F, F, F,
                                      P, P, P]
    L.kivi_decode_noalloc.restype = I
    return L


def _args(q, st, Hq, nps, ss):
    from int4_kivi import _native as N
    D = st["D"]
    khot = st["k_hot"].contiguous()
    return (N.ptr(q), q.stride(0), q.stride(1), N.ptr(st["k_packed"]), N.ptr(st["k_scale"]), nps,
            N.ptr(khot) if khot.shape[1] else None, khot.shape[1], N.ptr(st["v_packed"]),
            N.ptr(st["v_scale"]), ss, st["B"], Hq, st["H"], st["S"], D, 0, 1.0 / math.sqrt(D), 1.0, 1.0)


def _case(dev, seed, B, Hkv, Hq, S, D=128):
    from int4_kivi import store_kivi
    from int4_kivi.decode import stack_caches
    k, v, q = gen_kv(Hkv, S, D, seed=seed, Hq=Hq, B=B)
    st = stack_caches([store_kivi(k[b].to(dev), v[b].to(dev)) for b in range(B)])
    return q[:, :, 0].to(dev).contiguous(), st


def test_noalloc_matches_workspace_decode_twice(cuda_dev):
    from int4_kivi import _native as N
    from int4_kivi.cache import cache_geometry
    from int4_kivi.decode import decode_packed
    L = _lib()
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    # two calls in a row on different problems share the one scratch array
    for seed, (B, Hkv, Hq, S) in ((1, (2, 8, 32, 3000)), (2, (3, 4, 16, 1037))):
        q, st = _case(cuda_dev, seed, B, Hkv, Hq, S)

        nps, ss = cache_geometry((st["k_packed"], st["k_scale"], st["v_packed"], st["v_scale"]))
        want = decode_packed(q, st, Hq)
        got = torch.empty_like(want)
        rc = L.kivi_decode_noalloc(*_args(q, st, Hq, nps, ss), N.ptr(got), N.ptr(err), N.stream_of(q))
        assert rc == 0, L.kivi_status_string(rc)
        torch.cuda.synchronize()
        diff = (got.float() - want.float()).abs()
        assert bool((diff <= 2e-3 + want.float().abs() * 2.0 ** -8).all()), diff.max().item()
    assert int(err.item()) == 0


def test_noalloc_rejects_oversized_problem(cuda_dev):
    L = _lib()
    B, Hq, Hkv, S, D = 64, 32, 8, 1 << 20, 128
    assert L.kivi_decode_workspace_floats(B, Hq, Hkv, S, D) > NOALLOC_FLOATS
    rc = L.kivi_decode_noalloc(None, 0, 0, None, None, S // 16, None, 0, None, None, S, B, Hq, Hkv, S, D, 0,
                               0.1, 1.0, 1.0, None, None, None)
    assert rc == KIVI_ERR_SCRATCH
    assert b"scratch" in L.kivi_status_string(rc)
