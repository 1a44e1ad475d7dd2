"""CPU-only checks of the boundary: the C-ABI library loads, exports every
symbol include/kivi_sm100.h declares, and rejects bad arguments before any
device work (no compute calls here)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    names = []
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(kivi_\w+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from int4_kivi import _native
    L = _native.lib()
    decl = _declared()
    assert "kivi_decode" in decl and "kivi_store" in decl
    for n in decl:
        assert hasattr(L, n), f"{n} not exported"


def test_status_and_version():
    from int4_kivi import _native
    L = _native.lib()
    assert L.kivi_version() >= 100
    assert L.kivi_status_string(0) == b"ok"
    assert b"argument" in L.kivi_status_string(1)


def test_argument_errors_without_device_work():
    from int4_kivi import _native
    L = _native.lib()
    # D not a multiple of 16
    rc = L.kivi_store(None, None, 0, 0, 0, 0, 0, 0, 0, 1, 16, 16, 15, 0, 0, 0, None, 0, 1.0, 1.0,
                      None, None, 0, 1, None, None, 0, 16, None)
    assert rc == 1
    # bad format
    rc = L.kivi_roundtrip(None, None, 0, 1, 16, 16, 9, 0, 0, None, 0, None)
    assert rc == 1
    # Hq not a multiple of Hkv
    rc = L.kivi_decode(None, 0, 0, None, None, 16, None, 0, None, None, 16, 1, 6, 4, 32, 128, 0, 0.1,
                       1.0, 1.0, None, None, 0, None, None)
    assert rc == 1
    assert L.kivi_decode_workspace_floats(1, 6, 4, 32, 128) == 0


def test_no_cpu_fallback():
    """The product path raises on CPU tensors instead of computing on the host."""
    import torch
    from int4_kivi import store_kivi
    k = torch.zeros(2, 32, 128, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        store_kivi(k, k)
    if not torch.cuda.is_available():
        import kv_quant
        with pytest.raises(RuntimeError):
            kv_quant.roundtrip(k, "int4", "channel", "mse")


def test_paged_argument_errors_without_device_work():
    from int4_kivi import _native
    L = _native.lib()
    assert L.kivi_paged_full_dim(128) == 72 and L.kivi_paged_full_dim(15) == 0
    # D not a multiple of 16
    assert L.kivi_paged_store(None, None, 0, 0, 0, 0, 0, 0, 0, 4, 2, 24, 0, 1, None, None, 1, None, None) == 1
    # bad format
    assert L.kivi_paged_store(None, None, 0, 0, 0, 0, 0, 0, 0, 4, 2, 128, 7, 1, None, None, 1, None, None) == 1
    # zero tokens is a no-op
    assert L.kivi_paged_store(None, None, 0, 0, 0, 0, 0, 0, 0, 0, 2, 128, 0, 1, None, None, 1, None, None) == 0
    # Hq not a multiple of Hkv
    assert L.kivi_paged_decode(None, 0, 0, None, 1, None, 4, None, 1, 6, 4, 128, 0, 0.1,
                               None, None, 0, None, None) == 1
    assert L.kivi_paged_decode_workspace_floats(1, 6, 4, 4, 128) == 0
    assert L.kivi_paged_decode_workspace_floats(2, 32, 8, 64, 128) > 0
    assert L.kivi_paged_gather_dequant(None, 1, None, 4, None, 1, 2, 100, 0, 8, None, None, None, None) == 1


def test_paged_python_api_surface():
    from int4_kivi import paged
    for name in ("int4_kivi_store", "int4_kivi_gather_dequant", "int4_kivi_paged_decode",
                 "nvfp4_kivi_store", "nvfp4_kivi_gather_dequant", "nvfp4_kivi_paged_decode",
                 "int4_kivi_kv_cache_full_dim"):
        assert callable(getattr(paged, name))
    assert paged.BLOCK == 16 and paged.QMAX == 7 and paged.int4_kivi_kv_cache_full_dim(128) == 72


def test_peer_merge_argument_errors():
    from int4_kivi import _native as N
    L = N.lib()
    assert L.kivi_peer_buffer_bytes(32, 128, 2) == 256 + 2 * 32 * 130 * 4
    assert L.kivi_peer_buffer_bytes(32, 128, 17) == 0          # at most 16 ranks
    assert L.kivi_peer_publish(None, None, None, 32, 128, None, None, 2, 0, None, None) == 1
    assert L.kivi_peer_publish(None, None, None, 32, 128, None, None, 2, 2, None, None) == 1   # rank >= W
    assert L.kivi_peer_merge(None, 2, 32, 128, None, None, None, None, 0, None) == 1


def test_paged_api_rejects_host_tensors():
    """The paged functions run on CUDA tensors only (no CPU fallback)."""
    import torch
    from int4_kivi import paged
    kv = torch.zeros(2, 2, 16, 1, 72, dtype=torch.uint8)
    k = torch.zeros(4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        paged.int4_kivi_store(k, k, kv, torch.arange(4), 128)
    with pytest.raises(ValueError):
        paged.int4_kivi_paged_decode(torch.zeros(1, 2, 128, dtype=torch.bfloat16), kv,
                                     torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, dtype=torch.int32))


def test_device_index_spellings():
    """Every spelling of one GPU maps to one ordinal, so the error flag a kernel
    sets is the one device_status reads (no CUDA context needed for these)."""
    import torch
    from int4_kivi import _native as N
    assert N.device_index("cuda:1") == N.device_index(torch.device("cuda", 1)) == N.device_index(1) == 1
    assert N.device_index(torch.device("cuda:0")) == 0
    with pytest.raises(ValueError):
        N.device_index("cpu")


def test_fused_attention_mask_check():
    """The fused hf read path runs only when the mask is the plain causal mask
    over every stored key (a left-padded batch goes to SDPA over the
    dequantised K/V); single-token and multi-token steps."""
    import torch
    from int4_kivi.hf_cache import _causal_over_all
    assert _causal_over_all(None, 1) and _causal_over_all(None, 3)
    m = torch.ones(2, 1, 1, 9, dtype=torch.bool)
    assert _causal_over_all(m, 1)
    m[1, 0, 0, 0] = False                               # in place: the memo sees the new version
    assert not _causal_over_all(m, 1)
    f = torch.zeros(2, 1, 1, 9)
    assert _causal_over_all(f, 1)
    f[0, 0, 0, 3] = torch.finfo(torch.float32).min
    assert not _causal_over_all(f, 1)
    c = torch.tril(torch.ones(3, 9, dtype=torch.bool), diagonal=6)[None, None].repeat(2, 1, 1, 1)
    assert _causal_over_all(c, 3)
    assert not _causal_over_all(c[:, :, 1:].contiguous(), 3)    # wrong query count
    c2 = c.clone()
    c2[0, 0, 0, 0] = False                              # left padding
    assert not _causal_over_all(c2, 3)
    c3 = c.clone()
    c3[1, 0, 0, 7] = True                               # a future key visible
    assert not _causal_over_all(c3, 3)


def test_hf_cache_v_bits_and_mixed_layout_host_side():
    """Host-side checks of the mixed INT4-K / INT3-V cache (no GPU): the HF
    cache takes v_bits 4 or 3 only, the format id is the ABI's
    KIVI_FMT_MIX43, and a capacity buffer for it holds 12 bytes per pair of
    16-channel V blocks (144 bytes per token and kv head with its scales)."""
    import pytest
    import torch
    from int4_kivi import _native as N
    from int4_kivi.cache import alloc_packed, cache_geometry
    from int4_kivi.hf_cache import _Int4KiviLayer
    from int4_kivi.mixed import PACK3
    assert _Int4KiviLayer(v_bits=3).v_bits == 3 and _Int4KiviLayer().v_bits == 4
    with pytest.raises(ValueError):
        _Int4KiviLayer(v_bits=2)
    assert N.FMT["int4k_int3v"] == 3
    kp, ks, vp, vs = alloc_packed(2, 40, 128, "cpu", torch.float16, v_pack=PACK3)
    assert vp.shape[2:] == (4, 12) and vs.shape[2] == 8
    per_token = (vp[0, 0].numel() + vs[0, 0].numel() * 2 + kp[0, :, 0].numel() / 16 + ks[0, :, 0].numel() * 2 / 16)
    assert per_token == 48 + 16 + 64 + 16
    assert cache_geometry((kp[:, :, :2], ks[:, :, :2], vp[:, :40], vs[:, :40])) == (kp.shape[2], vp.shape[1])
