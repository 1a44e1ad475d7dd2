"""Pin the CPU oracle (oracle/) to the reference's own outputs (tests/golden/).

Bit-exact for quantised values, codes and scales; the decode oracle (double
precision) within 2e-6 of the reference's fp32 SDPA."""
import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits, load_golden

FMTS = ("int4", "int3", "nvfp4")
LAYOUTS = ("headdim", "channel")
CALIBS = ("absmax", "mse")


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("calib", CALIBS)
@pytest.mark.parametrize("name", ("k", "v"))
def test_roundtrip_bit_exact(fmt, layout, calib, name):
    g = load_golden("kvq_roundtrip.npz")
    x = bf16_from_bits(g[name])
    want = bf16_from_bits(g[f"{name}_{fmt}_{layout}_{calib}"])
    got = torch.from_numpy(oracle.roundtrip_f32(x, fmt, layout, calib)).to(torch.bfloat16)
    assert torch.equal(got, want)


def test_roundtrip_fp32_and_alpha_grid():
    g = load_golden("kvq_roundtrip.npz")
    xf = g["kf32"]
    assert np.array_equal(oracle.roundtrip_f32(xf, "int4", "channel", "mse", n_alphas=7),
                          g["kf32_int4_channel_mse_a7"])
    assert np.array_equal(oracle.roundtrip_f32(xf, "nvfp4", "headdim", "mse"),
                          g["kf32_nvfp4_headdim_mse"])


def test_alpha_grid_matches_linspace():
    c = load_golden("casts.npz")
    assert np.array_equal(oracle.alphas(32), c["linspace32"])
    assert np.array_equal(oracle.alphas(7), c["linspace7"])


@pytest.mark.parametrize("S", (40, 256))
@pytest.mark.parametrize("calib", CALIBS)
def test_int4_store_bit_exact(S, calib):
    g = load_golden("kivi_store.npz")
    k, v = bf16_from_bits(g[f"S{S}_k"]), bf16_from_bits(g[f"S{S}_v"])
    c = oracle.store_int4(k, v, calib, calib)
    pre = f"S{S}_{calib}_"
    assert np.array_equal(c["k_packed"], g[pre + "k_packed"])
    assert np.array_equal(c["v_packed"], g[pre + "v_packed"])
    assert np.array_equal(c["k_scale"].view(np.uint16), g[pre + "k_scale"])
    assert np.array_equal(c["v_scale"].view(np.uint16), g[pre + "v_scale"])
    kd, vd = oracle.dequant_int4(c)
    n_full = (S // 16) * 16
    assert torch.equal(torch.from_numpy(kd[:, :n_full]).bfloat16(), bf16_from_bits(g[pre + "k_deq"]))
    assert torch.equal(torch.from_numpy(vd).bfloat16(), bf16_from_bits(g[pre + "v_deq"]))
    # hot tail is verbatim bf16 (tests/test_int4_kivi.py:130-142)
    assert torch.equal(torch.from_numpy(kd[:, n_full:]).bfloat16(), k[:, n_full:])


@pytest.mark.parametrize("S", (40, 127, 300))
def test_decode_oracle_vs_reference_fp32(S):
    g = load_golden("decode_fp32.npz")
    pre = f"S{S}_"
    cache = dict(k_packed=g[pre + "k_packed"], v_packed=g[pre + "v_packed"],
                 k_scale=g[pre + "k_scale"].view(np.float16), v_scale=g[pre + "v_scale"].view(np.float16),
                 k_hot=bf16_from_bits(g[pre + "k_hot"]), H=2, S=S, D=128)
    k, v = oracle.dequant_int4(cache)
    q = bf16_from_bits(g[pre + "q"])                      # [Hq, 1, D]
    out = oracle.decode_attention(q[None, :, 0], k[None], v[None], 1.0 / np.sqrt(128))
    ref = g[pre + "out"][:, 0]
    assert np.abs(out[0] - ref).max() < 2e-6
    # and the oracle's own store reproduces the reference codes for this case
    kk, vv = bf16_from_bits(g[pre + "k"]), bf16_from_bits(g[pre + "v"])
    c = oracle.store_int4(kk, vv)
    assert np.array_equal(c["k_packed"], g[pre + "k_packed"])
    assert np.array_equal(c["v_packed"], g[pre + "v_packed"])


def test_scale_casts():
    c = load_golden("casts.npz")
    L = oracle.lib()
    f16 = np.array([L.orc_f32_to_f16(float(x)) for x in c["vals"]], np.uint16)
    assert np.array_equal(f16, c["f16"])
    e4 = np.array([L.orc_f32_to_e4m3(float(x)) for x in c["e4m3_in"]], np.uint8)
    assert np.array_equal(e4, c["e4m3"])
    # e4m3 decode is exact and inverts the encoder
    for b in range(0, 127):
        if (b & 0x7f) == 0x7f:
            continue
        assert L.orc_f32_to_e4m3(L.orc_e4m3_to_f32(b)) == b


def test_nvfp4_store_semantics():
    """NVFP4-KIVI store: codes are kv_quant's e2m1 rounding of x / sd where sd is
    the e4m3-rounded scale; absmax picks e4m3(absmax/6)."""
    import sys
    k = torch.randn(2, 48, 64, generator=torch.Generator().manual_seed(3)).bfloat16()
    v = torch.randn(2, 48, 64, generator=torch.Generator().manual_seed(4)).bfloat16()
    for calib in CALIBS:
        c = oracle.store_nvfp4(k, v, calib, calib)
        kd, vd = oracle.dequant_nvfp4(c)
        # every block: dequant == e2m1_grid(x/sd)*sd with sd from the stored byte
        sd = np.array([oracle.lib().orc_e4m3_to_f32(int(b)) for b in c["v_scale"].ravel()],
                      np.float32).reshape(c["v_scale"].shape)
        xb = v.float().numpy().reshape(2, 48, 4, 16)
        y = xb / sd[..., None]
        lv = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
        bd = np.array([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
        q = np.sign(y) * lv[np.searchsorted(bd, np.abs(y), side="left")]
        assert np.array_equal(q * sd[..., None], vd.reshape(2, 48, 4, 16))
        if calib == "absmax":
            am = np.abs(xb).max(-1)
            want = np.array([oracle.lib().orc_f32_to_e4m3(float(np.float32(a) / np.float32(6)))
                             for a in am.ravel()], np.uint8).reshape(am.shape)
            assert np.array_equal(want, c["v_scale"])
