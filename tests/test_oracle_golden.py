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


# ---------------------------------------------------------------------------
# Paged cache: the e4m3 calibration of scripts/diag_kernel_perchannel.py:30-53
# ---------------------------------------------------------------------------
def test_paged_calib_per_token_bit_exact():
    g = load_golden("paged_calib.npz")
    got = oracle.paged_calib(g["tok"], "int4", "mse")
    assert np.array_equal(got, g["tok_scale"])
    # dequantised values: rint(x / s) clamped to +-7, times s
    s = np.array([oracle.lib().orc_e4m3_to_f32(int(b)) for b in got], np.float32)[:, None]
    deq = np.clip(np.rint(g["tok"] / s), -7, 7) * s
    assert np.array_equal(deq.astype(np.float32), g["tok_deq"])


def test_paged_calib_per_channel_bit_exact():
    g = load_golden("paged_calib.npz")
    chan = g["chan"]                                            # [16 tokens, H, D]
    got = oracle.paged_calib(np.ascontiguousarray(chan.transpose(1, 2, 0)), "int4", "mse")
    assert np.array_equal(got, g["chan_scale"])


def _paged_prefill(L, H=2, D=128, seed=0, fmt="int4"):
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((L, H, D)) * np.exp(rng.uniform(-1, 2, (1, H, D)))).astype(np.float32)
    v = rng.standard_normal((L, H, D)).astype(np.float32)
    nb = (L + 15) // 16
    kv = np.zeros((nb + 2, 2, 16, H, oracle.paged_full_dim(D)), np.uint8)
    phys = np.arange(1, nb + 1)
    slots = np.array([phys[t // 16] * 16 + t % 16 for t in range(L)], np.int64)
    assert oracle.paged_store(k, v, slots, kv, fmt) == 0
    return k, v, kv, phys


@pytest.mark.parametrize("L", (15, 16, 40, 64))
def test_paged_oracle_store_geometry(L):
    """Full blocks carry per-channel K scales, the partial tail per-token ones;
    the gather reproduces the per-channel / per-token calibration exactly."""
    H, D = 2, 128
    k, v, kv, phys = _paged_prefill(L, H, D)
    kd, vd = oracle.paged_gather(kv, phys[None].astype(np.int32), [L], H, D, "int4", L)
    for h in range(H):
        for b in range(L // 16):
            blk = k[16 * b:16 * b + 16, h]                       # [16, D]
            sc = oracle.paged_calib(np.ascontiguousarray(blk.T), "int4", "mse")
            s = np.array([oracle.lib().orc_e4m3_to_f32(int(x)) for x in sc], np.float32)
            want = np.clip(np.rint(blk / s[None]), -7, 7) * s[None]
            assert np.array_equal(kd[0, h, 16 * b:16 * b + 16], want)
        for t in range((L // 16) * 16, L):
            blocks = k[t, h].reshape(-1, 16)
            sc = oracle.paged_calib(blocks, "int4", "mse")
            s = np.array([oracle.lib().orc_e4m3_to_f32(int(x)) for x in sc], np.float32)[:, None]
            want = (np.clip(np.rint(blocks / s), -7, 7) * s).reshape(-1)
            assert np.array_equal(kd[0, h, t], want)
    assert np.abs(vd[0] - v.transpose(1, 0, 2)).max() < 0.6


def test_paged_oracle_block_completion_across_calls():
    """A block grown token by token becomes per channel when its 16th slot is
    written; the earlier rows are requantised from their per-token values."""
    H, D = 1, 64
    rng = np.random.default_rng(3)
    k = rng.standard_normal((16, H, D)).astype(np.float32)
    v = rng.standard_normal((16, H, D)).astype(np.float32)
    kv = np.zeros((2, 2, 16, H, oracle.paged_full_dim(D)), np.uint8)
    for t in range(15):
        oracle.paged_store(k[t:t + 1], v[t:t + 1], np.array([16 + t]), kv)
    kd15, _ = oracle.paged_gather(kv, np.array([[1]], np.int32), [15], H, D, "int4", 15)
    oracle.paged_store(k[15:], v[15:], np.array([31]), kv)
    kd16, _ = oracle.paged_gather(kv, np.array([[1]], np.int32), [16], H, D, "int4", 16)
    src = np.concatenate([kd15[0, 0], k[15, 0][None]], 0)       # [16, D]
    sc = oracle.paged_calib(np.ascontiguousarray(src.T), "int4", "mse")
    s = np.array([oracle.lib().orc_e4m3_to_f32(int(x)) for x in sc], np.float32)
    assert np.array_equal(kd16[0, 0], np.clip(np.rint(src / s[None]), -7, 7) * s[None])


def test_paged_oracle_store_call_boundaries():
    """Chunked stores: chunks that end on block boundaries give the same bytes
    as one call; a chunk ending mid-block leaves that block per-token until a
    later call completes it (then it is requantised per channel from the
    dequantised rows, so the bytes differ from a one-call store); padding
    slots (-1) are skipped; an out-of-range slot is reported, the rest stored."""
    H, D, L = 2, 64, 48
    rng = np.random.default_rng(7)
    k = rng.standard_normal((L, H, D)).astype(np.float32)
    v = rng.standard_normal((L, H, D)).astype(np.float32)
    slots = np.arange(16, 16 + L, dtype=np.int64)
    shape = (5, 2, 16, H, oracle.paged_full_dim(D))
    one = np.zeros(shape, np.uint8)
    oracle.paged_store(k, v, slots, one)
    aligned = np.zeros(shape, np.uint8)
    for a, b in ((0, 16), (16, 48)):
        oracle.paged_store(k[a:b], v[a:b], slots[a:b], aligned)
    assert np.array_equal(one, aligned)
    ragged = np.zeros(shape, np.uint8)
    for a, b in ((0, 20), (20, 48)):
        oracle.paged_store(k[a:b], v[a:b], slots[a:b], ragged)
    assert np.array_equal(one[1], ragged[1])                  # block 1 complete within the first call
    assert not np.array_equal(one[2, 0], ragged[2, 0])        # block 2's K was requantised on completion
    assert np.array_equal(one[2, 1], ragged[2, 1])            # V is per token either way
    padded = np.zeros(shape, np.uint8)
    sl = slots.copy(); sl[5] = -1
    oracle.paged_store(k, v, sl, padded)
    assert not padded[1, 1, 5].any()                          # the padding token's V row is untouched
    bad = np.zeros(shape, np.uint8)
    sl = slots.copy(); sl[-1] = 10 ** 6
    assert oracle.paged_store(k, v, sl, bad) == 1
    assert np.array_equal(bad[1], one[1])


# ---------------- legacy page API (kv_quant.py:37-191) ----------------
@pytest.mark.parametrize("calib", CALIBS)
def test_legacy_page_oracle(calib):
    g = load_golden("legacy_page.npz")
    k, v = bf16_from_bits(g["k"])[:, :16], bf16_from_bits(g["v"])[:, :16]
    for name, x in (("k", k), ("v", v)):
        codes, sc = oracle.page_quantize(x, calib)
        assert np.array_equal(codes, g[f"page_{calib}_{name}_int4"])
        assert np.array_equal(sc.view(np.uint16), g[f"page_{calib}_{name}_scale"])
        assert torch.equal(oracle.page_dequant(codes, sc), bf16_from_bits(g[f"page_{calib}_{name}_deq"]))


def test_legacy_page_oracle_fp32_input():
    g = load_golden("legacy_page.npz")
    for name in ("k", "v"):
        codes, sc = oracle.page_quantize(g[f"f32_{name}"], "mse", n_alphas=7)
        assert np.array_equal(codes, g[f"f32_{name}_int4"])
        assert np.array_equal(sc.view(np.uint16), g[f"f32_{name}_scale"])


def test_legacy_page_error_oracle():
    g = load_golden("legacy_page.npz")
    a, o = oracle.page_error(g["err_x"])
    np.testing.assert_allclose([a, o], g["err"][:2], rtol=1e-6)


# ------------- heavy-tailed K of the reference test (randn**3) -------------
@pytest.mark.parametrize("calib", CALIBS)
def test_heavy_tail_store_oracle(calib):
    g = load_golden("heavy_tail.npz")
    k, v = bf16_from_bits(g["k"]), bf16_from_bits(g["v"])
    c = oracle.store_int4(k, v, calib, calib)
    assert np.array_equal(c["k_packed"], g[f"{calib}_k_packed"])
    assert np.array_equal(c["k_scale"].view(np.uint16), g[f"{calib}_k_scale"])
    assert np.array_equal(c["v_packed"], g[f"{calib}_v_packed"])
    assert np.array_equal(c["v_scale"].view(np.uint16), g[f"{calib}_v_scale"])
    rt = torch.from_numpy(oracle.roundtrip_f32(k, "int4", "channel", calib)).to(torch.bfloat16)
    assert torch.equal(rt, bf16_from_bits(g[f"{calib}_k_rt"]))


@pytest.mark.parametrize("calib", CALIBS)
def test_int3v_store_pinned_to_roundtrip(calib):
    """The mixed cache's INT3 V codes, times the fp32 block scale, are the
    reference's kv_quant.roundtrip(v, "int3", "headdim", calib) bit for bit;
    the stored fp16 scale is that fp32 scale rounded; dequant = code * scale."""
    g = load_golden("kvq_roundtrip.npz")
    k, v = bf16_from_bits(g["k"]), bf16_from_bits(g["v"])
    H, S, D = v.shape
    c = oracle.store_int3v(k, v, calib, calib)
    assert c["v_packed"].shape == (H, S, D // 32, 12)
    codes = oracle.unpack_int3(c["v_packed"]).astype(np.float32)
    assert codes.min() >= -3 and codes.max() <= 3
    s32 = oracle.calibrate(v.float().numpy().reshape(-1, 16), "int3", calib).reshape(H, S, D // 16, 1)
    got = torch.from_numpy((codes * s32).reshape(H, S, D)).to(torch.bfloat16)
    assert torch.equal(got, bf16_from_bits(g[f"v_int3_headdim_{calib}"]))
    assert np.array_equal(c["v_scale"], s32[..., 0].astype(np.float16))
    _, vd = oracle.dequant_int3v(c)
    assert np.array_equal(vd, (codes * c["v_scale"][..., None].astype(np.float32)).reshape(H, S, D))
    # K is the INT4 cache's K
    c4 = oracle.store_int4(k, v, calib, calib)
    assert np.array_equal(c["k_packed"], c4["k_packed"]) and np.array_equal(c["k_scale"], c4["k_scale"])
