"""The legacy page-level API of kv_quant (kv_quant.py:37-191) on the GPU:
quantize_page / QuantizedPage.dequantize / QuantizedKVLayer / QuantizedKVCache /
measure_page_error, compared with the reference's own outputs (golden fixture
made by running the reference's kv_quant) and with the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits, load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("use_mse", (False, True))
def test_quantize_page_matches_reference(cuda_dev, use_mse):
    import kv_quant
    g = load_golden("legacy_page.npz")
    tag = "mse" if use_mse else "absmax"
    k, v = bf16_from_bits(g["k"])[:, :16], bf16_from_bits(g["v"])[:, :16]
    pg = kv_quant.quantize_page(k.to(cuda_dev), v.to(cuda_dev), 0, use_mse=use_mse)
    assert pg.k_int4.dtype == torch.int8 and pg.k_scale.dtype == torch.float16
    assert np.array_equal(pg.k_int4.cpu().numpy(), g[f"page_{tag}_k_int4"])
    assert np.array_equal(pg.v_int4.cpu().numpy(), g[f"page_{tag}_v_int4"])
    assert np.array_equal(pg.k_scale.cpu().view(torch.int16).numpy().view(np.uint16), g[f"page_{tag}_k_scale"])
    assert np.array_equal(pg.v_scale.cpu().view(torch.int16).numpy().view(np.uint16), g[f"page_{tag}_v_scale"])
    kd, vd = pg.dequantize()
    assert torch.equal(kd.cpu(), bf16_from_bits(g[f"page_{tag}_k_deq"]))
    assert torch.equal(vd.cpu(), bf16_from_bits(g[f"page_{tag}_v_deq"]))
    assert [pg.mem_bytes(), pg.bf16_bytes()] == g[f"page_{tag}_mem"].tolist()


def test_quantize_page_fp32_input(cuda_dev):
    import kv_quant
    g = load_golden("legacy_page.npz")
    kf = torch.from_numpy(g["f32_k"]).to(cuda_dev)
    vf = torch.from_numpy(g["f32_v"]).to(cuda_dev)
    pg = kv_quant.quantize_page(kf, vf, 0, use_mse=True, n_alphas=7)
    assert np.array_equal(pg.k_int4.cpu().numpy(), g["f32_k_int4"])
    assert np.array_equal(pg.v_int4.cpu().numpy(), g["f32_v_int4"])
    assert np.array_equal(pg.k_scale.cpu().view(torch.int16).numpy().view(np.uint16), g["f32_k_scale"])


def test_quantized_kv_cache_ragged_appends(cuda_dev):
    """Two layers fed 5, 20, 1, 13, 9 tokens: get_kv after each append,
    memory accounting and compression ratio equal the reference's."""
    import kv_quant
    g = load_golden("legacy_page.npz")
    k, v = bf16_from_bits(g["k"]).to(cuda_dev), bf16_from_bits(g["v"]).to(cuda_dev)
    cache = kv_quant.QuantizedKVCache()
    t = 0
    for n in (5, 20, 1, 13, 9):
        for layer in (0, 1):
            sc = 1.0 if layer == 0 else 0.25
            cache.update(layer, (k[None, :, t:t + n] * sc).bfloat16(), (v[None, :, t:t + n] * sc).bfloat16())
        t += n
        kk, vv = cache.get_kv(1)
        assert torch.equal(kk.cpu(), bf16_from_bits(g[f"cache_t{t}_k"])), t
        assert torch.equal(vv.cpu(), bf16_from_bits(g[f"cache_t{t}_v"])), t
        assert [cache.mem_bytes(), cache.bf16_bytes()] == g[f"cache_t{t}_mem"].tolist()
        assert cache.compression_ratio() == pytest.approx(float(g[f"cache_t{t}_ratio"][0]), rel=1e-12)
        assert cache.layers[1].seq_len() == int(g[f"cache_t{t}_len"][0])
    kk, vv = cache.get_kv(0)
    assert torch.equal(kk.cpu(), bf16_from_bits(g["cache_l0_k"]))
    assert torch.equal(vv.cpu(), bf16_from_bits(g["cache_l0_v"]))
    # the page records the reference exposes as `layer.pages`
    pages = cache.layers[0].pages
    assert [p.start_pos for p in pages] == [0, 16, 32]
    kd, _ = pages[1].dequantize()
    assert torch.equal(kd.cpu(), bf16_from_bits(g["cache_l0_k"])[0, :, 16:32])


def test_quantized_kv_layer_empty_raises(cuda_dev):
    import kv_quant
    with pytest.raises(ValueError):
        kv_quant.QuantizedKVLayer().get_kv()


@pytest.mark.parametrize("use_mse", (False, True))
def test_quantized_kv_layer_vs_oracle(cuda_dev, use_mse):
    """A 4-head, 1000-token layer (62 pages + 8 hot tokens) grown in chunks
    that cross page boundaries and the buffer's capacity, against the oracle."""
    import kv_quant
    gen = torch.Generator().manual_seed(3)
    k = (torch.randn(4, 1000, 128, generator=gen) ** 3).bfloat16()
    v = torch.randn(4, 1000, 128, generator=gen).bfloat16()
    layer = kv_quant.QuantizedKVLayer(use_mse=use_mse)
    t = 0
    for n in (7, 300, 1, 500, 192):
        layer.append(k[:, t:t + n].to(cuda_dev), v[:, t:t + n].to(cuda_dev))
        t += n
    kk, vv = layer.get_kv()
    calib = "mse" if use_mse else "absmax"
    for x, got in ((k, kk), (v, vv)):
        codes, sc = oracle.page_quantize(x[:, :992], calib)
        want = torch.cat([oracle.page_dequant(codes, sc), x[:, 992:]], dim=1)
        assert torch.equal(got.cpu(), want)


def test_measure_page_error(cuda_dev):
    import kv_quant
    g = load_golden("legacy_page.npz")
    e = kv_quant.measure_page_error(torch.from_numpy(g["err_x"]).to(cuda_dev))
    np.testing.assert_allclose([e["absmax_mse"], e["optimal_mse"], e["reduction_pct"]], g["err"], rtol=1e-5)
