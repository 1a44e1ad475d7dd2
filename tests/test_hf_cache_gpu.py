"""Int4KiviCache (HF transformers Cache) on the B200 kernels: the values
returned by `update` equal the reference contract (int4_kivi/hf_cache.py:
157-190): completed pages dequantised from INT4-KIVI, the partial page bf16,
sliding layers trimmed to window - 1 + new tokens."""
import pytest
import torch

from conftest import gen_kv

pytestmark = pytest.mark.gpu


def test_update_matches_store_dequant(cuda_dev):
    from int4_kivi import dequant_kivi, store_kivi
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, D, S = 4, 128, 300
    k, v, _ = gen_kv(H, S, D, seed=3)
    layer = _Int4KiviLayer()
    pos = 0
    for n in (37, 1, 1, 14, 100, 147):
        kk, vv = layer.update(k[None, :, pos:pos + n].to(cuda_dev), v[None, :, pos:pos + n].to(cuda_dev))
        pos += n
        nf = (pos // 16) * 16
        ref = store_kivi(k[:, :nf].to(cuda_dev), v[:, :nf].to(cuda_dev)) if nf else None
        rk, rv = dequant_kivi(ref) if ref is not None else (k[:, :0].to(cuda_dev), v[:, :0].to(cuda_dev))
        want_k = torch.cat([rk, k[:, nf:pos].to(cuda_dev)], 1)
        want_v = torch.cat([rv, v[:, nf:pos].to(cuda_dev)], 1)
        assert kk.shape == (1, H, pos, D)
        assert torch.equal(kk[0], want_k) and torch.equal(vv[0], want_v)
    assert layer.get_seq_length() == S


def test_sliding_window_contract(cuda_dev):
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, D = 2, 128
    k, v, _ = gen_kv(H, 200, D, seed=4)
    layer = _Int4KiviLayer(is_sliding=True, sliding_window=64)
    pos = 0
    for n in (50, 30, 1, 1, 60, 58):
        kk, _ = layer.update(k[None, :, pos:pos + n].to(cuda_dev), v[None, :, pos:pos + n].to(cuda_dev))
        pos += n
        want = min(pos, 64 - 1 + n) if pos >= 64 else pos
        assert kk.shape[2] == want
        kv_len, off = layer.get_mask_sizes(1)
        assert off == max(pos - 64 + 1, 0)


def test_sliding_window_long_run_compacts(cuda_dev):
    """Thousands of single-token steps on a sliding layer: the returned window
    stays the last window-1+1 tokens and the store is compacted."""
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, D, W = 2, 128, 100
    k, v, _ = gen_kv(H, 2600, D, seed=5)
    kd, vd = k.to(cuda_dev), v.to(cuda_dev)
    layer = _Int4KiviLayer(is_sliding=True, sliding_window=W)
    layer.update(kd[None, :, :64], vd[None, :, :64])
    for t in range(64, 2600):
        kk, vv = layer.update(kd[None, :, t:t + 1], vd[None, :, t:t + 1])
    assert kk.shape[2] == W
    assert torch.equal(kk[0, :, -1], kd[:, 2599])          # newest token is bf16 verbatim
    assert layer.store.S <= 2048 + W + 64


def test_generate_with_tiny_random_model(cuda_dev):
    transformers = pytest.importorskip("transformers")
    from int4_kivi.hf_cache import Int4KiviCache
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).to(cuda_dev, torch.bfloat16).eval()
    ids = torch.randint(0, 128, (1, 40), device=cuda_dev)
    cache = Int4KiviCache(config=cfg)
    out = model.generate(ids, max_new_tokens=24, do_sample=False, past_key_values=cache)
    assert out.shape == (1, 64)
    assert cache.layers[0].get_seq_length() == 63
    assert cache.compression_ratio_vs_bf16() > 1.5
