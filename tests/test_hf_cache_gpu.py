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


def _ref_attention(q, k, v, scale):
    """fp32 attention of q [Hq, D] over k, v [H, S, D] (GQA by repeat)."""
    G = q.shape[0] // k.shape[0]
    kk = k.float().repeat_interleave(G, 0)
    vv = v.float().repeat_interleave(G, 0)
    p = torch.softmax((q.float()[:, None] @ kk.transpose(1, 2))[:, 0] * scale, -1)
    return (p[:, None] @ vv)[:, 0]


def _exact_kv(layer):
    """fp32 K/V a layer holds: packed pages dequantised exactly (code *
    fp32(scale), the oracle's dequant; `update` returns them rounded to bf16)
    followed by the bf16 partial page."""
    import oracle
    ks, vs = [], []
    if layer._frozen_len():
        c = layer.store
        d = dict(k_packed=c.k_packed.cpu().numpy(), k_scale=c.k_scale.cpu().numpy(),
                 v_packed=c.v_packed.cpu().numpy(), v_scale=c.v_scale.cpu().numpy(),
                 k_hot=c.k_hot.float().cpu().numpy(), H=c.H, S=c.S, D=c.D)
        k, v = oracle.dequant_int4(d) if c.fmt == "int4" else oracle.dequant_int3v(d)
        ks.append(torch.from_numpy(k)); vs.append(torch.from_numpy(v))
    if layer._hot_len():
        ks.append(layer.hot_k.float().cpu()); vs.append(layer.hot_v.float().cpu())
    return torch.cat(ks, 1), torch.cat(vs, 1)


def test_fused_decode_matches_dequant_path(cuda_dev):
    """The fused read path (packed pages + bf16 partial page, no bf16 K/V
    materialised) equals fp32 attention over the same stored tokens, and the
    plain layer's `update` returns those tokens (rounded to bf16):
    |out - ref| <= 2e-3 + |ref| * 2^-8, including steps with no full page yet
    and steps right after a page freezes."""
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, Hq, D = 2, 8, 128
    k, v, _ = gen_kv(H, 120, D, seed=8)
    kd, vd = k.to(cuda_dev), v.to(cuda_dev)
    g = torch.Generator().manual_seed(9)
    for pre in (5, 37):
        plain, fused = _Int4KiviLayer(), _Int4KiviLayer(fused_decode=True)
        plain.update(kd[None, :, :pre], vd[None, :, :pre])
        fused.update(kd[None, :, :pre], vd[None, :, :pre])
        for t in range(pre, 100):
            kk, vv = plain.update(kd[None, :, t:t + 1], vd[None, :, t:t + 1])
            stub, _ = fused.update(kd[None, :, t:t + 1], vd[None, :, t:t + 1])
            assert stub.shape[2] == 0 and stub._kivi_layer is fused
            q = torch.randn(1, Hq, 1, D, generator=g).bfloat16().to(cuda_dev)
            out = fused.fused_decode(q, D ** -0.5)[0].float().cpu()
            ek, ev = _exact_kv(fused)
            assert torch.equal(ek.bfloat16(), kk[0].cpu()) and torch.equal(ev.bfloat16(), vv[0].cpu())
            ref = _ref_attention(q[0, :, 0].cpu(), ek, ev, D ** -0.5)
            err = (out - ref).abs()
            assert bool((err <= 2e-3 + ref.abs() * 2.0 ** -8).all()), (pre, t, err.max().item())
        assert fused.get_seq_length() == plain.get_seq_length() == 100
        assert fused._deq_k is None                          # no bf16 copy kept in fused mode


def test_fused_multi_token_steps(cuda_dev):
    """Steps of 2..8 new tokens (speculative verify) on the fused read path:
    each query attends the stored tokens up to its own position, compared
    with fp32 attention over exactly those tokens, across page boundaries and
    from an empty cache."""
    from conftest import check_decode_bf16
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, Hq, D = 2, 8, 128
    k, v, _ = gen_kv(H, 160, D, seed=31)
    kd, vd = k.to(cuda_dev), v.to(cuda_dev)
    g = torch.Generator().manual_seed(32)
    fused = _Int4KiviLayer(fused_decode=True)
    pos = 0
    for n in (3, 8, 5, 2, 7, 16, 4, 6):
        stub, _ = fused.update(kd[None, :, pos:pos + n], vd[None, :, pos:pos + n])
        pos += n
        if n > 8:                                      # prefill-sized step: the dense path
            assert stub.shape[2] == pos
            continue
        assert stub.shape[2] == 0 and stub._kivi_layer is fused
        q = torch.randn(1, Hq, n, D, generator=g).bfloat16().to(cuda_dev)
        out = fused.fused_decode(q, D ** -0.5)[0].float().cpu()        # [n, Hq, D]
        ek, ev = _exact_kv(fused)
        ref = torch.stack([_ref_attention(q[0, :, j].cpu(), ek[:, :pos - n + j + 1], ev[:, :pos - n + j + 1],
                                          D ** -0.5) for j in range(n)])
        check_decode_bf16(out, ref, f"pos={pos} n={n}")


def test_fused_generate_tiny_random_model(cuda_dev):
    """Teacher-forced decode of a random tiny Llama: the fused path's logits
    track the dequantise + SDPA path's; greedy generate runs end to end."""
    transformers = pytest.importorskip("transformers")
    from int4_kivi.hf_cache import Int4KiviCache, enable_fused_decode
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).to(cuda_dev, torch.bfloat16).eval()
    ids = torch.randint(0, 128, (1, 80), device=cuda_dev)
    with torch.no_grad():
        c_ref = Int4KiviCache(config=cfg)
        ref = [model(ids[:, :40], past_key_values=c_ref).logits[:, -1]]
        for t in range(40, 80):
            ref.append(model(ids[:, t:t + 1], past_key_values=c_ref).logits[:, -1])
        enable_fused_decode(model)
        c_f = Int4KiviCache(config=cfg, fused_decode=True)
        got = [model(ids[:, :40], past_key_values=c_f).logits[:, -1]]
        for t in range(40, 80):
            got.append(model(ids[:, t:t + 1], past_key_values=c_f).logits[:, -1])
        # the same tokens fed 4 at a time (a speculative verify step): every
        # position's logits, through the multi-query fused path vs SDPA
        c_m = Int4KiviCache(config=cfg, fused_decode=True)
        model(ids[:, :40], past_key_values=c_m)
        multi = [model(ids[:, t:t + 4], past_key_values=c_m).logits[0] for t in range(40, 80, 4)]
        model.set_attn_implementation("sdpa")
        c_r = Int4KiviCache(config=cfg)
        model(ids[:, :40], past_key_values=c_r)
        multi_ref = [model(ids[:, t:t + 4], past_key_values=c_r).logits[0] for t in range(40, 80, 4)]
        enable_fused_decode(model)
    mr, mg = torch.cat(multi_ref).float(), torch.cat(multi).float()
    assert (mr - mg).abs().max().item() <= 0.02 * mr.abs().max().item()
    r, g_ = torch.stack(ref).float(), torch.stack(got).float()
    assert torch.equal(r[0], g_[0])                           # prefill takes the same path
    assert (r - g_).abs().max().item() <= 0.02 * r.abs().max().item()
    assert all(l._deq_k is None for l in c_f.layers)         # no bf16 copy of the prefix kept
    out = model.generate(ids[:, :40], max_new_tokens=16, do_sample=False,
                         past_key_values=Int4KiviCache(config=cfg, fused_decode=True))
    assert out.shape == (1, 56)
    model.set_attn_implementation("sdpa")


def test_batched_layer_equals_single_sequences(cuda_dev):
    """B = 2 sequences stored as stacked heads: `update` returns exactly what
    two batch-1 layers return, and the fused decode of each row equals fp32
    attention over that row's stored tokens."""
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, Hq, D, B = 2, 8, 128, 2
    k, v, _ = gen_kv(B * H, 90, D, seed=21)
    kd, vd = k.view(B, H, 90, D).to(cuda_dev), v.view(B, H, 90, D).to(cuda_dev)
    g = torch.Generator().manual_seed(22)
    batched, fused = _Int4KiviLayer(), _Int4KiviLayer(fused_decode=True)
    single = [_Int4KiviLayer() for _ in range(B)]
    pos = 0
    for n in (21, 1, 1, 10, 1, 40, 1):
        kk, vv = batched.update(kd[:, :, pos:pos + n], vd[:, :, pos:pos + n])
        fused.update(kd[:, :, pos:pos + n], vd[:, :, pos:pos + n])
        for b in range(B):
            sk, sv = single[b].update(kd[b:b + 1, :, pos:pos + n], vd[b:b + 1, :, pos:pos + n])
            assert torch.equal(kk[b:b + 1], sk) and torch.equal(vv[b:b + 1], sv)
        pos += n
        assert kk.shape == (B, H, pos, D) and batched.get_seq_length() == pos
        if n == 1:
            q = torch.randn(B, Hq, 1, D, generator=g).bfloat16().to(cuda_dev)
            out = fused.fused_decode(q, D ** -0.5).float().cpu()
            ek, ev = _exact_kv(fused)                       # [B*H, pos, D], sequence-major
            for b in range(B):
                ref = _ref_attention(q[b, :, 0].cpu(), ek[b * H:(b + 1) * H], ev[b * H:(b + 1) * H], D ** -0.5)
                err = (out[b] - ref).abs()
                assert bool((err <= 2e-3 + ref.abs() * 2.0 ** -8).all()), (pos, b, err.max().item())
    with pytest.raises(ValueError):
        batched.update(kd[:1, :, :1], vd[:1, :, :1])        # batch size may not change


def test_batched_generate_tiny_random_model(cuda_dev):
    """Batch 2 through a random tiny Llama: teacher-forced logits of the
    batch track each sequence run alone; fused and dequantise paths agree;
    a left-padded batch takes SDPA in the fused cache too (same tokens as the
    dequantise path, bit for bit)."""
    transformers = pytest.importorskip("transformers")
    from int4_kivi.hf_cache import Int4KiviCache, enable_fused_decode
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).to(cuda_dev, torch.bfloat16).eval()
    ids = torch.randint(0, 128, (2, 70), device=cuda_dev)

    def forced(x, **kw):
        c = Int4KiviCache(config=cfg, **kw)
        lg = [model(x[:, :40], past_key_values=c).logits[:, -1]]
        for t in range(40, 70):
            lg.append(model(x[:, t:t + 1], past_key_values=c).logits[:, -1])
        return torch.stack(lg, 1).float()                    # [B, 31, vocab]

    with torch.no_grad():
        both = forced(ids)
        alone = torch.cat([forced(ids[b:b + 1]) for b in range(2)])
        enable_fused_decode(model)
        fused = forced(ids, fused_decode=True)
    scale = both.abs().max().item()
    assert (both - alone).abs().max().item() <= 0.02 * scale
    assert (both - fused).abs().max().item() <= 0.02 * scale
    pad = torch.ones(2, 40, dtype=torch.long, device=cuda_dev)
    pad[1, :5] = 0                                           # left-padded second row
    x = ids[:, :40].clone()
    x[1, :5] = 0
    out_f = model.generate(x, attention_mask=pad, max_new_tokens=12, do_sample=False,
                           past_key_values=Int4KiviCache(config=cfg, fused_decode=True))
    model.set_attn_implementation("sdpa")
    out_d = model.generate(x, attention_mask=pad, max_new_tokens=12, do_sample=False,
                           past_key_values=Int4KiviCache(config=cfg))
    assert out_f.shape == (2, 52) and torch.equal(out_f, out_d)


def test_int3v_layer_update_and_fused_decode(cuda_dev):
    """v_bits=3 (K INT4, V INT3): `update` returns store_kivi_int3v +
    dequant of the completed pages and the bf16 partial page; the fused read
    path (single and multi-token steps) meets the decode bar against fp32
    attention over the exactly dequantised tokens."""
    from conftest import check_decode_bf16
    from int4_kivi.hf_cache import _Int4KiviLayer
    from int4_kivi.mixed import dequant_kivi_int3v, store_kivi_int3v
    H, Hq, D = 2, 8, 128
    k, v, _ = gen_kv(H, 200, D, seed=41)
    kd, vd = k.to(cuda_dev), v.to(cuda_dev)
    g = torch.Generator().manual_seed(42)
    plain, fused = _Int4KiviLayer(v_bits=3), _Int4KiviLayer(fused_decode=True, v_bits=3)
    pos = 0
    for n in (37, 1, 1, 3, 14, 8, 1, 60, 5, 1):
        kk, vv = plain.update(kd[None, :, pos:pos + n], vd[None, :, pos:pos + n])
        stub, _ = fused.update(kd[None, :, pos:pos + n], vd[None, :, pos:pos + n])
        pos += n
        nf = (pos // 16) * 16
        rk, rv = dequant_kivi_int3v(store_kivi_int3v(kd[:, :nf], vd[:, :nf])) if nf else (kd[:, :0], vd[:, :0])
        assert torch.equal(kk[0], torch.cat([rk, kd[:, nf:pos]], 1))
        assert torch.equal(vv[0], torch.cat([rv, vd[:, nf:pos]], 1))
        if n > 8:
            continue
        q = torch.randn(1, Hq, n, D, generator=g).bfloat16().to(cuda_dev)
        out = fused.fused_decode(q, D ** -0.5)
        out = (out[0] if n > 1 else out).float().cpu().reshape(n, Hq, D)
        ek, ev = _exact_kv(fused)
        ref = torch.stack([_ref_attention(q[0, :, j].cpu(), ek[:, :pos - n + j + 1], ev[:, :pos - n + j + 1],
                                          D ** -0.5) for j in range(n)])
        check_decode_bf16(out, ref, f"int3v pos={pos} n={n}")
    assert fused.store.fmt == "int4k_int3v" and fused.store.v_packed.shape[2:] == (D // 32, 12)


def test_int3v_generate_tiny_random_model(cuda_dev):
    """Int4KiviCache(v_bits=3): fused decode logits track the same cache's
    dequantise + SDPA path, greedy generate runs, and the cache is smaller
    than the INT4 one for the same tokens."""
    transformers = pytest.importorskip("transformers")
    from int4_kivi.hf_cache import Int4KiviCache, enable_fused_decode
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).to(cuda_dev, torch.bfloat16).eval()
    ids = torch.randint(0, 128, (1, 80), device=cuda_dev)
    with torch.no_grad():
        c_ref, c4 = Int4KiviCache(config=cfg, v_bits=3), Int4KiviCache(config=cfg)
        model(ids[:, :40], past_key_values=c4)
        ref = [model(ids[:, :40], past_key_values=c_ref).logits[:, -1]]
        for t in range(40, 80):
            ref.append(model(ids[:, t:t + 1], past_key_values=c_ref).logits[:, -1])
            model(ids[:, t:t + 1], past_key_values=c4)
        enable_fused_decode(model)
        c_f = Int4KiviCache(config=cfg, fused_decode=True, v_bits=3)
        got = [model(ids[:, :40], past_key_values=c_f).logits[:, -1]]
        for t in range(40, 80):
            got.append(model(ids[:, t:t + 1], past_key_values=c_f).logits[:, -1])
        out = model.generate(ids[:, :40], max_new_tokens=16, do_sample=False,
                             past_key_values=Int4KiviCache(config=cfg, fused_decode=True, v_bits=3))
        model.set_attn_implementation("sdpa")
    r, g_ = torch.stack(ref).float(), torch.stack(got).float()
    assert (r - g_).abs().max().item() <= 0.02 * r.abs().max().item()
    assert out.shape == (1, 56)
    assert c_ref.nbytes() < c4.nbytes()
