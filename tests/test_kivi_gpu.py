"""GPU parity tests: libkivi_sm100 (through the package API and its C ABI)
against the CPU oracle on identical seeded inputs.

Bars:
  * codes, scales, dequantised K/V, roundtrip outputs: bit-exact;
  * decode attention: the one decode bar of conftest.py (fp32 state max-abs
    <= 2e-3 and relative RMS <= 1e-3; bf16 output relative RMS <= 1e-3 vs the
    bf16-rounded oracle and |out - ref| <= 2e-3 + |ref| * 2^-8).
Mirrors the reference's tests/test_int4_kivi.py cases (code parity S in
{256, 512, 2048} x {absmax, mse}, dequant vs roundtrip, hot page S=40, memory
ratio) with the tolerance tightened to exact.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import check_decode_bf16, check_decode_fp32, gen_kv

pytestmark = pytest.mark.gpu

H, D = 8, 128


def _np(t):
    return t.detach().cpu().numpy()


# ---------------------------------------------------------------- store ----
@pytest.mark.parametrize("calib", ["absmax", "mse"])
@pytest.mark.parametrize("S", [256, 512, 2048, 40, 1, 15, 17])
def test_store_bit_exact(cuda_dev, S, calib):
    from int4_kivi import store_kivi
    k, v, _ = gen_kv(H, S, D, seed=S)
    c = store_kivi(k.to(cuda_dev), v.to(cuda_dev), k_calib=calib, v_calib=calib)
    o = oracle.store_int4(k, v, calib, calib)
    NP = S // 16
    assert c.k_packed.shape == (H, D, NP, 8) and c.v_packed.shape == (H, S, D // 16, 8)
    assert np.array_equal(_np(c.k_packed), o["k_packed"])
    assert np.array_equal(_np(c.v_packed), o["v_packed"])
    assert np.array_equal(_np(c.k_scale).view(np.uint16), o["k_scale"].view(np.uint16))
    assert np.array_equal(_np(c.v_scale).view(np.uint16), o["v_scale"].view(np.uint16))
    assert torch.equal(c.k_hot.cpu(), k[:, NP * 16:])


@pytest.mark.parametrize("calib", ["absmax", "mse"])
@pytest.mark.parametrize("S", [40, 2048])
def test_dequant_bit_exact(cuda_dev, S, calib):
    from int4_kivi import dequant_kivi, store_kivi
    k, v, _ = gen_kv(H, S, D, seed=1)
    c = store_kivi(k.to(cuda_dev), v.to(cuda_dev), k_calib=calib, v_calib=calib)
    kq, vq = dequant_kivi(c)
    kd, vd = oracle.dequant_int4(oracle.store_int4(k, v, calib, calib))
    assert torch.equal(kq.cpu(), torch.from_numpy(kd).bfloat16())
    assert torch.equal(vq.cpu(), torch.from_numpy(vd).bfloat16())


@pytest.mark.parametrize("calib", ["absmax", "mse"])
def test_dequant_tracks_roundtrip(cuda_dev, calib):
    """The reference's aggregate check (tests/test_int4_kivi.py:100-127)."""
    import kv_quant
    from int4_kivi import dequant_kivi, store_kivi
    S = 2048
    k, v, _ = gen_kv(H, S, D, seed=1)
    c = store_kivi(k.to(cuda_dev), v.to(cuda_dev), k_calib=calib, v_calib=calib)
    kq, vq = dequant_kivi(c)
    rk = kv_quant.roundtrip(k, "int4", "channel", calib)
    rv = kv_quant.roundtrip(v, "int4", "headdim", calib)

    def rel(a, b):
        return (((a.float().cpu() - b.float()) ** 2).mean().sqrt() / b.float().abs().mean()).item()
    assert rel(kq, rk) < 0.03 and rel(vq, rv) < 0.02


def test_hot_page_and_memory_ratio(cuda_dev):
    from int4_kivi import dequant_kivi, store_kivi
    k, v, _ = gen_kv(H, 40, D, seed=2)
    c = store_kivi(k.to(cuda_dev), v.to(cuda_dev))
    assert c.k_hot.shape == (H, 8, D)
    kq, _ = dequant_kivi(c)
    assert torch.equal(kq[:, 32:].cpu(), k[:, 32:])
    k, v, _ = gen_kv(H, 2048, D, seed=0)
    c = store_kivi(k.to(cuda_dev), v.to(cuda_dev))
    assert 3.0 <= c.compression_ratio_vs_bf16() <= 3.4
    data = c.k_packed.numel() + c.v_packed.numel()
    n_scales = c.k_scale.numel() + c.v_scale.numel()
    assert 3.45 <= c.bf16_nbytes() / (data + n_scales + c.k_hot.numel() * 2) <= 3.65


# ------------------------------------------------------------- kv_quant ----
@pytest.mark.parametrize("fmt", ["int4", "int3", "nvfp4"])
@pytest.mark.parametrize("layout", ["headdim", "channel"])
@pytest.mark.parametrize("calib", ["absmax", "mse"])
def test_roundtrip_bit_exact(cuda_dev, fmt, layout, calib):
    import kv_quant
    k, v, _ = gen_kv(4, 1000, D, seed=7)
    for x in (k, v.float()):
        got = kv_quant.roundtrip(x.to(cuda_dev), fmt, layout, calib).cpu()
        want = torch.from_numpy(oracle.roundtrip_f32(x, fmt, layout, calib)).to(x.dtype)
        assert torch.equal(got, want)
    # host tensors go through the device and come back
    got = kv_quant.roundtrip(k, fmt, layout, calib)
    assert got.device.type == "cpu"


def test_calibrate_matches_oracle(cuda_dev):
    import kv_quant
    k, _, _ = gen_kv(4, 256, D, seed=3)
    xb = kv_quant._to_blocks(k, "channel").float()
    for fmt in ("int4", "nvfp4"):
        for calib in ("absmax", "mse"):
            qmax, qfn = kv_quant._FORMATS[fmt]
            got = kv_quant._calibrate(xb.to(cuda_dev), qmax, qfn, calib).cpu().numpy()
            assert np.array_equal(got, oracle.calibrate(xb, fmt, calib))


# ----------------------------------------------------------------- NVFP4 ----
@pytest.mark.parametrize("calib", ["absmax", "mse"])
@pytest.mark.parametrize("g", [1.0, 0.01])
def test_nvfp4_store_dequant_bit_exact(cuda_dev, calib, g):
    from int4_kivi import dequant_nvfp4_kivi, store_nvfp4_kivi
    k, v, _ = gen_kv(4, 200, D, seed=9)
    c = store_nvfp4_kivi(k.to(cuda_dev), v.to(cuda_dev), calib, calib, g_k=g, g_v=g)
    o = oracle.store_nvfp4(k, v, calib, calib, g, g)
    for f in ("k_packed", "k_scale", "v_packed", "v_scale"):
        assert np.array_equal(_np(getattr(c, f)), o[f]), f
    kq, vq = dequant_nvfp4_kivi(c)
    kd, vd = oracle.dequant_nvfp4(o)
    assert torch.equal(kq.cpu(), torch.from_numpy(kd).bfloat16())
    assert torch.equal(vq.cpu(), torch.from_numpy(vd).bfloat16())


# ---------------------------------------------------------------- decode ----
def _oracle_decode(k, v, q, fmt, calib="mse", g=1.0):
    """q [B,Hq,D], k/v [B,Hkv,S,D] -> fp32 [B,Hq,D] on the oracle's dequant."""
    outs = []
    for b in range(k.shape[0]):
        if fmt == "int4":
            kd, vd = oracle.dequant_int4(oracle.store_int4(k[b], v[b], calib, calib))
        else:
            kd, vd = oracle.dequant_nvfp4(oracle.store_nvfp4(k[b], v[b], calib, calib, g, g))
        outs.append(oracle.decode_attention(q[b:b + 1], kd[None], vd[None], 1.0 / math.sqrt(k.shape[-1]))[0])
    return torch.from_numpy(np.stack(outs))


def _store(fmt, k, v, dev, calib="mse", g=1.0):
    from int4_kivi import store_kivi, store_nvfp4_kivi
    if fmt == "int4":
        return store_kivi(k.to(dev), v.to(dev), calib, calib)
    return store_nvfp4_kivi(k.to(dev), v.to(dev), calib, calib, g_k=g, g_v=g)


_check_fp32 = check_decode_fp32
_check_bf16 = check_decode_bf16


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
@pytest.mark.parametrize("B,Hkv,Hq,S", [(1, 8, 32, 1), (1, 8, 32, 15), (1, 8, 32, 16), (2, 8, 32, 17),
                                         (2, 2, 8, 127), (3, 4, 16, 300), (2, 8, 32, 1000),
                                         (1, 2, 2, 4096), (1, 2, 16, 2500), (2, 4, 24, 777)])
def test_decode_vs_oracle(cuda_dev, fmt, B, Hkv, Hq, S):
    from int4_kivi.decode import decode_packed, kivi_decode_attention_gqa, stack_caches
    k, v, q = gen_kv(Hkv, S, D, seed=S + Hq, Hq=Hq, B=B)
    q = q[:, :, 0]
    st = stack_caches([_store(fmt, k[b], v[b], cuda_dev) for b in range(B)])
    ref = _oracle_decode(k, v, q, fmt)
    out = kivi_decode_attention_gqa(q.to(cuda_dev), st, Hq).cpu()
    _check_bf16(out, ref)
    m, l, acc = decode_packed(q.to(cuda_dev), st, Hq, partial=True)
    full = (acc / l[:, None]).reshape(B, Hq, D).cpu()
    _check_fp32(full, ref)


def test_decode_single_sequence_api(cuda_dev):
    from int4_kivi.decode import kivi_decode_attention
    k, v, q = gen_kv(8, 999, D, seed=5, Hq=32)
    c = _store("int4", k, v, cuda_dev)
    out = kivi_decode_attention(q.to(cuda_dev), c)
    assert out.shape == (32, 1, D)
    _check_bf16(out[:, 0].cpu()[None], _oracle_decode(k[None], v[None], q[None, :, 0], "int4"))


def test_decode_generic_path(cuda_dev):
    """D = 64 and group 12 take the CUDA-core path; same bar."""
    from int4_kivi import store_kivi
    from int4_kivi.decode import kivi_decode_attention_gqa, stack_caches
    for (Hkv, Hq, S, Dd) in [(2, 24, 333, 64), (1, 4, 200, 256)]:
        k, v, q = gen_kv(Hkv, S, Dd, seed=11, Hq=Hq, B=2)
        q = q[:, :, 0]
        st = stack_caches([store_kivi(k[b].to(cuda_dev), v[b].to(cuda_dev)) for b in range(2)])
        out = kivi_decode_attention_gqa(q.to(cuda_dev), st, Hq).cpu()
        _check_bf16(out, _oracle_decode(k, v, q, "int4"))


def test_decode_nvfp4_global_scale(cuda_dev):
    from int4_kivi.decode import kivi_decode_attention_gqa, stack_caches
    k, v, q = gen_kv(4, 520, D, seed=21, Hq=16, B=2)
    q = q[:, :, 0]
    st = stack_caches([_store("nvfp4", k[b], v[b], cuda_dev, g=0.05) for b in range(2)])
    _check_bf16(kivi_decode_attention_gqa(q.to(cuda_dev), st, 16).cpu(), _oracle_decode(k, v, q, "nvfp4", g=0.05))


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
def test_append_matches_full_store(cuda_dev, fmt):
    """Streaming appends (1, 5, 16, 40 tokens) give the same cache as one store."""
    from int4_kivi import append_kivi
    k, v, _ = gen_kv(4, 300, D, seed=13)
    full = _store(fmt, k, v, cuda_dev)
    c = _store(fmt, k[:, :20], v[:, :20], cuda_dev)
    pos = 20
    for n in (1, 5, 16, 40, 218):
        append_kivi(c, k[:, pos:pos + n].to(cuda_dev), v[:, pos:pos + n].to(cuda_dev))
        pos += n
    assert c.S == 300
    for f in ("k_packed", "k_scale", "v_packed", "v_scale", "k_hot"):
        assert torch.equal(getattr(c, f).cpu(), getattr(full, f).cpu()), f


def test_lse_merge_of_sequence_shards(cuda_dev):
    """Split the KV sequence into page-aligned shards, decode each to (m,l,acc),
    merge: equals the single-shard decode (the cross-GPU merge, on one GPU)."""
    from int4_kivi.decode import decode_packed, lse_merge, stack_caches
    from int4_kivi.distributed import split_tokens
    k, v, q = gen_kv(8, 3000, D, seed=4, Hq=32, B=1)
    q = q[:, :, 0].to(cuda_dev)
    ms, ls, accs = [], [], []
    for r in range(4):
        a, b = split_tokens(3000, 4, r)
        st = stack_caches([_store("int4", k[0, :, a:b], v[0, :, a:b], cuda_dev)])
        m, l, acc = decode_packed(q, st, 32, sm_scale=1.0 / math.sqrt(D), partial=True)
        ms.append(m); ls.append(l); accs.append(acc)
    out = lse_merge(torch.stack(ms), torch.stack(ls), torch.stack(accs)).cpu()
    _check_bf16(out[None], _oracle_decode(k, v, q.cpu(), "int4"))


def test_decode_large_context_property(cuda_dev):
    """c1 shape at 64K context: compare two heads against the oracle and check
    the output is invariant to stacking order (sequence permutation)."""
    from int4_kivi.decode import kivi_decode_attention_gqa, stack_caches
    S = 65536
    k, v, q = gen_kv(8, S, D, seed=64, Hq=32, B=2)
    q = q[:, :, 0]
    cs = [_store("int4", k[b], v[b], cuda_dev) for b in range(2)]
    out = kivi_decode_attention_gqa(q.to(cuda_dev), stack_caches(cs), 32).cpu()
    out_rev = kivi_decode_attention_gqa(q.flip(0).to(cuda_dev), stack_caches(cs[::-1]), 32).cpu()
    assert torch.equal(out, out_rev.flip(0))
    sub = _oracle_decode(k[:1, :1], v[:1, :1], q[:1, :4], "int4")
    _check_bf16(out[:1, :4], sub)


def test_device_status_clear(cuda_dev):
    from int4_kivi import _native
    assert _native.device_status(cuda_dev) == 0


def test_decode_cuda_graph_replay(cuda_dev):
    """The decode step is sync-free: captured in a CUDA graph and replayed with
    new query values it matches the eager call bit for bit."""
    from int4_kivi.decode import decode_packed, stack_caches
    k, v, q = gen_kv(8, 2000, D, seed=31, Hq=32, B=2)
    st = stack_caches([_store("int4", k[b], v[b], cuda_dev) for b in range(2)])
    qd = q[:, :, 0].to(cuda_dev).contiguous()
    out = torch.empty(2, 32, D, dtype=torch.bfloat16, device=cuda_dev)
    decode_packed(qd, st, 32, out=out)          # warm-up allocates the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        decode_packed(qd, st, 32, out=out)
    q2 = torch.randn(2, 32, D, generator=torch.Generator().manual_seed(5)).bfloat16()
    qd.copy_(q2.to(cuda_dev))
    g.replay()
    torch.cuda.synchronize()
    want = decode_packed(qd, st, 32)
    assert torch.equal(out, want)


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
def test_decode_varlen_batch(cuda_dev, fmt):
    """Unequal sequence lengths in one launch (the config-3 serving shape):
    every batch entry attends only its own tokens, hot tails included."""
    from int4_kivi.decode import kivi_decode_attention_gqa, stack_caches
    lens = [1, 15, 16, 17, 300, 1000, 4097]
    Hkv, Hq = 8, 32
    ks, vs, qs, caches = [], [], [], []
    for i, L in enumerate(lens):
        k, v, q = gen_kv(Hkv, L, D, seed=500 + i, Hq=Hq)
        ks.append(k); vs.append(v); qs.append(q[:, 0])
        caches.append(_store(fmt, k, v, cuda_dev))
    st = stack_caches(caches)
    assert st["seq_lens"].tolist() == lens
    q = torch.stack(qs)
    out = kivi_decode_attention_gqa(q.to(cuda_dev), st, Hq).cpu()
    for i in range(len(lens)):
        ref = _oracle_decode(ks[i][None], vs[i][None], q[i:i + 1], fmt)
        _check_bf16(out[i:i + 1], ref)


def test_decode_varlen_generic_path(cuda_dev):
    from int4_kivi.decode import kivi_decode_attention_gqa, stack_caches
    lens = [40, 333, 7]
    ks, vs, qs, caches = [], [], [], []
    for i, L in enumerate(lens):
        k, v, q = gen_kv(2, L, 64, seed=700 + i, Hq=12)
        ks.append(k); vs.append(v); qs.append(q[:, 0])
        caches.append(_store("int4", k, v, cuda_dev))
    q = torch.stack(qs)
    out = kivi_decode_attention_gqa(q.to(cuda_dev), stack_caches(caches), 12).cpu()
    for i in range(len(lens)):
        _check_bf16(out[i:i + 1], _oracle_decode(ks[i][None], vs[i][None], q[i:i + 1], "int4"))
