"""Decode and store parity at the benchmark's own shapes and on the
reference's own inputs, against the CPU oracle, with the decode bar of
conftest.py on every output row:

* config 1 exactly: INT4, B=8, Hq=32, Hkv=8, D=128, S=8192;
* the 64K headline: INT4, B=8, S=65536 (the inputs bench.py times);
* config 2 exactly: NVFP4, B=8, S=65536, the cache built from 65520 tokens
  plus the 16-token store of the step, then decode -- as bench.py times it;
* the reference test's heavy-tailed K (k = randn**3 drawn on the device,
  tests/test_int4_kivi.py:51-56): store, dequant, decode;
* the S list of scripts/validate_int4_kivi_decode.py:131 with its inputs
  (H_KV=8, N_QH=48, D=128, k = randn**3, v/q = randn on the device, seed S,
  MSE store, :85-90).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits, check_decode_bf16, check_decode_fp32, load_golden

pytestmark = pytest.mark.gpu

D = 128


def _stacked(c, B):
    return dict(k_packed=c.k_packed, k_scale=c.k_scale, k_hot=c.k_hot, v_packed=c.v_packed,
                v_scale=c.v_scale, H=c.H // B, S=c.S, D=c.D, B=B)


def _oracle_rows(k, v, q, fmt="int4", calib="absmax"):
    """fp64 attention [B, Hq, D] over the oracle's own store of k/v [B, Hkv, S, D]
    (bf16 CPU tensors), one sequence at a time to bound host memory."""
    out = []
    for b in range(k.shape[0]):
        if fmt == "int4":
            kd, vd = oracle.dequant_int4(oracle.store_int4(k[b], v[b], calib, calib))
        else:
            kd, vd = oracle.dequant_nvfp4(oracle.store_nvfp4(k[b], v[b], calib, calib))
        out.append(oracle.decode_attention(q[b:b + 1].float(), kd[None], vd[None], 1.0 / math.sqrt(D))[0])
        del kd, vd
    return np.stack(out)


def _check_all_rows(q, st, Hq, ref, what):
    from int4_kivi.decode import decode_packed
    out = decode_packed(q, st, Hq)
    m, l, acc = decode_packed(q, st, Hq, partial=True)
    B = q.shape[0]
    check_decode_fp32((acc / l[:, None]).reshape(B, Hq, D), ref, what)
    check_decode_bf16(out, ref, what)


@pytest.mark.parametrize("S", (8192, 65536))
def test_int4_bench_shapes_every_row(cuda_dev, S):
    """Config 1 (S=8192) and the 64K headline, the exact inputs of bench.py."""
    import bench
    k, v, q = bench.make_inputs(S, seed=1234, device=cuda_dev)
    st = bench.build_stacked(k, v)
    ref = _oracle_rows(k.cpu(), v.cpu(), q.cpu())
    del k, v
    _check_all_rows(q, st, 32, ref, f"int4 S={S}")


def test_nvfp4_config2_store16_then_decode(cuda_dev):
    """Config 2 as bench.py times it: NVFP4 cache of 65520 tokens with room for
    65536, the step's 16-token store into it, then decode of every row."""
    import bench
    from int4_kivi import store_nvfp4_kivi
    from int4_kivi.cache import full_views, store_into
    S, B, Hkv = 65536, 8, 8
    BH = B * Hkv
    k, v, q = bench.make_inputs(S, seed=8, device=cuda_dev)
    kf, vf = k.reshape(BH, S, D), v.reshape(BH, S, D)
    c = store_nvfp4_kivi(kf[:, :S - 16].contiguous(), vf[:, :S - 16].contiguous(), "absmax", "absmax", capacity=S)
    kp, ks, vp, vs = full_views(c)
    store_into(kf[:, S - 16:].contiguous(), vf[:, S - 16:].contiguous(), "nvfp4", "absmax", "absmax",
               kp, ks, vp, vs, (S - 16) // 16, S - 16)
    st = dict(k_packed=kp[:, :, :S // 16], k_scale=ks[:, :, :S // 16],
              k_hot=torch.empty(BH, 0, D, dtype=torch.bfloat16, device=cuda_dev),
              v_packed=vp[:, :S], v_scale=vs[:, :S], H=Hkv, S=S, D=D, B=B, fmt="nvfp4", g_k=1.0, g_v=1.0)
    kc, vc = k.cpu(), v.cpu()
    del k, v, kf, vf
    # the cache bytes equal one oracle store of all 65536 tokens
    for b in (0, B - 1):
        o = oracle.store_nvfp4(kc[b], vc[b], "absmax", "absmax")
        sl = slice(b * Hkv, (b + 1) * Hkv)
        for name, t in (("k_packed", st["k_packed"]), ("k_scale", st["k_scale"]),
                        ("v_packed", st["v_packed"]), ("v_scale", st["v_scale"])):
            assert np.array_equal(t[sl].cpu().numpy(), o[name]), (b, name)
    ref = _oracle_rows(kc, vc, q.cpu(), fmt="nvfp4")
    _check_all_rows(q, st, 32, ref, "nvfp4 c2")


def _heavy(S, seed, dev, H=8, Hq=None):
    """tests/test_int4_kivi.py:51-56 / validate_int4_kivi_decode.py:85-89 inputs."""
    g = torch.Generator(device=dev).manual_seed(seed)
    k = (torch.randn(H, S, D, generator=g, device=dev) ** 3).to(torch.bfloat16)
    v = torch.randn(H, S, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(Hq, 1, D, generator=g, device=dev).to(torch.bfloat16) if Hq else None
    return k, v, q


@pytest.mark.parametrize("calib", ("absmax", "mse"))
@pytest.mark.parametrize("S", (256, 512, 2048))
def test_heavy_tail_store_dequant(cuda_dev, S, calib):
    """The reference test's code-parity cases, bit-exact here (the reference
    test allows 0.5 % off-by-one flips)."""
    from int4_kivi import dequant_kivi, store_kivi
    k, v, _ = _heavy(S, 0, cuda_dev)
    c = store_kivi(k, v, k_calib=calib, v_calib=calib)
    o = oracle.store_int4(k.cpu(), v.cpu(), calib, calib)
    for f in ("k_packed", "v_packed"):
        assert np.array_equal(getattr(c, f).cpu().numpy(), o[f]), f
    for f in ("k_scale", "v_scale"):
        assert np.array_equal(getattr(c, f).cpu().numpy().view(np.uint16), o[f].view(np.uint16)), f
    kq, vq = dequant_kivi(c)
    kd, vd = oracle.dequant_int4(o)
    assert torch.equal(kq.cpu(), torch.from_numpy(kd).bfloat16())
    assert torch.equal(vq.cpu(), torch.from_numpy(vd).bfloat16())


@pytest.mark.parametrize("calib", ("absmax", "mse"))
def test_heavy_tail_golden(cuda_dev, calib):
    """randn**3 K through the reference's own recipe (golden fixture)."""
    from int4_kivi import store_kivi
    g = load_golden("heavy_tail.npz")
    k, v = bf16_from_bits(g["k"]).to(cuda_dev), bf16_from_bits(g["v"]).to(cuda_dev)
    c = store_kivi(k, v, k_calib=calib, v_calib=calib)
    assert np.array_equal(c.k_packed.cpu().numpy(), g[f"{calib}_k_packed"])
    assert np.array_equal(c.v_packed.cpu().numpy(), g[f"{calib}_v_packed"])
    assert np.array_equal(c.k_scale.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{calib}_k_scale"])
    assert np.array_equal(c.v_scale.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{calib}_v_scale"])


@pytest.mark.parametrize("S", (127, 512, 1000, 2048, 4096, 8192, 16384, 32768))
def test_validate_decode_s_list(cuda_dev, S):
    """validate_int4_kivi_decode.py's cases with its own inputs: single
    sequence, 48 q heads over 8 kv heads (group 6), MSE store."""
    from int4_kivi import store_kivi
    from int4_kivi.decode import decode_packed, kivi_decode_attention
    k, v, q = _heavy(S, S, cuda_dev, Hq=48)
    c = store_kivi(k, v)
    out = kivi_decode_attention(q, c)                                  # [48, 1, D]
    o = oracle.store_int4(k.cpu(), v.cpu())
    kd, vd = oracle.dequant_int4(o)
    ref = oracle.decode_attention(q[:, 0].cpu().float()[None], kd[None], vd[None], 1.0 / math.sqrt(D))
    check_decode_bf16(out[:, 0][None], ref, f"S={S}")
    m, l, acc = decode_packed(q[:, 0][None], _stacked(c, 1), 48, partial=True)
    check_decode_fp32((acc / l[:, None])[None], ref, f"S={S}")
