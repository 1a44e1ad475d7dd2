"""Mixed-precision cache (K INT4, V INT3; int4_kivi.mixed) on the GPU against
the CPU oracle: store and dequant bit-exact, in-place appends, and the fused
decode (single and multi-query, equal and unequal lengths) with the decode
bar of conftest.py."""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import check_decode_bf16, check_decode_fp32, gen_kv

pytestmark = pytest.mark.gpu

D = 128


def _same_cache(c, o):
    H, S = c.H, c.S
    assert c.v_packed.shape == (H, S, c.D // 32, 12)
    assert np.array_equal(c.k_packed.cpu().numpy(), o["k_packed"])
    assert np.array_equal(c.k_scale.cpu().numpy().view(np.uint16), o["k_scale"].view(np.uint16))
    assert np.array_equal(c.v_packed.cpu().numpy(), o["v_packed"])
    assert np.array_equal(c.v_scale.cpu().numpy().view(np.uint16), o["v_scale"].view(np.uint16))


@pytest.mark.parametrize("calib", ("absmax", "mse"))
@pytest.mark.parametrize("S", (1, 15, 40, 256, 1000))
def test_store_and_dequant_bit_exact(cuda_dev, S, calib):
    from int4_kivi.mixed import dequant_kivi_int3v, store_kivi_int3v
    k, v, _ = gen_kv(4, S, D, seed=S)
    c = store_kivi_int3v(k.to(cuda_dev), v.to(cuda_dev), calib, calib)
    o = oracle.store_int3v(k, v, calib, calib)
    _same_cache(c, o)
    assert torch.equal(c.k_hot.cpu(), k[:, (S // 16) * 16:])
    kd, vd = dequant_kivi_int3v(c)
    okd, ovd = oracle.dequant_int3v(o)
    assert torch.equal(kd.cpu(), torch.from_numpy(okd).bfloat16())
    assert torch.equal(vd.cpu(), torch.from_numpy(ovd).bfloat16())
    assert c.nbytes == 4 * ((S // 16) * D * 10 + (S % 16) * D * 2 + S * (D // 16) * 8)


def test_append_in_place_matches_one_store(cuda_dev):
    from int4_kivi import append_kivi
    from int4_kivi.mixed import store_kivi_int3v
    k, v, _ = gen_kv(8, 300, D, seed=5)
    c = store_kivi_int3v(k[:, :100].to(cuda_dev), v[:, :100].to(cuda_dev), capacity=256)
    t = 100
    for n in (1, 7, 30, 120, 42):                  # crosses pages and the capacity
        c = append_kivi(c, k[:, t:t + n].to(cuda_dev), v[:, t:t + n].to(cuda_dev))
        t += n
    assert c.fmt == "int4k_int3v" and c.S == 300
    _same_cache(c, oracle.store_int3v(k, v))


def _oracle_decode(k, v, q, L=None):
    """fp64 attention [B, Hq, D] over the oracle's mixed cache of each sequence
    (k/v [B, Hkv, S, D]); L[b] limits sequence b to its first L[b] tokens."""
    out = []
    for b in range(k.shape[0]):
        S = k.shape[2] if L is None else L[b]
        kd, vd = oracle.dequant_int3v(oracle.store_int3v(k[b, :, :S], v[b, :, :S]))
        out.append(oracle.decode_attention(q[b:b + 1].float(), kd[None], vd[None], 1.0 / math.sqrt(D))[0])
    return np.stack(out)


@pytest.mark.parametrize("B,Hkv,Hq,S", [(2, 8, 32, 300), (1, 8, 48, 1000), (3, 2, 2, 40), (1, 4, 32, 17),
                                        (2, 8, 32, 4096)])
def test_decode_vs_oracle(cuda_dev, B, Hkv, Hq, S):
    from int4_kivi.decode import decode_packed, stack_caches
    from int4_kivi.mixed import store_kivi_int3v
    k, v, q = gen_kv(Hkv, S, D, seed=S + Hq, Hq=Hq, B=B)
    q = q[:, :, 0]
    st = stack_caches([store_kivi_int3v(k[b].to(cuda_dev), v[b].to(cuda_dev)) for b in range(B)])
    assert st["fmt"] == "int4k_int3v"
    ref = _oracle_decode(k, v, q)
    qd = q.to(cuda_dev)
    check_decode_bf16(decode_packed(qd, st, Hq), ref, f"mixed B={B} Hq={Hq} S={S}")
    m, l, acc = decode_packed(qd, st, Hq, partial=True)
    check_decode_fp32((acc / l[:, None]).reshape(B, Hq, D), ref, f"mixed fp32 S={S}")


def test_decode_single_sequence_api(cuda_dev):
    from int4_kivi.decode import kivi_decode_attention
    from int4_kivi.mixed import store_kivi_int3v
    k, v, q = gen_kv(8, 777, D, seed=11, Hq=32)
    out = kivi_decode_attention(q.to(cuda_dev), store_kivi_int3v(k.to(cuda_dev), v.to(cuda_dev)))
    check_decode_bf16(out[:, 0][None], _oracle_decode(k[None], v[None], q[:, 0][None]), "mixed single")


def test_decode_unequal_lengths(cuda_dev):
    from int4_kivi.decode import decode_packed, stack_caches
    from int4_kivi.mixed import store_kivi_int3v
    lens = [33, 700, 16, 257]
    k, v, q = gen_kv(8, max(lens), D, seed=21, Hq=32, B=len(lens))
    q = q[:, :, 0]
    st = stack_caches([store_kivi_int3v(k[b, :, :L].to(cuda_dev), v[b, :, :L].to(cuda_dev))
                       for b, L in enumerate(lens)])
    assert st.get("seq_lens") is not None
    check_decode_bf16(decode_packed(q.to(cuda_dev), st, 32), _oracle_decode(k, v, q, lens), "mixed varlen")


def test_multiquery(cuda_dev):
    from int4_kivi.decode import kivi_decode_attention_multiquery, stack_caches
    from int4_kivi.mixed import store_kivi_int3v
    B, Hkv, Hq, S, Tq = 2, 8, 32, 500, 4
    k, v, _ = gen_kv(Hkv, S, D, seed=3, B=B)
    q = torch.randn(B, Tq, Hq, D, generator=torch.Generator().manual_seed(4)).bfloat16()
    st = stack_caches([store_kivi_int3v(k[b].to(cuda_dev), v[b].to(cuda_dev)) for b in range(B)])
    out = kivi_decode_attention_multiquery(q.to(cuda_dev), st, Hq).cpu()
    want = np.zeros((B, Tq, Hq, D), np.float64)
    for b in range(B):
        kd, vd = oracle.dequant_int3v(oracle.store_int3v(k[b], v[b]))
        for j in range(Tq):
            L = S - Tq + j + 1
            want[b, j] = oracle.decode_attention(q[b:b + 1, j].float(), kd[None, :, :L], vd[None, :, :L],
                                                 1.0 / math.sqrt(D))[0]
    check_decode_bf16(out, want, "mixed multi-query")
