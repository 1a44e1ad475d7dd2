"""Multi-query decode (kivi_decode_multiquery): Tq query tokens per sequence,
query j at position q_pos + j attending tokens 0 .. q_pos + j, against the
oracle's attention over exactly those tokens of the same dequantised cache,
with the decode bar of conftest.py (bf16 output).  Tq = 1 at the last
position reproduces the plain decode bit for bit."""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import check_decode_bf16, gen_kv

pytestmark = pytest.mark.gpu

D = 128


def _store(fmt, k, v, dev):
    from int4_kivi import store_kivi, store_nvfp4_kivi
    if fmt == "int4":
        return store_kivi(k.to(dev), v.to(dev))
    return store_nvfp4_kivi(k.to(dev), v.to(dev))


def _oracle(k, v, q, q_pos, fmt):
    """q [B, Tq, Hq, D]; k/v [B, Hkv, S, D] -> fp32 [B, Tq, Hq, D]."""
    B, Tq, Hq, _ = q.shape
    out = np.zeros((B, Tq, Hq, D), np.float32)
    for b in range(B):
        c = oracle.store_int4(k[b], v[b]) if fmt == "int4" else oracle.store_nvfp4(k[b], v[b])
        kd, vd = oracle.dequant_int4(c) if fmt == "int4" else oracle.dequant_nvfp4(c)
        for j in range(Tq):
            L = q_pos + j + 1
            out[b, j] = oracle.decode_attention(q[b:b + 1, j], kd[None, :, :L], vd[None, :, :L],
                                                1.0 / math.sqrt(D))[0]
    return out


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
@pytest.mark.parametrize("B,Hkv,Hq,S,Tq", [(2, 8, 32, 300, 2), (1, 8, 32, 4096, 4), (2, 2, 2, 1000, 8),
                                            (1, 4, 32, 777, 3), (3, 8, 8, 40, 5), (1, 8, 32, 17, 2)])
def test_multiquery_vs_oracle(cuda_dev, fmt, B, Hkv, Hq, S, Tq):
    from int4_kivi.decode import kivi_decode_attention_multiquery, stack_caches
    k, v, _ = gen_kv(Hkv, S, D, seed=S + Tq, B=B)
    q = torch.randn(B, Tq, Hq, D, generator=torch.Generator().manual_seed(S)).bfloat16()
    st = stack_caches([_store(fmt, k[b], v[b], cuda_dev) for b in range(B)])
    out = kivi_decode_attention_multiquery(q.to(cuda_dev), st, Hq)
    assert out.shape == (B, Tq, Hq, D)
    check_decode_bf16(out, _oracle(k, v, q, S - Tq, fmt), f"{fmt} S={S} Tq={Tq}")


def test_multiquery_inside_the_cache(cuda_dev):
    """Queries that sit before the end of the cache (q_pos + Tq < S) see only
    their causal prefix, across a page boundary and inside packed pages."""
    from int4_kivi.decode import kivi_decode_attention_multiquery, stack_caches
    k, v, _ = gen_kv(8, 500, D, seed=3, B=2)
    q = torch.randn(2, 6, 32, D, generator=torch.Generator().manual_seed(4)).bfloat16()
    st = stack_caches([_store("int4", k[b], v[b], cuda_dev) for b in range(2)])
    for q_pos in (0, 13, 250, 480):
        out = kivi_decode_attention_multiquery(q.to(cuda_dev), st, 32, q_pos=q_pos)
        check_decode_bf16(out, _oracle(k, v, q, q_pos, "int4"), f"q_pos={q_pos}")
    with pytest.raises(ValueError):
        kivi_decode_attention_multiquery(q.to(cuda_dev), st, 32, q_pos=495)


@pytest.mark.parametrize("S", [16, 300, 4096])
def test_single_query_at_the_end_equals_decode(cuda_dev, S):
    from int4_kivi.decode import decode_packed, kivi_decode_attention_multiquery, stack_caches
    k, v, q = gen_kv(8, S, D, seed=9, Hq=32, B=2)
    st = stack_caches([_store("int4", k[b], v[b], cuda_dev) for b in range(2)])
    q3 = q[:, :, 0].to(cuda_dev)
    want = decode_packed(q3, st, 32)
    got = kivi_decode_attention_multiquery(q3[:, None], st, 32)[:, 0]
    assert torch.equal(got, want)


@pytest.mark.parametrize("n", [1, 2, 3, 7])
def test_hf_layer_tail_only_noncontiguous_inputs(cuda_dev, n):
    """The HF cache layer with fewer than 16 tokens (no packed page yet), fed
    K/V as strided views: the bf16 tail rows must be read at their own row
    stride.  Query j attends tokens 0 .. j in exact bf16 (fp32 reference)."""
    from int4_kivi.hf_cache import _Int4KiviLayer
    H, Hq = 2, 8
    k, v, _ = gen_kv(H, 40, D, seed=31)
    layer = _Int4KiviLayer(fused_decode=True)
    layer.update(k[None, :, :n].to(cuda_dev), v[None, :, :n].to(cuda_dev))   # views with row stride 40 * D
    q = torch.randn(1, Hq, n, D, generator=torch.Generator().manual_seed(1)).bfloat16()
    out = layer.fused_decode(q.to(cuda_dev), D ** -0.5)
    out = (out[0] if n > 1 else out).float().cpu().reshape(n, Hq, D)
    for j in range(n):
        kk = k[:, :j + 1].float().repeat_interleave(Hq // H, 0)
        vv = v[:, :j + 1].float().repeat_interleave(Hq // H, 0)
        p = torch.softmax((q[0, :, j].float()[:, None] @ kk.transpose(1, 2))[:, 0] * D ** -0.5, -1)
        want = (p[:, None] @ vv)[:, 0]
        torch.testing.assert_close(out[j], want, atol=2e-2, rtol=2e-2, msg=f"query {j}")
