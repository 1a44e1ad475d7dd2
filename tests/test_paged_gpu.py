"""Paged (vLLM block layout) cache on the GPU vs the CPU oracle.

Cases follow the reference's own harnesses for the fork kernels:
scripts/validate_store_equiv.py:87-96 (prefill L = 512, 500, 257, 33, 16, 15
and scattered decode-style stores), scripts/validate_paged_decode.py:108-116
(decode: exact block, partial tail, short, tiny, mixed batch, long, long
mixed; Hq = 48, Hkv = 8, D = 128, block 0 left unused) and
scripts/validate_nvfp4_kivi.py:126-160 (NVFP4 decode at 512 / 500 / 33).
Store and gather are compared byte for byte; decode against the oracle's
double-precision attention over the same cache with the decode bar of
conftest.py, on the bf16 output and on the fp32 state (kivi_paged_decode_f32).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import check_decode_bf16, check_decode_fp32

pytestmark = pytest.mark.gpu

D = 128


def _prefill_layout(seq_lens, first_block=1):
    nblk = [(L + 15) // 16 for L in seq_lens]
    bt = np.zeros((len(seq_lens), max(max(nblk), 1)), np.int32)
    slots, cur = [], first_block
    for b, L in enumerate(seq_lens):
        phys = list(range(cur, cur + nblk[b]))
        cur += nblk[b]
        bt[b, :nblk[b]] = phys
        slots.append(np.array([phys[t // 16] * 16 + t % 16 for t in range(L)], np.int64))
    return bt, slots, cur + 2


def _kv_inputs(n, H, seed, dtype=torch.bfloat16, Dh=D):
    g = torch.Generator().manual_seed(seed)
    f = torch.exp(torch.empty(1, H, Dh).uniform_(math.log(0.5), math.log(8.0), generator=g))
    k = (torch.randn(n, H, Dh, generator=g) * f).to(dtype)
    v = torch.randn(n, H, Dh, generator=g).to(dtype)
    return k, v


_BUILT = {}


def _build(seq_lens, H, fmt, seed, dev, calib="mse", Dh=D):
    """The same prefill stores on the GPU and in the oracle (cached per case)."""
    from int4_kivi import paged
    key = (tuple(seq_lens), H, fmt, seed, calib, Dh)
    if key in _BUILT:
        kv_gpu, kv_cpu, bt = _BUILT[key]
        return kv_gpu.clone(), kv_cpu.copy(), bt.copy()
    bt, slots, nb = _prefill_layout(seq_lens)
    kv_gpu = torch.zeros(nb, 2, 16, H, paged.int4_kivi_kv_cache_full_dim(Dh), dtype=torch.uint8, device=dev)
    kv_cpu = np.zeros(tuple(kv_gpu.shape), np.uint8)
    store = paged.int4_kivi_store if fmt == "int4" else paged.nvfp4_kivi_store
    for b, L in enumerate(seq_lens):
        if L == 0:
            continue
        k, v = _kv_inputs(L, H, seed + b, Dh=Dh)
        store(k.to(dev), v.to(dev), kv_gpu, torch.from_numpy(slots[b]).to(dev), Dh, calib=calib)
        assert oracle.paged_store(k.float(), v.float(), slots[b], kv_cpu, fmt, calib) == 0
    torch.cuda.synchronize()
    if sum(seq_lens) >= 4000:
        _BUILT[key] = (kv_gpu, kv_cpu, bt)
    return kv_gpu, kv_cpu, bt


def _assert_bytes_equal(kv_gpu, kv_cpu):
    got = kv_gpu.cpu().numpy()
    bad = np.argwhere(got != kv_cpu)
    assert bad.size == 0, f"{len(bad)} bytes differ, first at {bad[:4].tolist()}"


@pytest.mark.parametrize("fmt", ("int4", "nvfp4"))
@pytest.mark.parametrize("calib", ("mse", "absmax"))
@pytest.mark.parametrize("L", (512, 500, 257, 33, 16, 15, 1))
def test_paged_store_prefill_bit_exact(cuda_dev, fmt, calib, L):
    kv_gpu, kv_cpu, _ = _build([L], 8, fmt, 1234 + L, cuda_dev, calib)
    _assert_bytes_equal(kv_gpu, kv_cpu)


@pytest.mark.parametrize("fmt", ("int4", "nvfp4"))
@pytest.mark.parametrize("B", (16, 40))
def test_paged_store_scattered_bit_exact(cuda_dev, fmt, B):
    """Decode-style store: token 3 of B distinct blocks, all per-token K
    (scripts/validate_store_equiv.py:68-78)."""
    from int4_kivi import paged
    H = 8
    k, v = _kv_inputs(B, H, 77 + B)
    slots = (np.arange(B, dtype=np.int64) + 1) * 16 + 3
    kv_gpu = torch.zeros(B + 2, 2, 16, H, 72, dtype=torch.uint8, device=cuda_dev)
    kv_cpu = np.zeros(tuple(kv_gpu.shape), np.uint8)
    store = paged.int4_kivi_store if fmt == "int4" else paged.nvfp4_kivi_store
    store(k.to(cuda_dev), v.to(cuda_dev), kv_gpu, torch.from_numpy(slots).to(cuda_dev), D)
    oracle.paged_store(k.float(), v.float(), slots, kv_cpu, fmt)
    _assert_bytes_equal(kv_gpu, kv_cpu)


@pytest.mark.parametrize("fmt", ("int4", "nvfp4"))
def test_paged_store_decode_growth_and_chunks(cuda_dev, fmt):
    """Chunked prefill that stops mid-block, then one token per step across two
    block boundaries; padding slots (-1) in a batch are skipped."""
    from int4_kivi import paged
    H, total = 4, 70
    k, v = _kv_inputs(total, H, 5)
    bt, slots, nb = _prefill_layout([total])
    slots = slots[0]
    kv_gpu = torch.zeros(nb, 2, 16, H, 72, dtype=torch.uint8, device=cuda_dev)
    kv_cpu = np.zeros(tuple(kv_gpu.shape), np.uint8)
    store = paged.int4_kivi_store if fmt == "int4" else paged.nvfp4_kivi_store
    chunks = [(0, 21), (21, 40)] + [(t, t + 1) for t in range(40, total)]
    for a, b in chunks:
        sl = slots[a:b]
        kk, vv = k[a:b], v[a:b]
        if b - a == 1:                                   # a padded batch of 3
            sl = np.array([-1, sl[0], -1], np.int64)
            kk = torch.cat([kk, kk, kk]); vv = torch.cat([vv, vv, vv])
        store(kk.to(cuda_dev), vv.to(cuda_dev), kv_gpu, torch.from_numpy(sl).to(cuda_dev), D)
        oracle.paged_store(kk.float(), vv.float(), sl, kv_cpu, fmt)
    _assert_bytes_equal(kv_gpu, kv_cpu)


@pytest.mark.parametrize("fmt", ("int4", "nvfp4"))
def test_paged_gather_bit_exact(cuda_dev, fmt):
    from int4_kivi import paged
    seq_lens = [128, 257, 64, 1000, 16, 999, 0]
    H = 8
    kv_gpu, kv_cpu, bt = _build(seq_lens, H, fmt, 11, cuda_dev)
    max_seq = 1024
    gather = paged.int4_kivi_gather_dequant if fmt == "int4" else paged.nvfp4_kivi_gather_dequant
    kd, vd = gather(kv_gpu, torch.from_numpy(bt).to(cuda_dev),
                    torch.tensor(seq_lens, dtype=torch.int32, device=cuda_dev), D, H, max_seq)
    kw, vw = oracle.paged_gather(kv_cpu, bt, seq_lens, H, D, fmt, max_seq)
    assert torch.equal(kd.float().cpu(), torch.from_numpy(kw))
    assert torch.equal(vd.float().cpu(), torch.from_numpy(vw))


def _check_decode(out, want):
    """The decode bar of conftest.py, on the bf16 output (or, for an fp32
    `out`, on the normalised state before the bf16 cast)."""
    if out.dtype == torch.float32:
        check_decode_fp32(out, want)
    else:
        check_decode_bf16(out, want)


DECODE_CASES = {
    "exact-block": [512],
    "partial-tail": [500],
    "short": [33],
    "tiny": [1],
    "mixed": [128, 257, 64, 1000, 16, 999],
    "long": [12000],
    "long-mixed": [12000, 8001, 16000, 4096],
}


@pytest.mark.parametrize("fmt", ("int4", "nvfp4"))
@pytest.mark.parametrize("case", list(DECODE_CASES))
@pytest.mark.parametrize("Hq", (48, 32))
def test_paged_decode_vs_oracle(cuda_dev, fmt, case, Hq):
    from int4_kivi import paged
    seq_lens = DECODE_CASES[case]
    H = 8
    kv_gpu, kv_cpu, bt = _build(seq_lens, H, fmt, 100 + len(case), cuda_dev)
    g = torch.Generator().manual_seed(999)
    q = torch.randn(len(seq_lens), Hq, D, generator=g).bfloat16()
    sm = 1.0 / math.sqrt(D)
    dec = paged.int4_kivi_paged_decode if fmt == "int4" else paged.nvfp4_kivi_paged_decode
    btd, sld = torch.from_numpy(bt).to(cuda_dev), torch.tensor(seq_lens, dtype=torch.int32, device=cuda_dev)
    out = dec(q.to(cuda_dev), kv_gpu, btd, sld, sm)
    out32 = dec(q.to(cuda_dev), kv_gpu, btd, sld, sm,
                out=torch.empty(len(seq_lens), Hq, D, dtype=torch.float32, device=cuda_dev))
    torch.cuda.synchronize()
    want = oracle.paged_decode(q.float(), kv_cpu, bt, seq_lens, sm, fmt)
    _check_decode(out, want)
    _check_decode(out32, want)
    assert torch.equal(out, out32.bfloat16())


@pytest.mark.parametrize("H,Hq,Dh", ((16, 32, 128), (2, 6, 64), (4, 4, 256)))
def test_paged_decode_other_shapes(cuda_dev, H, Hq, Dh):
    """16 KV heads (the wide fast kernel) and head_dims of the generic path."""
    from int4_kivi import paged
    seq_lens = [300, 17, 64]
    kv_gpu, kv_cpu, bt = _build(seq_lens, H, "int4", 3, cuda_dev, Dh=Dh)
    g = torch.Generator().manual_seed(4)
    q = torch.randn(len(seq_lens), Hq, Dh, generator=g).bfloat16()
    btd, sld = torch.from_numpy(bt).to(cuda_dev), torch.tensor(seq_lens, dtype=torch.int32, device=cuda_dev)
    out = paged.int4_kivi_paged_decode(q.to(cuda_dev), kv_gpu, btd, sld)
    out32 = paged.int4_kivi_paged_decode(q.to(cuda_dev), kv_gpu, btd, sld,
                                         out=torch.empty(3, Hq, Dh, dtype=torch.float32, device=cuda_dev))
    torch.cuda.synchronize()
    want = oracle.paged_decode(q.float(), kv_cpu, bt, seq_lens, 1.0 / math.sqrt(Dh), "int4")
    _check_decode(out, want)
    _check_decode(out32, want)


def test_paged_decode_empty_sequence_and_graph(cuda_dev):
    """A zero-length sequence yields zeros; the call replays under a CUDA graph
    with new seq_lens and queries written in place."""
    from int4_kivi import paged
    seq_lens = [700, 0, 45]
    H, Hq = 8, 32
    kv_gpu, kv_cpu, bt = _build(seq_lens, H, "int4", 21, cuda_dev)
    btd = torch.from_numpy(bt).to(cuda_dev)
    sld = torch.tensor(seq_lens, dtype=torch.int32, device=cuda_dev)
    q = torch.randn(3, Hq, D, generator=torch.Generator().manual_seed(1)).bfloat16().to(cuda_dev)
    out = torch.empty(3, Hq, D, dtype=torch.bfloat16, device=cuda_dev)
    paged.int4_kivi_paged_decode(q, kv_gpu, btd, sld, out=out)          # warm-up / workspace
    torch.cuda.synchronize()
    assert torch.count_nonzero(out[1]).item() == 0
    gr = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        paged.int4_kivi_paged_decode(q, kv_gpu, btd, sld, out=out)
        with torch.cuda.graph(gr, stream=s):
            paged.int4_kivi_paged_decode(q, kv_gpu, btd, sld, out=out)
    torch.cuda.current_stream().wait_stream(s)
    new_lens = [600, 30, 0]
    q2 = torch.randn(3, Hq, D, generator=torch.Generator().manual_seed(2)).bfloat16()
    sld.copy_(torch.tensor(new_lens, dtype=torch.int32))
    q.copy_(q2.to(cuda_dev))
    gr.replay()
    torch.cuda.synchronize()
    want = oracle.paged_decode(q2.float(), kv_cpu, bt, new_lens, 1.0 / math.sqrt(D), "int4")
    _check_decode(out, want)
    del gr


def test_paged_bad_block_id_sets_error_flag(cuda_dev):
    """A block id outside the cache is reported through the error flag and
    read as block 0, never dereferenced."""
    from int4_kivi import _native as N
    from int4_kivi import paged
    kv_gpu, _, bt = _build([64], 8, "int4", 2, cuda_dev)
    bt[0, 1] = 10 ** 6
    N.device_status(cuda_dev)
    paged.int4_kivi_paged_decode(torch.randn(1, 32, D, device=cuda_dev).bfloat16(), kv_gpu,
                                 torch.from_numpy(bt).to(cuda_dev),
                                 torch.tensor([64], dtype=torch.int32, device=cuda_dev))
    assert N.device_status(cuda_dev) == 1
