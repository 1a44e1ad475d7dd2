"""kivi_peer_publish / kivi_peer_merge on one GPU (no peer process needed).

* W = 1: the merge of a single published state equals its normalisation.
* W = 2 with both buffer addresses pointing at this GPU's buffer and nobody
  publishing for rank 1: the merge's bounded wait runs out and reports
  KIVI_ERR_TIMEOUT through the error flag instead of hanging; the context
  stays usable.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(dev, W, rows=32, D=128):
    from int4_kivi import _native as N
    L = N.lib()
    nbytes = L.kivi_peer_buffer_bytes(rows, D, W)
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    peers = torch.tensor([buf.data_ptr()] * W, dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    g = torch.Generator().manual_seed(3)
    m = (torch.randn(rows, generator=g) * 4).to(dev)
    l = (torch.rand(rows, generator=g) * 10 + 1).to(dev)
    acc = torch.randn(rows, D, generator=g).to(dev)
    return N, L, buf, peers, epoch, m, l, acc


def test_peer_merge_single_rank(cuda_dev):
    N, L, buf, peers, epoch, m, l, acc = _setup(cuda_dev, 1)
    out = torch.empty(32, 128, dtype=torch.bfloat16, device=cuda_dev)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    s = N.stream_of(acc)
    for step in range(3):                           # both slots, epoch advancing
        acc.mul_(1.5)
        N.check(L.kivi_peer_publish(N.ptr(m), N.ptr(l), N.ptr(acc), 32, 128, N.ptr(buf), N.ptr(peers), 1, 0,
                                    N.ptr(epoch), s), "publish")
        N.check(L.kivi_peer_merge(N.ptr(peers), 1, 32, 128, N.ptr(epoch), N.ptr(buf), N.ptr(out), N.ptr(err),
                                  ctypes.c_longlong(int(2e9)), s), "merge")
        torch.cuda.synchronize()
        want = (acc / l[:, None]).bfloat16()
        assert torch.equal(out, want)
    assert int(err.item()) == 0 and int(epoch.item()) == 3


def test_peer_merge_wait_times_out(cuda_dev):
    N, L, buf, peers, epoch, m, l, acc = _setup(cuda_dev, 2)
    out = torch.zeros(32, 128, dtype=torch.bfloat16, device=cuda_dev)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    s = N.stream_of(acc)
    N.check(L.kivi_peer_publish(N.ptr(m), N.ptr(l), N.ptr(acc), 32, 128, N.ptr(buf), N.ptr(peers), 2, 0,
                                N.ptr(epoch), s), "publish")
    N.check(L.kivi_peer_merge(N.ptr(peers), 2, 32, 128, N.ptr(epoch), N.ptr(buf), N.ptr(out), N.ptr(err),
                              ctypes.c_longlong(int(5e7)), s), "merge")
    torch.cuda.synchronize()
    assert int(err.item()) == 5                      # KIVI_ERR_TIMEOUT
    assert torch.count_nonzero(out).item() == 0      # rows left unwritten
    torch.ones(4, device=cuda_dev).sum().item()      # context still usable


def _seqpar_case(dev, W):
    from conftest import gen_kv
    from int4_kivi import _native as N
    from int4_kivi import store_kivi
    k, v, q = gen_kv(8, 3000, 128, seed=12, Hq=32)
    c = store_kivi(k.to(dev), v.to(dev))
    st = dict(k_packed=c.k_packed, k_scale=c.k_scale, k_hot=c.k_hot, v_packed=c.v_packed, v_scale=c.v_scale,
              H=8, S=3000, D=128, B=1)
    L = N.lib()
    xbuf = torch.zeros(L.kivi_seqpar_buffer_bytes(32, 128, W), dtype=torch.uint8, device=dev)

    class X:                                        # the fields decode_packed reads from an exchange
        pass
    x = X()
    x.own = ctypes.c_void_p(xbuf.data_ptr())
    x.peers = torch.tensor([xbuf.data_ptr()] * W, dtype=torch.int64, device=dev)
    x.world, x.rank = W, 0
    x.row_epoch = torch.zeros(32, dtype=torch.int32, device=dev)
    x.timeout_ns = int(2e9) if W == 1 else int(5e7)
    x.rows, x.D, x.closed = 32, 128, False
    x.device = torch.device("cuda", N.device_index(dev))
    return q[None, :, 0].to(dev), st, x, xbuf


def test_fused_seqpar_single_rank_equals_decode(cuda_dev):
    """kivi_decode_seqpar with one rank: the exchange tail publishes and
    re-reads the row's own state; the result is kivi_decode's (the W = 1
    merge divides the same accumulator by the same l)."""
    from int4_kivi import _native as N
    from int4_kivi.decode import decode_packed
    q, st, x, _ = _seqpar_case(cuda_dev, 1)
    want = decode_packed(q, st, 32)
    for it in range(3):
        got = decode_packed(q, st, 32, exchange=x)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (it, int(torch.count_nonzero(got != want)))
    assert N.device_status(cuda_dev) == 0
    assert int(x.row_epoch.min().item()) == 3 == int(x.row_epoch.max().item())


def test_fused_seqpar_wait_times_out(cuda_dev):
    """Two ranks declared, the second never publishes: every row's bounded
    wait ends with KIVI_ERR_TIMEOUT, rows stay unwritten, context usable."""
    from int4_kivi import _native as N
    from int4_kivi.decode import decode_packed
    q, st, x, _ = _seqpar_case(cuda_dev, 2)
    N.device_status(cuda_dev)
    out = torch.zeros(1, 32, 128, dtype=torch.bfloat16, device=cuda_dev)
    decode_packed(q, st, 32, exchange=x, out=out)
    torch.cuda.synchronize()
    assert N.device_status(cuda_dev) == 5
    assert torch.count_nonzero(out).item() == 0


def test_timeout_raises_through_python_api(cuda_dev):
    """The same silent second rank, seen from the Python API: decode_packed
    (check=True) raises KiviError with status KIVI_ERR_TIMEOUT, and the
    sync-free per-step poll raises it once the step has finished."""
    from int4_kivi import _native as N
    from int4_kivi.decode import decode_packed
    q, st, x, _ = _seqpar_case(cuda_dev, 2)
    N.device_status(cuda_dev)
    with pytest.raises(N.KiviError) as ei:
        decode_packed(q, st, 32, exchange=x, check=True)
    assert ei.value.status == N.KIVI_ERR_TIMEOUT
    assert N.device_status(cuda_dev) == 0                # raised and cleared
    decode_packed(q, st, 32, exchange=x)                 # fails on the device again
    N.poll_errors(cuda_dev)                              # queues the flag copy, returns at once
    torch.cuda.synchronize()
    with pytest.raises(N.KiviError) as ei:
        N.poll_errors(cuda_dev)
    assert ei.value.status == N.KIVI_ERR_TIMEOUT
    N.poll_errors(cuda_dev)                              # cleared: nothing more to report
    torch.cuda.synchronize()
    N.poll_errors(cuda_dev)
    assert N.device_status(cuda_dev) == 0
