"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once, in a container that has the reference checkout (it is NOT needed at
test time and never travels to the GPU box):

    python tests/golden/make_golden.py --reference /path/to/poolside-hackathon

Everything here is computed by the reference's OWN Python code on CPU:
  * kv_quant.roundtrip / _calibrate / _to_blocks / _FORMATS     (kv_quant.py:206-321)
  * the reference test's code/scale recipe `_ref_codes`          (tests/test_int4_kivi.py:43-48)
  * the fp32-exact decode reference `ref_decode_fp32` and its
    `dequant_fp32_exact` helper                                  (scripts/validate_int4_kivi_decode.py:37-84)
  * torch's float16 / float8_e4m3fn casts, the scale storage the
    reference uses (int4_kivi/cache.py:54,59; scripts/diag_kernel_perchannel.py:30-31)
  * the paged cache's e4m3 MSE calibration `fp8` / `mse_scale` / `rt`
    (scripts/diag_kernel_perchannel.py:30-53), taken from the script's source
    text (its module-level vLLM import and GPU code are not executed)
  * the legacy page-level API quantize_page / QuantizedPage /
    QuantizedKVCache / measure_page_error                       (kv_quant.py:37-191)
  * the reference test's heavy-tailed K (randn**3) through `_ref_codes`
    and roundtrip                                                (tests/test_int4_kivi.py:43-56)

The only code of ours is the nibble packer (element 2j -> low nibble of byte j,
int4_kivi/triton_kernels.py:21-24) and the input generator.
Inputs follow the seeded generator used by bench.py and the tests:
k = randn * per-channel log-uniform[0.5, 8] factors, v = randn, q = randn.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def gen_kv(H, S, D, seed, Hq=None):
    g = torch.Generator().manual_seed(seed)
    k0 = torch.randn(1, H, S, D, generator=g)
    f = torch.exp(torch.empty(1, H, 1, D).uniform_(float(np.log(0.5)), float(np.log(8.0)), generator=g))
    k = (k0 * f).bfloat16()[0]
    v = torch.randn(1, H, S, D, generator=g).bfloat16()[0]
    q = torch.randn(1, Hq or H, 1, D, generator=g).bfloat16()[0] if Hq else None
    return k, v, q


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def pack_codes(codes: torch.Tensor) -> np.ndarray:
    c = codes.to(torch.int32) & 0xF
    c = c.reshape(*c.shape[:-1], 8, 2)
    return (c[..., 0] | (c[..., 1] << 4)).to(torch.uint8).numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KIVI_REFERENCE"),
                    help="checkout of a1exxd0/poolside-hackathon (or set KIVI_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or KIVI_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    sys.path.insert(0, os.path.join(args.reference, "scripts"))
    import kv_quant  # noqa: E402
    from kv_quant import _FORMATS, _calibrate, _to_blocks  # noqa: E402

    # ---------------- 1. kv_quant.roundtrip over every cell ----------------
    H, S, D = 2, 40, 64
    k, v, _ = gen_kv(H, S, D, seed=11)
    rt = {"k": bits16(k), "v": bits16(v)}
    for fmt in ("int4", "int3", "nvfp4"):
        for layout in ("headdim", "channel"):
            for calib in ("absmax", "mse"):
                for name, x in (("k", k), ("v", v)):
                    rt[f"{name}_{fmt}_{layout}_{calib}"] = bits16(kv_quant.roundtrip(x, fmt, layout, calib))
    # fp32 input keeps the cast out of the picture; odd n_alphas exercises linspace
    xf = k.float()[:, :32]
    rt["kf32"] = xf.numpy()
    rt["kf32_int4_channel_mse_a7"] = kv_quant.roundtrip(xf, "int4", "channel", "mse", n_alphas=7).numpy()
    rt["kf32_nvfp4_headdim_mse"] = kv_quant.roundtrip(xf, "nvfp4", "headdim", "mse").numpy()
    np.savez_compressed(os.path.join(HERE, "kvq_roundtrip.npz"), **rt)

    # ---------------- 2. INT4-KIVI store: codes + fp16 scales ----------------
    # int4_kivi/cache.py:52-63 layout, codes per tests/test_int4_kivi.py:43-48.
    st = {}
    qmax, qfn = _FORMATS["int4"]
    for S2, seed in ((40, 2), (256, 0)):
        k, v, _ = gen_kv(2, S2, 128, seed=seed)
        st[f"S{S2}_k"], st[f"S{S2}_v"] = bits16(k), bits16(v)
        n_full = (S2 // 16) * 16
        for calib in ("absmax", "mse"):
            kb = _to_blocks(k[:, :n_full], "channel").float()          # [H, D, NP, 16]
            ks = _calibrate(kb, qmax, qfn, calib)
            kc = qfn(kb / ks)
            vb = _to_blocks(v, "headdim").float()                      # [H, S, ND, 16]
            vs = _calibrate(vb, qmax, qfn, calib)
            vc = qfn(vb / vs)
            st[f"S{S2}_{calib}_k_packed"] = pack_codes(kc)
            st[f"S{S2}_{calib}_k_scale"] = bits16(ks[..., 0].to(torch.float16))
            st[f"S{S2}_{calib}_k_scale_f32"] = ks[..., 0].numpy()
            st[f"S{S2}_{calib}_v_packed"] = pack_codes(vc)
            st[f"S{S2}_{calib}_v_scale"] = bits16(vs[..., 0].to(torch.float16))
            st[f"S{S2}_{calib}_v_scale_f32"] = vs[..., 0].numpy()
            # dequantised bf16: code * fp32(fp16 scale) (triton_kernels.py:201-210,277-286)
            kd = (kc * ks.to(torch.float16).float()).reshape(2, 128, n_full).transpose(1, 2)
            st[f"S{S2}_{calib}_k_deq"] = bits16(kd.contiguous().to(torch.bfloat16))
            vd = (vc * vs.to(torch.float16).float()).reshape(2, S2, 128)
            st[f"S{S2}_{calib}_v_deq"] = bits16(vd.to(torch.bfloat16))
    np.savez_compressed(os.path.join(HERE, "kivi_store.npz"), **st)

    # ---------------- 3. fused decode vs the reference's fp32-exact SDPA ------
    import validate_int4_kivi_decode as vdec  # noqa: E402
    from int4_kivi.cache import KIVICache  # noqa: E402

    dec = {}
    Hkv, Hq, Dd = 2, 8, 128
    for S3 in (40, 127, 300):
        k, v, q = gen_kv(Hkv, S3, Dd, seed=100 + S3, Hq=Hq)
        n_full = (S3 // 16) * 16
        NP = n_full // 16
        kb = _to_blocks(k[:, :n_full], "channel").float()
        ks = _calibrate(kb, qmax, qfn, "mse")
        kc = qfn(kb / ks).to(torch.int32)
        vb = _to_blocks(v, "headdim").float()
        vs = _calibrate(vb, qmax, qfn, "mse")
        vc = qfn(vb / vs).to(torch.int32)
        cache = KIVICache(
            k_packed=torch.from_numpy(pack_codes(kc)),
            k_scale=ks[..., 0].to(torch.float16),
            k_hot=k[:, n_full:].contiguous(),
            v_packed=torch.from_numpy(pack_codes(vc)),
            v_scale=vs[..., 0].to(torch.float16),
            H=Hkv, S=S3, D=Dd,
        )
        assert cache.k_packed.shape == (Hkv, Dd, NP, 8)
        out = vdec.ref_decode_fp32(q, cache)                           # [Hq, 1, D] fp32
        pre = f"S{S3}"
        dec[pre + "_q"] = bits16(q)
        dec[pre + "_k"], dec[pre + "_v"] = bits16(k), bits16(v)
        for f_ in ("k_packed", "v_packed"):
            dec[pre + "_" + f_] = getattr(cache, f_).numpy()
        dec[pre + "_k_scale"] = bits16(cache.k_scale)
        dec[pre + "_v_scale"] = bits16(cache.v_scale)
        dec[pre + "_k_hot"] = bits16(cache.k_hot)
        dec[pre + "_out"] = out.numpy()
    np.savez_compressed(os.path.join(HERE, "decode_fp32.npz"), **dec)

    # ---------------- 4. scale-storage casts (fp16, e4m3fn) -------------------
    g = torch.Generator().manual_seed(5)
    vals = torch.cat([
        torch.exp(torch.empty(20000).uniform_(-25.0, 12.0, generator=g)),
        torch.tensor([0.0, 2.0 ** -10, 2.0 ** -9, 3 * 2.0 ** -11, 0.0009765625, 0.001953125,
                      448.0, 440.0, 464.0 - 1e-3, 65504.0, 65519.0, 6.1e-5, 5.96e-8, 1e-9]),
    ]).float()
    fin = vals[vals < 460.0]
    casts = {
        "vals": vals.numpy(),
        "f16": bits16(vals.to(torch.float16)),
        "e4m3_in": fin.numpy(),
        "e4m3": fin.to(torch.float8_e4m3fn).view(torch.uint8).numpy(),
        "linspace32": torch.linspace(0.5, 1.0, 32).numpy(),
        "linspace7": torch.linspace(0.5, 1.0, 7).numpy(),
    }
    np.savez_compressed(os.path.join(HERE, "casts.npz"), **casts)

    # ---------------- 5. paged-cache e4m3 calibration -------------------------
    import ast
    src_path = os.path.join(args.reference, "scripts", "diag_kernel_perchannel.py")
    tree = ast.parse(open(src_path).read())
    defs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in ("fp8", "mse_scale", "rt")]
    ns = {"torch": torch, "QMAX": qmax, "BLOCK": 16}
    exec(compile(ast.Module(body=defs, type_ignores=[]), src_path, "exec"), ns)
    g = torch.Generator().manual_seed(9)
    tok = (torch.randn(3000, 16, generator=g) *
           torch.exp(torch.empty(3000, 1).uniform_(-4.0, 4.0, generator=g))).bfloat16().float()
    s_tok = ns["mse_scale"](tok, -1)                                  # per token: blocks of 16 channels
    chan = (torch.randn(16, 4, 128, generator=g) *
            torch.exp(torch.empty(1, 4, 128).uniform_(-2.0, 2.0, generator=g))).bfloat16().float()
    s_ch = ns["mse_scale"](chan, 0)                                   # per channel over 16 tokens
    paged = {
        "tok": tok.numpy(),
        "tok_scale": s_tok.to(torch.float8_e4m3fn).view(torch.uint8).numpy()[:, 0],
        "tok_deq": ns["rt"](tok, s_tok).numpy(),
        "chan": chan.numpy(),
        "chan_scale": s_ch.to(torch.float8_e4m3fn).view(torch.uint8).numpy()[0],
        "chan_deq": ns["rt"](chan, s_ch).numpy(),
    }
    np.savez_compressed(os.path.join(HERE, "paged_calib.npz"), **paged)

    # ---------------- 6. legacy page-level API (kv_quant.py:37-191) ---------
    leg = {}
    k, v, _ = gen_kv(2, 48, 64, seed=21)
    leg["k"], leg["v"] = bits16(k), bits16(v)
    for use_mse in (False, True):
        tag = "mse" if use_mse else "absmax"
        pg = kv_quant.quantize_page(k[:, :16], v[:, :16], 0, use_mse=use_mse)
        leg[f"page_{tag}_k_int4"] = pg.k_int4.numpy()
        leg[f"page_{tag}_v_int4"] = pg.v_int4.numpy()
        leg[f"page_{tag}_k_scale"] = bits16(pg.k_scale)
        leg[f"page_{tag}_v_scale"] = bits16(pg.v_scale)
        kd, vd = pg.dequantize()
        leg[f"page_{tag}_k_deq"], leg[f"page_{tag}_v_deq"] = bits16(kd), bits16(vd)
        leg[f"page_{tag}_mem"] = np.array([pg.mem_bytes(), pg.bf16_bytes()])
    # fp32 input page (the calibration sees the full fp32 values)
    xf = torch.randn(2, 16, 64, generator=torch.Generator().manual_seed(4)) * 3
    leg["f32_k"], leg["f32_v"] = xf.numpy(), (xf * 0.5).numpy()
    pg = kv_quant.quantize_page(xf, xf * 0.5, 0, use_mse=True, n_alphas=7)
    leg["f32_k_int4"], leg["f32_k_scale"] = pg.k_int4.numpy(), bits16(pg.k_scale)
    leg["f32_v_int4"], leg["f32_v_scale"] = pg.v_int4.numpy(), bits16(pg.v_scale)
    # a two-layer cache fed in ragged appends (5, 20, 1, 13, 9 tokens = 48)
    cache = kv_quant.QuantizedKVCache()
    t = 0
    for n in (5, 20, 1, 13, 9):
        for layer in (0, 1):
            sc = 1.0 if layer == 0 else 0.25
            cache.update(layer, (k[None, :, t:t + n] * sc).bfloat16(), (v[None, :, t:t + n] * sc).bfloat16())
        t += n
        kk, vv = cache.get_kv(1)
        leg[f"cache_t{t}_k"], leg[f"cache_t{t}_v"] = bits16(kk), bits16(vv)
        leg[f"cache_t{t}_mem"] = np.array([cache.mem_bytes(), cache.bf16_bytes()])
        leg[f"cache_t{t}_ratio"] = np.array([cache.compression_ratio()])
        leg[f"cache_t{t}_len"] = np.array([cache.layers[1].seq_len()])
    kk, vv = cache.get_kv(0)
    leg["cache_l0_k"], leg["cache_l0_v"] = bits16(kk), bits16(vv)
    xe = (torch.randn(4, 80, 128, generator=torch.Generator().manual_seed(6)) *
          torch.exp(torch.empty(1, 1, 128).uniform_(-1.0, 2.0, generator=torch.Generator().manual_seed(7))))
    leg["err_x"] = xe.numpy()
    e = kv_quant.measure_page_error(xe)
    leg["err"] = np.array([e["absmax_mse"], e["optimal_mse"], e["reduction_pct"]])
    np.savez_compressed(os.path.join(HERE, "legacy_page.npz"), **leg)

    # ------- 7. heavy-tailed K (randn**3, tests/test_int4_kivi.py:51-56) -------
    # the reference test's input distribution, drawn here on the CPU generator;
    # codes and scales from the reference test's recipe (`_ref_codes`)
    ht = {}
    g = torch.Generator().manual_seed(0)
    k = (torch.randn(2, 72, 128, generator=g) ** 3).to(torch.bfloat16)
    v = torch.randn(2, 72, 128, generator=g).to(torch.bfloat16)
    ht["k"], ht["v"] = bits16(k), bits16(v)
    for calib in ("absmax", "mse"):
        kb = _to_blocks(k[:, :64], "channel").float()
        ks = _calibrate(kb, qmax, qfn, calib)
        vb = _to_blocks(v, "headdim").float()
        vs = _calibrate(vb, qmax, qfn, calib)
        ht[f"{calib}_k_packed"] = pack_codes(qfn(kb / ks))
        ht[f"{calib}_k_scale"] = bits16(ks[..., 0].to(torch.float16))
        ht[f"{calib}_v_packed"] = pack_codes(qfn(vb / vs))
        ht[f"{calib}_v_scale"] = bits16(vs[..., 0].to(torch.float16))
        ht[f"{calib}_k_rt"] = bits16(kv_quant.roundtrip(k, "int4", "channel", calib))
    np.savez_compressed(os.path.join(HERE, "heavy_tail.npz"), **ht)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
