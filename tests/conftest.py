"""Shared pytest setup: markers, import paths, seeded input generators."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "poolside-hackathon_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name))


def bf16_from_bits(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def gen_kv(H, S, D, seed, Hq=None, B=None):
    """Seeded inputs: k = randn * per-channel log-uniform[0.5, 8] factors,
    v = randn, q = randn; drawn on CPU so every device sees the same bits."""
    import torch
    g = torch.Generator().manual_seed(seed)
    b = B or 1
    k0 = torch.randn(b, H, S, D, generator=g)
    f = torch.exp(torch.empty(1, H, 1, D).uniform_(float(np.log(0.5)), float(np.log(8.0)), generator=g))
    k = (k0 * f).bfloat16()
    v = torch.randn(b, H, S, D, generator=g).bfloat16()
    q = torch.randn(b, Hq or H, 1, D, generator=g).bfloat16() if Hq else None
    if B is None:
        return k[0], v[0], (q[0] if q is not None else None)
    return k, v, q


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    return torch.device("cuda:0")


# ---------------------------------------------------------------------------
# The decode bar, one definition for every decode path (contiguous, varlen,
# paged, the fused hf read path, multi-GPU), against the oracle's
# double-precision attention on the same dequantised values:
#   * fp32 state (the normalised output before the bf16 cast):
#       max-abs <= 2e-3 and relative RMS <= 1e-3;
#   * bf16 output: relative RMS <= 1e-3 against the oracle rounded to bf16,
#       and elementwise |out - ref| <= 2e-3 + |ref| * 2^-8 (the fp32 bar plus
#       one bf16 rounding step of the value).
# ---------------------------------------------------------------------------
FP32_MAX_ABS, REL_RMS = 2e-3, 1e-3


def _f64(x):
    import torch
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().double().numpy()
    return np.asarray(x, dtype=np.float64)


def check_decode_fp32(got, ref, what=""):
    g, r = _f64(got), _f64(ref)
    err = np.abs(g - r).max() if g.size else 0.0
    rel = np.sqrt(((g - r) ** 2).sum() / max((r ** 2).sum(), 1e-300))
    assert err <= FP32_MAX_ABS and rel <= REL_RMS, f"{what} fp32 max-abs {err:.3e} rel-rms {rel:.3e}"
    return err, rel


def check_decode_bf16(got, ref, what=""):
    import torch
    g, r = _f64(got), _f64(ref)
    rb = torch.from_numpy(r).to(torch.bfloat16).double().numpy()
    err = np.abs(g - r)
    ok = err <= 2e-3 + np.abs(r) * 2.0 ** -8
    assert bool(ok.all()), f"{what} bf16 max-abs {err.max():.3e} ({int((~ok).sum())} elements over the bound)"
    rel = np.sqrt(((g - rb) ** 2).sum() / max((r ** 2).sum(), 1e-300))
    assert rel <= REL_RMS, f"{what} bf16 rel-rms {rel:.3e} vs the bf16-rounded oracle"
    return float(err.max()) if err.size else 0.0, rel
