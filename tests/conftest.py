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
