import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "nano-vllm-spec-decode_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libnvattn.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def load_golden(name):
    import numpy as np
    z = np.load(os.path.join(REPO, "tests", "golden", name), allow_pickle=False)
    cases = {}
    for key in z.files:
        case, field = key.split("/", 1)
        cases.setdefault(case, {})[field] = z[key]
    return cases


# Attention tolerance of the north star: BF16 output vs the FP32 oracle, max-abs 2e-2 / relative 1e-2.
ATOL, RTOL = 2e-2, 1e-2


def assert_attn_close(got, ref, what=""):
    import torch
    got = got.float().cpu()
    ref = ref.float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs()
    bound = ATOL + RTOL * ref.abs()
    bad = err > bound
    assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance, max abs err {float(err.max()):.4g}"
