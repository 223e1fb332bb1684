import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "llm.cpp_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu on a B200)")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def llmk_lib():
    """libllmk.so built in-tree (builds it when missing or stale)."""
    import build as llmk_build  # llm.cpp_b200/build.py
    llmk_build.ensure_built()
    import llmk
    return llmk.lib()


@pytest.fixture(scope="session")
def cuda_dev(llmk_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    cc = torch.cuda.get_device_capability(0)
    assert cc[0] == 10, f"needs sm_100 (B200), found sm_{cc[0]}{cc[1]}"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _as_double(x):
    import numpy as np
    import torch
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x)).double()
    return x.detach().double().cpu()


def max_rel_err(x, y) -> float:
    """max_i |x_i - y_i| / max_j |y_j| (the parity metric of the hot path)."""
    x = _as_double(x)
    y = _as_double(y)
    den = y.abs().max().item()
    return (x - y).abs().max().item() / max(den, 1e-30)


def norm_rel_err(x, y) -> float:
    """||x - y||_2 / ||y||_2 (the reference tests' Eigen isApprox metric)."""
    x = _as_double(x)
    y = _as_double(y)
    return ((x - y).norm() / max(y.norm().item(), 1e-30)).item()
