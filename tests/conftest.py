"""Test configuration: markers and import paths.

-m "not gpu": oracle, golden fixtures, C-ABI symbol/argument checks, work
partition and multi-rank host logic (gloo) - no GPU needed.
-m gpu: parity of the CUDA kernels (called through the C ABI) against the
oracle on a B200.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "gpullama3.java_b200"), os.path.join(REPO, "oracle"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as _oracle  # noqa: WPS433 - test infrastructure

    _oracle.build()
    return _oracle


def _cuda_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gla_ctx():
    if not _cuda_available():
        pytest.skip("no CUDA device")
    import torch
    import gpullama_attn as gla

    torch.cuda.init()
    ctx = gla.Context(0, torch.cuda.current_stream().cuda_stream)
    yield ctx
    ctx.close()
