from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls the sm_100a kernels")


@pytest.fixture(scope="session")
def oracle():
    from oracle import kv_oracle

    kv_oracle.build()
    return kv_oracle


@pytest.fixture(scope="session")
def golden():
    return torch.load(os.path.join(GOLDEN, "reference_cases.pt"), weights_only=True)


@pytest.fixture(scope="session")
def config1_golden():
    return torch.load(os.path.join(GOLDEN, "config1_writes.pt"), weights_only=True)


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests; these tests fail (not skip) without one."""
    assert torch.cuda.is_available(), "gpu-marked tests need a CUDA device"
    from augur_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def bits(t: torch.Tensor) -> torch.Tensor:
    """Bit view for exact comparison: NaNs and -0.0 compare by their bits."""
    t = t.detach().contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def assert_bits_equal(a: torch.Tensor, b: torch.Tensor, what: str = "") -> None:
    assert a.shape == b.shape, f"{what}: shape {tuple(a.shape)} != {tuple(b.shape)}"
    assert a.dtype == b.dtype, f"{what}: dtype {a.dtype} != {b.dtype}"
    ab, bb = bits(a.cpu()), bits(b.cpu())
    if not torch.equal(ab, bb):
        diff = (ab != bb).nonzero()
        mask = (1 << (8 * a.element_size())) - 1
        shown = ", ".join(f"{idx}: {int(ab[tuple(idx)]) & mask:#x} vs {int(bb[tuple(idx)]) & mask:#x}"
                          for idx in diff[:8].tolist())
        raise AssertionError(f"{what}: {diff.shape[0]} elements differ, first at {diff[0].tolist()} "
                             f"(got vs want bits: {shown})")


def poison_(t: torch.Tensor) -> torch.Tensor:
    t.view(torch.uint8).fill_(0xFF)
    return t
