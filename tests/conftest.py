"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; the rest run on CPU."""
import importlib
import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
GOLDEN = REPO / "tests" / "golden" / "golden.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_pkg():
    return importlib.import_module("pytorch-implementation-of-screening-attention_b200")


@pytest.fixture(scope="session")
def ms():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    from oracle import screening_oracle
    return screening_oracle


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    return torch.device("cuda:0")


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / max |b| (0 when both are all-zero)."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = b.abs().max().item()
    num = (a - b).abs().max().item()
    if den == 0.0:
        return num
    return num / den
