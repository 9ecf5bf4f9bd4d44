"""Shared test set-up.

- `-m gpu` marks tests that need a CUDA GPU (a B200); everything else runs on the CPU.
- The product package lives in `mini-llm-inference-server_b200/`, a directory name that is not a Python
  identifier, so it is imported with `importlib` (`load_package`).
- Golden fixtures and their seeded input builders are in `tests/golden/`.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)

PACKAGE = "mini-llm-inference-server_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run on the B200 box with -m gpu)")


def load_package():
    return importlib.import_module(PACKAGE)


@pytest.fixture(scope="session")
def mlb():
    return load_package()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test is marked gpu and needs CUDA")
    return torch.device("cuda", 0)
