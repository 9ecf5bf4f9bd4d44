"""Shared test set-up.

- `-m gpu` marks tests that need a CUDA GPU (a B200); everything else runs on the CPU.
- The product package lives in `mini-llm-inference-server_b200/`, a directory name that is not a Python
  identifier, so it is imported with `importlib` (`load_package`).
- Golden fixtures and their seeded input builders are in `tests/golden/`.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)

PACKAGE = "mini-llm-inference-server_b200"


def reference_src() -> Path | None:
    """The reference's `src/` directory, when its source tree is at hand (MINILLM_REF_SRC, or a checkout named
    `reference` beside this repository): CPU tests then pin fixtures and adapters against the reference's
    live objects.  The GPU box has no copy, and no GPU test uses it."""
    env = os.environ.get("MINILLM_REF_SRC")
    cand = Path(env) if env else REPO.parent / "reference" / "src"
    return cand if (cand / "minillm" / "attention" / "metadata.py").is_file() else None


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
