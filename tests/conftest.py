"""Shared pytest setup: the `gpu` marker, repo-root imports, and seeding."""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _reference_import_path() -> str | None:
    """Where `import strands_decider` (the reference package) comes from: the directory named
    by STRANDS_DECIDER_SRC (a checkout root with src/strands_decider, or a directory holding
    the installed package), else this repository's baseline/_ref install (`pip install
    --target baseline/_ref <reference>`), when present."""
    root = os.environ.get("STRANDS_DECIDER_SRC") or os.path.join(ROOT, "baseline", "_ref")
    for cand in (os.path.join(root, "src"), root):
        if os.path.isdir(os.path.join(cand, "strands_decider")):
            return cand
    return None


REFERENCE_PATH = _reference_import_path()
if REFERENCE_PATH and REFERENCE_PATH not in sys.path:
    sys.path.append(REFERENCE_PATH)


def require_reference():
    """Skip the calling test unless the reference package is importable."""
    if REFERENCE_PATH is None:
        pytest.skip("the reference package is not installed (set STRANDS_DECIDER_SRC or install it into "
                    "baseline/_ref)")
    return pytest.importorskip("strands_decider.infer")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on the CPU")


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield
