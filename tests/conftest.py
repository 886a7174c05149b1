"""Shared pytest setup: the `gpu` marker and golden-fixture access."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def case_names(golden_dict):
    return [str(n) for n in golden_dict["cases"]]


def load_case(g, name):
    """Collect one fixture case as a plain dict (keys without the prefix)."""
    p = f"{name}/"
    return {k[len(p):]: v for k, v in g.items() if k.startswith(p)}


def golden_case_list():
    with np.load(GOLDEN) as z:
        return [str(n) for n in z["cases"]]
