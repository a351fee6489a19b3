"""Shared test setup: the `gpu` marker, the package import, the oracle import."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    """The product package, imported under its Python name."""
    from __graft_entry__ import import_package

    return import_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import paged_attention_oracle

    return paged_attention_oracle
