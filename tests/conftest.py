"""Shared pytest configuration.

``-m gpu`` tests need a B200 and the built native library; everything else
runs on CPU (the oracle against the golden vectors, host-side argument
validation, the C-ABI export table, and the gloo multi-rank sharding logic).
"""
from __future__ import annotations

import importlib
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG_NAME = "fused-quantized-kv-decode-attention_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


def load_package():
    """Import the product package (its directory name is not an identifier)."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def fqkv():
    return load_package()


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
