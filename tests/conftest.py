"""Shared test setup: the `gpu` marker, repo-root imports and fixtures."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libwllm_mulmat.so")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def runtime():
    """JSEP-style runtime bound to cuda:0. Fails (does not skip) when the
    CUDA library or the GPU is missing: GPU tests must run the native path."""
    from webllm_b200 import jsep
    from webllm_b200.build_ext import build

    build()
    rt = jsep.install_jsep_callbacks(0)
    yield rt
    jsep.destroy_jsep_callbacks()
