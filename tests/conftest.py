"""Shared pytest setup: the `gpu` marker, the package import (its directory name has
a hyphen, so it is imported with importlib), and the golden-fixture loader."""
import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and libmkv.so")


def pytest_collection_modifyitems(config, items):
    # GPU tests must not pass silently on a machine without a GPU: fail them instead.
    import torch
    if torch.cuda.is_available():
        return
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(pytest.mark.usefixtures("_require_gpu"))


@pytest.fixture
def _require_gpu():
    pytest.fail("this test needs a CUDA GPU")


def mkv_module(name=""):
    return importlib.import_module("mini-kvllm_b200" + (("." + name) if name else ""))


@pytest.fixture(scope="session")
def mkv():
    return mkv_module()


@pytest.fixture(scope="session")
def attn():
    return mkv_module("layers.attention")


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))
