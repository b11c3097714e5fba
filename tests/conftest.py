"""Shared pytest setup: the `gpu` marker, repo import path, golden fixtures."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture
def repo_tmp(request):
    """A scratch directory inside the repository (git-ignored `.test_tmp/`),
    removed after the test, so that file-writing tests stay in the tree."""
    import shutil
    import uuid
    d = os.path.join(ROOT, ".test_tmp", f"{request.node.name[:40]}-{uuid.uuid4().hex[:8]}")
    os.makedirs(d)
    yield __import__("pathlib").Path(d)
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN, "gemm_path.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cfg0_digests():
    out = {}
    with open(os.path.join(GOLDEN, "cfg0_sha256.txt")) as f:
        for line in f:
            if line.startswith("#") or not line.strip():
                continue
            k, v = line.split()
            out[k] = v
    return out


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests need a CUDA device; on a GPU box the extension must load
    (no fallback), so a missing library fails instead of skipping."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ovnative_b200 as ovb
    ovb.lib()
    return torch.device("cuda", 0)
