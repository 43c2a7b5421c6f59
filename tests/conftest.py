"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "universal-ai-inference_b200")
for p in (REPO, PKG, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def um():
    import uaii_moe
    return uaii_moe


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("reference build oracle/_ref/libuaii_ref.so not present")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(REPO, "tests", "golden", "golden.npz")
    return dict(np.load(path))


@pytest.fixture(scope="session")
def backend(um):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    b = um.Backend(0)
    yield b
    b.close()
