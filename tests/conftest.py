"""Shared test setup.

Markers: `gpu` tests need a CUDA device and call the engine through the C ABI; all other
tests run on CPU (oracle vs reference, golden vectors, host logic, library exports).
"""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "minicpm5.cpp_b200")
for p in (PKG, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build(reference=True)
    return O.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle as O
    O.build(reference=True)
    if not O.have_ref():
        pytest.skip("reference library not built (reference tree absent)")
    return O.Ref()


@pytest.fixture(scope="session")
def model_path():
    from mcpm import synth
    return synth.ensure_model("q4_k_m", 0)


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def rand_tensor_bytes(ggml_type, rows, cols, seed):
    from mcpm import spec, synth
    t = spec.TensorInfo("w", ggml_type, (cols, rows))
    return synth.tensor_bytes(t, np.random.Generator(np.random.PCG64([seed, 99])))
