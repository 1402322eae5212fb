"""Shared test set-up.

`-m "not gpu"` runs on any machine: the oracle restatement against the
compiled reference and the reference's golden vectors, the host logic, and
the C ABI's symbol table. `-m gpu` runs the parity tests proper on a B200,
calling libsllm_cuda.so through its C ABI.
"""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device of compute capability 10.x (B200)")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("saphira-llm_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("saphira-llm_b200.synth")


@pytest.fixture(scope="session")
def orc():
    import oracle
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(ref=False)
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.reference_available():
        if os.path.isdir(os.path.join(oracle.REFERENCE_DIR, "src")):
            oracle.build(ref=True)
        else:
            pytest.skip("reference library oracle/_ref/libsllm_ref.so not built and the reference tree is absent")
    return oracle.Reference()


@pytest.fixture(scope="session")
def cuda(pkg):
    """The CUDA backend on a real device. A GPU test fails (never skips) when
    the library is missing or the device is unusable: the product has no CPU
    fallback, so a silent skip would hide exactly that."""
    rc, n, cc = pkg.probe()
    assert rc == 0, f"sllm_cuda_probe: {rc} ({pkg.lib().sllm_cuda_last_error().decode()})"
    assert cc[0] == 10, f"compute capability {cc}"
    import torch
    assert torch.cuda.is_available()
    return pkg


@pytest.fixture(scope="session")
def cuda_absent(pkg):
    """For CPU tests of behaviour without a device: skipped where one exists."""
    rc, n, cc = pkg.probe()
    if rc == 0:
        pytest.skip("a CUDA device is present")
    return pkg


def bits(a):
    """Bit patterns of a float32 array, for exact comparisons. Every NaN maps
    to one pattern: x86 produces the negative default NaN (0xffc00000) where a
    GPU produces 0x7fffffff, and both mean the same value."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).copy()
    u[np.isnan(a)] = 0x7FC00000
    return u
