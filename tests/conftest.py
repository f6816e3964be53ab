"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref_strict():
    from oracle.oracle import REF_STRICT_SO, RefLib
    if not REF_STRICT_SO.exists():
        pytest.skip("reference library not built here (oracle/_ref)")
    return RefLib(REF_STRICT_SO)


@pytest.fixture(scope="session")
def ref_native():
    from oracle.oracle import REF_NATIVE_SO, RefLib
    if not REF_NATIVE_SO.exists():
        pytest.skip("reference library not built here (oracle/_ref)")
    return RefLib(REF_NATIVE_SO)


@pytest.fixture(scope="session")
def gpu():
    """The CUDA library bound to torch's current stream (fails loudly without it)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from gncx_b200 import core
    lib = core.load()
    torch.cuda.init()
    lib.gncx_set_synchronous(1)
    core.bind_torch_stream(lib)
    return lib


def golden(name: str) -> dict:
    with np.load(ROOT / "tests" / "golden" / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}
