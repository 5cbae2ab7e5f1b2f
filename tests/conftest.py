"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import kvl_pkg  # noqa: E402

kvl_pkg.load()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA C-ABI library)")


@pytest.fixture(scope="session")
def K():
    import kvl_b200.kvl_mla as K  # noqa: N812
    K.load()
    return K


@pytest.fixture(scope="session")
def S():
    import kvl_b200.synth as S  # noqa: N812
    return S


@pytest.fixture(scope="session")
def orc():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref not built (reference sources absent when building)")
    return Reference()


@pytest.fixture(scope="session")
def ref_scalar():
    from oracle.oracle import REF_SCALAR_SO, Reference, reference_available
    if not reference_available(scalar=True):
        pytest.skip("oracle/_ref not built")
    return Reference(REF_SCALAR_SO)


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA")
    torch.cuda.init()
    return torch
