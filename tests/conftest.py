"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import load_oracle
    return load_oracle()


@pytest.fixture(scope="session")
def ref_lib():
    from oracle_lib import load_reference
    lib = load_reference()
    if lib is None:
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    return lib


@pytest.fixture(scope="session")
def golden():
    import json
    return json.loads((TESTS / "golden" / "reference_vectors.json").read_text())
