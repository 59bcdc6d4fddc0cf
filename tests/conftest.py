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
    # CPU runs bind the test link of the library, which adds the fake-device seam to the
    # product exports; `-m gpu` runs bind the product library itself.
    import os
    if config.getoption("markexpr", "") != "gpu" and not os.environ.get("XVRAM_B200_LIBRARY"):
        from fake_device import testing_library
        os.environ["XVRAM_B200_LIBRARY"] = str(testing_library())


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
