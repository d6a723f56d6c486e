"""Shared pytest setup.

* puts the package directory (``tile-ascendnpu-ops_b200``) and the repo root
  (for ``oracle``) on ``sys.path``;
* registers the markers: ``gpu`` (needs a B200; the parity tests proper),
  plus the reference's ``smoke`` / ``full`` / ``packaging`` tiers;
* seeds torch with 1235 before every test, like the reference conftest
  (examples/TileOPs/tests/conftest.py:8-12);
* attaches the checked op and its max abs error to the JUnit properties.
"""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "tile-ascendnpu-ops_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

from tileops.testing.test_base import get_check_result  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the native kernels")
    config.addinivalue_line("markers", "smoke: quick reference-tier case")
    config.addinivalue_line("markers", "full: larger reference-tier case")
    config.addinivalue_line("markers", "packaging: packaging sanity case")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def setup() -> None:
    torch.manual_seed(1235)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(1235)


@pytest.hookimpl(hookwrapper=True)
def pytest_runtest_call(item):
    yield
    cr = get_check_result()
    if cr.op_name:
        item.user_properties.append(("op", cr.op_name))
        if cr.op_module:
            item.user_properties.append(("op_module", cr.op_module))
        if cr.max_abs_err is not None:
            item.user_properties.append(("max_abs_err", f"{cr.max_abs_err:.2e}"))
        cr.op_name = None
        cr.op_module = None
        cr.max_abs_err = None
