"""Pytest configuration.

* ``gpu`` marks tests that need a CUDA device (run with ``-m gpu`` on a B200);
  everything else runs on CPU.
* The package under test is ``associative_scan_triton`` from
  ``associative-scan-triton_b200/``; the oracle is ``oracle/`` at the repo root.
* Device-side error checking (a sync after every op) is switched on for the
  whole session so that a device-detected problem fails the test that caused it.
"""

from __future__ import annotations

import gc
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
DIST = REPO / "associative-scan-triton_b200"
for p in (str(REPO), str(DIST), str(Path(__file__).resolve().parent)):
  if p not in sys.path:
    sys.path.insert(0, p)

os.environ.setdefault("ASCAN_SYNC_CHECK", "1")


def _build_native() -> None:
  """Build the oracle and, when nvcc exists, the native library if stale."""
  from oracle import oracle as _oracle

  _oracle.build()
  import build_native

  if not build_native.up_to_date():
    try:
      build_native._nvcc()
    except RuntimeError:
      return
    build_native.build()


_build_native()

import torch  # noqa: E402

import associative_scan_triton as ast  # noqa: E402

ast.set_sync_check(True)


def pytest_configure(config):
  config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
  config.addinivalue_line("markers", "slow: large-shape test")


def pytest_collection_modifyitems(config, items):
  if torch.cuda.is_available():
    return
  skip = pytest.mark.skip(reason="CUDA device required")
  for item in items:
    if "gpu" in item.keywords:
      item.add_marker(skip)


@pytest.fixture(autouse=True)
def _cuda_hygiene():
  yield
  if torch.cuda.is_available():
    torch.cuda.synchronize()
  gc.collect()


@pytest.fixture(params=["tma", "simple"])
def impl(request):
  """Run a test under both kernel families (persistent TMA and plain)."""
  from associative_scan_triton import _lib

  _lib.set_implementation(request.param)
  yield request.param
  _lib.set_implementation("auto")


def first_order_op(fl, xl, fr, xr):
  """Plain-Python combine operator (reference tests/conftest.py:67-71)."""
  return fr * fl, fr * xl + xr
