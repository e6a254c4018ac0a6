"""Failure detection without a GPU fault.

The kernels' waits are bounded: a wait that is never satisfied gives up,
reports, and every other wait of the launch returns at once, so a lost
predecessor turns into an error status instead of a hang.  Here the waits
are run on conditions that nothing ever satisfies (a flag nobody sets), with
a short limit, through ``ascan_selftest_waits``; then an ordinary scan checks
that the context is still usable.  Malformed ``cu_seqlens`` -- the failure a
caller can actually plant -- are covered in ``test_scan_kernels.py`` with
sync checking on, and here with it off: the host-visible error flag makes a
later op raise without any synchronisation in the ops themselves.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from associative_scan_triton import _lib
from oracle import oracle
from scan_testlib import assert_close_to_gold, cu_of, make_inputs


def test_selftest_refuses_bad_arguments_without_a_gpu():
  lib = _lib.load()
  res = (ctypes.c_longlong * 4)()
  assert lib.ascan_selftest_waits(None, 512, 10_000_000, res, None) == -1
  assert lib.ascan_selftest_waits(256, 100, 10_000_000, res, None) == -1  # too small
  assert lib.ascan_selftest_waits(257, 512, 10_000_000, res, None) == -1  # misaligned


@pytest.mark.gpu
@pytest.mark.parametrize("limit_ms", [20, 100])
def test_unsatisfied_waits_give_up_and_the_context_survives(limit_ms):
  lib = _lib.load()
  ws = torch.empty(512, dtype=torch.uint8, device="cuda")
  res = (ctypes.c_longlong * 4)()
  stream = torch.cuda.current_stream().cuda_stream
  rc = lib.ascan_selftest_waits(ws.data_ptr(), ws.numel(), limit_ms * 1_000_000, res, stream)
  assert rc == 0, _lib.strerror(rc)
  assert res[0] == 0, "a stage barrier nobody arrives on reported success"
  assert res[1] == 0, "a hand-off slot nobody tags reported success"
  assert res[2] == 1, "a look-back with an unpublished predecessor did not give up"
  elapsed_ms = res[3] / 1e6
  assert 3 * limit_ms * 0.9 <= elapsed_ms <= 3 * limit_ms + 1000, elapsed_ms
  # the sticky error word is untouched and the context still runs scans
  _lib.check_device_error()
  g, x = make_inputs(4, 9000, gate="long")
  cu = cu_of([5000, 4000])
  y = torch.empty_like(x)
  _lib.forward(g, x, y, None, cu, 2, 4, False)
  torch.cuda.synchronize()
  gold, _ = oracle.scan_fwd(g, x, cu)
  assert_close_to_gold(y, gold, torch.float32, "scan after the self-test")


@pytest.mark.gpu
def test_device_error_surfaces_without_sync_checking():
  """A cu_seqlens that does not end at BL, passed with sync checking off: the
  call itself returns (the kernel runs asynchronously, stays in bounds and
  reports), and once it has run the following op raises ScanError from the
  host-visible flag.  The reference reads out of bounds silently here
  (reference tests/test_scan_kernels.py:45-83)."""
  g, x = make_inputs(3, 1000, gate="long")
  y = torch.empty_like(x)
  bad = cu_of([400, 700])  # ends at 1100 > BL = 1000
  good = cu_of([400, 600])
  was = _lib.sync_check_enabled()
  _lib.set_sync_check(False)
  try:
    _lib.clear_device_error()
    assert _lib.error_flag() == 0
    _lib.forward(g, x, y, None, bad, 2, 3, False)  # no exception: nothing synchronised
    torch.cuda.synchronize()                       # the failing kernel has run
    assert _lib.error_flag() & _lib.DEV_ERR_CU_END
    with pytest.raises(_lib.ScanError, match="cu_seqlens"):
      _lib.forward(g, x, y, None, good, 2, 3, False)
    # reading the error cleared it: the next ops run and are right
    assert _lib.error_flag() == 0
    _lib.forward(g, x, y, None, good, 2, 3, False)
    torch.cuda.synchronize()
    assert _lib.error_flag() == 0
  finally:
    _lib.set_sync_check(was)
  gold, _ = oracle.scan_fwd(g, x, good)
  assert_close_to_gold(y, gold, torch.float32, "scan after the reported error")
