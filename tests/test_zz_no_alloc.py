"""GPU: ascan_forward_noalloc, the forward scan that allocates nothing.

Some callers cannot allocate device memory at call time (a serving loop on a
fixed memory budget without an allocator, a plugin that is only handed its
input and output buffers, a foreign-language binding of the C ABI with no
access to torch's caching allocator).  For them the library keeps the
look-back scratch in a fixed device array and exposes this entry point.

The test calls it through the C ABI with ctypes and compares each result
with the regular entry point (``ascan_forward`` with a caller-provided
workspace), within the suite's fp32 tolerance, on two calls in a row -- the
second reuses the array that the first one left behind.  The file is named
so that pytest collects it last, and it needs nothing from earlier tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from associative_scan_triton import _lib
from scan_testlib import assert_close_to_gold, cu_of, make_inputs

ASCAN_ETOOLARGE = -5
MAX_ELEMENTS = 536805376


def _noalloc():
  lib = _lib.load()
  fn = lib.ascan_forward_noalloc
  p, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
  fn.restype = ci
  fn.argtypes = [p, p, p, p, p, ci, i64, i64, i64, ci, ci, p]
  return fn


def _call(fn, g, x, y, gout, cu, reverse):
  C, BL = g.shape
  return fn(g.data_ptr(), x.data_ptr(), y.data_ptr(),
            gout.data_ptr() if gout is not None else None, cu.data_ptr(),
            _lib.INDEX_CODES[cu.dtype], cu.numel() - 1, C, BL, _lib.DTYPE_CODES[g.dtype],
            int(reverse), torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
def test_forward_noalloc_matches_forward_on_two_calls_in_a_row():
  fn = _noalloc()
  cases = [
    # (C, seqlens, reverse, gate products): a long sequence that needs look-back,
    # then a different packing that reuses the scratch the first call left
    (64, [20000, 4096, 77, 9000], False, True),
    (300, [5, 4096, 1, 2500], True, False),
  ]
  for i, (C, seqlens, reverse, want_gates) in enumerate(cases):
    g, x = make_inputs(C, sum(seqlens), gate="long", seed=100 + i)
    cu = cu_of(seqlens, dtype=torch.int32 if i else torch.int64)
    y_ref = torch.empty_like(x)
    g_ref = g.clone() if want_gates else None
    _lib.forward(g, x, y_ref, g_ref, cu, len(seqlens), C, reverse)
    y = torch.full_like(x, float("nan"))
    g_out = torch.full_like(g, float("nan")) if want_gates else None
    rc = _call(fn, g, x, y, g_out, cu, reverse)
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    _lib.check_device_error()
    assert_close_to_gold(y, y_ref.double().cpu().numpy(), torch.float32, f"call {i} y")
    if want_gates:
      assert_close_to_gold(g_out, g_ref.double().cpu().numpy(), torch.float32,
                           f"call {i} gate products")


@pytest.mark.gpu
def test_forward_noalloc_rejects_sizes_beyond_its_scratch():
  fn = _noalloc()
  cu = torch.tensor([0, 1], dtype=torch.int64, device="cuda")
  # one element more than the fixed scratch can serve: refused before any launch
  dummy = torch.empty(16, device="cuda")
  rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None, cu.data_ptr(), 1, 1,
          MAX_ELEMENTS + 1, 1, 0, 0, torch.cuda.current_stream().cuda_stream)
  assert rc == ASCAN_ETOOLARGE
  assert "fixed scratch" in _lib.strerror(rc)
  assert np.int64(MAX_ELEMENTS) // 4096 == 131056  # whole 4096-element status slots
