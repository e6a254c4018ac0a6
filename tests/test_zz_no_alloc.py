"""GPU: ascan_forward_noalloc, the forward scan that allocates nothing.

Some callers cannot allocate device memory at call time (a serving loop on a
fixed memory budget without an allocator, a plugin that is only handed its
input and output buffers, a foreign-language binding of the C ABI with no
access to torch's caching allocator).  For them the library keeps the
look-back scratch in a fixed device array and exposes this entry point.

The test calls it through the C ABI with ctypes and compares each result with
the regular entry point (``ascan_forward`` with a caller-provided workspace)
and with the fp64 oracle, within the suite's tolerance of each dtype, on calls
in a row -- each later call reuses the array that the earlier ones left
behind.  The last call is a bfloat16 problem just under the array's limit at
a shape where the forward runs 8192-element tiles, whose status records are
counted in the array's 4096-element slots.  The file is named so that pytest
collects it last, and it needs nothing from earlier tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from associative_scan_triton import _lib
from oracle import oracle
from scan_testlib import assert_close_to_gold, cu_of, in_sequence_mask, make_inputs

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


def _device_inputs(C, BL, dtype, seed):
  gen = torch.Generator(device="cuda").manual_seed(seed)
  g = (0.9 + 0.1 * torch.rand(C, BL, device="cuda", generator=gen)).to(dtype)
  x = torch.randn(C, BL, device="cuda", generator=gen).to(dtype)
  return g, x


@pytest.mark.gpu
def test_forward_noalloc_matches_forward_and_oracle_on_calls_in_a_row():
  fn = _noalloc()
  big_c, big_bl = 16380, 32768  # 536,739,840 elements: just under MAX_ELEMENTS
  assert big_c * big_bl <= MAX_ELEMENTS
  cases = [
    # (C, seqlens, dtype, reverse, gate products): a long sequence that needs
    # look-back, a different packing that reuses the scratch the first call
    # left, then bf16 near the limit (wide tiles in row order)
    (64, [20000, 4096, 77, 9000], torch.float32, False, True),
    (300, [5, 4096, 1, 2500], torch.float32, True, False),
    (big_c, [20000, big_bl - 20000], torch.bfloat16, False, False),
  ]
  for i, (C, seqlens, dtype, reverse, want_gates) in enumerate(cases):
    BL = sum(seqlens)
    if C * BL > 10**7:
      g, x = _device_inputs(C, BL, dtype, seed=100 + i)
    else:
      g, x = make_inputs(C, BL, dtype=dtype, gate="long", seed=100 + i)
    cu = cu_of(seqlens, dtype=torch.int32 if i % 2 else torch.int64)
    y_ref = torch.empty_like(x)
    g_ref = g.clone() if want_gates else None
    _lib.forward(g, x, y_ref, g_ref, cu, len(seqlens), C, reverse)
    y = torch.full_like(x, float("nan"))
    g_out = torch.full_like(g, float("nan")) if want_gates else None
    rc = _call(fn, g, x, y, g_out, cu, reverse)
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    _lib.check_device_error()
    # against the regular entry point (whole tensors; the same kernels run)
    if C * BL > 10**7:  # on the device: |y - y_ref| <= rtol (|y_ref| + rms(y_ref))
      yr = y_ref.float()
      bound = 2e-2 * (yr.abs() + yr.square().mean().sqrt())
      bad = int(((y.float() - yr).abs() > bound).sum())
      assert bad == 0, f"call {i}: {bad} elements differ from ascan_forward"
    else:
      assert_close_to_gold(y, y_ref.double().cpu().numpy(), dtype, f"call {i} y vs ascan_forward")
      if want_gates:
        assert_close_to_gold(g_out, g_ref.double().cpu().numpy(), dtype,
                             f"call {i} gate products vs ascan_forward")
    # against the fp64 oracle (a seeded sample of rows for the large call)
    rows = (np.arange(C) if C <= 512 else
            np.unique(np.r_[0, 1, C // 2, C - 1,
                            np.random.default_rng(i).integers(0, C, 4)]))
    idx = torch.as_tensor(rows, device="cuda")
    gold_y, gold_a = oracle.scan_fwd(g[idx], x[idx], cu, reverse=reverse)
    mask = in_sequence_mask(len(rows), BL, cu)
    assert_close_to_gold(y[idx], gold_y, dtype, f"call {i} y vs oracle", mask=mask)
    if want_gates:
      assert_close_to_gold(g_out[idx], gold_a, dtype, f"call {i} gate products vs oracle",
                           mask=mask)
    del g, x, y, y_ref, g_ref, g_out
    torch.cuda.empty_cache()


@pytest.mark.gpu
def test_forward_noalloc_rejects_sizes_beyond_its_scratch():
  fn = _noalloc()
  cu = torch.tensor([0, 1], dtype=torch.int64, device="cuda")
  # one element more than the fixed scratch can serve: refused on the host
  # before anything else is looked at -- the data pointers are NULL, so if the
  # size check ever regressed the call would fail with EINVAL, not launch
  rc = fn(None, None, None, None, cu.data_ptr(), 1, 1, MAX_ELEMENTS + 1, 1, 0, 0,
          torch.cuda.current_stream().cuda_stream)
  assert rc == ASCAN_ETOOLARGE
  assert "fixed scratch" in _lib.strerror(rc)
  assert np.int64(MAX_ELEMENTS) // 4096 == 131056  # whole 4096-element status slots
