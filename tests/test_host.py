"""CPU: host-side logic and the C ABI boundary (no compute calls without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import associative_scan_triton as ast
from associative_scan_triton import _lib
from conftest import REPO

HEADER = REPO / "include" / "ascan.h"


def _header_functions() -> list[str]:
  text = HEADER.read_text()
  return re.findall(r"^ASCAN_API\s+[\w\s\*]+?\b(ascan_\w+)\s*\(", text, flags=re.M)


def test_library_exports_every_header_symbol():
  names = _header_functions()
  assert len(names) >= 9, names
  assert set(names) == set(_lib.EXPORTED_SYMBOLS)
  lib = ctypes.CDLL(str(_lib.LIB_PATH))
  for n in names:
    assert hasattr(lib, n), f"{n} declared in {HEADER.name} but not exported"


def test_library_identity():
  lib = _lib.load()
  assert lib.ascan_abi_version() == 1
  assert b"sm_100a" in lib.ascan_build_info()
  assert _lib.strerror(0) == "ok"
  assert "workspace" in _lib.strerror(-2)


def test_workspace_size_grows_with_problem():
  lib = _lib.load()
  small = lib.ascan_workspace_size(4, 128, 0)
  big = lib.ascan_workspace_size(1536, 8 * 65536, 0)
  assert small >= 256 and big > small
  # one 16-byte status slot per 4096 elements plus a 256-byte header
  tiles = (1536 * 8 * 65536 + 4095) // 4096
  assert big == 256 + 16 * tiles
  # rows that are not whole tiles: one slot per tile of every row (row order
  # cuts each row into whole tiles and a partial last one)
  assert lib.ascan_workspace_size(7, 4097, 0) == 256 + 16 * 7 * 2
  assert lib.ascan_workspace_size(3, 100, 0) == 256 + 16 * 1  # flat count is larger


def test_abi_rejects_bad_arguments_without_a_gpu():
  lib = _lib.load()
  # no pointers at all -> EINVAL before any CUDA call
  rc = lib.ascan_forward(None, None, None, None, None, 0, 1, 1, 4, 0, 0, None, 0, None)
  assert rc == -1
  rc = lib.ascan_backward(None, None, None, None, None, None, 0, 1, 1, 4, 0, 1, None, 0, None)
  assert rc == -1
  # unknown dtype
  rc = lib.ascan_forward(1, 1, 1, None, 1, 0, 1, 1, 4, 7, 0, None, 0, None)
  assert rc == -1
  # aliasing d_gates with gates is refused
  rc = lib.ascan_backward(16, 32, 48, 64, 32, 80, 0, 1, 1, 4, 0, 1, None, 0, None)
  assert rc == -1
  # a valid call shape without a workspace is refused before launching
  rc = lib.ascan_forward(16, 32, 48, None, 64, 0, 1, 1, 4, 0, 0, None, 0, None)
  assert rc == -2


def test_bidi_abi_refuses_crossed_buffers_without_a_gpu():
  """The two directions of ascan_*_bidi run at the same time, so an output of
  one may not be a buffer the other reads or writes; all checks come before
  any CUDA call."""
  lib = _lib.load()
  gf, xf, yf, gb, xb, yb, cu = 16, 32, 48, 64, 80, 96, 112
  fwd = lambda *p, ws=None: lib.ascan_forward_bidi(*p, cu, 0, 1, 1, 4, 0, ws, 0, None)
  assert fwd(gf, xf, yf, gb, xb, xf) == -1          # reverse output over the causal tokens
  assert fwd(gf, xf, xb, gb, xb, yb) == -1          # causal output over the reverse tokens
  assert fwd(gf, xf, yf, gb, xb, yf) == -1          # one output for both
  assert fwd(gf, xf, yf, gb, xb, yb) == -2          # valid shape, no workspace
  assert fwd(gf, xf, xf, gb, xb, xb) == -2          # in place in each direction is allowed
  dyf, hf, dxf, dgf, dyb, hb, dxb, dgb = 128, 144, 160, 176, 192, 208, 224, 240
  bwd = lambda *p: lib.ascan_backward_bidi(*p, cu, 0, 1, 1, 4, 0, None, 0, None)
  assert bwd(dyf, gf, hf, dxf, dgf, dyb, gb, hb, dxb, dgb) == -2
  assert bwd(dyf, gf, hf, dxf, dgf, dyb, gb, hb, dxb, hf) == -1   # over the causal states
  assert bwd(dyf, gf, hf, dxf, dgf, dyb, gb, hb, dyf, dgb) == -1  # over the causal grad
  assert bwd(dyf, gf, hf, dxf, dgf, dyb, gb, hb, dxf, dgb) == -1  # two outputs in one buffer
  assert bwd(dyf, gf, hf, dyf, dgf, dyb, gb, hb, dyb, dgb) == -2  # d_tokens over own grad: ok
  assert lib.ascan_workspace_size_bidi(7, 4097, 0) == 2 * 512  # two 256-aligned halves


def test_tile_width_knob_without_a_gpu():
  assert _lib.get_tile_width() == 0
  with pytest.raises(ValueError):
    _lib.set_tile_width(24)
  _lib.set_tile_width(32)
  assert _lib.get_tile_width() == 32
  _lib.set_tile_width(0)


def test_ops_refuse_cpu_tensors():
  g = torch.rand(2, 8)
  x = torch.rand(2, 8)
  cu = torch.tensor([0, 8])
  args = {"cu_seqlens": cu, "chunk_size": 8, "grid": ast.get_grid(2, 8, 8, 2)}
  with pytest.raises(ValueError, match="CUDA tensors only"):
    ast.scan_causal(g, x, args)
  with pytest.raises(ValueError, match="CUDA tensors only"):
    ast.forward_scan_full(g, x, cu, args["grid"], REVERSE=False, CHUNK_SIZE=8)
  with pytest.raises(ValueError, match="CUDA tensors only"):
    ast.shift_pad(g, cu, 0.0, True)


def test_dispatcher_grid_assertion():
  g = torch.rand(1, 8)
  with pytest.raises(AssertionError, match="cu_seqlens do not match grid"):
    ast.forward_scan_full(g, g, torch.tensor([0, 4, 8]), (1, 1, 1), REVERSE=False, CHUNK_SIZE=4)


def test_shift_pad_zero_length_assertion():
  # reference tests/test_shift_pad.py:120-132 (checked before any kernel runs)
  data = torch.tensor([[1.0, 2.0, 3.0]])
  with pytest.raises(AssertionError, match="can't shift_pad zero-length seqments"):
    ast.shift_pad(data, torch.tensor([0, 0, 1, 1, 3]), -1, True)


# --- grid helpers: same results as the reference (src/associative_scan_triton/_grid.py) ---

def _ref_next_power_of_2(n: int) -> int:
  # bit-smearing restatement of the reference's function, for comparison
  n -= 1
  for s in (1, 2, 4, 8, 16, 32):
    n |= n >> s
  return n + 1


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 5, 7, 8, 9, 100, 512, 513, 4096, 65535, 65536,
                               2**31 - 1, 2**31, 2**40 + 3])
def test_next_power_of_2(n):
  assert ast.next_power_of_2(n) == _ref_next_power_of_2(n)


def test_get_grid_matches_reference():
  assert ast.get_grid(9, 4096, 512, 1536) == (8, 8, 1536)
  assert ast.get_grid(33, 8192, 512, 2048) == (32, 16, 2048)
  assert ast.get_grid(2, 128, 128, 4) == (1, 1, 4)
  assert ast.get_grid(2, 5, 4, 1) == (1, 2, 1)
  assert ast.get_grid(2, 9, 4, 1) == (1, 4, 1)  # 3 chunks padded to 4
  with pytest.raises(AssertionError, match="chunk size must be divisible by 2"):
    ast.get_grid(2, 8, 3, 1)
  assert ast.get_static_grid(4096, 512, 1536) == (8, 1536)


def test_get_num_stages_table():
  from associative_scan_triton._grid import get_num_stages
  assert get_num_stages(1) == 1
  assert get_num_stages(4, "fwd") == 1
  assert get_num_stages(8, "fwd") == 3
  assert get_num_stages(4, "bwd") == 2
  assert get_num_stages(8, "bwd") == 3


def test_public_api_surface():
  expected = {
    "op", "forward_scan_chunked", "forward_scan_onepass_pipelined", "forward_scan_full",
    "backward_scan_fused", "backward_scan_fused_single_chunk", "backward_scan_fused_full",
    "shift_pad", "shift_pad_compiled", "next_power_of_2", "get_grid", "get_static_grid",
    "scan_causal", "scan_causal_compiled", "scan_bidirectional_branched",
    "scan_bidirectional_branched_compiled",
  }
  assert set(ast.__all__) == expected
  assert ast.__version__ == "1.0.0"
  for name in expected:
    assert hasattr(ast, name)
  assert hasattr(ast, "get_num_stages")


def test_custom_ops_registered():
  ops = torch.ops.associative_scan_triton
  for name in ("scan_causal_fwd", "scan_causal_bwd", "scan_bidi_fwd", "scan_bidi_bwd",
               "shift_pad", "scan_causal_fwd_noclone", "scan_bidi_fwd_noclone"):
    assert hasattr(ops, name), name
  # the reference-named forward ops keep the reference's outputs: states + gates copies
  # (reference src/associative_scan_triton/scan_compiled.py:89-97, :208-218)
  assert len(ops.scan_causal_fwd.default._schema.returns) == 2
  assert len(ops.scan_bidi_fwd.default._schema.returns) == 4
  assert len(ops.scan_causal_fwd_noclone.default._schema.returns) == 1


def test_custom_ops_have_fake_kernels():
  # shape propagation works on meta tensors without touching a GPU
  from torch._subclasses.fake_tensor import FakeTensorMode
  with FakeTensorMode():
    g = torch.empty(3, 16, device="cuda")
    x = torch.empty(3, 16, device="cuda")
    cu = torch.empty(2, dtype=torch.int32, device="cuda")
    y, g_copy = torch.ops.associative_scan_triton.scan_causal_fwd(g, x, cu, 1, 3, 16)
    assert y.shape == g_copy.shape == (3, 16)
    y = torch.ops.associative_scan_triton.scan_causal_fwd_noclone(g, x, cu, 1, 3, 16)
    assert y.shape == (3, 16)
    dg, dx = torch.ops.associative_scan_triton.scan_causal_bwd(y, g, y, cu, 1, 3, 16)
    assert dg.shape == dx.shape == (3, 16)


def test_op_is_the_combine_operator():
  assert ast.op(2.0, 3.0, 0.5, 1.0) == (1.0, 2.5)


def test_kernel_launchers_are_indexable():
  launch = ast.forward_scan_chunked[(1, 1, 2)]
  assert callable(launch)
  assert "sm_100a" in repr(ast.backward_scan_fused)
