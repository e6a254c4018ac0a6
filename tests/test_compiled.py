"""GPU: the torch.compile-safe custom ops -- reference tests/test_compiled.py,
plus a fullgraph torch.compile run through them."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import TEST_SEED, assert_close_to_gold

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _seed():
  torch.manual_seed(TEST_SEED)


def _cu(batch, seq_len):
  cu = torch.zeros(batch + 1, device=DEV, dtype=torch.int32)
  cu[1:] = torch.full((batch,), seq_len, device=DEV, dtype=torch.int32).cumsum(0)
  return cu


@pytest.mark.parametrize("batch_size", [1, 4])
@pytest.mark.parametrize("seq_len", [64, 256])
def test_scan_matches_original(batch_size, seq_len):
  # reference tests/test_compiled.py:49-89
  C = 64
  cu = _cu(batch_size, seq_len)
  total = int(cu[-1])
  grid = ast.get_grid(len(cu), seq_len, 128, C)
  t = [torch.rand(C, total, device=DEV), torch.randn(C, total, device=DEV),
       torch.rand(C, total, device=DEV), torch.randn(C, total, device=DEV)]
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": grid}
  ref_fwd, ref_bwd = ast.scan_bidirectional_branched(*[x.clone() for x in t], args)
  test_fwd, test_bwd = ast.scan_bidirectional_branched_compiled(*[x.clone() for x in t], args)
  torch.testing.assert_close(ref_fwd, test_fwd, rtol=0, atol=0)
  torch.testing.assert_close(ref_bwd, test_bwd, rtol=0, atol=0)


@pytest.mark.parametrize("backward", [True, False])
@pytest.mark.parametrize("pad_value", [0.0, 1.0])
def test_shift_pad_matches_original(backward, pad_value):
  # reference tests/test_compiled.py:91-104
  cu = _cu(4, 64)
  data = torch.randn(64, 256, device=DEV)
  ref = ast.shift_pad(data, cu, pad_value=pad_value, backward=backward)
  test = ast.shift_pad_compiled(data, cu, pad_value=pad_value, backward=backward)
  torch.testing.assert_close(ref, test, rtol=0, atol=0)


def test_compiled_autograd_matches_eager():
  C, cu = 32, _cu(3, 1000)
  total = int(cu[-1])
  args = {"cu_seqlens": cu, "chunk_size": 512, "grid": ast.get_grid(len(cu), 1000, 512, C)}
  base = [torch.rand(C, total, device=DEV), torch.randn(C, total, device=DEV)]
  dy = torch.randn(C, total, device=DEV)
  a = [t.clone().requires_grad_(True) for t in base]
  b = [t.clone().requires_grad_(True) for t in base]
  ast.scan_causal(*a, args).backward(dy)
  ast.scan_causal_compiled(*b, args).backward(dy)
  for x, y in zip(a, b):
    torch.testing.assert_close(x.grad, y.grad, rtol=0, atol=0)
  # bidi compiled autograd
  four = [torch.rand(C, total, device=DEV) for _ in range(4)]
  la = [t.clone().requires_grad_(True) for t in four]
  lb = [t.clone().requires_grad_(True) for t in four]
  fa, ba = ast.scan_bidirectional_branched(*la, args)
  (fa * dy).sum().add_((ba * dy).sum()).backward()
  fb, bb = ast.scan_bidirectional_branched_compiled(*lb, args)
  (fb * dy).sum().add_((bb * dy).sum()).backward()
  for x, y in zip(la, lb):
    torch.testing.assert_close(x.grad, y.grad, rtol=0, atol=0)


def test_torch_compile_fullgraph():
  C, cu = 16, _cu(2, 300)
  total = int(cu[-1])
  args = {"cu_seqlens": cu, "chunk_size": 512, "grid": ast.get_grid(len(cu), 300, 512, C)}
  w = torch.randn(C, 1, device=DEV)

  def model(g, x):
    y = ast.scan_causal_compiled(torch.sigmoid(g), x * w, args)
    return (y * y).sum()

  compiled = torch.compile(model, fullgraph=True)
  g0 = torch.randn(C, total, device=DEV)
  x0 = torch.randn(C, total, device=DEV)
  ge, xe = g0.clone().requires_grad_(True), x0.clone().requires_grad_(True)
  gc_, xc = g0.clone().requires_grad_(True), x0.clone().requires_grad_(True)
  le = model(ge, xe)
  le.backward()
  lc = compiled(gc_, xc)
  lc.backward()
  torch.testing.assert_close(le, lc, rtol=1e-5, atol=1e-4)
  torch.testing.assert_close(ge.grad, gc_.grad, rtol=1e-5, atol=1e-5)
  torch.testing.assert_close(xe.grad, xc.grad, rtol=1e-5, atol=1e-5)


def test_compiled_causal_vs_oracle():
  C, seqlens = 8, [100, 4096, 1, 4500]
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV)
  total = int(cu[-1])
  g = torch.rand(C, total, device=DEV, requires_grad=True)
  x = torch.randn(C, total, device=DEV, requires_grad=True)
  dy = torch.randn(C, total, device=DEV)
  y = ast.scan_causal_compiled(g, x, {"cu_seqlens": cu, "chunk_size": 512,
                                      "grid": ast.get_grid(len(cu), 4500, 512, C)})
  y.backward(dy)
  gy, gdx, gdg = oracle.scan_fwd_bwd(g, x, dy, cu)
  assert_close_to_gold(y, gy, torch.float32, "y")
  assert_close_to_gold(x.grad, gdx, torch.float32, "dx")
  assert_close_to_gold(g.grad, gdg, torch.float32, "dg")


def test_reference_named_ops_keep_the_reference_schema():
  """torch.ops.associative_scan_triton.scan_causal_fwd / scan_bidi_fwd return
  what the reference's triton_ops return (reference
  src/associative_scan_triton/scan_compiled.py:89-113, :208-240): the states
  plus a copy of the gates, and gradients flow to gates and tokens."""
  C, cu = 16, _cu(2, 300)
  total = int(cu[-1])
  grid = ast.get_grid(len(cu), 300, 128, C)
  g = torch.rand(C, total, device=DEV, requires_grad=True)
  x = torch.randn(C, total, device=DEV, requires_grad=True)
  y, g_copy = torch.ops.associative_scan_triton.scan_causal_fwd(g, x, cu, grid[1], C, 128)
  assert torch.equal(g_copy, g.detach()) and g_copy.data_ptr() != g.data_ptr()
  gold, _ = oracle.scan_fwd(g, x, cu)
  assert_close_to_gold(y, gold, torch.float32, "scan_causal_fwd states")
  y.sum().backward()
  want_dg, want_dx = g.grad.clone(), x.grad.clone()
  g.grad = x.grad = None
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": grid}
  ast.scan_causal_compiled(g, x, args).sum().backward()
  torch.testing.assert_close(g.grad, want_dg, rtol=0, atol=0)
  torch.testing.assert_close(x.grad, want_dx, rtol=0, atol=0)
  t = [torch.rand(C, total, device=DEV), torch.randn(C, total, device=DEV),
       torch.rand(C, total, device=DEV), torch.randn(C, total, device=DEV)]
  outs = torch.ops.associative_scan_triton.scan_bidi_fwd(*t, cu, grid[1], C, 128)
  assert len(outs) == 4
  assert torch.equal(outs[2], t[0]) and torch.equal(outs[3], t[2])
  ref_fwd, ref_bwd = ast.scan_bidirectional_branched_compiled(*t, args)
  torch.testing.assert_close(outs[0], ref_fwd, rtol=0, atol=0)
  torch.testing.assert_close(outs[1], ref_bwd, rtol=0, atol=0)
