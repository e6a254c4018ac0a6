"""GPU: scan_bidirectional_branched -- reference tests/test_scan_bidi.py, with
the fp64 oracle in place of JAX."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import (
  TEST_SEED, assert_close_to_gold, golden_cases, golden_tensor, make_inputs,
)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(num_channels, seqlens, chunk_size, testing):
  torch.manual_seed(TEST_SEED)
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV)
  BL = int(cu[-1])
  leaves = [torch.rand(num_channels, BL, device=DEV, requires_grad=True) for _ in range(4)]
  grid = ast.get_grid(len(cu), max(seqlens), chunk_size, num_channels)
  args = {"cu_seqlens": cu, "chunk_size": chunk_size, "grid": grid}
  yf, yb = ast.scan_bidirectional_branched(*leaves, args, testing=testing)
  (yf.sum() + yb.sum()).backward()
  ones = np.ones((num_channels, BL))
  gf, xf, gb, xb = leaves
  oy_f, odx_f, odg_f = oracle.scan_fwd_bwd(gf, xf, ones, cu, causal=True)
  oy_b, odx_b, odg_b = oracle.scan_fwd_bwd(gb, xb, ones, cu, causal=False)
  assert_close_to_gold(yf, oy_f, torch.float32, "states fwd")
  assert_close_to_gold(yb, oy_b, torch.float32, "states bwd")
  assert_close_to_gold(gf.grad, odg_f, torch.float32, "gates grad fwd")
  assert_close_to_gold(xf.grad, odx_f, torch.float32, "tokens grad fwd")
  assert_close_to_gold(gb.grad, odg_b, torch.float32, "gates grad bwd")
  assert_close_to_gold(xb.grad, odx_b, torch.float32, "tokens grad bwd")


@pytest.mark.parametrize(
  ("chunk_size", "num_channels", "seqlen"),
  [(cs, c, t) for cs in [2**i for i in range(1, 9)] for c in (1, 2, 32) for t in (1, 5, 32, 128)],
)
def test_scan_bidirectional_branched(chunk_size, num_channels, seqlen):
  # reference tests/test_scan_bidi.py:21-124
  _run(num_channels, [seqlen], chunk_size, testing=True)


@pytest.mark.parametrize(
  ("chunk_size", "num_channels", "seqlen"),
  [(cs, c, t) for cs in [2**i for i in range(1, 9)] for c in (1, 2, 32) for t in (1, 5, 32, 128)
   if cs >= t],
)
def test_scan_bidirectional_branched_micro(chunk_size, num_channels, seqlen):
  # reference tests/test_scan_bidi.py:126-233 (testing=False)
  _run(num_channels, [seqlen], chunk_size, testing=False)


def test_bidi_varlen_packed():
  _run(16, [5000, 33, 1, 4096, 700], 512, testing=False)


@pytest.mark.parametrize("C", [8, 300])
def test_bidi_long_memory(C):
  """Both scans of the pair with gates of 1 or 1 - 2^-8 over sequences of many
  tiles: a tile's gate product stays near 1, so a wrong carry would show on
  whole tiles (row order for C = 300, flat order for C = 8)."""
  seqlens = [40_000, 4096 * 6, 777]
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV)
  BL = int(cu[-1])
  gf, xf = make_inputs(C, BL, gate="nearone", seed=C)
  gb, xb = make_inputs(C, BL, gate="nearone", seed=C + 1)
  leaves = [t.clone().requires_grad_(True) for t in (gf, xf, gb, xb)]
  args = {"cu_seqlens": cu, "chunk_size": 512,
          "grid": ast.get_grid(len(cu), max(seqlens), 512, C)}
  yf, yb = ast.scan_bidirectional_branched(*leaves, args)
  (yf.sum() + yb.sum()).backward()
  ones = np.ones((C, BL))
  oy_f, odx_f, odg_f = oracle.scan_fwd_bwd(gf, xf, ones, cu, causal=True)
  oy_b, odx_b, odg_b = oracle.scan_fwd_bwd(gb, xb, ones, cu, causal=False)
  assert_close_to_gold(yf, oy_f, torch.float32, "states fwd")
  assert_close_to_gold(yb, oy_b, torch.float32, "states bwd")
  assert_close_to_gold(leaves[0].grad, odg_f, torch.float32, "gates grad fwd")
  assert_close_to_gold(leaves[1].grad, odx_f, torch.float32, "tokens grad fwd")
  assert_close_to_gold(leaves[2].grad, odg_b, torch.float32, "gates grad bwd")
  assert_close_to_gold(leaves[3].grad, odx_b, torch.float32, "tokens grad bwd")


def test_bidi_matches_reference_golden():
  z, _ = golden_cases()
  c = "bidi_f32"
  names = ("gates_fwd", "tokens_fwd", "gates_bwd", "tokens_bwd")
  leaves = [golden_tensor(z, c, n).requires_grad_(True) for n in names]
  cu = golden_tensor(z, c, "cu_seqlens")
  args = {"cu_seqlens": cu, "chunk_size": 8, "grid": ast.get_grid(len(cu), 31, 8, 3)}
  yf, yb = ast.scan_bidirectional_branched(*leaves, args)
  dyf, dyb = golden_tensor(z, c, "grad_fwd"), golden_tensor(z, c, "grad_bwd")
  ((yf * dyf).sum() + (yb * dyb).sum()).backward()
  got = {"y_fwd": yf, "y_bwd": yb, "d_gates_fwd": leaves[0].grad, "d_tokens_fwd": leaves[1].grad,
         "d_gates_bwd": leaves[2].grad, "d_tokens_bwd": leaves[3].grad}
  for name, t in got.items():
    assert_close_to_gold(t, z[f"{c}/{name}"].astype(np.float64), torch.float32, name, rtol=2e-5)


BIDI_FUSED_CASES = [
  # C, seqlens
  (64, [2048] * 8),          # configs[3] geometry, fewer channels
  (33, [5000, 20000, 77]),   # look-back across tiles
  (7, [4097]),               # ragged rows (row order, partial last tiles)
  (300, [4096 * 3]),         # aligned row order
  (3, [100]),                # one tile
]


def _bidi_inputs(C, BL, dtype, seed):
  gen = torch.Generator().manual_seed(seed)
  ts = [torch.rand(C, BL, generator=gen) * 0.5 + 0.5 if k % 2 == 0 else torch.randn(C, BL, generator=gen)
        for k in range(6)]
  return [t.to(DEV, dtype) for t in ts]  # gf, xf, gb, xb, dyf, dyb


@pytest.mark.parametrize("width", [0, 16, 32])
@pytest.mark.parametrize("impl", ["auto", "tma-flat", "simple"])
@pytest.mark.parametrize(("C", "seqlens"), BIDI_FUSED_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_fused_bidi_launch_matches_two_launches(width, impl, C, seqlens, dtype):
  """One launch for both directions (ascan_forward_bidi / ascan_backward_bidi)
  against the two single-direction launches it replaces; bit for bit where no
  tile needs a look-back (the same arithmetic), else to float rounding."""
  from associative_scan_triton import _lib
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV, dtype=torch.int32)
  S, BL = len(seqlens), int(sum(seqlens))
  gf, xf, gb, xb, dyf, dyb = _bidi_inputs(C, BL, dtype, seed=C + BL)
  e = torch.empty_like
  try:
    _lib.set_implementation(impl)
    _lib.set_tile_width(width)
    yf, yb = e(xf), e(xb)
    _lib.forward_bidi(gf, xf, yf, gb, xb, yb, cu, S, C)
    d = [e(xf) for _ in range(4)]
    _lib.backward_bidi(dyf, gf, yf, d[0], d[1], dyb, gb, yb, d[2], d[3], cu, S, C)
    yf2, yb2 = e(xf), e(xb)
    _lib.forward(gf, xf, yf2, None, cu, S, C, False)
    _lib.forward(gb, xb, yb2, None, cu, S, C, True)
    d2 = [e(xf) for _ in range(4)]
    _lib.backward(dyf, gf, yf2, d2[0], d2[1], cu, S, C, True)
    _lib.backward(dyb, gb, yb2, d2[2], d2[3], cu, S, C, False)
    torch.cuda.synchronize()
  finally:
    _lib.set_tile_width(0)
    _lib.set_implementation("auto")
  _lib.check_device_error()
  got, want = [yf, yb, *d], [yf2, yb2, *d2]
  if all(L <= 4096 and 4096 % L == 0 for L in seqlens):
    for k, (a, b) in enumerate(zip(got, want)):
      assert torch.equal(a, b), k
  else:
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    for a, b in zip(got, want):
      torch.testing.assert_close(a.float(), b.float(), rtol=tol, atol=tol)
  # and against the oracle, through the reference-facing API
  oy_f, odx_f, odg_f = oracle.scan_fwd_bwd(gf, xf, dyf, cu, causal=True)
  oy_b, odx_b, odg_b = oracle.scan_fwd_bwd(gb, xb, dyb, cu, causal=False)
  for t, gold, name in ((yf, oy_f, "y fwd"), (yb, oy_b, "y bwd"), (d[0], odx_f, "dx fwd"),
                        (d[1], odg_f, "dg fwd"), (d[2], odx_b, "dx bwd"), (d[3], odg_b, "dg bwd")):
    assert_close_to_gold(t, gold, dtype, name)


def test_fused_bidi_graph_replay():
  """The fused launches are stream operations like the single ones: a CUDA
  graph of one bidirectional fwd+bwd step replays to the eager result."""
  from associative_scan_triton import _lib
  C, seqlens = 96, [2048] * 4
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV, dtype=torch.int32)
  S, BL = len(seqlens), int(sum(seqlens))
  ins = _bidi_inputs(C, BL, torch.float32, seed=3)
  gf, xf, gb, xb, dyf, dyb = ins
  outs = [torch.empty_like(xf) for _ in range(6)]

  def step():
    _lib.forward_bidi(gf, xf, outs[0], gb, xb, outs[1], cu, S, C)
    _lib.backward_bidi(dyf, gf, outs[0], outs[2], outs[3], dyb, gb, outs[1], outs[4], outs[5],
                       cu, S, C)

  was = _lib.sync_check_enabled()
  _lib.set_sync_check(False)
  try:
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
      for _ in range(2):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
      step()
    fresh = _bidi_inputs(C, BL, torch.float32, seed=4)
    for t, f in zip(ins, fresh):
      t.copy_(f)
    graph.replay()
    torch.cuda.synchronize()
    replayed = [o.clone() for o in outs]
    step()
    torch.cuda.synchronize()
    for a, b in zip(replayed, outs):
      assert torch.equal(a, b)
    del graph
  finally:
    _lib.set_sync_check(was)
  _lib.check_device_error()
