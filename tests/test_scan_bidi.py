"""GPU: scan_bidirectional_branched -- reference tests/test_scan_bidi.py, with
the fp64 oracle in place of JAX."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import TEST_SEED, assert_close_to_gold, golden_cases, golden_tensor

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
