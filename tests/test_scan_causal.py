"""GPU: scan_causal (autograd) -- reference tests/test_scan_causal.py.

The reference compares against JAX's associative_scan; JAX is not part of this
build, so the fp64 sequential oracle (oracle/) takes its place with the same
sweep of chunk sizes, channel counts and lengths.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import TEST_SEED, assert_close_to_gold, golden_cases, golden_tensor

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("chunk_size", [2, 4, 8])
def test_causal_scan_known_answer(chunk_size):
  # reference tests/test_scan_causal.py:33-71
  torch.manual_seed(TEST_SEED)
  seqlens = torch.tensor([4, 4])
  cu = torch.cat((torch.tensor([0]), seqlens.cumsum(dim=0))).to(DEV)
  grid = ast.get_grid(len(cu), 4, chunk_size, 1)
  gates = torch.tensor([[1.0, 1.5, 0.8, 2.0, 1.0, 1.5, 0.8, 2.0]], device=DEV,
                       requires_grad=True)
  tokens = torch.tensor([[1.0, -1.0, 0.5, 2.0, 1.0, -1.0, 0.5, 2.0]], device=DEV,
                        requires_grad=True)
  args = {"cu_seqlens": cu, "chunk_size": chunk_size, "grid": grid}
  result = ast.scan_causal(gates, tokens, args)
  assert torch.allclose(result, torch.tensor([[1, 0.5, 0.9, 3.8] * 2], device=DEV),
                        rtol=1e-4, atol=1e-4)
  result.sum().backward()
  assert torch.allclose(gates.grad, torch.tensor([[0.0, 3.4, 1.5, 0.9] * 2], device=DEV),
                        rtol=1e-4, atol=1e-4)
  assert torch.allclose(tokens.grad, torch.tensor([[6.1, 3.4, 3.0, 1.0] * 2], device=DEV),
                        rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize(
  ("chunk_size", "num_channels", "seqlen"),
  [(cs, c, t) for cs in [2**i for i in range(1, 9)] for c in (1, 2, 32) for t in (1, 5, 32, 128)],
)
def test_scan_causal_vs_oracle(chunk_size, num_channels, seqlen):
  # reference tests/test_scan_causal.py:75-136, JAX replaced by the fp64 oracle
  torch.manual_seed(TEST_SEED)
  cu = torch.tensor([0, seqlen], device=DEV)
  grid = ast.get_grid(len(cu), seqlen, chunk_size, num_channels)
  gates = torch.rand(num_channels, seqlen, device=DEV).requires_grad_(True)
  tokens = torch.randn(num_channels, seqlen, device=DEV).requires_grad_(True)
  args = {"cu_seqlens": cu, "chunk_size": chunk_size, "grid": grid}
  result = ast.scan_causal(gates, tokens, args)
  result.sum().backward()
  y, dx, dg = oracle.scan_fwd_bwd(gates, tokens, np.ones((num_channels, seqlen)), cu)
  assert_close_to_gold(result, y, torch.float32, "y")
  assert_close_to_gold(gates.grad, dg, torch.float32, "d_gates")
  assert_close_to_gold(tokens.grad, dx, torch.float32, "d_tokens")


def test_config0_matches_reference_golden():
  # C=4, T=128, one sequence, seed 0 -- outputs of the reference itself
  z, _ = golden_cases()
  c = "config0_scan_causal"
  g = golden_tensor(z, c, "gates").requires_grad_(True)
  x = golden_tensor(z, c, "tokens").requires_grad_(True)
  cu = golden_tensor(z, c, "cu_seqlens")
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": ast.get_grid(2, 128, 128, 4)}
  y = ast.scan_causal(g, x, args)
  y.sum().backward()
  for ours, name in ((y, "y"), (g.grad, "d_gates"), (x.grad, "d_tokens")):
    ref = z[f"{c}/{name}"].astype(np.float64)
    assert_close_to_gold(ours, ref, torch.float32, name, rtol=2e-5)
  gy, gdx, gdg = oracle.scan_fwd_bwd(g, x, np.ones((4, 128)), cu)
  assert_close_to_gold(y, gy, torch.float32, "y vs oracle")
  assert_close_to_gold(g.grad, gdg, torch.float32, "dg vs oracle")
  assert_close_to_gold(x.grad, gdx, torch.float32, "dx vs oracle")


@pytest.mark.parametrize("seqlens", [[4096] * 8, [300, 9000, 1, 77, 4096, 12000]])
def test_scan_causal_packed_batches(seqlens):
  C = 64
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV, dtype=torch.int32)
  BL = int(cu[-1])
  grid = ast.get_grid(len(cu), max(seqlens), 512, C)
  gen = torch.Generator(device="cpu").manual_seed(3)
  g = (0.9 + 0.1 * torch.rand(C, BL, generator=gen)).to(DEV).requires_grad_(True)
  x = torch.randn(C, BL, generator=gen).to(DEV).requires_grad_(True)
  dy = torch.randn(C, BL, generator=gen).to(DEV)
  y = ast.scan_causal(g, x, {"cu_seqlens": cu, "chunk_size": 512, "grid": grid})
  y.backward(dy)
  gy, gdx, gdg = oracle.scan_fwd_bwd(g, x, dy, cu)
  assert_close_to_gold(y, gy, torch.float32, "y")
  assert_close_to_gold(x.grad, gdx, torch.float32, "dx")
  assert_close_to_gold(g.grad, gdg, torch.float32, "dg")


def test_scan_causal_no_grad_saves_nothing():
  g = torch.rand(2, 50, device=DEV)
  x = torch.rand(2, 50, device=DEV)
  y = ast.scan_causal(g, x, {"cu_seqlens": torch.tensor([0, 50], device=DEV), "chunk_size": 64,
                             "grid": (1, 1, 2)})
  assert not y.requires_grad
