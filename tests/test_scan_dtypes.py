"""GPU: float32 / float16 / bfloat16 against the fp64 sequential gold label.

Reference tests/test_scan_dtypes.py compares against ``sequential_scan_gold``
with per-dtype tolerances; this build is held to the tighter tolerances of the
project goal (rtol 1e-5 for fp32, 2e-2 for fp16/bf16 with fp32 accumulation;
see scan_testlib.assert_close_to_gold) and also checks the backward values,
not only their finiteness.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import TEST_SEED, assert_close_to_gold

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(autouse=True)
def _seed():
  torch.manual_seed(TEST_SEED)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 128, 512, 1024, 8192])
@pytest.mark.parametrize("num_channels", [1, 4])
def test_forward_vs_gold(dtype, seqlen, num_channels):
  # reference tests/test_scan_dtypes.py:62-90
  chunk_size = min(seqlen, 512)
  gates = torch.rand(num_channels, seqlen, device=DEV).to(dtype)
  tokens = torch.randn(num_channels, seqlen, device=DEV).to(dtype)
  cu = torch.tensor([0, seqlen], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": chunk_size,
          "grid": ast.get_grid(2, seqlen, chunk_size, num_channels)}
  result = ast.scan_causal(gates.clone(), tokens.clone(), args)
  assert result.dtype == dtype
  gold, _ = oracle.scan_fwd(gates, tokens, cu)
  assert_close_to_gold(result, gold, dtype, f"forward {dtype} T={seqlen}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 128, 512, 1024, 8192])
def test_backward_vs_gold(dtype, seqlen):
  # reference tests/test_scan_dtypes.py:92-113 checks finiteness only
  num_channels = 4
  chunk_size = min(seqlen, 512)
  gates = torch.rand(num_channels, seqlen, device=DEV, dtype=dtype, requires_grad=True)
  tokens = torch.randn(num_channels, seqlen, device=DEV, dtype=dtype, requires_grad=True)
  dy = torch.randn(num_channels, seqlen, device=DEV, dtype=dtype)
  cu = torch.tensor([0, seqlen], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": chunk_size,
          "grid": ast.get_grid(2, seqlen, chunk_size, num_channels)}
  result = ast.scan_causal(gates, tokens, args)
  result.backward(dy)
  assert torch.isfinite(gates.grad).all() and torch.isfinite(tokens.grad).all()
  assert gates.grad.dtype == dtype and tokens.grad.dtype == dtype
  # gradients of sum(y * dy) at the given (rounded) inputs, states in fp64
  _y, gdx, gdg = oracle.scan_fwd_bwd(gates, tokens, dy, cu)
  assert_close_to_gold(tokens.grad, gdx, dtype, f"d_tokens {dtype}")
  # d_gates uses the stored (rounded) forward states, like the reference
  gdx2, gdg2 = oracle.scan_bwd(dy, gates, result, cu)
  assert_close_to_gold(gates.grad, gdg2, dtype, f"d_gates {dtype}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_multi_chunk_rmse(dtype):
  # reference tests/test_scan_dtypes.py:115-142 (RMSE bounds fp16 < 1e-3, bf16 < 5e-3)
  gates = torch.rand(4, 1024, device=DEV).to(dtype)
  tokens = torch.randn(4, 1024, device=DEV).to(dtype)
  cu = torch.tensor([0, 1024], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": 512, "grid": ast.get_grid(2, 1024, 512, 4)}
  result = ast.scan_causal(gates.clone(), tokens.clone(), args)
  gold, _ = oracle.scan_fwd(gates, tokens, cu)
  rmse = float(np.sqrt(np.mean((result.double().cpu().numpy() - gold) ** 2)))
  assert rmse < (1e-3 if dtype == torch.float16 else 5e-3), rmse


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [64, 256, 1024])
def test_bidi_forward_vs_gold(dtype, seqlen):
  # reference tests/test_scan_dtypes.py:148-189
  C = 4
  leaves = [torch.rand(C, seqlen, device=DEV, dtype=dtype),
            torch.randn(C, seqlen, device=DEV, dtype=dtype),
            torch.rand(C, seqlen, device=DEV, dtype=dtype),
            torch.randn(C, seqlen, device=DEV, dtype=dtype)]
  cu = torch.tensor([0, seqlen], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": min(seqlen, 512),
          "grid": ast.get_grid(2, seqlen, min(seqlen, 512), C)}
  yf, yb = ast.scan_bidirectional_branched(*[t.clone() for t in leaves], args)
  gf, _ = oracle.scan_fwd(leaves[0], leaves[1], cu)
  # flip / scan / flip, as the reference builds its reverse gold label
  gb_flip, _ = oracle.scan_fwd(leaves[2].flip(-1), leaves[3].flip(-1), cu)
  assert_close_to_gold(yf, gf, dtype, "bidi fwd")
  assert_close_to_gold(yb, gb_flip[:, ::-1].copy(), dtype, "bidi bwd")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("seqlen", [64, 512, 1024])
def test_bidi_backward_vs_gold(dtype, seqlen):
  # reference tests/test_scan_dtypes.py:191-215 checks finiteness only
  C = 4
  leaves = [torch.rand(C, seqlen, device=DEV, dtype=dtype, requires_grad=True),
            torch.randn(C, seqlen, device=DEV, dtype=dtype, requires_grad=True),
            torch.rand(C, seqlen, device=DEV, dtype=dtype, requires_grad=True),
            torch.randn(C, seqlen, device=DEV, dtype=dtype, requires_grad=True)]
  cu = torch.tensor([0, seqlen], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": min(seqlen, 512),
          "grid": ast.get_grid(2, seqlen, min(seqlen, 512), C)}
  yf, yb = ast.scan_bidirectional_branched(*leaves, args)
  (yf.sum() + yb.sum()).backward()
  for t in leaves:
    assert t.grad is not None and torch.isfinite(t.grad).all()
  ones = np.ones((C, seqlen))
  _, dxf, _ = oracle.scan_fwd_bwd(leaves[0], leaves[1], ones, cu, causal=True)
  _, dxb, _ = oracle.scan_fwd_bwd(leaves[2], leaves[3], ones, cu, causal=False)
  assert_close_to_gold(leaves[1].grad, dxf, dtype, "tokens grad fwd")
  assert_close_to_gold(leaves[3].grad, dxb, dtype, "tokens grad bwd")
  _, dgf = oracle.scan_bwd(ones, leaves[0], yf, cu, causal=True)
  _, dgb = oracle.scan_bwd(ones, leaves[2], yb, cu, causal=False)
  assert_close_to_gold(leaves[0].grad, dgf, dtype, "gates grad fwd")
  assert_close_to_gold(leaves[2].grad, dgb, dtype, "gates grad bwd")


@pytest.mark.parametrize("dtype", DTYPES)
def test_varlen_packed(dtype):
  # reference tests/test_scan_dtypes.py:221-256
  seqlens = [32, 64, 128]
  C, total = 2, sum(seqlens)
  gates = torch.rand(C, total, device=DEV, dtype=dtype)
  tokens = torch.randn(C, total, device=DEV, dtype=dtype)
  cu = torch.tensor([0, 32, 96, 224], device=DEV, dtype=torch.int32)
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": ast.get_grid(4, 128, 128, C)}
  result = ast.scan_causal(gates.clone(), tokens.clone(), args)
  for i, sl in enumerate(seqlens):
    s = sum(seqlens[:i])
    gold, _ = oracle.scan_fwd(gates[:, s:s + sl], tokens[:, s:s + sl], [0, sl])
    assert_close_to_gold(result[:, s:s + sl], gold, dtype, f"varlen seq {i}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_boundaries_exact(dtype):
  # the first element of every sequence is its token, bit for bit, in any dtype
  seqlens = [5000, 1, 3000, 8192]
  cu = torch.tensor([0, *np.cumsum(seqlens)], device=DEV)
  C, BL = 3, int(cu[-1])
  g = torch.rand(C, BL, device=DEV).to(dtype)
  x = torch.randn(C, BL, device=DEV).to(dtype)
  y = torch.empty_like(x)
  ast.forward_scan_full(g, x, cu, (4, 1, C), REVERSE=False, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y)
  assert torch.equal(y[:, cu[:-1]], x[:, cu[:-1]])
