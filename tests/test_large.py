"""GPU: the benchmark configurations at full size.

The kernels run on the full tensors; the fp64 oracle checks a seeded sample of
channels (every channel is an independent row, so a sample is a faithful
check), and size-independent properties (linearity in the tokens, the
reverse scan as flip / scan / flip) cover the whole tensor.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import assert_close_to_gold

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
DEV = "cuda"


def _data(C, BL, dtype, gate, seed):
  gen = torch.Generator(device=DEV).manual_seed(seed)
  if gate == "long":
    g = 0.9 + 0.1 * torch.rand(C, BL, device=DEV, generator=gen)
  elif gate == "verylong":
    g = 0.99 + 0.01 * torch.rand(C, BL, device=DEV, generator=gen)
  elif gate == "sigmoid":
    g = torch.sigmoid(2.0 + torch.randn(C, BL, device=DEV, generator=gen))
  else:
    g = torch.rand(C, BL, device=DEV, generator=gen)
  x = torch.randn(C, BL, device=DEV, generator=gen)
  dy = torch.randn(C, BL, device=DEV, generator=gen)
  return g.to(dtype), x.to(dtype), dy.to(dtype)


def _check_rows(rows, g, x, dy, y, dx, dg, cu, dtype, causal=True, tag=""):
  cu_h = cu.cpu()
  for r in rows:
    sl = slice(int(r), int(r) + 1)
    gy, gdx, _ = oracle.scan_fwd_bwd(g[sl], x[sl], dy[sl], cu_h, causal=causal)
    _, gdg = oracle.scan_bwd(dy[sl], g[sl], y[sl], cu_h, causal=causal)
    assert_close_to_gold(y[sl], gy, dtype, f"{tag} y row {r}")
    assert_close_to_gold(dx[sl], gdx, dtype, f"{tag} dx row {r}")
    assert_close_to_gold(dg[sl], gdg, dtype, f"{tag} dg row {r}")


def _run(g, x, dy, cu, causal=True):
  C = g.shape[0]
  grid = (len(cu) - 1, 1, C)
  y = torch.empty_like(x)
  ast.forward_scan_full(g, x, cu, grid, REVERSE=not causal, CHUNK_SIZE=512, TESTING=False,
                        tokens_out=y)
  dx, dg = torch.empty_like(x), torch.empty_like(x)
  ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, grid, CHUNK_SIZE=512, CAUSAL=causal)
  return y, dx, dg


def test_config2_packed_causal():
  # B=8 x T=4096 packed, C=1536, fp32, gates U(0.9, 1)
  C, B, T = 1536, 8, 4096
  cu = torch.arange(B + 1, device=DEV, dtype=torch.int32) * T
  g, x, dy = _data(C, B * T, torch.float32, "long", 2)
  y, dx, dg = _run(g, x, dy, cu)
  rows = np.random.default_rng(2).choice(C, 12, replace=False)
  _check_rows(rows, g, x, dy, y, dx, dg, cu, torch.float32, tag="config2")
  # linearity over the whole tensor: scan(g, 2x + dy) == 2 scan(g, x) + scan(g, dy)
  y2 = torch.empty_like(x)
  y3 = torch.empty_like(x)
  grid = (B, 1, C)
  ast.forward_scan_full(g, 2 * x + dy, cu, grid, REVERSE=False, CHUNK_SIZE=512, TESTING=False,
                        tokens_out=y2)
  ast.forward_scan_full(g, dy, cu, grid, REVERSE=False, CHUNK_SIZE=512, TESTING=False,
                        tokens_out=y3)
  lin = 2 * y + y3
  scale = lin.square().mean().sqrt()
  assert ((y2 - lin).abs() <= 1e-5 * (lin.abs() + scale) + 1e-6).all()


def test_config3_varlen_bf16():
  # C=2048, 32 lengths U[64, 8192] (seed 0), bf16 in / fp32 accumulate, sigmoid(N(2,1)) gates
  gen = torch.Generator().manual_seed(0)
  lens = torch.randint(64, 8193, (32,), generator=gen)
  cu = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)]).to(DEV)
  C, BL = 2048, int(cu[-1])
  g, x, dy = _data(C, BL, torch.bfloat16, "sigmoid", 3)
  y, dx, dg = _run(g, x, dy, cu)
  rows = np.random.default_rng(3).choice(C, 8, replace=False)
  _check_rows(rows, g, x, dy, y, dx, dg, cu, torch.bfloat16, tag="config3")


def test_config4_bidi_fp16():
  # B=8, C=1536, T=2048, fp16, independent pairs per direction
  C, B, T = 1536, 8, 2048
  cu = torch.arange(B + 1, device=DEV, dtype=torch.int32) * T
  gf, xf, dyf = _data(C, B * T, torch.float16, "uniform", 4)
  gb, xb, dyb = _data(C, B * T, torch.float16, "uniform", 5)
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": ast.get_grid(B + 1, T, 128, C)}
  leaves = [t.clone().requires_grad_(True) for t in (gf, xf, gb, xb)]
  yf, yb = ast.scan_bidirectional_branched(*leaves, args)
  torch.autograd.backward([yf, yb], [dyf, dyb])
  rows = np.random.default_rng(4).choice(C, 6, replace=False)
  _check_rows(rows, gf, xf, dyf, yf.detach(), leaves[1].grad, leaves[0].grad, cu, torch.float16,
              causal=True, tag="bidi fwd")
  _check_rows(rows, gb, xb, dyb, yb.detach(), leaves[3].grad, leaves[2].grad, cu, torch.float16,
              causal=False, tag="bidi bwd")


def test_config5a_long_sequences():
  # B=8, C=1536, T=65536, fp32: 16 tiles per sequence, every tile but the first looks back
  C, B, T = 1536, 8, 65536
  cu = torch.arange(B + 1, device=DEV, dtype=torch.int64) * T
  g, x, dy = _data(C, B * T, torch.float32, "long", 5)
  y, dx, dg = _run(g, x, dy, cu)
  rows = np.random.default_rng(5).choice(C, 3, replace=False)
  _check_rows(rows, g, x, dy, y, dx, dg, cu, torch.float32, tag="config5a")


def test_config5b_single_long_sequence_and_reverse_symmetry():
  # C=256, one sequence of 2^20, gates U(0.99, 1): 256 tiles per row in one chain
  C, T = 256, 1 << 20
  cu = torch.tensor([0, T], device=DEV)
  g, x, dy = _data(C, T, torch.float32, "verylong", 6)
  y, dx, dg = _run(g, x, dy, cu)
  rows = np.random.default_rng(6).choice(C, 2, replace=False)
  _check_rows(rows, g, x, dy, y, dx, dg, cu, torch.float32, tag="config5b")
  # reverse scan of the flipped input equals the flipped forward scan
  yr = torch.empty_like(x)
  ast.forward_scan_full(g.flip(-1).contiguous(), x.flip(-1).contiguous(), cu, (1, 1, C),
                        REVERSE=True, CHUNK_SIZE=512, TESTING=False, tokens_out=yr)
  torch.testing.assert_close(yr.flip(-1), y, rtol=1e-5, atol=1e-4)
