"""GPU: kernel-level launches and the dispatchers against known answers, the
reference's own golden outputs and the fp64 oracle.

Follows reference tests/test_scan_kernels.py: the same launch syntax
(``kernel[grid](...)``), the same hand-computed vectors, plus edge cases the
B200 tiling makes interesting (tile and row boundaries, misaligned views,
int32/int64 cu_seqlens, empty sequences, positions outside every sequence).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import (
  RTOL_F32, TEST_SEED, assert_close_to_gold, cu_of, golden_case_names, golden_cases,
  golden_tensor, in_sequence_mask, make_inputs, rtol_of,
)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _grid_from_cu(cu, chunk_size, C):
  lens = (cu[1:] - cu[:-1])
  return ast.get_grid(len(cu), int(lens.max().item()) if len(lens) else 0, chunk_size, C)


# --- known-answer vectors (reference tests/test_scan_kernels.py) ------------------------

@pytest.mark.parametrize("chunk_size", [4, 8, 16])
def test_fwd_chunk_numeric_single_chunks(chunk_size):
  # :130-170
  cu = torch.tensor([0, 4], device=DEV)
  grid = _grid_from_cu(cu, chunk_size, 1)
  gates = torch.tensor([1.0, 1.5, 0.8, 2.0], device=DEV)
  tokens = torch.tensor([1.0, -1.0, 0.5, 2.0], device=DEV)
  ast.forward_scan_chunked[grid](gates_ptr=gates, tokens_ptr=tokens, tokens_out_ptr=tokens,
                                 cu_seqlens_ptr=cu, REVERSE=False, CHUNK_SIZE=chunk_size,
                                 TESTING=True, INPLACE=True)
  assert torch.allclose(torch.tensor([1.0, 1.5, 1.2, 2.4], device=DEV), gates)
  assert torch.allclose(torch.tensor([1.0, 0.5, 0.9, 3.8], device=DEV), tokens)


@pytest.mark.parametrize("chunk_size", [4, 8, 16])
def test_fwd_chunk_numeric_single_chunks_reverse(chunk_size):
  # :183-222
  cu = torch.tensor([0, 4], device=DEV)
  grid = _grid_from_cu(cu, chunk_size, 1)
  gates = torch.tensor([1.0, 1.5, 0.8, 2.0], device=DEV)
  tokens = torch.tensor([1.0, -1.0, 0.5, 2.0], device=DEV)
  ast.forward_scan_chunked[grid](gates_ptr=gates, tokens_ptr=tokens, tokens_out_ptr=tokens,
                                 cu_seqlens_ptr=cu, REVERSE=True, CHUNK_SIZE=chunk_size,
                                 TESTING=True, INPLACE=True)
  assert torch.allclose(torch.tensor([2.4, 2.4, 1.6, 2.0], device=DEV), gates)
  assert torch.allclose(torch.tensor([3.15, 2.15, 2.1, 2.0], device=DEV), tokens)


@pytest.mark.parametrize("reverse", [False, True])
def test_fwd_multi_chunk_numeric(reverse):
  # :224-295
  cu = torch.tensor([0, 8], device=DEV)
  gates = torch.tensor([1.0, 1.5, 0.8, 2.0, 1.0, 1.5, 0.8, 2.0], device=DEV)
  tokens = torch.tensor([1.0, -1.0, 0.5, 2.0, 1.0, -1.0, 0.5, 2.0], device=DEV)
  grid = _grid_from_cu(cu, 4, 1)
  ast.forward_scan_full(gates, tokens, cu, grid, REVERSE=reverse, CHUNK_SIZE=4, TESTING=True)
  exp = ([10.71, 9.71, 7.14, 8.3, 3.15, 2.15, 2.1, 2.0] if reverse
         else [1.0, 0.5, 0.9, 3.8, 4.8, 6.2, 5.46, 12.92])
  assert torch.allclose(torch.tensor(exp, device=DEV), tokens)


@pytest.mark.parametrize(("seqlen", "chunk_size", "no_channels"),
                         [(4, 2, 2), (8, 4, 1), (8, 4, 2), (8, 4, 3), (8, 2, 1), (8, 2, 2),
                          (8, 2, 3), (16, 8, 2), (16, 4, 2), (16, 2, 2)])
@pytest.mark.parametrize("reverse", [False, True])
def test_one_vs_multiple_chunks(seqlen, chunk_size, no_channels, reverse):
  # :297-458 -- the reference compares without asserting; here it is asserted,
  # both against the single-chunk launch and against the oracle.
  torch.manual_seed(TEST_SEED)
  mult = 10
  gates = torch.rand(no_channels, seqlen * mult, device=DEV)
  tokens = torch.rand(no_channels, seqlen * mult, device=DEV)
  cu = torch.arange(mult + 1, device=DEV) * seqlen
  g1, x1 = gates.clone(), tokens.clone()
  ast.forward_scan_full(gates=g1, tokens=x1, cu_seqlens=cu, CHUNK_SIZE=chunk_size,
                        grid=_grid_from_cu(cu, chunk_size, no_channels), REVERSE=reverse)
  g2, x2 = gates.clone(), tokens.clone()
  ast.forward_scan_full(gates=g2, tokens=x2, cu_seqlens=cu, CHUNK_SIZE=seqlen,
                        grid=_grid_from_cu(cu, seqlen, no_channels), REVERSE=reverse)
  assert torch.allclose(g1, g2) and torch.allclose(x1, x2)
  y, a = oracle.scan_fwd(gates, tokens, cu, reverse=reverse)
  assert_close_to_gold(x1, y, torch.float32, "tokens")
  assert_close_to_gold(g1, a, torch.float32, "gate products")


@pytest.mark.parametrize("chunk_size", [2, 4, 8])
def test_copied_sequences(chunk_size):
  # :460-507
  cu = torch.tensor([0, 4, 8], device=DEV)
  gates = torch.tensor([1.0, 1.5, 0.8, 2.0] * 2, device=DEV)
  tokens = torch.tensor([1.0, -1.0, 0.5, 2.0] * 2, device=DEV)
  ast.forward_scan_full(gates=gates, tokens=tokens, cu_seqlens=cu, CHUNK_SIZE=chunk_size,
                        grid=_grid_from_cu(cu, chunk_size, 1), REVERSE=False, TESTING=True)
  assert torch.allclose(torch.tensor([1, 1.5, 1.2, 2.4] * 2, device=DEV), gates)
  assert torch.allclose(torch.tensor([1, 0.5, 0.9, 3.8] * 2, device=DEV), tokens)


@pytest.mark.parametrize("chunk_size", [2, 4, 8])
def test_multiple_varlen_sequences(chunk_size):
  # :509-563
  cu = torch.tensor([0, 4, 9], device=DEV)
  gates = torch.tensor([[1.0, 1.5, 0.8, 2.0, 0.3, 0.4, 0.9, 0.5, 0.45]], device=DEV)
  tokens = torch.tensor([[1.0, -1.0, 0.5, 2.0, 1.0, -0.7, 0.8, 0.6, 0.33]], device=DEV)
  ast.forward_scan_full(gates=gates, tokens=tokens, cu_seqlens=cu, CHUNK_SIZE=chunk_size,
                        grid=_grid_from_cu(cu, chunk_size, 1), REVERSE=False, TESTING=True)
  exp_g = torch.tensor([[1, 1.5, 1.2, 2.4, 0.3, 0.12, 0.108, 0.054, 0.0243]], device=DEV)
  exp_x = torch.tensor([[1.0, 0.5, 0.9, 3.8, 1.0, -0.3, 0.53, 0.865, 0.7192]], device=DEV)
  assert torch.allclose(exp_x, tokens, rtol=1e-4, atol=1e-7)
  assert torch.allclose(exp_g, gates, rtol=1e-4, atol=1e-7)


_VL_G = [[0.3, 0.4, 0.9, 0.5, 0.45, 1.0, 1.5, 0.8, 2.0],
         [0.3, 0.55, 0.96, 0.35, 0.7, 0.35, 0.85, 0.45, 1.3]]
_VL_X = [[1.0, -0.7, 0.8, 0.6, 0.33, 1.0, -1.0, 0.5, 2.0],
         [0.6, -0.75, 0.4, 0.65, 0.8, 1.0, -0.55, 0.65, 0.4]]


@pytest.mark.parametrize("chunk_size", [2, 4, 8])
@pytest.mark.parametrize("reverse", [False, True])
def test_varlen_sequences_and_channels(chunk_size, reverse):
  # :565-727
  cu = torch.tensor([0, 5, 9], device=DEV)
  gates = torch.tensor(_VL_G, device=DEV)
  tokens = torch.tensor(_VL_X, device=DEV)
  ast.forward_scan_full(gates=gates, tokens=tokens, cu_seqlens=cu,
                        grid=_grid_from_cu(cu, chunk_size, 2), CHUNK_SIZE=chunk_size,
                        REVERSE=reverse)
  if reverse:
    exp_g = [[0.0243, 0.081, 0.2025, 0.225, 0.45, 2.4, 2.4, 1.6, 2.0],
             [0.038808, 0.12936, 0.2352, 0.245, 0.7, 0.174038, 0.49725, 0.585, 1.3]]
    exp_x = [[0.96862, -0.1046, 1.4885, 0.765, 0.33, 3.15, 2.15, 2.1, 2.0],
             [0.588312, -0.03896, 1.2928, 0.93, 0.8, 1.054425, 0.1555, 0.83, 0.4]]
  else:
    exp_g = [[0.3, 0.12, 0.108, 0.054, 0.0243, 1.0, 1.5, 1.2, 2.4],
             [0.3, 0.165, 0.1584, 0.05544, 0.0388, 0.35, 0.2975, 0.1339, 0.174]]
    exp_x = [[1.0, -0.3, 0.53, 0.865, 0.71925, 1.0, 0.5, 0.9, 3.8],
             [0.60, -0.42, -0.0032, 0.6489, 1.25422, 1.0, 0.3, 0.7850, 1.4205]]
  assert torch.allclose(torch.tensor(exp_g, device=DEV), gates, rtol=1e-3, atol=1e-5)
  assert torch.allclose(torch.tensor(exp_x, device=DEV), tokens, rtol=1e-3, atol=1e-5)


def test_onepass_and_backward_launchers():
  # the remaining launcher objects, with the reference's keyword arguments
  g, x = make_inputs(3, 1000)
  cu = torch.tensor([0, 300, 301, 1000], device=DEV, dtype=torch.int32)
  y = torch.empty_like(x)
  ast.forward_scan_onepass_pipelined[(3, 3)](
    gates_ptr=g, tokens_ptr=x, tokens_out_ptr=y, cu_seqlens_ptr=cu, REVERSE=False,
    CHUNK_SIZE=256, NUM_CHUNKS=4, TESTING=False, NUM_STAGES=3, INPLACE=False)
  gold_y, _ = oracle.scan_fwd(g, x, cu)
  assert_close_to_gold(y, gold_y, torch.float32, "onepass y")
  dy = torch.randn_like(x)
  dx, dg = torch.empty_like(x), torch.empty_like(x)
  ast.backward_scan_fused[(3, 3)](grad_ptr=dy, gates_ptr=g, states_ptr=y, d_tokens_ptr=dx,
                                  d_gates_ptr=dg, cu_seqlens_ptr=cu, CHUNK_SIZE=256,
                                  NUM_CHUNKS=4, NUM_STAGES=3, CAUSAL=True)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=True)
  assert_close_to_gold(dx, gdx, torch.float32, "dx")
  assert_close_to_gold(dg, gdg, torch.float32, "dg")
  dx2, dg2 = torch.empty_like(x), torch.empty_like(x)
  ast.backward_scan_fused_single_chunk[(3, 1, 3)](
    grad_ptr=dy, gates_ptr=g, states_ptr=y, d_tokens_ptr=dx2, d_gates_ptr=dg2,
    cu_seqlens_ptr=cu, CHUNK_SIZE=1024, CAUSAL=True)
  assert torch.equal(dx, dx2) and torch.equal(dg, dg2)


# --- the reference's own outputs (tests/golden, made by running the reference) ---------

@pytest.mark.parametrize("case", golden_case_names("fwd"))
def test_forward_matches_reference_golden(case, impl):
  z, meta = golden_cases()
  m = meta[case]
  dtype = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[m["dtype"]]
  g = golden_tensor(z, case, "gates", dtype)
  x = golden_tensor(z, case, "tokens", dtype)
  cu = golden_tensor(z, case, "cu_seqlens")
  grid = ast.get_grid(len(cu), max(m["seqlens"]), m["chunk_size"], m["C"])
  # out of place, TESTING=False
  y = torch.empty_like(x)
  ast.forward_scan_full(g.clone(), x.clone(), cu, grid, REVERSE=m["reverse"],
                        CHUNK_SIZE=m["chunk_size"], TESTING=False, tokens_out=y)
  # in place, TESTING=True
  g_ip, x_ip = g.clone(), x.clone()
  ast.forward_scan_full(g_ip, x_ip, cu, grid, REVERSE=m["reverse"], CHUNK_SIZE=m["chunk_size"],
                        TESTING=True)
  assert torch.equal(y, x_ip)
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=m["reverse"])
  assert_close_to_gold(y, gold_y, dtype, f"{case} y vs oracle")
  assert_close_to_gold(g_ip, gold_a, dtype, f"{case} gate products vs oracle")
  # and against the reference's outputs, at the output dtype's resolution
  ref_y = z[f"{case}/y"].astype(np.float64)
  ref_a = z[f"{case}/gate_products"].astype(np.float64)
  tol = {torch.float32: 1e-5, torch.float16: 4e-3, torch.bfloat16: 3e-2}[dtype]
  assert_close_to_gold(y, ref_y, dtype, f"{case} y vs reference", rtol=tol)
  assert_close_to_gold(g_ip, ref_a, dtype, f"{case} gates vs reference", rtol=tol)


@pytest.mark.parametrize("case", golden_case_names("bwd"))
def test_backward_matches_reference_golden(case, impl):
  z, meta = golden_cases()
  m = meta[case]
  dtype = {"float32": torch.float32, "float16": torch.float16}[m["dtype"]]
  t = {k: golden_tensor(z, case, k, dtype) for k in ("gates", "grad", "states")}
  cu = golden_tensor(z, case, "cu_seqlens")
  grid = ast.get_grid(len(cu), max(m["seqlens"]), m["chunk_size"], m["C"])
  dx, dg = torch.empty_like(t["grad"]), torch.empty_like(t["grad"])
  ast.backward_scan_fused_full(t["grad"], t["gates"], t["states"], dx, dg, cu, grid,
                               CHUNK_SIZE=m["chunk_size"], CAUSAL=m["causal"])
  gdx, gdg = oracle.scan_bwd(t["grad"], t["gates"], t["states"], cu, causal=m["causal"])
  assert_close_to_gold(dx, gdx, dtype, f"{case} dx vs oracle")
  assert_close_to_gold(dg, gdg, dtype, f"{case} dg vs oracle")
  tol = {torch.float32: 1e-5, torch.float16: 4e-3}[dtype]
  assert_close_to_gold(dx, z[f"{case}/d_tokens"].astype(np.float64), dtype, "dx vs ref", rtol=tol)
  assert_close_to_gold(dg, z[f"{case}/d_gates"].astype(np.float64), dtype, "dg vs ref", rtol=tol)


# --- tiling edge cases against the oracle ---------------------------------------------

EDGE_CASES = [
  # C, seqlens
  (1, [1]),
  (1, [2]),
  (3, [1, 1, 1, 1, 1]),
  (5, [7, 3, 1, 9]),              # odd row length: rows start unaligned
  (2, [4095, 1, 4097]),           # sequences around the tile size
  (1, [4096 * 3]),                # one sequence over three tiles
  (1, [4096 * 40 + 17]),          # long chain of look-backs
  (7, [100, 5000, 13, 2048]),
  (33, [129]),                    # many short rows per tile
  (2, [512] * 24),
  (1, [0, 5, 0, 0, 9, 0]),        # empty sequences
  (300, [3, 2]),                  # rows of 5 elements, tile spans 800+ rows
  (3, [4096 * 5 + 31]),           # ragged tail shorter than one 128-byte row
  (1, [12345, 54321]),
  (2, [1] * 700 + [9000]),        # hundreds of heads in one tile
]


@pytest.mark.parametrize(("C", "seqlens"), EDGE_CASES)
@pytest.mark.parametrize("reverse", [False, True])
@pytest.mark.parametrize("cu_dtype", [torch.int32, torch.int64])
def test_forward_edge_cases(C, seqlens, reverse, cu_dtype, impl):
  BL = sum(seqlens)
  g, x = make_inputs(C, BL, gate="long", seed=C * 7 + BL)
  cu = cu_of(seqlens, dtype=cu_dtype)
  y = torch.full_like(x, float("nan"))
  gp = torch.full_like(x, float("nan"))
  ast.forward_scan_chunked[(len(seqlens), 1, C)](
    gates_ptr=g, tokens_ptr=x, tokens_out_ptr=y, cu_seqlens_ptr=cu, REVERSE=reverse,
    CHUNK_SIZE=2, TESTING=False, INPLACE=False)
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, torch.float32, "y")
  gcopy = g.clone()
  ast.forward_scan_full(gcopy, x.clone(), cu, (len(seqlens), 1, C), REVERSE=reverse,
                        CHUNK_SIZE=2, TESTING=True)
  assert_close_to_gold(gcopy, gold_a, torch.float32, "gate products")


@pytest.mark.parametrize(("C", "seqlens"), EDGE_CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_backward_edge_cases(C, seqlens, causal, impl):
  BL = sum(seqlens)
  g, x = make_inputs(C, BL, gate="long", seed=C * 11 + BL)
  dy = torch.randn_like(x)
  cu = cu_of(seqlens)
  gold_y, _ = oracle.scan_fwd(g, x, cu, reverse=not causal)
  h = torch.from_numpy(gold_y.astype(np.float32)).to(DEV)
  dx, dg = torch.empty_like(x), torch.empty_like(x)
  ast.backward_scan_fused_full(dy, g, h, dx, dg, cu, (len(seqlens), 1, C), CHUNK_SIZE=2,
                               CAUSAL=causal)
  gdx, gdg = oracle.scan_bwd(dy, g, h, cu, causal=causal)
  assert_close_to_gold(dx, gdx, torch.float32, "dx")
  assert_close_to_gold(dg, gdg, torch.float32, "dg")


@pytest.mark.parametrize("offset", [1, 2, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_misaligned_views(offset, dtype):
  # contiguous views that start off a 16-byte boundary take the scalar-load path
  C, BL = 3, 777
  base_g, base_x = make_inputs(1, C * BL + offset, dtype=dtype, gate="long")
  g = base_g.view(-1)[offset:].view(C, BL)
  x = base_x.view(-1)[offset:].view(C, BL)
  cu = cu_of([300, 477])
  y = torch.empty(C * BL + offset, dtype=dtype, device=DEV)[offset:].view(C, BL)
  ast.forward_scan_full(g, x, cu, (2, 1, C), REVERSE=False, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y)
  gold_y, _ = oracle.scan_fwd(g, x, cu)
  assert_close_to_gold(y, gold_y, dtype, "misaligned y")
  dy = torch.randn(C, BL, device=DEV).to(dtype)
  dx, dg = torch.empty_like(dy), torch.empty_like(dy)
  dx = torch.empty(C * BL + offset, dtype=dtype, device=DEV)[offset:].view(C, BL)
  ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (2, 1, C), CHUNK_SIZE=2, CAUSAL=True)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=True)
  assert_close_to_gold(dx, gdx, dtype, "misaligned dx")
  assert_close_to_gold(dg, gdg, dtype, "misaligned dg")


def test_positions_outside_sequences_are_untouched(impl):
  # cu[0] > 0: the head of every row belongs to no sequence (reference: masked)
  C, BL = 4, 5000
  g, x = make_inputs(C, BL)
  cu = torch.tensor([10, 2000, 5000], device=DEV)
  y = torch.full_like(x, 123.0)
  ast.forward_scan_full(g, x, cu, (2, 1, C), REVERSE=True, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y)
  assert (y[:, :10] == 123.0).all()
  gold_y, _ = oracle.scan_fwd(g, x, cu, reverse=True)
  mask = in_sequence_mask(C, BL, cu)
  assert_close_to_gold(y, gold_y, torch.float32, "y", mask=mask)


@pytest.mark.parametrize("reverse", [False, True])
def test_boundaries_are_bit_exact_and_isolated(reverse, impl):
  # the first element of a sequence (in scan order) is its token, bit for bit,
  # and nothing -- not even Inf/NaN -- leaks across a boundary
  C, seqlens = 5, [1000, 3000, 4096, 123, 9000]
  BL = sum(seqlens)
  g, x = make_inputs(C, BL, gate="long")
  cu = cu_of(seqlens)
  y1 = torch.empty_like(x)
  ast.forward_scan_full(g, x, cu, (5, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y1)
  starts = cu[:-1] if not reverse else cu[1:] - 1
  assert torch.equal(y1[:, starts], x[:, starts])
  # poison sequence 2 with Inf/NaN: the other sequences must not change at all
  g2, x2 = g.clone(), x.clone()
  s, e = int(cu[2]), int(cu[3])
  g2[:, s:e] = float("inf")
  x2[:, s + 5] = float("nan")
  y2 = torch.empty_like(x)
  ast.forward_scan_full(g2, x2, cu, (5, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y2)
  keep = torch.ones(BL, dtype=torch.bool, device=DEV)
  keep[s:e] = False
  assert torch.equal(y1[:, keep], y2[:, keep])


@pytest.mark.parametrize("causal", [True, False])
def test_backward_boundaries_exact(causal, impl):
  C, seqlens = 3, [700, 5000, 1]
  BL = sum(seqlens)
  g, x = make_inputs(C, BL)
  cu = cu_of(seqlens)
  y = torch.empty_like(x)
  ast.forward_scan_full(g, x, cu, (3, 1, C), REVERSE=not causal, CHUNK_SIZE=2, TESTING=False,
                        tokens_out=y)
  dy = torch.randn_like(x)
  dx, dg = torch.empty_like(x), torch.empty_like(x)
  ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (3, 1, C), CHUNK_SIZE=2, CAUSAL=causal)
  first = cu[1:] - 1 if causal else cu[:-1]     # first element of the adjoint scan
  last = cu[:-1] if causal else cu[1:] - 1      # its last element
  assert torch.equal(dx[:, first], dy[:, first])
  assert (dg[:, last] == 0).all()


def test_device_error_on_cu_mismatch():
  # reference tests/test_scan_kernels.py:45-83 launches with a cu_seqlens whose
  # total exceeds the tensor and reads out of bounds; here the kernel stays in
  # bounds and the mismatch is reported.
  g = torch.rand(8, device=DEV)
  x = torch.rand(8, device=DEV)
  cu = torch.cumsum(torch.tensor([0, 3, 5, 3, 8, 2]), 0).to(DEV)
  grid = _grid_from_cu(cu, 8, 2)
  with pytest.raises(ast.ScanError, match="cu_seqlens"):
    ast.forward_scan_chunked[grid](gates_ptr=g, tokens_ptr=x, tokens_out_ptr=x,
                                   cu_seqlens_ptr=cu, REVERSE=False, CHUNK_SIZE=8, TESTING=True,
                                   INPLACE=True)
  # the context stays usable and the error word was cleared
  y = torch.empty_like(x)
  ast.forward_scan_full(g, x, torch.tensor([0, 8], device=DEV), (1, 1, 1), REVERSE=False,
                        CHUNK_SIZE=8, TESTING=False, tokens_out=y)


def test_device_error_on_non_monotone_cu():
  g, x = make_inputs(2, 100)
  cu = torch.tensor([0, 60, 40, 100], device=DEV)
  y = torch.empty_like(x)
  with pytest.raises(ast.ScanError, match="monotone"):
    ast.forward_scan_full(g, x, cu, (3, 1, 2), REVERSE=False, CHUNK_SIZE=2, TESTING=False,
                          tokens_out=y)


def test_backward_refuses_aliased_outputs():
  g, x = make_inputs(2, 100)
  cu = torch.tensor([0, 100], device=DEV)
  with pytest.raises(ast.ScanError, match="invalid argument"):
    ast.backward_scan_fused_full(x, g, x, x.clone(), g, cu, (1, 1, 2), CHUNK_SIZE=2, CAUSAL=True)


def test_nonzero_stream_and_second_device_index():
  # work goes on torch's current stream
  g, x = make_inputs(4, 10000)
  cu = torch.tensor([0, 10000], device=DEV)
  s = torch.cuda.Stream()
  y = torch.empty_like(x)
  with torch.cuda.stream(s):
    ast.forward_scan_full(g, x, cu, (1, 1, 4), REVERSE=False, CHUNK_SIZE=2, TESTING=False,
                          tokens_out=y)
  s.synchronize()
  gold_y, _ = oracle.scan_fwd(g, x, cu)
  assert_close_to_gold(y, gold_y, torch.float32, "y on side stream")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
def test_both_kernel_families_agree(dtype, reverse):
  # the persistent TMA kernels and the plain kernels compute the same scan
  # (different association order, so compare both to the oracle and to each other)
  from associative_scan_triton import _lib
  seqlens = [5000, 77, 4096, 1, 20000, 333]
  C = 9
  BL = sum(seqlens)
  g, x = make_inputs(C, BL, dtype=dtype, gate="long")
  cu = cu_of(seqlens)
  outs = {}
  try:
    for name in ("tma", "simple"):
      _lib.set_implementation(name)
      y = torch.empty_like(x)
      gp = g.clone()
      ast.forward_scan_full(gp, x, cu, (len(seqlens), 1, C), REVERSE=reverse, CHUNK_SIZE=2,
                            TESTING=True, tokens_out=y)
      dy = torch.ones_like(x)
      dx, dg = torch.empty_like(x), torch.empty_like(x)
      ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (len(seqlens), 1, C), CHUNK_SIZE=2,
                                   CAUSAL=not reverse)
      outs[name] = (y, gp, dx, dg)
  finally:
    _lib.set_implementation("auto")
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=reverse)
  for name, (y, gp, dx, dg) in outs.items():
    assert_close_to_gold(y, gold_y, dtype, f"{name} y")
    assert_close_to_gold(gp, gold_a, dtype, f"{name} gate products")
    gdx, gdg = oracle.scan_bwd(torch.ones_like(x), g, outs["tma"][0], cu, causal=not reverse)
    assert_close_to_gold(dx, gdx, dtype, f"{name} dx")
  # the two families against each other, with the oracle tests' scale-aware bound
  for i in range(4):
    ref = outs["simple"][i].double().cpu().numpy()
    assert_close_to_gold(outs["tma"][i], ref, dtype, f"tma vs simple output {i}",
                         rtol=2 * rtol_of(dtype))


# --- tile orders of the persistent kernels ---------------------------------------------

TILE_ORDER_CASES = [
  # C, cu_seqlens -- every row a whole number of 4096-element tiles, so the
  # row order applies; 300 rows is the automatic choice on a 148-SM B200
  (300, [0, 8192]),
  (300, [0, 4096, 4173, 12288]),
  (5, [0, 4096 * 6]),                 # row order with fewer rows than CTAs
  (2, [100, 300, 12288]),             # positions before cu[0] lie in no sequence
  (7, [0, 1, 4097, 4098, 8192]),
  (160, [0, 4096 * 4]),
  # equal sequences of whole tiles: the segment order (one row per
  # (channel, sequence) pair)
  (160, [0, 16384, 32768, 49152]),
  # the same BL and S, but unequal sequences: the launch offers the segment
  # order and the kernels' cu_seqlens check turns it down
  (160, [0, 8192, 32768, 49152]),
  (3, [0, 16384, 32768, 40960, 49152]),
  (20, [0, 4096, 8192, 12288]),       # segments of one narrow tile each
]


@pytest.mark.parametrize("order", ["tma-row", "tma-flat"])
@pytest.mark.parametrize(("C", "cu_list"), TILE_ORDER_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
def test_tile_orders_match_oracle(order, C, cu_list, dtype, reverse):
  from associative_scan_triton import _lib
  BL = cu_list[-1]
  S = len(cu_list) - 1
  g, x = make_inputs(C, BL, dtype=dtype, gate="long", seed=C + BL + S)
  cu = torch.tensor(cu_list, dtype=torch.int64, device=DEV)
  mask = in_sequence_mask(C, BL, cu)
  dy = torch.randn(C, BL, generator=torch.Generator().manual_seed(5)).to(DEV, dtype)
  try:
    _lib.set_implementation(order)
    y = torch.full_like(x, 7.0)
    gp = g.clone()
    ast.forward_scan_full(gp, x, cu, (S, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=True,
                          tokens_out=y)
    dx, dg = torch.full_like(x, 7.0), torch.full_like(x, 7.0)
    ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (S, 1, C), CHUNK_SIZE=2,
                                 CAUSAL=not reverse)
    torch.cuda.synchronize()
  finally:
    _lib.set_implementation("auto")
  _lib.check_device_error()
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, dtype, f"{order} y", mask=mask)
  assert_close_to_gold(gp, gold_a, dtype, f"{order} gate products", mask=mask)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=not reverse)
  assert_close_to_gold(dx, gdx, dtype, f"{order} dx", mask=mask)
  assert_close_to_gold(dg, gdg, dtype, f"{order} dg", mask=mask)
  # positions outside every sequence are never written
  assert (y[:, ~mask[0]] == 7.0).all() and (dx[:, ~mask[0]] == 7.0).all()


@pytest.mark.parametrize("width", [16, 32])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
def test_segment_order_long_chains(width, dtype, reverse):
  """One rank's share of the 8-GPU headline split, scaled down: 192 rows of
  4 equal sequences of 32768 (segment order, a chain of 4 or 8 tiles per
  segment, 768 segments over the SMs), forward and fused backward against the
  oracle, and again with one sequence 4096 longer than the next, which the
  kernels must scan in the plain row order."""
  from associative_scan_triton import _lib
  C, S, T = 192, 4, 32768
  BL = S * T
  g, x = make_inputs(C, BL, dtype=dtype, gate="verylong", seed=77)
  dy = torch.randn(C, BL, generator=torch.Generator().manual_seed(8)).to(DEV, dtype)
  for cu_list in ([i * T for i in range(S + 1)], [0, T + 4096, 2 * T, 3 * T, 4 * T]):
    cu = torch.tensor(cu_list, dtype=torch.int32, device=DEV)
    try:
      _lib.set_tile_width(width)
      y = torch.empty_like(x)
      ast.forward_scan_full(g.clone(), x, cu, (S, 1, C), REVERSE=reverse, CHUNK_SIZE=2,
                            TESTING=True, tokens_out=y)
      dx, dg = torch.empty_like(x), torch.empty_like(x)
      ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (S, 1, C), CHUNK_SIZE=2,
                                   CAUSAL=not reverse)
      torch.cuda.synchronize()
    finally:
      _lib.set_tile_width(0)
    _lib.check_device_error()
    gold_y, _ = oracle.scan_fwd(g, x, cu, reverse=reverse)
    assert_close_to_gold(y, gold_y, dtype, f"segment order y, cu={cu_list}")
    gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=not reverse)
    assert_close_to_gold(dx, gdx, dtype, f"segment order dx, cu={cu_list}")
    assert_close_to_gold(dg, gdg, dtype, f"segment order dg, cu={cu_list}")


RAGGED_ROW_CASES = [
  # C, cu_seqlens -- rows that are not whole tiles: the row order cuts each
  # row into whole tiles and a partial last one, and tiles start anywhere
  # inside a 128-byte line
  (3, [0, 5000]),
  (7, [0, 4097]),                     # the array ends inside a 128-byte line
  (33, [0, 1, 5000, 9001]),
  (2, [100, 300, 12289]),             # positions before cu[0] lie in no sequence
  (1, [0, 70001]),                    # one long row: a chain of 18 tiles
  (200, [0, 4100]),                   # more tiles than CTAs, tiny last tiles
  (5, [0, 4096 * 2 + 31, 4096 * 3]),
]


@pytest.mark.parametrize(("C", "cu_list"), RAGGED_ROW_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
@pytest.mark.parametrize("inplace", [False, True])
def test_ragged_row_order_matches_oracle(C, cu_list, dtype, reverse, inplace):
  from associative_scan_triton import _lib
  BL = cu_list[-1]
  S = len(cu_list) - 1
  g, x = make_inputs(C, BL, dtype=dtype, gate="long", seed=C + BL + S)
  cu = torch.tensor(cu_list, dtype=torch.int32, device=DEV)
  mask = in_sequence_mask(C, BL, cu)
  dy = torch.randn(C, BL, generator=torch.Generator().manual_seed(6)).to(DEV, dtype)
  try:
    _lib.set_implementation("tma-row")
    y = x.clone() if inplace else torch.full_like(x, 7.0)
    gp = g.clone()
    ast.forward_scan_full(gp, y if inplace else x, cu, (S, 1, C), REVERSE=reverse,
                          CHUNK_SIZE=2, TESTING=True, tokens_out=y)
    dx, dg = torch.full_like(x, 7.0), torch.full_like(x, 7.0)
    ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (S, 1, C), CHUNK_SIZE=2,
                                 CAUSAL=not reverse)
    torch.cuda.synchronize()
  finally:
    _lib.set_implementation("auto")
  _lib.check_device_error()
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, dtype, "ragged rows y", mask=mask)
  assert_close_to_gold(gp, gold_a, dtype, "ragged rows gate products", mask=mask)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=not reverse)
  assert_close_to_gold(dx, gdx, dtype, "ragged rows dx", mask=mask)
  assert_close_to_gold(dg, gdg, dtype, "ragged rows dg", mask=mask)
  assert (dx[:, ~mask[0]] == 7.0).all() and (dg[:, ~mask[0]] == 7.0).all()
  if not inplace:
    assert (y[:, ~mask[0]] == 7.0).all()


@pytest.mark.parametrize("reverse", [False, True])
def test_flat_sized_workspace_is_accepted(reverse):
  """A caller that sized the workspace for the flat tile order (one status
  slot per 4096 elements) still gets correct results: the library then keeps
  the flat order instead of cutting ragged rows."""
  import ctypes

  from associative_scan_triton import _lib
  C, BL = 9, 5000
  g, x = make_inputs(C, BL, gate="long", seed=11)
  cu = torch.tensor([0, BL], dtype=torch.int64, device=DEV)
  f32 = _lib.DTYPE_CODES[torch.float32]
  flat_bytes = 256 + 16 * ((C * BL + 4095) // 4096)
  assert flat_bytes < _lib.load().ascan_workspace_size(C, BL, f32)
  ws = torch.empty(flat_bytes, dtype=torch.uint8, device=DEV)
  y = torch.empty_like(x)
  stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

  def call(nbytes):
    return _lib.load().ascan_forward(
      g.data_ptr(), x.data_ptr(), y.data_ptr(), None, cu.data_ptr(), _lib.INDEX_CODES[cu.dtype],
      1, C, BL, f32, int(reverse), ws.data_ptr(), nbytes, stream)

  try:
    _lib.set_implementation("tma-row")
    rc = call(flat_bytes)
    torch.cuda.synchronize()
  finally:
    _lib.set_implementation("auto")
  assert rc == 0, _lib.strerror(rc)
  _lib.check_device_error()
  gold_y, _ = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, torch.float32, "flat-sized workspace")
  assert call(flat_bytes - 1) == -2  # ASCAN_EWORKSPACE: one byte short of the flat size


LONG_MEMORY_CASES = [
  # C, cu_seqlens
  (300, [0, 4096 * 8]),                    # row order, more rows than CTAs
  (5, [0, 4096 * 24]),                     # row order, fewer rows than CTAs
  (3, [0, 16384, 32768, 49152]),           # segment order
  (2, [0, 100_003]),                       # ragged rows
  (40, [0, 3, 70_000, 70_001, 131_072]),   # boundaries inside
]


@pytest.mark.parametrize(("order", "width"), [
  ("simple", 0), ("tma", 16), ("tma", 32), ("tma-row", 16), ("tma-row", 32),
  ("tma-flat", 16), ("tma-flat", 32),
])
@pytest.mark.parametrize(("C", "cu_list"), LONG_MEMORY_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
def test_long_memory_gates(order, width, C, cu_list, dtype, reverse):
  """Gates of exactly 1 or 1 - 2^-8: a tile's gate product stays near 1, so
  every earlier tile of a sequence reaches its last element.  A carry put
  together from the wrong look-back records then shows on the whole tile;
  with gates below 0.99 a tile's product is under 1e-9 and such an error
  would only touch its first few elements."""
  from associative_scan_triton import _lib
  BL = cu_list[-1]
  S = len(cu_list) - 1
  g, x = make_inputs(C, BL, dtype=dtype, gate="nearone", seed=C + S)
  cu = torch.tensor(cu_list, dtype=torch.int64, device=DEV)
  dy = torch.randn(C, BL, generator=torch.Generator().manual_seed(9)).to(DEV, dtype)
  try:
    _lib.set_implementation(order)
    _lib.set_tile_width(width)
    y, gp = torch.empty_like(x), g.clone()
    ast.forward_scan_full(gp, x, cu, (S, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=True,
                          tokens_out=y)
    y2 = torch.empty_like(x)
    ast.forward_scan_full(g, x, cu, (S, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=False,
                          tokens_out=y2)
    dx, dg = torch.empty_like(x), torch.empty_like(x)
    ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (S, 1, C), CHUNK_SIZE=2,
                                 CAUSAL=not reverse)
    torch.cuda.synchronize()
  finally:
    _lib.set_tile_width(0)
    _lib.set_implementation("auto")
  _lib.check_device_error()
  gold_y, gold_a = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, dtype, f"{order}/{width} y (gate-product launch)")
  assert_close_to_gold(gp, gold_a, dtype, f"{order}/{width} gate products")
  assert_close_to_gold(y2, gold_y, dtype, f"{order}/{width} y")
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=not reverse)
  assert_close_to_gold(dx, gdx, dtype, f"{order}/{width} dx")
  assert_close_to_gold(dg, gdg, dtype, f"{order}/{width} dg")


WIDE_TILE_CASES = [
  # C, cu_seqlens: flat order, row order (aligned and ragged), look-back
  (64, [0, 8192 * 2]),
  (300, [0, 4096, 8192 * 2 + 5, 8192 * 3]),
  (5, [0, 8192 * 3 + 77]),
  (33, [0, 1, 5000, 9001, 30000]),
  (3, [0, 100]),
  (2, [100, 300, 16389]),
]


@pytest.mark.parametrize("order", ["tma", "tma-row", "tma-flat"])
@pytest.mark.parametrize(("C", "cu_list"), WIDE_TILE_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("reverse", [False, True])
def test_wide_tiles_match_oracle(order, C, cu_list, dtype, reverse):
  """8192-element tiles (32 elements per consumer thread), forced: the forward
  of every dtype and the 16-bit backward run them (the fp32 backward and the
  gate-product forward stay at 4096), against the oracle."""
  from associative_scan_triton import _lib
  BL = cu_list[-1]
  S = len(cu_list) - 1
  g, x = make_inputs(C, BL, dtype=dtype, gate="long", seed=C + BL + 7)
  cu = torch.tensor(cu_list, dtype=torch.int64, device=DEV)
  mask = in_sequence_mask(C, BL, cu)
  dy = torch.randn(C, BL, generator=torch.Generator().manual_seed(8)).to(DEV, dtype)
  try:
    _lib.set_implementation(order)
    _lib.set_tile_width(32)
    y = torch.full_like(x, 7.0)
    ast.forward_scan_full(g, x, cu, (S, 1, C), REVERSE=reverse, CHUNK_SIZE=2, TESTING=False,
                          tokens_out=y)
    dx, dg = torch.full_like(x, 7.0), torch.full_like(x, 7.0)
    ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, (S, 1, C), CHUNK_SIZE=2,
                                 CAUSAL=not reverse)
    torch.cuda.synchronize()
  finally:
    _lib.set_tile_width(0)
    _lib.set_implementation("auto")
  _lib.check_device_error()
  gold_y, _ = oracle.scan_fwd(g, x, cu, reverse=reverse)
  assert_close_to_gold(y, gold_y, dtype, "wide tiles y", mask=mask)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu, causal=not reverse)
  assert_close_to_gold(dx, gdx, dtype, "wide tiles dx", mask=mask)
  assert_close_to_gold(dg, gdg, dtype, "wide tiles dg", mask=mask)
  assert (y[:, ~mask[0]] == 7.0).all() and (dx[:, ~mask[0]] == 7.0).all()
