"""GPU: shift_pad -- reference tests/test_shift_pad.py (run on CUDA tensors)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import associative_scan_triton as ast
from oracle import oracle
from scan_testlib import golden_case_names, golden_cases, golden_tensor

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(params=[True, False])
def backward(request):
  return request.param


@pytest.fixture(params=[-1])
def pad_value(request):
  return request.param


def test_shift_pad_single_sequence(backward, pad_value):
  data = torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0]], device=DEV)
  result = ast.shift_pad(data, torch.tensor([0, 5], device=DEV), pad_value, backward)
  exp = [[pad_value, 1.0, 2.0, 3.0, 4.0]] if backward else [[2.0, 3.0, 4.0, 5.0, pad_value]]
  assert torch.allclose(result, torch.tensor(exp, device=DEV))


def test_shift_pad_multiple_sequences(backward, pad_value):
  data = torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0]], device=DEV)
  result = ast.shift_pad(data, torch.tensor([0, 3, 7], device=DEV), pad_value, backward)
  exp = ([[pad_value, 1.0, 2.0, pad_value, 4.0, 5.0, 6.0]] if backward
         else [[2.0, 3.0, pad_value, 5.0, 6.0, 7.0, pad_value]])
  assert torch.allclose(result, torch.tensor(exp, device=DEV))


def test_shift_pad_multi_dimensional(backward, pad_value):
  data = torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 0.0],
                       [7.0, 8.0, 9.0, 10.0, 11.0, 12.0, 0.0]], device=DEV)
  result = ast.shift_pad(data, torch.tensor([0, 2, 4, 7], device=DEV), pad_value, backward)
  p = pad_value
  exp = ([[p, 1.0, p, 3.0, p, 5.0, 6.0], [p, 7.0, p, 9.0, p, 11.0, 12.0]] if backward
         else [[2.0, p, 4.0, p, 6.0, 0.0, p], [8.0, p, 10.0, p, 12.0, 0.0, p]])
  assert torch.allclose(result, torch.tensor(exp, device=DEV))


def test_shift_pad_single_element_sequences(backward, pad_value):
  data = torch.tensor([[1.0, 2.0, 3.0, 4.0]], device=DEV)
  result = ast.shift_pad(data, torch.tensor([0, 1, 2, 3, 4], device=DEV), pad_value, backward)
  assert torch.allclose(result, torch.full_like(data, pad_value))


def test_shift_pad_empty_sequences(backward, pad_value):
  data = torch.tensor([[1.0, 2.0, 3.0]], device=DEV)
  with pytest.raises(AssertionError, match="can't shift_pad zero-length seqments"):
    ast.shift_pad(data, torch.tensor([0, 0, 1, 1, 3], device=DEV), pad_value, backward)


@pytest.mark.parametrize("case", golden_case_names("shift_pad"))
def test_shift_pad_matches_reference_golden(case):
  z, meta = golden_cases()
  m = meta[case]
  out = ast.shift_pad(golden_tensor(z, case, "data"), golden_tensor(z, case, "cu_seqlens"),
                      m["pad_value"], m["backward"])
  np.testing.assert_array_equal(out.cpu().numpy(), z[f"{case}/out"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("wrap_variant", [True, False])
def test_shift_pad_large_vs_oracle(dtype, wrap_variant, backward):
  C, seqlens = 5, [7, 1000, 1, 33]
  cu = torch.tensor([3, *(3 + np.cumsum(seqlens))], device=DEV)  # row head outside sequences
  BL = int(cu[-1])
  data = torch.randn(C, BL, device=DEV).to(dtype)
  if wrap_variant:
    out = ast.shift_pad(data, cu, 0.5, backward)
  else:
    out = ast.shift_pad_compiled(data, cu, 0.5, backward)
  gold = oracle.shift_pad(data, cu, 0.5, backward, wrap=wrap_variant)
  np.testing.assert_array_equal(out.float().cpu().numpy(), gold.astype(np.float32))
