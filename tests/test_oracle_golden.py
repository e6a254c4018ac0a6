"""CPU: pin the fp64 oracle to the reference before trusting it.

Three independent anchors:
1. hand-computed known-answer vectors from the reference's own tests
   (file:line cited per test);
2. golden outputs produced by running the reference implementation itself
   (tests/golden/make_golden.py, Triton interpreter on CPU);
3. a second, pure-Python restatement of the recurrence.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from scan_testlib import golden_case_names, golden_cases

# --- 1. known-answer vectors --------------------------------------------------

KAT_G = [1.0, 1.5, 0.8, 2.0]
KAT_X = [1.0, -1.0, 0.5, 2.0]


def test_kat_single_sequence_forward():
  # reference tests/test_scan_kernels.py:146-170
  y, a = oracle.scan_fwd([KAT_G], [KAT_X], [0, 4])
  np.testing.assert_allclose(y[0], [1.0, 0.5, 0.9, 3.8], rtol=1e-6)
  np.testing.assert_allclose(a[0], [1.0, 1.5, 1.2, 2.4], rtol=1e-6)


def test_kat_single_sequence_reverse():
  # reference tests/test_scan_kernels.py:199-222
  y, a = oracle.scan_fwd([KAT_G], [KAT_X], [0, 4], reverse=True)
  np.testing.assert_allclose(y[0], [3.15, 2.15, 2.1, 2.0], rtol=1e-6)
  np.testing.assert_allclose(a[0], [2.4, 2.4, 1.6, 2.0], rtol=1e-6)


def test_kat_multi_chunk_forward_and_reverse():
  # reference tests/test_scan_kernels.py:238-258 and :273-295
  g, x = [KAT_G * 2], [KAT_X * 2]
  y, _ = oracle.scan_fwd(g, x, [0, 8])
  np.testing.assert_allclose(y[0], [1.0, 0.5, 0.9, 3.8, 4.8, 6.2, 5.46, 12.92], rtol=1e-6)
  y, _ = oracle.scan_fwd(g, x, [0, 8], reverse=True)
  np.testing.assert_allclose(y[0], [10.71, 9.71, 7.14, 8.3, 3.15, 2.15, 2.1, 2.0], rtol=1e-6)


def test_kat_copied_sequences():
  # reference tests/test_scan_kernels.py:481-507
  y, a = oracle.scan_fwd([KAT_G * 2], [KAT_X * 2], [0, 4, 8])
  np.testing.assert_allclose(y[0], [1, 0.5, 0.9, 3.8] * 2, rtol=1e-6)
  np.testing.assert_allclose(a[0], [1, 1.5, 1.2, 2.4] * 2, rtol=1e-6)


def test_kat_varlen():
  # reference tests/test_scan_kernels.py:530-563
  g = [[1.0, 1.5, 0.8, 2.0, 0.3, 0.4, 0.9, 0.5, 0.45]]
  x = [[1.0, -1.0, 0.5, 2.0, 1.0, -0.7, 0.8, 0.6, 0.33]]
  y, a = oracle.scan_fwd(g, x, [0, 4, 9])
  np.testing.assert_allclose(y[0], [1.0, 0.5, 0.9, 3.8, 1.0, -0.3, 0.53, 0.865, 0.7192],
                             rtol=1e-4, atol=1e-7)
  np.testing.assert_allclose(a[0], [1, 1.5, 1.2, 2.4, 0.3, 0.12, 0.108, 0.054, 0.0243],
                             rtol=1e-4, atol=1e-7)


VL_G = [[0.3, 0.4, 0.9, 0.5, 0.45, 1.0, 1.5, 0.8, 2.0],
        [0.3, 0.55, 0.96, 0.35, 0.7, 0.35, 0.85, 0.45, 1.3]]
VL_X = [[1.0, -0.7, 0.8, 0.6, 0.33, 1.0, -1.0, 0.5, 2.0],
        [0.6, -0.75, 0.4, 0.65, 0.8, 1.0, -0.55, 0.65, 0.4]]


def test_kat_varlen_two_channels():
  # reference tests/test_scan_kernels.py:591-645 (tolerance rtol 1e-3, atol 1e-5)
  y, a = oracle.scan_fwd(VL_G, VL_X, [0, 5, 9])
  np.testing.assert_allclose(a, [[0.3, 0.12, 0.108, 0.054, 0.0243, 1.0, 1.5, 1.2, 2.4],
                                 [0.3, 0.165, 0.1584, 0.05544, 0.0388, 0.35, 0.2975, 0.1339,
                                  0.174]], rtol=1e-3, atol=1e-5)
  np.testing.assert_allclose(y, [[1.0, -0.3, 0.53, 0.865, 0.71925, 1.0, 0.5, 0.9, 3.8],
                                 [0.60, -0.42, -0.0032, 0.6489, 1.25422, 1.0, 0.3, 0.7850,
                                  1.4205]], rtol=1e-3, atol=1e-5)


def test_kat_varlen_two_channels_reverse():
  # reference tests/test_scan_kernels.py:672-727
  y, a = oracle.scan_fwd(VL_G, VL_X, [0, 5, 9], reverse=True)
  np.testing.assert_allclose(a, [[0.0243, 0.081, 0.2025, 0.225, 0.45, 2.4, 2.4, 1.6, 2.0],
                                 [0.038808, 0.12936, 0.2352, 0.245, 0.7, 0.174038, 0.49725,
                                  0.585, 1.3]], rtol=1e-3, atol=1e-5)
  np.testing.assert_allclose(y, [[0.96862, -0.1046, 1.4885, 0.765, 0.33, 3.15, 2.15, 2.1, 2.0],
                                 [0.588312, -0.03896, 1.2928, 0.93, 0.8, 1.054425, 0.1555, 0.83,
                                  0.4]], rtol=1e-3, atol=1e-5)


def test_kat_causal_autograd_values():
  # reference tests/test_scan_causal.py:33-71 (y, dL/dg, dL/dx for L = sum(y))
  g, x = [KAT_G * 2], [KAT_X * 2]
  y, dx, dg = oracle.scan_fwd_bwd(g, x, np.ones((1, 8)), [0, 4, 8])
  np.testing.assert_allclose(y[0], [1, 0.5, 0.9, 3.8] * 2, rtol=1e-4, atol=1e-4)
  np.testing.assert_allclose(dg[0], [0.0, 3.4, 1.5, 0.9] * 2, rtol=1e-4, atol=1e-4)
  np.testing.assert_allclose(dx[0], [6.1, 3.4, 3.0, 1.0] * 2, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize(("gates", "tokens"), [([0.5, 0.6, 0.7], [1.0, 2.0, 3.0]),
                                               ([0.3, 0.45, 0.6], [1.0, 1.4, 0.3])])
def test_manual_gradients(gates, tokens):
  # reference tests/test_scan_kernels.py:873-933: hand-derived dg, dx
  g, t = gates, tokens
  h1 = t[0]
  h2 = g[1] * h1 + t[1]
  d3 = 1.0
  d2 = 1.0 + d3 * g[2]
  d1 = 1.0 + d2 * g[1]
  _, dx, dg = oracle.scan_fwd_bwd([g], [t], np.ones((1, 3)), [0, 3])
  np.testing.assert_allclose(dx[0], [d1, d2, d3], rtol=1e-6)
  np.testing.assert_allclose(dg[0], [0.0, d2 * h1, d3 * h2], rtol=1e-6)


@pytest.mark.parametrize(("a", "b", "c"), [((0.5, 0.3), (0.6, 0.9), (0.7, 0.8)),
                                           ((0.6, 0.9), (0.5, 0.3), (0.7, 0.8)),
                                           ((0.6, 0.9), (0.7, 0.8), (0.5, 0.3))])
def test_combine_is_associative(a, b, c):
  # reference tests/test_scan_kernels.py:23-43
  ab = oracle.combine(*a, *b)
  abc1 = oracle.combine(*ab, *c)
  bc = oracle.combine(*b, *c)
  abc2 = oracle.combine(*a, *bc)
  assert np.allclose(abc1, abc2)


SP_DATA = [[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0]]


@pytest.mark.parametrize("backward", [True, False])
def test_kat_shift_pad(backward):
  # reference tests/test_shift_pad.py:24-118 (pad_value -1)
  p = -1.0
  out = oracle.shift_pad([[1.0, 2.0, 3.0, 4.0, 5.0]], [0, 5], p, backward)
  exp = [[p, 1, 2, 3, 4]] if backward else [[2, 3, 4, 5, p]]
  np.testing.assert_array_equal(out, exp)
  out = oracle.shift_pad(SP_DATA, [0, 3, 7], p, backward)
  exp = [[p, 1, 2, p, 4, 5, 6]] if backward else [[2, 3, p, 5, 6, 7, p]]
  np.testing.assert_array_equal(out, exp)
  data = [[1, 2, 3, 4, 5, 6, 0.0], [7, 8, 9, 10, 11, 12, 0.0]]
  out = oracle.shift_pad(data, [0, 2, 4, 7], p, backward)
  exp = ([[p, 1, p, 3, p, 5, 6], [p, 7, p, 9, p, 11, 12]] if backward
         else [[2, p, 4, p, 6, 0, p], [8, p, 10, p, 12, 0, p]])
  np.testing.assert_array_equal(out, exp)
  out = oracle.shift_pad([[1.0, 2, 3, 4]], [0, 1, 2, 3, 4], p, backward)
  np.testing.assert_array_equal(out, [[p] * 4])


# --- 2. golden outputs of the reference itself ------------------------------------

def _tol(dtype: str):
  # The reference computes in fp32 (fp16/bf16 inputs upcast, outputs rounded
  # back), the oracle in fp64: allow fp32 rounding, or the output dtype's.
  return {"float32": 2e-6, "float16": 2e-3, "bfloat16": 1.6e-2}[dtype]


@pytest.mark.parametrize("case", golden_case_names("fwd"))
def test_oracle_matches_reference_forward(case):
  z, meta = golden_cases()
  m = meta[case]
  y, a = oracle.scan_fwd(z[f"{case}/gates"], z[f"{case}/tokens"], z[f"{case}/cu_seqlens"],
                         reverse=m["reverse"])
  tol = _tol(m["dtype"])
  for ours, ref in ((y, z[f"{case}/y"]), (y, z[f"{case}/y_inplace"]),
                    (a, z[f"{case}/gate_products"])):
    scale = max(1.0, float(np.abs(ref).max()))
    np.testing.assert_allclose(ours, ref, rtol=tol, atol=tol * scale)


@pytest.mark.parametrize("case", golden_case_names("bwd"))
def test_oracle_matches_reference_backward(case):
  z, meta = golden_cases()
  m = meta[case]
  dx, dg = oracle.scan_bwd(z[f"{case}/grad"], z[f"{case}/gates"], z[f"{case}/states"],
                           z[f"{case}/cu_seqlens"], causal=m["causal"])
  tol = _tol(m["dtype"])
  for ours, ref in ((dx, z[f"{case}/d_tokens"]), (dg, z[f"{case}/d_gates"])):
    scale = max(1.0, float(np.abs(ref).max()))
    np.testing.assert_allclose(ours, ref, rtol=tol, atol=tol * scale)


def test_oracle_matches_reference_config0_autograd():
  z, _ = golden_cases()
  c = "config0_scan_causal"
  y, dx, dg = oracle.scan_fwd_bwd(z[f"{c}/gates"], z[f"{c}/tokens"],
                                  np.ones_like(z[f"{c}/tokens"]), z[f"{c}/cu_seqlens"])
  np.testing.assert_allclose(y, z[f"{c}/y"], rtol=2e-6, atol=2e-6)
  np.testing.assert_allclose(dx, z[f"{c}/d_tokens"], rtol=2e-6, atol=2e-5)
  np.testing.assert_allclose(dg, z[f"{c}/d_gates"], rtol=2e-6, atol=2e-5)


def test_oracle_matches_reference_bidi():
  z, _ = golden_cases()
  c = "bidi_f32"
  k = lambda n: z[f"{c}/{n}"]  # noqa: E731
  yf, dxf, dgf = oracle.scan_fwd_bwd(k("gates_fwd"), k("tokens_fwd"), k("grad_fwd"),
                                     k("cu_seqlens"), causal=True)
  yb, dxb, dgb = oracle.scan_fwd_bwd(k("gates_bwd"), k("tokens_bwd"), k("grad_bwd"),
                                     k("cu_seqlens"), causal=False)
  for ours, name in ((yf, "y_fwd"), (dxf, "d_tokens_fwd"), (dgf, "d_gates_fwd"), (yb, "y_bwd"),
                     (dxb, "d_tokens_bwd"), (dgb, "d_gates_bwd")):
    np.testing.assert_allclose(ours, k(name), rtol=2e-6, atol=2e-6, err_msg=name)


@pytest.mark.parametrize("case", golden_case_names("shift_pad"))
def test_oracle_matches_reference_shift_pad(case):
  z, meta = golden_cases()
  m = meta[case]
  out = oracle.shift_pad(z[f"{case}/data"], z[f"{case}/cu_seqlens"], m["pad_value"],
                         m["backward"], wrap=True)
  np.testing.assert_array_equal(out, z[f"{case}/out"])


# --- 3. C oracle vs pure-Python restatement -------------------------------------------

@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("direction", [True, False])
def test_c_oracle_matches_python_loops(seed, direction):
  rng = np.random.default_rng(seed)
  seqlens = rng.integers(1, 9, size=rng.integers(1, 5))
  cu = np.concatenate([[0], np.cumsum(seqlens)])
  C, BL = 3, int(cu[-1])
  g = rng.uniform(0, 1.2, size=(C, BL)).astype(np.float32)
  x = rng.normal(size=(C, BL)).astype(np.float32)
  dy = rng.normal(size=(C, BL)).astype(np.float32)
  y, a = oracle.scan_fwd(g, x, cu, reverse=not direction)
  py_y, py_a = oracle.py_scan_fwd(g, x, cu, reverse=not direction)
  np.testing.assert_allclose(y, py_y, rtol=1e-12, atol=1e-12)
  np.testing.assert_allclose(a, py_a, rtol=1e-12, atol=1e-12)
  h = y.astype(np.float32)
  dx, dg = oracle.scan_bwd(dy, g, h, cu, causal=direction)
  py_dx, py_dg = oracle.py_scan_bwd(dy, g, h, cu, causal=direction)
  np.testing.assert_allclose(dx, py_dx, rtol=1e-12, atol=1e-12)
  np.testing.assert_allclose(dg, py_dg, rtol=1e-12, atol=1e-12)


def test_oracle_leaves_positions_outside_sequences():
  # positions before cu[0] are not part of any sequence and are not written
  y, _ = oracle.scan_fwd([[0.5] * 6], [[1.0] * 6], [2, 4, 6])
  assert np.isnan(y[0, :2]).all()
  np.testing.assert_allclose(y[0, 2:], [1.0, 1.5, 1.0, 1.5])
