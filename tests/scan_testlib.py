"""Shared helpers of the test suite: data factories, golden fixtures, tolerances.

Tolerances are the ones the build is held to, measured against the fp64
sequential oracle (oracle/ascan_oracle.c):

* float32 outputs: |ours - gold| <= RTOL_F32 * |gold| + RTOL_F32 * scale
* float16 / bfloat16 outputs (fp32 accumulation): the same with RTOL_HALF,

where ``scale`` is the RMS of the gold tensor (so the absolute floor follows
the magnitude of the data instead of being a fixed number).  Sequence
boundaries are checked bit-exactly elsewhere.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_cases.npz"

RTOL_F32 = 1e-5
RTOL_HALF = 2e-2
TEST_SEED = 1155

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def rtol_of(dtype: torch.dtype) -> float:
  return RTOL_F32 if dtype == torch.float32 else RTOL_HALF


def assert_close_to_gold(ours: torch.Tensor, gold: np.ndarray, dtype: torch.dtype, what: str,
                         mask: np.ndarray | None = None, rtol: float | None = None) -> None:
  """Elementwise |ours - gold| <= rtol * (|gold| + rms(gold)) over ``mask``."""
  rtol = rtol_of(dtype) if rtol is None else rtol
  o = ours.detach().float().cpu().numpy().astype(np.float64).reshape(gold.shape)
  g = gold
  if mask is not None:
    o, g = o[mask], g[mask]
  assert np.isfinite(g).all(), f"{what}: gold has non-finite values"
  scale = float(np.sqrt(np.mean(g * g))) if g.size else 0.0
  err = np.abs(o - g)
  bound = rtol * (np.abs(g) + scale)
  bad = ~(err <= bound)
  if bad.any():
    i = int(np.argmax(np.where(bad, err - bound, -np.inf)))
    raise AssertionError(
      f"{what}: {int(bad.sum())}/{bad.size} elements off (dtype {dtype}, rtol {rtol}); "
      f"worst at flat {i}: ours {o.flat[i]!r} gold {g.flat[i]!r} err {err.flat[i]:.3e} "
      f"bound {bound.flat[i]:.3e}; max err {err.max():.3e}, scale {scale:.3e}")


def cu_of(seqlens, dtype=torch.int64, device="cuda") -> torch.Tensor:
  return torch.tensor([0, *np.cumsum(seqlens).tolist()], dtype=dtype, device=device)


def make_inputs(C: int, BL: int, dtype=torch.float32, gate="uniform", seed=TEST_SEED,
                device="cuda"):
  """(gates, tokens) [C, BL]; gates U(0,1) / U(0.9,1) / U(0.99,1) / sigmoid(N(2,1)), or
  "nearone": 1 - 2^-8 with probability 0.02 and exactly 1 otherwise (exact in
  every dtype; a 4096-element tile's gate product is about 0.73, so carries
  reach across whole sequences); tokens N(0,1)."""
  gen = torch.Generator(device="cpu").manual_seed(seed)
  if gate == "uniform":
    g = torch.rand(C, BL, generator=gen)
  elif gate == "nearone":
    g = 1.0 - (torch.rand(C, BL, generator=gen) < 0.02).float() / 256
  elif gate == "long":
    g = 0.9 + 0.1 * torch.rand(C, BL, generator=gen)
  elif gate == "verylong":
    g = 0.99 + 0.01 * torch.rand(C, BL, generator=gen)
  elif gate == "sigmoid":
    g = torch.sigmoid(2.0 + torch.randn(C, BL, generator=gen))
  else:
    raise ValueError(gate)
  x = torch.randn(C, BL, generator=gen)
  return g.to(dtype).to(device).contiguous(), x.to(dtype).to(device).contiguous()


def in_sequence_mask(C: int, BL: int, cu) -> np.ndarray:
  """True where a position of a [C, BL] row belongs to a sequence."""
  cu = np.asarray(cu.cpu() if hasattr(cu, "cpu") else cu, dtype=np.int64)
  m = np.zeros(BL, dtype=bool)
  for i in range(len(cu) - 1):
    m[max(cu[i], 0):max(cu[i + 1], 0)] = True
  return np.broadcast_to(m, (C, BL))


def golden_cases():
  z = np.load(GOLDEN)
  meta = json.loads(bytes(z["__meta__"]).decode())
  return z, meta


def golden_case_names(kind: str | None = None):
  _, meta = golden_cases()
  return sorted(k for k, m in meta.items() if kind is None or m["kind"] == kind)


def golden_tensor(z, case: str, name: str, dtype=None, device="cuda") -> torch.Tensor:
  a = z[f"{case}/{name}"]
  t = torch.from_numpy(np.ascontiguousarray(a))
  if dtype is not None:
    t = t.to(dtype)
  return t.to(device).contiguous()


def oracle_fwd(g, x, cu, reverse=False):
  return oracle.scan_fwd(g, x, cu, reverse=reverse)


def oracle_fwd_bwd(g, x, dy, cu, causal=True):
  return oracle.scan_fwd_bwd(g, x, dy, cu, causal=causal)
