"""CPU oracle for the scan path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of bench.py import this module.  The product package
never imports it and has no CPU fallback.

Two restatements of the reference's semantics live here:

* ``ascan_oracle.c`` (compiled by :func:`build`), an fp64 sequential scan that
  is threaded over channels.  It is the checker for every parity test and the
  timed CPU baseline.
* ``py_scan_fwd`` / ``py_scan_bwd``, pure-Python loops for tiny cases, used to
  cross-check the C code.

Reference semantics followed (file:line in the reference project):

* forward gold label: tests/test_scan_dtypes.py:26-38
  (``sequential_scan_gold``), identical at bench/bench_accuracy.py:40-49;
* reverse scan: tests/test_scan_kernels.py:281-286, tests/test_scan_dtypes.py:173-177;
* gate products written back with TESTING: src/associative_scan_triton/_kernels.py:74-76;
* backward: tests/test_scan_kernels.py:850-897, src/associative_scan_triton/_kernels.py:184-196;
* shift_pad: src/associative_scan_triton/_shift_pad.py:18-55 and :63-118.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "ascan_oracle.c"
_LIB_PATH = _HERE / "build" / "libascan_oracle.so"

_lib = None


def build(force: bool = False) -> Path:
  """Compile ascan_oracle.c into oracle/build/libascan_oracle.so."""
  out = _LIB_PATH
  if out.exists() and not force and out.stat().st_mtime >= _SRC.stat().st_mtime:
    return out
  out.parent.mkdir(parents=True, exist_ok=True)
  tmp = out.with_suffix(f".{os.getpid()}.tmp")
  cmd = [
    "gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
    "-fvisibility=hidden", "-o", str(tmp), str(_SRC),
  ]
  subprocess.run(cmd, check=True)
  os.replace(tmp, out)
  return out


def _load():
  global _lib
  if _lib is not None:
    return _lib
  path = build()
  lib = ctypes.CDLL(str(path))
  p = ctypes.c_void_p
  i64 = ctypes.c_int64
  ci = ctypes.c_int
  lib.oracle_scan_fwd.argtypes = [p, p, p, p, p, i64, i64, i64, ci, ci]
  lib.oracle_scan_bwd.argtypes = [p, p, p, p, p, p, i64, i64, i64, ci, ci]
  lib.oracle_scan_fwd_bwd.argtypes = [p, p, p, p, p, p, p, i64, i64, i64, ci, ci]
  lib.oracle_shift_pad.argtypes = [p, p, p, i64, i64, i64, ctypes.c_double, ci, ci, ci]
  lib.oracle_num_threads.restype = ci
  for f in ("oracle_scan_fwd", "oracle_scan_bwd", "oracle_scan_fwd_bwd", "oracle_shift_pad"):
    getattr(lib, f).restype = None
  _lib = lib
  return lib


def num_threads() -> int:
  return int(_load().oracle_num_threads())


def _f32(a) -> np.ndarray:
  """Any array-like / torch tensor -> C-contiguous 2-D float32 numpy array."""
  if hasattr(a, "detach"):
    a = a.detach().to("cpu")
    import torch

    if a.dtype in (torch.bfloat16, torch.float16):
      a = a.float()
    a = a.numpy()
  a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
  if a.ndim == 1:
    a = a[None, :]
  return a


def _cu(cu) -> np.ndarray:
  if hasattr(cu, "detach"):
    cu = cu.detach().to("cpu").numpy()
  return np.ascontiguousarray(np.asarray(cu, dtype=np.int64))


def _ptr(a: np.ndarray):
  return a.ctypes.data_as(ctypes.c_void_p)


def scan_fwd(g, x, cu, reverse: bool = False, nthreads: int = 0, fill=np.nan):
  """fp64 forward scan.  Returns (y, gate_products), both float64 [C, BL].

  Positions that lie in no sequence keep ``fill``.
  """
  g, x, cu = _f32(g), _f32(x), _cu(cu)
  assert g.shape == x.shape
  C, BL = g.shape
  y = np.full((C, BL), fill, dtype=np.float64)
  a = np.full((C, BL), fill, dtype=np.float64)
  _load().oracle_scan_fwd(_ptr(g), _ptr(x), _ptr(y), _ptr(a), _ptr(cu),
                          len(cu) - 1, C, BL, int(bool(reverse)), int(nthreads))
  return y, a


def scan_bwd(dy, g, h, cu, causal: bool = True, nthreads: int = 0, fill=np.nan):
  """fp64 backward given forward states ``h``.  Returns (dx, dg) float64."""
  dy, g, h, cu = _f32(dy), _f32(g), _f32(h), _cu(cu)
  C, BL = g.shape
  dx = np.full((C, BL), fill, dtype=np.float64)
  dg = np.full((C, BL), fill, dtype=np.float64)
  _load().oracle_scan_bwd(_ptr(dy), _ptr(g), _ptr(h), _ptr(dx), _ptr(dg), _ptr(cu),
                          len(cu) - 1, C, BL, int(bool(causal)), int(nthreads))
  return dx, dg


def scan_fwd_bwd(g, x, dy, cu, causal: bool = True, nthreads: int = 0, fill=np.nan):
  """fp64 forward + backward with the states kept in fp64.

  ``causal=False`` is the reverse scan and its adjoint.  Returns (y, dx, dg).
  """
  g, x, dy, cu = _f32(g), _f32(x), _f32(dy), _cu(cu)
  C, BL = g.shape
  y = np.full((C, BL), fill, dtype=np.float64)
  dx = np.full((C, BL), fill, dtype=np.float64)
  dg = np.full((C, BL), fill, dtype=np.float64)
  _load().oracle_scan_fwd_bwd(_ptr(g), _ptr(x), _ptr(dy), _ptr(y), _ptr(dx), _ptr(dg),
                              _ptr(cu), len(cu) - 1, C, BL, int(bool(causal)), int(nthreads))
  return y, dx, dg


def shift_pad(data, cu, pad_value: float = 0.0, backward: bool = True, wrap: bool = True,
              nthreads: int = 0):
  """fp64 shift_pad; ``wrap`` selects the torch.roll (True) or clamped (False) variant."""
  d, cu = _f32(data), _cu(cu)
  C, BL = d.shape
  out = np.empty((C, BL), dtype=np.float64)
  _load().oracle_shift_pad(_ptr(d), _ptr(out), _ptr(cu), len(cu) - 1, C, BL,
                           float(pad_value), int(bool(backward)), int(bool(wrap)), int(nthreads))
  return out


# ---------------------------------------------------------------------------
# Pure-Python loops (tiny cases only) -- an independent restatement used to
# cross-check the C oracle.
# ---------------------------------------------------------------------------


def combine(fl, xl, fr, xr):
  """The reference's combine operator (src/associative_scan_triton/_kernels.py:6-16)."""
  return fr * fl, fr * xl + xr


def py_scan_fwd(g, x, cu, reverse=False):
  g = [list(map(float, row)) for row in _f32(g)]
  x = [list(map(float, row)) for row in _f32(x)]
  cu = [int(v) for v in _cu(cu)]
  y = [[float("nan")] * len(r) for r in g]
  a = [[float("nan")] * len(r) for r in g]
  for c in range(len(g)):
    for i in range(len(cu) - 1):
      idx = list(range(cu[i], cu[i + 1]))
      if reverse:
        idx = idx[::-1]
      acc = (1.0, 0.0)
      for t in idx:
        acc = combine(acc[0], acc[1], g[c][t], x[c][t])
        a[c][t], y[c][t] = acc
  return np.array(y), np.array(a)


def py_scan_bwd(dy, g, h, cu, causal=True):
  dy = [list(map(float, row)) for row in _f32(dy)]
  g = [list(map(float, row)) for row in _f32(g)]
  h = [list(map(float, row)) for row in _f32(h)]
  cu = [int(v) for v in _cu(cu)]
  dx = [[float("nan")] * len(r) for r in g]
  dg = [[float("nan")] * len(r) for r in g]
  for c in range(len(g)):
    for i in range(len(cu) - 1):
      s, e = cu[i], cu[i + 1]
      order = range(e - 1, s - 1, -1) if causal else range(s, e)
      d = 0.0
      for t in order:
        nxt = t + 1 if causal else t - 1  # the element the adjoint came from
        prv = t - 1 if causal else t + 1  # the forward state that fed h[t]
        gate = g[c][nxt] if s <= nxt < e else 1.0
        d = dy[c][t] + gate * d
        dx[c][t] = d
        dg[c][t] = d * h[c][prv] if s <= prv < e else 0.0
  return np.array(dx), np.array(dg)
