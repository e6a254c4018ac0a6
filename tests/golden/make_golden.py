"""Generate golden input/output vectors by running the REFERENCE implementation.

Run in a container that has the reference project checked out (its ``src/``
directory on ``--ref-src``).  The reference's Triton kernels execute on CPU
tensors under ``TRITON_INTERPRET=1``, so no GPU is needed.  The output,
``reference_cases.npz``, is committed and is what tests/test_oracle_golden.py
pins the CPU oracle against and what the GPU parity tests compare with; the
reference itself is never needed at test time.

Usage::

    python tests/golden/make_golden.py --ref-src <reference>/src

Each case stores its inputs (float32, or the raw fp16 bits widened to float32)
and the reference outputs, keyed ``<case>/<name>``.  Entry points exercised
(file:line in the reference):

* ``forward_scan_full`` src/associative_scan_triton/_dispatcher.py:12-70
  (single-chunk kernel _kernels.py:19-81, multi-chunk kernel :84-168), in place
  with TESTING=True (gate products written back) and out of place;
* ``backward_scan_fused_full`` _dispatcher.py:73-117 (kernels :171-374);
* ``scan_causal`` / ``scan_bidirectional_branched`` scan_eager.py:67-85, :181-210;
* ``shift_pad`` _shift_pad.py:18-55.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> None:
  ap = argparse.ArgumentParser()
  ap.add_argument("--ref-src", required=True, help="the reference's src/ directory")
  ap.add_argument("--out", default=str(HERE / "reference_cases.npz"))
  args = ap.parse_args()

  os.environ["TRITON_INTERPRET"] = "1"
  sys.path.insert(0, args.ref_src)
  import torch
  import associative_scan_triton as ref

  torch.manual_seed(1155)
  out: dict[str, np.ndarray] = {}
  meta: dict[str, dict] = {}

  def cu_of(seqlens):
    return torch.tensor([0, *np.cumsum(seqlens).tolist()], dtype=torch.int64)

  def grid_of(seqlens, cs, C):
    return ref.get_grid(len(seqlens) + 1, max(seqlens), cs, C)

  def put(case, **arrays):
    for k, v in arrays.items():
      if isinstance(v, torch.Tensor):
        v = v.detach().to(torch.float32).numpy() if v.is_floating_point() else v.numpy()
      out[f"{case}/{k}"] = np.ascontiguousarray(v)

  def gen(C, BL, dtype, kind):
    if kind == "gate":
      t = torch.rand(C, BL)
    elif kind == "gate_long":
      t = 0.9 + 0.1 * torch.rand(C, BL)
    else:
      t = torch.randn(C, BL)
    return t.to(dtype).contiguous()

  # ---- forward kernels through the dispatcher ------------------------------
  fwd_cases = [
    # name, C, seqlens, chunk, dtype, reverse
    ("fwd_causal_f32_single", 3, [5, 8, 3], 8, torch.float32, False),
    ("fwd_reverse_f32_single", 3, [5, 8, 3], 8, torch.float32, True),
    ("fwd_causal_f32_multi", 3, [37, 64, 5, 100], 16, torch.float32, False),
    ("fwd_reverse_f32_multi", 3, [37, 64, 5, 100], 16, torch.float32, True),
    ("fwd_causal_f32_long", 2, [300, 211], 32, torch.float32, False),
    ("fwd_causal_f16_multi", 2, [70, 33], 16, torch.float16, False),
    ("fwd_reverse_f16_multi", 2, [70, 33], 16, torch.float16, True),
    ("fwd_causal_bf16_multi", 2, [70, 33], 16, torch.bfloat16, False),
  ]
  for name, C, seqlens, cs, dtype, reverse in fwd_cases:
    BL = sum(seqlens)
    g = gen(C, BL, dtype, "gate")
    x = gen(C, BL, dtype, "token")
    cu = cu_of(seqlens)
    grid = grid_of(seqlens, cs, C)
    # in place, TESTING=True: tokens and gate products written back
    g_ip, x_ip = g.clone(), x.clone()
    ref.forward_scan_full(g_ip, x_ip, cu, grid, REVERSE=reverse, CHUNK_SIZE=cs, TESTING=True)
    # out of place, TESTING=False
    y = torch.empty_like(x)
    ref.forward_scan_full(g.clone(), x.clone(), cu, grid, REVERSE=reverse, CHUNK_SIZE=cs,
                          TESTING=False, tokens_out=y)
    put(name, gates=g, tokens=x, cu_seqlens=cu, y_inplace=x_ip, gate_products=g_ip, y=y)
    meta[name] = {"kind": "fwd", "C": C, "seqlens": seqlens, "chunk_size": cs,
                  "dtype": str(dtype).split(".")[-1], "reverse": reverse}

  # ---- fused backward kernels through the dispatcher -----------------------
  bwd_cases = [
    ("bwd_causal_f32_single", 3, [5, 8, 3], 8, torch.float32, True),
    ("bwd_anticausal_f32_single", 3, [5, 8, 3], 8, torch.float32, False),
    ("bwd_causal_f32_multi", 3, [37, 64, 5, 100], 16, torch.float32, True),
    ("bwd_anticausal_f32_multi", 3, [37, 64, 5, 100], 16, torch.float32, False),
    ("bwd_causal_f16_multi", 2, [70, 33], 16, torch.float16, True),
  ]
  for name, C, seqlens, cs, dtype, causal in bwd_cases:
    BL = sum(seqlens)
    g = gen(C, BL, dtype, "gate")
    x = gen(C, BL, dtype, "token")
    dy = gen(C, BL, dtype, "token")
    cu = cu_of(seqlens)
    grid = grid_of(seqlens, cs, C)
    h = torch.empty_like(x)
    ref.forward_scan_full(g.clone(), x.clone(), cu, grid, REVERSE=not causal, CHUNK_SIZE=cs,
                          TESTING=False, tokens_out=h)
    dx = torch.empty_like(dy)
    dg = torch.empty_like(g)
    ref.backward_scan_fused_full(dy, g, h, dx, dg, cu, grid, CHUNK_SIZE=cs, CAUSAL=causal)
    put(name, gates=g, tokens=x, grad=dy, states=h, cu_seqlens=cu, d_tokens=dx, d_gates=dg)
    meta[name] = {"kind": "bwd", "C": C, "seqlens": seqlens, "chunk_size": cs,
                  "dtype": str(dtype).split(".")[-1], "causal": causal}

  # ---- autograd API ---------------------------------------------------------
  # configs[0] of the benchmark plan: C=4, T=128, one sequence, seed 0.
  torch.manual_seed(0)
  C, T = 4, 128
  g = torch.rand(C, T)
  x = torch.randn(C, T)
  cu = torch.tensor([0, T])
  gr, xr = g.clone().requires_grad_(True), x.clone().requires_grad_(True)
  args_ = {"cu_seqlens": cu, "chunk_size": 128, "grid": ref.get_grid(2, T, 128, C)}
  y = ref.scan_causal(gr, xr, args_)
  y.sum().backward()
  put("config0_scan_causal", gates=g, tokens=x, cu_seqlens=cu, y=y, d_gates=gr.grad,
      d_tokens=xr.grad)
  meta["config0_scan_causal"] = {"kind": "autograd_causal", "C": C, "seqlens": [T],
                                 "chunk_size": 128, "dtype": "float32"}

  torch.manual_seed(1155)
  seqlens, cs, C = [20, 13, 31], 8, 3
  BL = sum(seqlens)
  cu = cu_of(seqlens)
  grid = grid_of(seqlens, cs, C)
  gf, xf, gb, xb = (gen(C, BL, torch.float32, k) for k in ("gate", "token", "gate", "token"))
  dyf, dyb = gen(C, BL, torch.float32, "token"), gen(C, BL, torch.float32, "token")
  leaves = [t.clone().requires_grad_(True) for t in (gf, xf, gb, xb)]
  yf, yb = ref.scan_bidirectional_branched(*leaves, {"cu_seqlens": cu, "chunk_size": cs,
                                                     "grid": grid})
  ((yf * dyf).sum() + (yb * dyb).sum()).backward()
  put("bidi_f32", gates_fwd=gf, tokens_fwd=xf, gates_bwd=gb, tokens_bwd=xb, grad_fwd=dyf,
      grad_bwd=dyb, cu_seqlens=cu, y_fwd=yf, y_bwd=yb, d_gates_fwd=leaves[0].grad,
      d_tokens_fwd=leaves[1].grad, d_gates_bwd=leaves[2].grad, d_tokens_bwd=leaves[3].grad)
  meta["bidi_f32"] = {"kind": "autograd_bidi", "C": C, "seqlens": seqlens, "chunk_size": cs,
                      "dtype": "float32"}

  # ---- shift_pad (torch.roll variant) ---------------------------------------
  for backward in (True, False):
    for pad in (0.0, 1.0):
      name = f"shift_pad_{'right' if backward else 'left'}_pad{int(pad)}"
      seqlens = [3, 1, 6, 2]
      C, BL = 2, sum(seqlens)
      d = torch.randn(C, BL)
      cu = cu_of(seqlens)
      o = ref.shift_pad(d, cu, pad, backward)
      put(name, data=d, cu_seqlens=cu, out=o)
      meta[name] = {"kind": "shift_pad", "backward": backward, "pad_value": pad,
                    "seqlens": seqlens, "C": C}

  out["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
  np.savez_compressed(args.out, **out)
  print(f"wrote {len(meta)} cases to {args.out}")


if __name__ == "__main__":
  main()
