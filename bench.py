"""Benchmark of the packed-varlen linear scan on B200 (one JSON line on stdout).

Headline workload: configs[4] case 5a of the north star (the reference's
kernel-benchmark shape at its longest T, reference bench/bench_kernels.py:42-46
and README.md:155,170): causal fwd+bwd over B=8 packed sequences of T=65536,
C=1536 channels, float32, gates ~ U(0.9, 1), tokens ~ N(0, 1), upstream
gradient ~ N(0, 1), seeded synthetic data (each block of 64 channels seeded by
its index, so the problem is the same at every N).  One fixed problem of
805,306,368 elements: under torchrun rank k of N owns the channel block
``sharding.channel_block(1536, N, k)`` with the full cu_seqlens and no
collective on the data path (strong scaling).  One step = one forward kernel +
one fused backward kernel on every rank; ``value`` = algorithmic bytes of the
whole problem (fwd 3 x 4 B + bwd 5 x 4 B = 32 B per element) / the slowest
rank's CUDA-event time per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --profile-case NAME [--steps K] [--warmup W]

Secondary keys, each with its own fp64 parity check of a seeded sample of rows
(``parity``; a failed check makes the run exit non-zero):
  configs1_replicas        configs[1] (B=8 x T=4096, C=1536, fp32), one full
                           copy per rank (weak scaling)
  sequence_shard_configs2  configs[2] (varlen, C=2048, 32 seeded lengths, bf16)
                           split into whole-sequence shards across the ranks
  time_shard               configs[4] case 5b (C=256, one sequence of 2^20)
                           time-sharded across the ranks (carry exchange over
                           NVLink peer memory, one kernel per direction)
  time_shard_nccl          the same with the NCCL all-gather exchange (N > 1)
and, on one GPU, a T sweep, the small-T graph replay, configs[3] and the CPU
baseline.

``--impl reference`` times the reference's CPU algorithm -- the fp64 sequential
scan of its tests (oracle/ascan_oracle.c restates it) -- on the host cores
with every available thread, on the headline configuration.

``--profile-case`` runs one workload W + K times for an ncu capture and prints
one line (no contract JSON): headline_rank8 (the per-rank block of the
headline at 8 GPUs: C=192), configs1, varlen_bf16, bidi_fp16,
time_shard_emulated (all 8 slabs of case 5b on one GPU).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
REF_TREE = REPO / "baseline" / "_ref"  # the unmodified reference package (git-ignored)
if "--reference-triton-child" in sys.argv:
  # the reference's package has the same name as ours: this child process
  # sees only the reference's tree
  sys.path.insert(0, str(REF_TREE))
else:
  sys.path.insert(0, str(REPO / "associative-scan-triton_b200"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "fwd & fwd+bwd ms and achieved HBM GB/s at B=8,C=1536,T=128..65536"
B, C = 8, 1536
T_HEAD = 65536                 # configs[4] case 5a
T_C1 = 4096                    # configs[1]
FWD_BYTES_PER_ELEM = 3 * 4     # read g, x; write y (fp32)
BWD_BYTES_PER_ELEM = 5 * 4     # read dy, g, h; write dx, dg
STEP_BYTES_PER_ELEM = FWD_BYTES_PER_ELEM + BWD_BYTES_PER_ELEM
L2_BYTES = 126 * 2**20
RTOL_F32, RTOL_HALF = 1e-5, 2e-2
# ncu summary of the headline's backward at the per-rank shape of 8 GPUs
# (C=192); its DRAM bytes scale with the elements of a launch
PROFILE_SUMMARY = REPO / "profiles" / "scan_bwd_tma_kernel_B8_T65536_C192_f32.md"
TS_C, TS_T, TS_CHUNK = 256, 1 << 20, 1 << 17  # configs[4] case 5b


def _peaks() -> tuple[float, str]:
  p = REPO / "MEASURED_PEAKS.json"
  try:
    return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
  except Exception:
    return 6650.0, "fallback"


def _profile_traffic(elements: int) -> float | None:
  """DRAM bytes of one backward launch over `elements`, scaled from the
  committed ncu summary (bytes per element of the captured launch)."""
  try:
    for line in PROFILE_SUMMARY.read_text().splitlines():
      if line.startswith("traffic_bytes_per_element:"):
        return round(float(line.split(":", 1)[1].strip()) * elements, 0)
  except OSError:
    pass
  return None


class ClockSampler:
  """nvidia-smi clock / throttle-reason sampling while the GPU is busy."""

  FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

  def __init__(self, device_index: int):
    self.proc = None
    self.path = None
    try:
      uuid = str(torch.cuda.get_device_properties(device_index).uuid)
      self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
      self.gpu = None

  def start(self):
    if self.gpu is None:
      return self
    import tempfile
    fd, self.path = tempfile.mkstemp(prefix="ascan_clocks_", suffix=".csv")
    os.close(fd)
    try:
      self.proc = subprocess.Popen(
        ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
         "--format=csv,noheader,nounits", "-lms", "50"],
        stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
    except OSError:
      self.proc = None
    return self

  def stop(self) -> dict:
    if self.proc is None:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    self.proc.terminate()
    try:
      self.proc.wait(timeout=5)
    except subprocess.TimeoutExpired:
      self.proc.kill()
    rows = []
    for line in Path(self.path).read_text().splitlines():
      parts = [p.strip() for p in line.split(",")]
      if len(parts) == 8:
        rows.append(parts)
    os.unlink(self.path)
    if not rows:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
    mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
    pw = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
    names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
    loaded = sorted(sm)[len(sm) // 2:] if sm else []  # upper half = under load
    return {"sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max(mx) if mx else None,
            "power_w_max": max(pw) if pw else None,
            "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


def _dist_setup():
  world = int(os.environ.get("WORLD_SIZE", "1"))
  if world > 1:
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist, dist.get_rank(), world, local
  return None, 0, 1, 0


def _barrier(dist, device):
  if dist is not None:
    dist.barrier(device_ids=[device.index])


def _reduce(dist, value: float, device, op: str = "max") -> float:
  if dist is None:
    return value
  t = torch.tensor([value], dtype=torch.float64, device=device)
  dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM,
                         "min": dist.ReduceOp.MIN}[op])
  return float(t.item())


# ---------------------------------------------------------------------------
# seeded inputs (the same global problem at every N)
# ---------------------------------------------------------------------------


ROW_BLOCK = 64  # rows drawn per generator call


def _rows_rand(rows, width, device, seed, law, dtype):
  """[len(rows), width] tensor for the contiguous rows ``rows``; each block of
  64 rows is drawn from a generator seeded by (seed, block index), so a row's
  values do not depend on how the rows are split across ranks.  law "u09" =
  U(0.9,1), "u099" = U(0.99,1), "n" = N(0,1), "sig" = sigmoid(N(2,1))."""
  r0, r1 = rows[0], rows[-1] + 1
  out = torch.empty(r1 - r0, width, device=device, dtype=torch.float32)
  gen = torch.Generator(device=device)
  for b in range(r0 // ROW_BLOCK, (r1 + ROW_BLOCK - 1) // ROW_BLOCK):
    gen.manual_seed(seed * 1_000_003 + b)
    blk = (torch.randn if law in ("n", "sig") else torch.rand)(
      ROW_BLOCK, width, device=device, generator=gen)
    a, z = max(b * ROW_BLOCK, r0), min((b + 1) * ROW_BLOCK, r1)
    out[a - r0:z - r0] = blk[a - b * ROW_BLOCK:z - b * ROW_BLOCK]
    del blk
  if law == "sig":
    out.add_(2.0).sigmoid_()
  elif law in ("u09", "u099"):
    lo = 0.9 if law == "u09" else 0.99
    out.mul_(1.0 - lo).add_(lo)
  return out if dtype == torch.float32 else out.to(dtype)


def _packed_problem(device, c0, c1, T_, seed, B_=B):
  """Channels [c0, c1) of a packed causal problem of B_ sequences of T_."""
  rows = range(c0, c1)
  BL = B_ * T_
  g = _rows_rand(rows, BL, device, seed, "u09", torch.float32)
  x = _rows_rand(rows, BL, device, seed + 1, "n", torch.float32)
  dy = _rows_rand(rows, BL, device, seed + 2, "n", torch.float32)
  cu = torch.arange(B_ + 1, device=device, dtype=torch.int32) * T_
  return g, x, dy, cu


# ---------------------------------------------------------------------------
# fp64 parity check of sampled rows (restates the reference's sequential gold
# label, tests/test_scan_dtypes.py:26-38, and the hand-derived backward,
# tests/test_scan_kernels.py:850-897, in blocks of 32 steps: inside a block
# h[t] = P[t] (h_in + sum_{s<=t} x[s] / P[s]) with P the running gate product;
# exact up to fp64 rounding for gates well above zero, which every checked
# config has)
# ---------------------------------------------------------------------------


def _fp64_scan_seg(a, b, K=32):
  """Inclusive scan h[t] = a[t] h[t-1] + b[t] from h = 0, fp64 [R, L]."""
  R, L = a.shape
  out = np.empty((R, L))
  h = np.zeros(R)
  for k0 in range(0, L, K):
    k1 = min(k0 + K, L)
    P = np.cumprod(a[:, k0:k1], axis=1)
    out[:, k0:k1] = P * (h[:, None] + np.cumsum(b[:, k0:k1] / P, axis=1))
    h = out[:, k1 - 1]
  return out


def _fp64_fwd_bwd(g, x, dy, cu):
  """(y, dx, dg) in fp64 for rows [R, BL]; the backward uses the fp64 states."""
  g, x, dy = (np.asarray(v, dtype=np.float64) for v in (g, x, dy))
  assert g.min() > 1e-3, "the blocked check needs gates well above zero"
  y = np.full(g.shape, np.nan)
  dx = np.full(g.shape, np.nan)
  dg = np.full(g.shape, np.nan)
  for s, e in zip(cu[:-1], cu[1:]):
    s, e = int(s), int(e)
    if e <= s:
      continue
    y[:, s:e] = _fp64_scan_seg(g[:, s:e], x[:, s:e])
    c = np.ones((g.shape[0], e - s))
    c[:, 1:] = g[:, s + 1:e][:, ::-1]          # coefficient of dh[t+1] is g[t+1]
    d = _fp64_scan_seg(c, dy[:, s:e][:, ::-1])[:, ::-1]
    dx[:, s:e] = d
    dg[:, s] = 0.0
    dg[:, s + 1:e] = d[:, 1:] * y[:, s:e - 1]
  return y, dx, dg


def _worst_rel(ours: np.ndarray, gold: np.ndarray) -> float:
  """max |ours - gold| / (|gold| + rms(gold)) over the positions gold covers."""
  m = np.isfinite(gold)
  o, gg = np.asarray(ours, dtype=np.float64)[m], gold[m]
  if gg.size == 0:
    return 0.0
  scale = float(np.sqrt(np.mean(gg * gg)))
  return float(np.max(np.abs(o - gg) / (np.abs(gg) + scale)))


def _check_rows(g, x, dy, y, dx, dg, cu, rows) -> float:
  """Worst relative error of y, dx, dg over `rows` (device tensors, any dtype)."""
  idx = torch.as_tensor(list(rows), device=g.device, dtype=torch.long)
  host = [t.index_select(0, idx).double().cpu().numpy() for t in (g, x, dy, y, dx, dg)]
  cu_h = cu.cpu().numpy() if isinstance(cu, torch.Tensor) else np.asarray(cu)
  gy, gdx, gdg = _fp64_fwd_bwd(host[0], host[1], host[2], cu_h)
  return max(_worst_rel(host[3], gy), _worst_rel(host[4], gdx), _worst_rel(host[5], gdg))


def _sample_rows(n_rows: int, k: int, seed: int) -> list[int]:
  if n_rows <= k:
    return list(range(n_rows))
  rng = np.random.default_rng(seed)
  extra = rng.choice(np.arange(1, n_rows - 1), size=k - 2, replace=False).tolist()
  return sorted({0, n_rows - 1, *extra})


def _parity(dist, device, worst: float, rows: int, rtol: float) -> dict:
  worst = _reduce(dist, worst, device, "max")
  rows = int(_reduce(dist, float(rows), device, "sum"))
  return {"rows": rows, "outputs": ["y", "dx", "dg"], "max_err_rel": float(f"{worst:.3e}"),
          "rtol": rtol, "ok": bool(worst <= rtol),
          "gold": "fp64 sequential scan and its adjoint (blocked), same inputs"}


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------


def _time_steps(steps, fwd, bwd, device, dist):
  """K steps of fwd+bwd bracketed by barrier + synchronize; (step, fwd, bwd)
  ms, each the max over ranks."""
  ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
  _barrier(dist, device)
  torch.cuda.synchronize()
  start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  start.record()
  for i in range(steps):
    ev[i][0].record()
    fwd()
    ev[i][1].record()
    bwd()
    ev[i][2].record()
  stop.record()
  torch.cuda.synchronize()
  _barrier(dist, device)
  step_ms = start.elapsed_time(stop) / steps
  fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / steps
  bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / steps
  return (_reduce(dist, step_ms, device), _reduce(dist, fwd_ms, device),
          _reduce(dist, bwd_ms, device))


def _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, n_seq, chunk=512):
  grid = (n_seq, 1, g.shape[0])

  def fwd():
    ast.forward_scan_full(g, x, cu, grid, REVERSE=False, CHUNK_SIZE=chunk, TESTING=False,
                          tokens_out=y)

  def bwd():
    ast.backward_scan_fused_full(dy, g, y, dx, dg, cu, grid, CHUNK_SIZE=chunk, CAUSAL=True)

  return fwd, bwd


# ---------------------------------------------------------------------------
# legs of our arm
# ---------------------------------------------------------------------------


def _e2e(ast, device, g_dev, x_dev, dy_dev, cu, T_, steps: int) -> dict:
  """scan_causal fwd+bwd through the public API with host buffers every step.

  Every step uploads its three inputs from pinned host memory, runs
  ``scan_causal`` forward and ``backward``, and downloads y, d_gates and
  d_tokens into pinned host memory -- all inside the timed region.  As in a
  training input pipeline, the copies of neighbouring steps overlap: the
  uploads of step i+1 (copy-in stream) and the downloads of step i-1
  (copy-out stream) run while step i computes, on two input buffer sets."""
  def pinned_copy(t):
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h

  g_h, x_h, dy_h = pinned_copy(g_dev), pinned_copy(x_dev), pinned_copy(dy_dev)
  y_h = torch.empty(g_h.shape, dtype=g_h.dtype, pin_memory=True)
  dg_h = torch.empty(g_h.shape, dtype=g_h.dtype, pin_memory=True)
  dx_h = torch.empty(g_h.shape, dtype=g_h.dtype, pin_memory=True)
  bufs = [(torch.empty_like(g_dev), torch.empty_like(x_dev), torch.empty_like(dy_dev))
          for _ in range(2)]
  Cr = g_dev.shape[0]
  args = {"cu_seqlens": cu, "chunk_size": 512, "grid": ast.get_grid(len(cu), T_, 512, Cr)}
  compute = torch.cuda.current_stream(device)
  copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
  in_ready = [torch.cuda.Event() for _ in range(2)]
  slot_free = [torch.cuda.Event() for _ in range(2)]
  for ev in slot_free:
    ev.record(compute)

  def run(n_steps):
    for i in range(n_steps):
      k = i % 2
      g_b, x_b, dy_b = bufs[k]
      with torch.cuda.stream(copy_in):
        copy_in.wait_event(slot_free[k])   # step i-2 is done with this buffer set
        g_b.copy_(g_h, non_blocking=True)
        x_b.copy_(x_h, non_blocking=True)
        dy_b.copy_(dy_h, non_blocking=True)
        in_ready[k].record(copy_in)
      compute.wait_event(in_ready[k])
      g_l = g_b.detach().requires_grad_(True)
      x_l = x_b.detach().requires_grad_(True)
      y = ast.scan_causal(g_l, x_l, args)
      y.backward(dy_b)
      slot_free[k].record(compute)
      outs = (y.detach(), g_l.grad, x_l.grad)
      with torch.cuda.stream(copy_out):
        copy_out.wait_stream(compute)
        for t in outs:
          t.record_stream(copy_out)     # keep the results alive until they are read back
        y_h.copy_(outs[0], non_blocking=True)
        dg_h.copy_(outs[1], non_blocking=True)
        dx_h.copy_(outs[2], non_blocking=True)
    compute.wait_stream(copy_out)

  run(2)
  torch.cuda.synchronize()
  s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  s.record(compute)
  copy_in.wait_stream(compute)
  run(steps)
  e.record(compute)
  e.synchronize()
  ms = s.elapsed_time(e) / steps
  nbytes = g_dev.numel() * g_dev.element_size()
  del bufs, g_h, x_h, dy_h, y_h, dg_h, dx_h
  return {"ms_per_step": ms, "steps": steps, "h2d_bytes_per_step": 3 * nbytes,
          "d2h_bytes_per_step": 3 * nbytes,
          "overlap": "uploads of step i+1 and downloads of step i-1 overlap step i "
                     "(two input buffer sets, copy-in and copy-out streams)"}


def _configs1_replicas(ast, dist, rank, world, device, steps, warmup) -> dict:
  """configs[1] (B=8 x T=4096, C=1536, fp32), one full copy per rank: weak scaling."""
  g, x, dy, cu = _packed_problem(device, 0, C, T_C1, seed=4000 + 7 * rank)
  y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
  fwd, bwd = _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, B)
  for _ in range(warmup):
    fwd()
    bwd()
  step_ms, fwd_ms, bwd_ms = _time_steps(steps, fwd, bwd, device, dist)
  worst = _check_rows(g, x, dy, y, dx, dg, cu, _sample_rows(C, 6, 11 + rank))
  n = C * B * T_C1
  out = {"workload": f"causal fwd+bwd, B=8 packed x T=4096, C=1536, fp32 (configs[1]); "
                     f"one full copy per rank x{world} (weak scaling)",
         "ms_per_step": round(step_ms, 5), "fwd_ms": round(fwd_ms, 5), "bwd_ms": round(bwd_ms, 5),
         "gbs": round(STEP_BYTES_PER_ELEM * n * world / (step_ms * 1e-3) / 1e9, 1),
         "parity": _parity(dist, device, worst, min(C, 6), RTOL_F32)}
  del g, x, dy, y, dx, dg
  torch.cuda.empty_cache()
  return out


def _configs2_lengths():
  gen = torch.Generator().manual_seed(0)
  lens = torch.randint(64, 8193, (32,), generator=gen).tolist()
  return lens, [0, *np.cumsum(lens).tolist()]


def _sequence_shard_configs2(ast, dist, rank, world, device, steps, warmup) -> dict:
  """configs[2] (varlen, C=2048, 32 seeded lengths in [64, 8192], bf16 with fp32
  accumulation) split into whole-sequence shards (sharding.sequence_shards):
  rank k scans its own columns with rebased cu_seqlens, no collective.
  scan_causal + backward per step; GB/s counts 16 B per element (3 x 2 B fwd +
  5 x 2 B bwd) of the whole batch over the slowest rank's time."""
  from associative_scan_triton import sharding
  lens, cu_g = _configs2_lengths()
  C2 = 2048
  sh = sharding.sequence_shards(cu_g, world)[rank]
  width = sh.t1 - sh.t0
  n_total = C2 * cu_g[-1]
  step_ms, worst, checked = 0.0, 0.0, 0
  if width > 0:
    parts = {"g": [], "x": [], "dy": []}
    for i in range(sh.s0, sh.s1):  # each sequence seeded by its index: same data at every N
      L = lens[i]
      parts["g"].append(_rows_rand(range(C2), L, device, 7000 + 3 * i, "sig", torch.bfloat16))
      parts["x"].append(_rows_rand(range(C2), L, device, 7001 + 3 * i, "n", torch.bfloat16))
      parts["dy"].append(_rows_rand(range(C2), L, device, 7002 + 3 * i, "n", torch.bfloat16))
    g = torch.cat(parts["g"], 1).contiguous()
    x = torch.cat(parts["x"], 1).contiguous()
    dy = torch.cat(parts["dy"], 1).contiguous()
    del parts
    cu = torch.tensor(sh.local_cu, dtype=torch.int64, device=device)
    args = {"cu_seqlens": cu, "chunk_size": 512,
            "grid": ast.get_grid(len(cu), max(lens[sh.s0:sh.s1]), 512, C2)}
    res = {}

    def step():
      gl = g.detach().requires_grad_(True)
      xl = x.detach().requires_grad_(True)
      y = ast.scan_causal(gl, xl, args)
      y.backward(dy)
      res["y"], res["dg"], res["dx"] = y.detach(), gl.grad, xl.grad

    for _ in range(warmup):
      step()
  else:
    def step():
      return None

  _barrier(dist, device)
  torch.cuda.synchronize()
  s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  s.record()
  for _ in range(steps):
    step()
  e.record()
  torch.cuda.synchronize()
  _barrier(dist, device)
  step_ms = _reduce(dist, s.elapsed_time(e) / steps, device)
  if width > 0:
    rows = _sample_rows(C2, 4, 21 + rank)
    worst = _check_rows(g, x, dy, res["y"], res["dx"], res["dg"], cu, rows)
    checked = len(rows)
    del g, x, dy, res
    torch.cuda.empty_cache()
  return {"workload": f"causal fwd+bwd, C=2048, 32 sequences of seeded lengths in [64, 8192] "
                      f"(BL={cu_g[-1]}), bf16, scan_causal + backward; whole-sequence shards "
                      f"over {world} GPU(s), no collective",
          "shard_columns": width,
          "ms_per_step": round(step_ms, 4),
          "gbs": round(16 * n_total / (step_ms * 1e-3) / 1e9, 1),
          "parity": _parity(dist, device, worst, checked, RTOL_HALF)}


def _time_shard_5b(dist, rank: int, world: int, device, steps: int = 10,
                   exchange: str = "peer") -> dict:
  """configs[4]'s time-sharded case: C=256 channels of one sequence of T=2^20
  fp32 steps, gates ~ U(0.99, 1); rank k scans columns [kT/W, (k+1)T/W) and
  exchanges per-row carries once per direction (``exchange``: "peer", one
  kernel over NVLink peer memory that publishes, waits and folds; or "nccl",
  an all-gather and a fold kernel).  At W=1 the same
  workload runs as an ordinary single-GPU scan.  Device time per fwd+bwd step,
  max over ranks; GB/s counts the single-device algorithmic bytes (32 B per
  element), so the second reads of the two passes show up as a lower rate.
  The slabs of a sample of rows are gathered on rank 0 and checked against the
  fp64 scan of the whole axis."""
  import associative_scan_triton as ast
  from associative_scan_triton import time_shard as ts
  bounds = ts.even_bounds(TS_T, world, align=64)
  t0, t1 = bounds[rank], bounds[rank + 1]
  L = t1 - t0

  def slab(seed, law):  # columns [t0, t1) of every row, seeded per 2^17-column chunk
    out = torch.empty(TS_C, L, device=device)
    gen = torch.Generator(device=device)
    for c0 in range(t0 - t0 % TS_CHUNK, t1, TS_CHUNK):
      a, b = max(c0, t0), min(c0 + TS_CHUNK, t1)
      gen.manual_seed(seed * 1_000_003 + c0 // TS_CHUNK)
      chunk = (torch.rand if law == "u" else torch.randn)(TS_C, TS_CHUNK, device=device,
                                                          generator=gen)
      out[:, a - t0:b - t0] = chunk[:, a - c0:b - c0]
      del chunk
    if law == "u":
      out.mul_(0.01).add_(0.99)
    return out

  g, x, dy = slab(99, "u"), slab(98, "n"), slab(97, "n")
  plans = ts.plan_slabs([0, TS_T], bounds)
  res = {}
  step_obj = None
  if world > 1:
    step_obj = ts.TimeShardStep(g.shape, g.dtype, plans, rank, device, exchange=exchange,
                                timeout_s=10.0)

    def fwd():
      res["y"] = step_obj.forward(g, x)

    def bwd():
      res["dg"], res["dx"] = step_obj.backward(dy, g, res["y"])
  else:
    cu = torch.tensor([0, TS_T], dtype=torch.int32, device=device)
    grid = (1, 1, TS_C)
    y1, dx1, dg1 = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    res.update(y=y1, dx=dx1, dg=dg1)

    def fwd():
      ast.forward_scan_full(g, x, cu, grid, REVERSE=False, CHUNK_SIZE=512, TESTING=False,
                            tokens_out=y1)

    def bwd():
      ast.backward_scan_fused_full(dy, g, y1, dx1, dg1, cu, grid, CHUNK_SIZE=512, CAUSAL=True)
  for _ in range(3):
    fwd()
    bwd()
  phases, graph, mode = None, None, "eager"
  if world > 1:
    # one eager step with an event after every phase (CUDA events) and host
    # timestamps around the enqueue, then the step captured in a CUDA graph
    # (kernels and NCCL collectives replayed without host work)
    marks = [torch.cuda.Event(enable_timing=True)]
    torch.cuda.synchronize()
    _barrier(dist, device)
    h0 = time.perf_counter()
    marks[0].record()
    y_ph = step_obj.forward(g, x, marks=marks)
    step_obj.backward(dy, g, y_ph, marks=marks)
    h1 = time.perf_counter()
    torch.cuda.synchronize()
    if exchange == "peer":
      names = ["fwd_aggregate", "fwd_exchange_and_fold", "fwd_none", "fwd_seeded",
               "bwd_aggregate", "bwd_edges_exchange_and_fold", "bwd_none", "bwd_seeded"]
    else:
      names = ["fwd_aggregate", "fwd_all_gather", "fwd_fold", "fwd_seeded",
               "bwd_aggregate_and_edges", "bwd_all_gather", "bwd_fold", "bwd_seeded"]
    phases = {n: round(_reduce(dist, 1e3 * a.elapsed_time(b), device), 1)
              for n, a, b in zip(names, marks, marks[1:]) if not n.endswith("_none")}
    phases["host_enqueue"] = round(_reduce(dist, 1e6 * (h1 - h0), device), 1)
    phases["unit"] = "us, max over ranks"
    try:
      side = torch.cuda.Stream(device)
      side.wait_stream(torch.cuda.current_stream(device))
      with torch.cuda.stream(side):
        fwd()
        bwd()
      torch.cuda.current_stream(device).wait_stream(side)
      graph = torch.cuda.CUDAGraph()
      with torch.cuda.graph(graph):
        fwd()
        bwd()
      mode = "cuda_graph"
    except Exception as e:  # eager steps remain valid
      graph, mode = None, f"eager (graph capture failed: {type(e).__name__})"
  if graph is not None:
    step_ms, fwd_ms, _ = _time_steps(steps, graph.replay, lambda: None, device, dist)
    fwd_ms = None  # one replay per step: no fwd/bwd split
  else:
    step_ms, fwd_ms, _ = _time_steps(steps, fwd, bwd, device, dist)
  # parity: rank 0 checks a sample of rows over the whole axis
  rows = _sample_rows(TS_C, 4, 5)
  idx = torch.as_tensor(rows, device=device)
  pieces = [t.index_select(0, idx).contiguous() for t in (g, x, dy, res["y"], res["dx"], res["dg"])]
  if dist is not None:
    full = []
    for p in pieces:
      bufs = [torch.empty_like(p) for _ in range(world)]
      dist.all_gather(bufs, p)  # equal slabs: 2^20 splits evenly
      full.append(torch.cat(bufs, 1))
    pieces = full
  worst = 0.0
  if rank == 0:
    cu_all = np.array([0, TS_T])
    h = [p.double().cpu().numpy() for p in pieces]
    gy, gdx, gdg = _fp64_fwd_bwd(h[0], h[1], h[2], cu_all)
    worst = max(_worst_rel(h[3], gy), _worst_rel(h[4], gdx), _worst_rel(h[5], gdg))
  parity = _parity(dist, device, worst, len(rows) if rank == 0 else 0, RTOL_F32)
  n = TS_C * TS_T
  del graph  # released before the process group is destroyed
  if step_obj is not None:
    step_obj.close()  # collective: unmaps the peers' exchange buffers, frees this rank's
  del g, x, dy, res, pieces
  torch.cuda.empty_cache()
  out = {"workload": f"causal fwd+bwd, C={TS_C}, one sequence of T=2^20, fp32, "
                     f"time-sharded over {world} GPU(s) (configs[4] case 5b)",
         "ms_per_step": round(step_ms, 4),
         "fwd_ms": round(fwd_ms, 4) if fwd_ms is not None else None,
         "step_mode": mode}
  if phases is not None:
    out["phases_eager_step"] = phases
  return {**out,
          "gbs": round(STEP_BYTES_PER_ELEM * n / (step_ms * 1e-3) / 1e9, 1),
          "exchange": ("one kernel per direction over NVLink peer memory (CUDA IPC): "
                       "publishes this rank's [C,2] fwd / [C,4] bwd record, waits for the "
                       "ranks it depends on, reads their records and folds the carry; no "
                       "collective" if exchange == "peer" else
                       "one NCCL all-gather into a preallocated buffer per direction "
                       "([C,2] fwd, [C,4] bwd floats per rank); carries folded on the device")
          if world > 1 else "none (single GPU)",
          "parity": parity}


def _sweep(ast, device) -> list[dict]:
  """fwd and fwd+bwd at B=8, C=1536, T=128..65536 (fp32), L2 flushed when inputs fit in it."""
  out = []
  flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
  for Tn in [2**i for i in range(7, 17)]:
    gen = torch.Generator(device=device).manual_seed(100 + Tn)
    BL = B * Tn
    g = 0.9 + 0.1 * torch.rand(C, BL, device=device, generator=gen)
    x = torch.randn(C, BL, device=device, generator=gen)
    dy = torch.randn(C, BL, device=device, generator=gen)
    cu = torch.arange(B + 1, device=device, dtype=torch.int32) * Tn
    y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    fwd, bwd = _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, B)
    n = C * BL
    small = 3 * n * 4 < L2_BYTES * 2
    reps = 30 if Tn <= 8192 else 10
    res = {}
    for name, fns in (("fwd", (fwd,)), ("fwdbwd", (fwd, bwd))):
      for _ in range(3):
        for f in fns:
          f()
      times = []
      for _ in range(reps):
        if small:
          flush.fill_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for f in fns:
          f()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
      ms = statistics.median(times)
      bpe = FWD_BYTES_PER_ELEM if name == "fwd" else STEP_BYTES_PER_ELEM
      res[f"{name}_ms"] = round(ms, 5)
      res[f"{name}_gbs"] = round(bpe * n / (ms * 1e-3) / 1e9, 1)
    out.append({"T": Tn, **res})
    del g, x, dy, y, dx, dg
    torch.cuda.empty_cache()
  return out


def _small_t_graph(ast, device, reps: int = 200) -> dict:
  """The launch-bound end of the sweep: B=8 sequences of T=128, C=1536 fp32,
  one causal fwd+bwd step through the dispatcher API, called eagerly and
  replayed from a CUDA graph captured once (same work, no host overhead)."""
  from associative_scan_triton import _lib
  Tn = 128
  g, x, dy, cu = _packed_problem(device, 0, C, Tn, seed=7)
  y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
  fwd, bwd = _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, B, chunk=128)

  def step():
    fwd()
    bwd()

  def timed(fn):
    for _ in range(10):
      fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
      fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / reps

  eager_ms = timed(step)
  side = torch.cuda.Stream(device)
  side.wait_stream(torch.cuda.current_stream(device))
  with torch.cuda.stream(side):
    step()
  torch.cuda.current_stream(device).wait_stream(side)
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph):
    step()
  graph_ms = timed(graph.replay)
  _lib.check_device_error(device)
  del graph
  n = g.numel()
  return {"workload": "causal fwd+bwd, B=8 x T=128, C=1536, fp32", "eager_ms_per_step":
          round(eager_ms, 4), "graph_ms_per_step": round(graph_ms, 4),
          "graph_gbs": round(STEP_BYTES_PER_ELEM * n / (graph_ms * 1e-3) / 1e9, 1)}


def _bidi_inputs(device):
  Tn, C3 = 2048, 1536
  BL = B * Tn
  gen = torch.Generator(device=device).manual_seed(4)
  ts_ = [torch.rand(C3, BL, device=device, generator=gen).half() if k in (0, 2) else
         torch.randn(C3, BL, device=device, generator=gen).half() for k in range(6)]
  cu = torch.arange(B + 1, device=device, dtype=torch.int32) * Tn
  return ts_, cu, Tn, C3


def _bidi_configs3(ast, device, reps: int = 20) -> dict:
  """configs[3] through the public autograd API (device-resident inputs, fwd +
  backward per step, CUDA events; 3s fwd + 5s bwd bytes per element and
  direction, s = 2)."""
  (gf, xf, gb, xb, dyf, dyb), cu, Tn, C3 = _bidi_inputs(device)
  args = {"cu_seqlens": cu, "chunk_size": 128, "grid": ast.get_grid(len(cu), Tn, 128, C3)}

  def bidi_step():
    ins = [t.detach().requires_grad_(True) for t in (gf, xf, gb, xb)]
    yf, yb = ast.scan_bidirectional_branched(*ins, args)
    torch.autograd.backward([yf, yb], [dyf, dyb])

  for _ in range(3):
    bidi_step()
  torch.cuda.synchronize()
  s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  s.record()
  for _ in range(reps):
    bidi_step()
  e.record()
  e.synchronize()
  ms = s.elapsed_time(e) / reps
  from associative_scan_triton import _lib
  _lib.check_device_error(device)
  n = gf.numel()
  return {"workload": "scan_bidirectional_branched fwd+bwd, B=8 x T=2048, C=1536, fp16, "
                      "independent gate/token pairs per direction",
          "ms_per_step": round(ms, 4), "gbs": round(2 * 16 * n / (ms * 1e-3) / 1e9, 1)}


def _cpu_sample(threads: int, seconds: float, seed: int = 0) -> dict:
  """The reference's CPU algorithm (fp64 sequential scan, oracle port) on a
  channel sample of the headline workload, timed on `threads` host threads."""
  from oracle import oracle
  BL = B * T_HEAD
  rng = np.random.default_rng(seed)
  cu = np.arange(B + 1, dtype=np.int64) * T_HEAD

  def inputs(c):
    return (rng.uniform(0.9, 1.0, size=(c, BL)).astype(np.float32),
            rng.standard_normal((c, BL), dtype=np.float32),
            rng.standard_normal((c, BL), dtype=np.float32))

  g, x, dy = inputs(threads)
  t0 = time.perf_counter()
  oracle.scan_fwd_bwd(g, x, dy, cu, nthreads=threads)  # warm + per-channel cost
  per_pass = time.perf_counter() - t0
  c_sample = int(min(C, max(threads, threads * round(seconds / max(per_pass, 1e-6)))))
  g, x, dy = inputs(c_sample)
  t0 = time.perf_counter()
  oracle.scan_fwd_bwd(g, x, dy, cu, nthreads=threads)
  dt = time.perf_counter() - t0
  return {"c_sample": c_sample, "seconds": dt, "elements": c_sample * BL}


def _cpu_baseline(seconds: float = 10.0) -> dict:
  threads = os.cpu_count() or 1
  r = _cpu_sample(threads, seconds)
  return {"value": round(STEP_BYTES_PER_ELEM * r["elements"] / r["seconds"] / 1e9, 3),
          "unit": "GB/s", "cores": threads, "kind": "port",
          "sample": (f"one fwd+bwd pass over {r['c_sample']} of {C} channels x B*T={B * T_HEAD} "
                     f"(fp32 in, fp64 sequential, OpenMP over channels on {threads} threads), "
                     f"{r['seconds']:.1f} s; same 32 B/elem accounting"),
          "ms_per_full_step_equiv": round(r["seconds"] / r["elements"] * C * B * T_HEAD * 1e3, 1)}


def _headline_config(world: int) -> dict:
  return {
    "workload": f"causal fwd+bwd, B={B} packed x T={T_HEAD}, C={C}, fp32 (configs[4] case 5a)",
    "elements": C * B * T_HEAD, "bytes_per_element_fwd_bwd": STEP_BYTES_PER_ELEM,
    "api": "forward_scan_full + backward_scan_fused_full -> C ABI",
    "l2": "inputs larger than L2 (3.2 GB per tensor at N=1, 403 MB per rank at N=8); no flush",
    "parallelism": f"channel blocks x{world} (one fixed problem, no collective on the data path)",
  }


def run_ours(args) -> tuple[dict | None, bool]:
  dist, rank, world, local = _dist_setup()
  device = torch.device("cuda", local)
  torch.cuda.set_device(device)
  import associative_scan_triton as ast
  from associative_scan_triton import _lib, sharding
  _lib.load()
  _lib.set_sync_check(False)

  c0, c1 = sharding.channel_block(C, world, rank)
  g, x, dy, cu = _packed_problem(device, c0, c1, T_HEAD, seed=1234)
  y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
  n_rank = (c1 - c0) * B * T_HEAD
  n_total = C * B * T_HEAD
  fwd, bwd = _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, B)

  sampler = ClockSampler(local).start() if rank == 0 else None
  for _ in range(args.warmup):
    fwd()
    bwd()
  torch.cuda.synchronize()
  _lib.check_device_error(device)
  ms_per_step, fwd_ms, bwd_ms = _time_steps(args.steps, fwd, bwd, device, dist)
  _lib.check_device_error(device)
  clocks = sampler.stop() if sampler else None
  worst = _check_rows(g, x, dy, y, dx, dg, cu, _sample_rows(c1 - c0, 8, 31 + rank))
  head_parity = _parity(dist, device, worst, min(8, c1 - c0), RTOL_F32)
  value = STEP_BYTES_PER_ELEM * n_total / (ms_per_step * 1e-3) / 1e9
  del y, dx, dg
  torch.cuda.empty_cache()

  e2e_steps = max(3, min(args.steps, 5))
  e2e = _e2e(ast, device, g, x, dy, cu, T_HEAD, e2e_steps)
  e2e_ms = _reduce(dist, e2e["ms_per_step"], device)
  del g, x, dy
  torch.cuda.empty_cache()

  extra = {}
  if not args.no_secondary:
    extra["configs1_replicas"] = _configs1_replicas(ast, dist, rank, world, device,
                                                    min(args.steps, 50), 3)
    extra["sequence_shard_configs2"] = _sequence_shard_configs2(ast, dist, rank, world, device,
                                                                min(args.steps, 20), 3)
    extra["time_shard"] = _time_shard_5b(dist, rank, world, device, exchange="peer")
    if world > 1:  # the same step with the collective exchange, for comparison
      extra["time_shard_nccl"] = _time_shard_5b(dist, rank, world, device, exchange="nccl")

  if dist is not None:
    _barrier(dist, device)
    dist.destroy_process_group()
  parities = [head_parity] + [v["parity"] for v in extra.values()]
  all_ok = all(p["ok"] for p in parities)
  if rank != 0:
    return None, all_ok

  peak, peak_kind = _peaks()
  bwd_achieved = BWD_BYTES_PER_ELEM * n_rank / (bwd_ms * 1e-3) / 1e9
  fwd_achieved = FWD_BYTES_PER_ELEM * n_rank / (fwd_ms * 1e-3) / 1e9
  line = {
    "metric": METRIC,
    "value": round(value, 1),
    "unit": "GB/s",
    "n_gpus": world,
    "steps": args.steps,
    "warmup": args.warmup,
    "ms_per_step": round(ms_per_step, 5),
    "higher_is_better": True,
    "scaling": "strong",
    "vs_baseline": None,
    "dtype": "f32",
    "data": "synthetic (seeded per 64-channel block; gates U(0.9,1), tokens N(0,1), dy N(0,1))",
    "config": _headline_config(world),
    "fwd_ms": round(fwd_ms, 5),
    "fwd_gbs": round(FWD_BYTES_PER_ELEM * n_total / (fwd_ms * 1e-3) / 1e9, 1),
    "bwd_ms": round(bwd_ms, 5),
    "roofline": {
      "bound": "hbm", "kernel": "scan_bwd_tma_kernel (fused backward, persistent TMA)",
      "achieved": round(bwd_achieved, 1), "peak": peak, "unit": "GB/s",
      "frac": round(bwd_achieved / peak, 4), "peak_kind": f"{peak_kind} copy bandwidth",
      "traffic": _profile_traffic(n_rank),
      "algorithmic_bytes_per_launch": BWD_BYTES_PER_ELEM * n_rank,
      "elements_per_launch": n_rank,
      "fwd_achieved": round(fwd_achieved, 1),
      "fwd_frac": round(fwd_achieved / peak, 4),
      "frac_of_8000_nominal": round(bwd_achieved / 8000.0, 4),
    },
    "parity": head_parity,
    "e2e": {
      "value": round(STEP_BYTES_PER_ELEM * n_total / (e2e_ms * 1e-3) / 1e9, 2),
      "unit": "GB/s", "ms_per_step": round(e2e_ms, 3), "steps": e2e["steps"],
      "h2d_bytes_per_step": e2e["h2d_bytes_per_step"] * world,
      "d2h_bytes_per_step": e2e["d2h_bytes_per_step"] * world,
      "api": "scan_causal(g, x, args) + y.backward(dy), pinned host buffers",
      "overlap": e2e["overlap"],
    },
    "gpu_launches": 2 * args.steps,
    "clocks": clocks,
  }
  line.update(extra)
  if not args.no_sweep and world == 1:
    line["sweep_B8_C1536_fp32"] = _sweep(ast, device)
    line["small_t_graph"] = _small_t_graph(ast, device)
    line["bidi_configs3"] = _bidi_configs3(ast, device)
  if not args.no_cpu_baseline and world == 1:
    line["cpu_baseline"] = _cpu_baseline(args.cpu_seconds)
  if not args.no_reference_triton and world == 1:
    line["reference_triton_b200"] = _reference_triton_context()
  return line, all_ok


# ---------------------------------------------------------------------------
# context: the reference's own Triton kernels on the same GPU
# ---------------------------------------------------------------------------


def _reference_triton_child(args) -> int:
  """Runs in a child process whose sys.path holds only the reference's
  unmodified package (baseline/_ref): times its forward_scan_full +
  backward_scan_fused_full (reference src/associative_scan_triton/
  _dispatcher.py:12-117, Triton kernels of _kernels.py:84-287) at configs[1]
  and at the headline shape, fp32, chunk_size 512, one GPU; prints one JSON."""
  import associative_scan_triton as ref
  device = torch.device("cuda", 0)
  out = {"source": "reference package " + str(Path(ref.__file__).parent.relative_to(REPO)),
         "api": "forward_scan_full(TESTING=False, tokens_out=y) + backward_scan_fused_full",
         "chunk_size": 512}
  for name, Tn in (("configs1_T4096", T_C1), ("headline_T65536", T_HEAD)):
    g, x, dy, cu = _packed_problem(device, 0, C, Tn, seed=1234)
    y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    grid = ref.get_grid(len(cu), Tn, 512, C)

    def fwd():
      ref.forward_scan_full(g, x, cu, grid, REVERSE=False, CHUNK_SIZE=512, TESTING=False,
                            tokens_out=y)

    def bwd():
      ref.backward_scan_fused_full(dy, g, y, dx, dg, cu, grid, CHUNK_SIZE=512, CAUSAL=True)

    for _ in range(3):  # includes Triton's compilation
      fwd()
      bwd()
    torch.cuda.synchronize()
    reps = 20 if Tn == T_C1 else 5
    res = {}
    for key, fns in (("fwd", (fwd,)), ("fwdbwd", (fwd, bwd))):
      times = []
      for _ in range(reps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        for f in fns:
          f()
        e_.record()
        e_.synchronize()
        times.append(s_.elapsed_time(e_))
      ms = statistics.median(times)
      bpe = FWD_BYTES_PER_ELEM if key == "fwd" else STEP_BYTES_PER_ELEM
      res[f"{key}_ms"] = round(ms, 4)
      res[f"{key}_gbs"] = round(bpe * g.numel() / (ms * 1e-3) / 1e9, 1)
    worst = _check_rows(g, x, dy, y, dx, dg, cu, [0, C // 2, C - 1])
    res["max_err_rel_vs_fp64"] = float(f"{worst:.3e}")
    out[name] = res
    del g, x, dy, y, dx, dg
    torch.cuda.empty_cache()
  print(json.dumps(out), flush=True)
  return 0


def _reference_triton_context() -> dict:
  """The reference's Triton kernels timed on this GPU (context for the
  comparison; the reference arm of the contract is its CPU algorithm)."""
  if not (REF_TREE / "associative_scan_triton" / "__init__.py").exists():
    return {"unavailable": "baseline/_ref holds no copy of the reference package"}
  torch.cuda.empty_cache()
  try:
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--reference-triton-child"],
                       capture_output=True, text=True, timeout=600)
  except subprocess.TimeoutExpired:
    return {"unavailable": "the reference's Triton run exceeded 600 s"}
  lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
  if r.returncode != 0 or not lines:
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"reference Triton run failed (rc {r.returncode}): {tail[0][:200]}"}
  return json.loads(lines[-1])


# ---------------------------------------------------------------------------
# profile cases (one workload, no contract line; for ncu captures)
# ---------------------------------------------------------------------------


def run_profile_case(args) -> int:
  import associative_scan_triton as ast
  from associative_scan_triton import _lib
  device = torch.device("cuda", 0)
  torch.cuda.set_device(device)
  _lib.load()
  _lib.set_sync_check(False)
  name = args.profile_case
  if name in ("headline_rank8", "configs1"):
    Cn, Tn = (C // 8, T_HEAD) if name == "headline_rank8" else (C, T_C1)
    g, x, dy, cu = _packed_problem(device, 0, Cn, Tn, seed=1234)
    y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    fwd, bwd = _dispatcher_ops(ast, g, x, dy, cu, y, dx, dg, B)

    def step():
      fwd()
      bwd()
  elif name == "varlen_bf16":
    lens, cu_g = _configs2_lengths()
    C2 = 2048
    g = torch.sigmoid(2.0 + torch.randn(C2, cu_g[-1], device=device)).to(torch.bfloat16)
    x = torch.randn(C2, cu_g[-1], device=device).to(torch.bfloat16)
    dy = torch.randn(C2, cu_g[-1], device=device).to(torch.bfloat16)
    cu = torch.tensor(cu_g, dtype=torch.int64, device=device)
    sargs = {"cu_seqlens": cu, "chunk_size": 512, "grid": ast.get_grid(len(cu), max(lens), 512, C2)}

    def step():
      gl, xl = g.detach().requires_grad_(True), x.detach().requires_grad_(True)
      ast.scan_causal(gl, xl, sargs).backward(dy)
  elif name == "bidi_fp16":
    (gf, xf, gb, xb, dyf, dyb), cu, Tn, C3 = _bidi_inputs(device)
    sargs = {"cu_seqlens": cu, "chunk_size": 128, "grid": ast.get_grid(len(cu), Tn, 128, C3)}

    def step():
      ins = [t.detach().requires_grad_(True) for t in (gf, xf, gb, xb)]
      yf, yb = ast.scan_bidirectional_branched(*ins, sargs)
      torch.autograd.backward([yf, yb], [dyf, dyb])
  elif name == "time_shard_emulated":
    from associative_scan_triton import time_shard as ts
    bounds = ts.even_bounds(TS_T, 8, align=64)
    plans = ts.plan_slabs([0, TS_T], bounds)
    gs = [0.99 + 0.01 * torch.rand(TS_C, TS_T // 8, device=device) for _ in range(8)]
    xs = [torch.randn(TS_C, TS_T // 8, device=device) for _ in range(8)]
    dys = [torch.randn(TS_C, TS_T // 8, device=device) for _ in range(8)]

    def step():
      ys = ts.emulate_forward(gs, xs, plans)
      ts.emulate_backward(dys, gs, ys, plans)
  else:
    raise SystemExit(f"unknown profile case {name!r}")
  for _ in range(args.warmup):
    step()
  torch.cuda.synchronize()
  s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  s.record()
  for _ in range(args.steps):
    step()
  e.record()
  e.synchronize()
  _lib.check_device_error(device)
  print(f"profile case {name}: {s.elapsed_time(e) / args.steps:.4f} ms per step "
        f"({args.steps} steps after {args.warmup} warm-up)", flush=True)
  return 0


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm (oracle port) on host cores
# ---------------------------------------------------------------------------


def run_reference(args) -> dict | None:
  rank = int(os.environ.get("RANK", "0"))
  world = int(os.environ.get("WORLD_SIZE", "1"))
  if rank != 0:
    return None
  from oracle import oracle
  # every host thread (torchrun sets OMP_NUM_THREADS=1 for its ranks; the
  # other ranks of this arm exit at once, so the cores are free)
  threads = os.cpu_count() or 1
  BL = B * T_HEAD
  cu = np.arange(B + 1, dtype=np.int64) * T_HEAD
  rng = np.random.default_rng(0)
  budget_s = 90.0
  probe_c = threads
  g = rng.uniform(0.9, 1.0, size=(probe_c, BL)).astype(np.float32)
  x = rng.standard_normal((probe_c, BL), dtype=np.float32)
  dy = rng.standard_normal((probe_c, BL), dtype=np.float32)
  t0 = time.perf_counter()
  oracle.scan_fwd_bwd(g, x, dy, cu, nthreads=threads)
  per_wave = time.perf_counter() - t0      # one pass over `threads` channels
  per_step_s = min(4.0, budget_s / max(1, args.steps + args.warmup))
  waves = int(max(1, min(C // threads if C >= threads else 1, per_step_s / max(per_wave, 1e-9))))
  c_sample = min(C, waves * threads)
  g = rng.uniform(0.9, 1.0, size=(c_sample, BL)).astype(np.float32)
  x = rng.standard_normal((c_sample, BL), dtype=np.float32)
  dy = rng.standard_normal((c_sample, BL), dtype=np.float32)
  for _ in range(args.warmup):
    oracle.scan_fwd_bwd(g, x, dy, cu, nthreads=threads)
  t0 = time.perf_counter()
  for _ in range(args.steps):
    oracle.scan_fwd_bwd(g, x, dy, cu, nthreads=threads)
  dt = time.perf_counter() - t0
  ms_per_step = dt / args.steps * 1e3
  elems = c_sample * BL
  value = STEP_BYTES_PER_ELEM * elems / (ms_per_step * 1e-3) / 1e9
  sample = (f"each step: causal fwd+bwd over {c_sample} of {C} channels x B*T={BL} "
            f"(fp32 in, fp64 sequential scan, OpenMP over channels on {threads} threads); "
            f"GB/s of the same 32 B/elem accounting")
  return {
    "impl": "reference",
    "metric": METRIC,
    "value": round(value, 3),
    "unit": "GB/s",
    "n_gpus": world,
    "steps": args.steps,
    "warmup": args.warmup,
    "ms_per_step": round(ms_per_step, 3),
    "higher_is_better": True,
    "scaling": "strong",
    "vs_baseline": None,
    "dtype": "f64",
    "data": "synthetic (seeded; gates U(0.9,1), tokens N(0,1), dy N(0,1))",
    "config": _headline_config(world),
    "implementation": "reference CPU algorithm (sequential_scan_gold + hand-derived backward), "
                      "restated in C (oracle/ascan_oracle.c), rank 0 only",
    "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                     "sample": sample},
    "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
            "d2h_bytes_per_step": 0},
  }


def main(argv=None) -> int:
  ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=100)
  ap.add_argument("--warmup", type=int, default=10)
  ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
  ap.add_argument("--no-sweep", action="store_true")
  ap.add_argument("--no-cpu-baseline", action="store_true")
  ap.add_argument("--no-secondary", action="store_true",
                  help="skip configs1_replicas, sequence_shard_configs2 and time_shard")
  ap.add_argument("--cpu-seconds", type=float, default=10.0)
  ap.add_argument("--profile-case", default=None)
  ap.add_argument("--no-reference-triton", action="store_true",
                  help="skip timing the reference's Triton kernels (context key)")
  ap.add_argument("--reference-triton-child", action="store_true", help=argparse.SUPPRESS)
  args = ap.parse_args(argv)
  args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
  if args.reference_triton_child:
    return _reference_triton_child(args)
  if args.profile_case:
    return run_profile_case(args)
  if args.impl == "reference":
    line = run_reference(args)
    if line is not None:
      print(json.dumps(line), flush=True)
    return 0
  line, ok = run_ours(args)
  if line is not None:
    print(json.dumps(line), flush=True)
  if not ok:
    print("bench: parity check FAILED (see the parity objects)", file=sys.stderr, flush=True)
    return 3
  return 0


if __name__ == "__main__":
  sys.exit(main())
