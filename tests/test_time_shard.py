"""Time-sharded causal scan: slabs of one long sequence axis.

GPU tests run every slab of a problem on one device through the same passes
and carry folds as the multi-rank driver (``emulate_forward`` /
``emulate_backward``) and compare the concatenated slabs with the fp64 oracle
on the whole axis.  CPU tests run the exchange and the folds as 2-4 ``gloo``
ranks on aggregates computed in numpy from their definitions, and check the
carries against the oracle's states at the slab edges.  A real multi-GPU run
(NCCL, one rank per GPU) is ``test_nccl_ranks_match_oracle`` and needs at
least two GPUs.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from associative_scan_triton import time_shard as ts
from oracle import oracle
from scan_testlib import assert_close_to_gold, make_inputs

REPO = Path(__file__).resolve().parent.parent


# --- host geometry ---------------------------------------------------------------------

def test_plan_slabs_rebases_boundaries():
  plans = ts.plan_slabs([0, 100, 256, 300, 512], [0, 256, 512])
  assert plans[0].local_cu == (0, 100, 256) and plans[0].starts_new and plans[0].inner_boundary
  assert plans[1].local_cu == (0, 44, 256) and plans[1].starts_new and plans[1].inner_boundary
  one = ts.plan_slabs([0, 1000], [0, 256, 512, 1000])
  assert [p.starts_new for p in one] == [True, False, False]
  assert [p.last_piece_continues for p in one] == [False, True, True]
  with pytest.raises(ValueError):
    ts.plan_slabs([0, 5, 3, 10], [0, 10])
  with pytest.raises(ValueError):
    ts.plan_slabs([0, 10], [0, 4, 4, 10])


def test_even_bounds():
  assert ts.even_bounds(1 << 20, 8) == [k * (1 << 17) for k in range(9)]
  b = ts.even_bounds(1000, 3, align=8)
  assert b[0] == 0 and b[-1] == 1000 and all(x % 8 == 0 for x in b[:-1])
  with pytest.raises(ValueError):
    ts.even_bounds(10, 4, align=8)


# --- numpy definitions of the per-slab records (fp64) ----------------------------------

def _fwd_aggregate(g, x, plan):
  """(P, Y) per row: gate product since the last local boundary, state from 0."""
  C, L = g.shape
  last = max(b for b in plan.local_cu if b < L)
  P = np.prod(g[:, last:], axis=1)
  y = np.zeros(C)
  for t in range(last, L):
    y = g[:, t] * y + x[:, t]
  return np.stack([P, y], axis=1)


def _bwd_aggregate(dy, g, plan):
  """(Q, D) per row at column 0 from a zero carry: the adjoint and the product
  of the coefficients g[t+1] since the nearest sequence end at or after it
  (that end's own coefficient included; the slab's last column counts 1)."""
  C, L = g.shape
  ends = {b - 1 for b in plan.local_cu[1:]}
  dh = np.zeros(C)
  q = np.ones(C)
  for t in range(L - 1, -1, -1):
    coeff = g[:, t + 1] if t + 1 < L else np.ones(C)
    if t in ends:  # a sequence ends at t: the recurrence restarts
      dh = dy[:, t].copy()
      q = coeff.copy()
    else:
      dh = dy[:, t] + coeff * dh
      q = q * coeff
  return np.stack([q, dh], axis=1)


def _protocol_worker(rank, world, port, C, T, cu, seed, errq):
  import torch.distributed as dist
  try:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(seed)
    g = rng.uniform(0.9, 1.0, size=(C, T))
    x = rng.standard_normal((C, T))
    dy = rng.standard_normal((C, T))
    bounds = ts.even_bounds(T, world, align=8)
    plans = ts.plan_slabs(cu, bounds)
    t0, t1 = bounds[rank], bounds[rank + 1]
    gather = ts._all_gather
    agg = torch.from_numpy(_fwd_aggregate(g[:, t0:t1], x[:, t0:t1], plans[rank]))
    carry = ts.forward_carry(plans, gather(agg), rank)
    bagg = torch.from_numpy(_bwd_aggregate(dy[:, t0:t1], g[:, t0:t1], plans[rank]))
    firsts = [r.reshape(-1) for r in gather(torch.from_numpy(g[:, t0].copy()))]
    bcarry = ts.backward_carry(plans, gather(bagg), firsts, rank)
    # oracle on the whole axis: the state before t0 and the adjoint after t1
    cu_t = torch.tensor(cu, dtype=torch.int64)
    y_full, a_full = oracle.scan_fwd(torch.from_numpy(g).float(), torch.from_numpy(x).float(), cu_t)
    h_prev = y_full[:, t0 - 1] if (rank > 0 and not plans[rank].starts_new) else np.zeros(C)
    np.testing.assert_allclose(carry[:, 1].numpy(), h_prev, rtol=1e-5, atol=1e-5)
    if rank > 0 and not plans[rank].starts_new:
      np.testing.assert_allclose(carry[:, 0].numpy(), a_full[:, t0 - 1], rtol=1e-5, atol=1e-12)
    dx_full, _ = oracle.scan_bwd(torch.from_numpy(dy).float(), torch.from_numpy(g).float(),
                                 torch.from_numpy(y_full).float(), cu_t)
    if rank < world - 1 and not plans[rank + 1].starts_new:
      want = g[:, t1].astype(np.float32).astype(np.float64) * dx_full[:, t1]
    else:
      want = np.zeros(C)
    np.testing.assert_allclose(bcarry.numpy(), want, rtol=1e-5, atol=1e-5)
    dist.destroy_process_group()
  except BaseException as e:  # reported to the parent
    errq.put(f"rank {rank}: {type(e).__name__}: {e}")
    raise


def _free_port() -> int:
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


@pytest.mark.parametrize(("world", "cu"), [
  (2, [0, 512]),                       # one sequence across both slabs
  (4, [0, 512]),
  (4, [0, 100, 128, 300, 512]),        # boundaries inside slabs and on a slab edge
  (3, [0, 17, 400, 401, 512]),
])
def test_exchange_and_folds_on_gloo_ranks(world, cu):
  import multiprocessing as mp
  ctx = mp.get_context("spawn")
  errq = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_protocol_worker, args=(r, world, port, 3, 512, cu, 7, errq))
           for r in range(world)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(timeout=120)
  errors = []
  while not errq.empty():
    errors.append(errq.get())
  for p in procs:
    if p.is_alive():
      p.kill()
      errors.append("a rank did not finish")
  assert not errors and all(p.exitcode == 0 for p in procs), errors


SLAB_CONTRACT_CASES = [
  ([0, 600], [0, 200, 400, 600]),
  ([0, 200, 250, 600], [0, 200, 400, 600]),        # a start on a slab edge, one inside
  (list(range(0, 600, 48)) + [600], [0, 200, 400, 600]),
  ([0, 1, 199, 200, 201, 599, 600], [0, 200, 400, 600]),  # one-element pieces at the edges
]


@pytest.mark.parametrize(("cu", "bounds"), SLAB_CONTRACT_CASES)
@pytest.mark.parametrize("r2l", [False, True])
def test_seeded_slab_contract_in_fp64(cu, bounds, r2l):
  """The row I/O contract of ascan_forward_slab / ascan_backward_slab restated
  with the oracle on each slab alone: the row carry folded into the row's
  first element in scan order (forward x' = x + g Y and g' = g A; backward an
  additive adjoint term), the state halo as the edge element's neighbour, and
  the row aggregate (``_slab_agg_reference``) reproduce the oracle of the
  whole axis, with the carries and halos read off that oracle as the GPU test
  of the seeded passes reads them."""
  C, L = 3, bounds[-1]
  rng = np.random.default_rng(len(cu))
  g = (1 - (rng.random((C, L)) < 0.1) / 256).astype(np.float32)
  x = rng.standard_normal((C, L)).astype(np.float32)
  dy = rng.standard_normal((C, L)).astype(np.float32)
  starts = set(cu)
  y, A = oracle.scan_fwd(g, x, cu, reverse=r2l)
  h = y.astype(np.float32)
  dx, dg = oracle.scan_bwd(dy, g, h, cu, causal=not r2l)
  tol = dict(rtol=1e-5, atol=1e-5)
  for p in ts.plan_slabs(cu, bounds):
    a, b = p.t0, p.t1
    n, lcu = b - a, list(p.local_cu)
    gs, xs, dys = (t[:, a:b].astype(np.float64) for t in (g, x, dy))
    # forward: the carry enters at column n-1 (reverse) or 0
    src = b if r2l else a - 1
    if 0 <= src < L and (b if r2l else a) not in starts:
      carry = np.stack([A[:, src], y[:, src]], 1)
    else:
      carry = np.stack([np.ones(C), np.zeros(C)], 1)
    first = n - 1 if r2l else 0
    gs2, xs2 = gs.copy(), xs.copy()
    xs2[:, first] += gs[:, first] * carry[:, 1]
    gs2[:, first] *= carry[:, 0]
    ys, As = oracle.scan_fwd(gs2, xs2, lcu, reverse=r2l)
    np.testing.assert_allclose(ys, y[:, a:b], **tol, err_msg=f"forward slab {a}")
    np.testing.assert_allclose(As, A[:, a:b], **tol, err_msg=f"gate products slab {a}")
    last = 0 if r2l else n - 1
    agg = _slab_agg_reference(gs, xs, lcu, True, r2l, carry)
    np.testing.assert_allclose(agg, np.stack([A[:, a + last], y[:, a + last]], 1), **tol,
                               err_msg=f"forward aggregate slab {a}")
    # backward: the adjoint term from column b (causal) or a - 1, the state
    # neighbour from column a - 1 (causal) or b
    nb = a - 1 if r2l else b
    linked = 0 <= nb < L and (a if r2l else b) not in starts
    bcarry = g[:, nb].astype(np.float64) * dx[:, nb] if linked else np.zeros(C)
    hn = b if r2l else a - 1
    halo = h[:, hn].astype(np.float64) if 0 <= hn < L and (b if r2l else a) not in starts \
        else np.zeros(C)
    dys2 = dys.copy()
    dys2[:, 0 if r2l else n - 1] += bcarry
    dxs, dgs = oracle.scan_bwd(dys2, g[:, a:b], h[:, a:b], lcu, causal=not r2l)
    edge = n - 1 if r2l else 0  # the element whose state neighbour is the halo
    dgs[:, edge] = dxs[:, edge] * halo
    np.testing.assert_allclose(dxs, dx[:, a:b], **tol, err_msg=f"d_tokens slab {a}")
    np.testing.assert_allclose(dgs, dg[:, a:b], **tol, err_msg=f"d_gates slab {a}")
    bagg = _slab_agg_reference(gs, dys, lcu, False, not r2l, bcarry)
    np.testing.assert_allclose(bagg[:, 1], dx[:, a + (n - 1 if r2l else 0)], **tol,
                               err_msg=f"backward aggregate slab {a}")


def _connect_worker(rank, world, port, fail, outq):
  """PeerExchange.connect on gloo with the library's buffer calls replaced by
  fakes that log what they do; ``fail``: "import" (the last rank cannot map
  the last peer's buffer) or "export" (one rank cannot export its handle)."""
  import torch.distributed as dist
  from associative_scan_triton import _lib
  try:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    calls, own = [], 0x1000 * (rank + 1)

    def create(C, device):
      calls.append(("create", own))
      return own

    def export(buf):
      if fail == "export":
        raise _lib.ScanError("fake export failure")
      return bytes([rank]) * _lib.IPC_HANDLE_BYTES

    def import_(h, device):
      src = h[0]
      if fail == "import" and rank == world - 1 and src == world - 2:
        raise _lib.ScanError("fake import failure")
      calls.append(("import", src))
      return 0x100000 + src

    _lib.exchange_create, _lib.exchange_export, _lib.exchange_import = create, export, import_
    _lib.exchange_close = lambda p: calls.append(("close", p))
    _lib.exchange_destroy = lambda b: calls.append(("destroy", b))
    try:
      ex = ts.PeerExchange.connect(4, "cpu")
      outq.put((rank, "ok", ex.table.tolist(), ex.mapped, calls))
    except _lib.ScanError:
      outq.put((rank, "failed", None, None, calls))
    dist.destroy_process_group()
  except BaseException as e:  # reported to the parent
    outq.put((rank, f"error {type(e).__name__}: {e}", None, None, None))
    raise


def _run_connect(world, fail):
  import multiprocessing as mp
  ctx = mp.get_context("spawn")
  outq = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_connect_worker, args=(r, world, port, fail, outq))
           for r in range(world)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(timeout=120)
  for p in procs:
    if p.is_alive():
      p.kill()
  got = {}
  while not outq.empty():
    r, *rest = outq.get()
    got[r] = rest
  assert sorted(got) == list(range(world)), got
  return got


def test_peer_exchange_connect_on_gloo_ranks():
  """Host side of PeerExchange.connect: every rank's table holds its own
  buffer and the other ranks' mapped buffers; a rank that fails to map a
  peer unmaps what it had mapped and keeps its own buffer (the handles went
  round); a rank whose export fails frees its buffer (nobody saw it)."""
  world = 3
  got = _run_connect(world, "none")
  for r in range(world):
    status, table, mapped, _ = got[r]
    assert status == "ok"
    assert table == [0x1000 * (r + 1) if j == r else 0x100000 + j for j in range(world)]
    assert mapped == [0x100000 + j for j in range(world) if j != r]
  got = _run_connect(world, "import")
  status, _, _, calls = got[world - 1]
  assert status == "failed"
  assert ("close", 0x100000) in calls and not any(c[0] == "destroy" for c in calls)
  assert all(got[r][0] == "ok" for r in range(world - 1))
  got = _run_connect(1, "export")
  status, _, _, calls = got[0]
  assert status == "failed" and ("destroy", 0x1000) in calls


# --- GPU: emulated slabs against the oracle on the whole axis ---------------------------

CASES = [
  # C, T, world, cu_seqlens
  (8, 1 << 16, 4, [0, 1 << 16]),                       # one long sequence (the 5b shape, small)
  (4, 1 << 15, 8, [0, 1 << 15]),
  (5, 3 * 4096 * 4, 4, [0, 5000, 12288, 20000, 49152]),  # boundaries inside, one on an edge
  (3, 8192 * 3, 3, [0, 1, 8191, 8192, 24575, 24576]),   # pieces of one element at the edges
  (2, 4096 * 6 + 64, 5, [0, 4096 * 6 + 64]),            # slabs not multiples of a tile
]


@pytest.mark.gpu
@pytest.mark.parametrize("width", [0, 32])
@pytest.mark.parametrize(("C", "T", "world", "cu"), CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gate", ["verylong", "nearone"])
def test_emulated_slabs_match_oracle(C, T, world, cu, dtype, width, gate):
  """gate "nearone" keeps gate products near 1 over whole slabs, so every
  slab's carry reaches the end of the axis."""
  from associative_scan_triton import _lib
  _lib.set_tile_width(width)  # 32: the slab kernels on 8192-element tiles
  try:
    _emulated_slabs_match_oracle(C, T, world, cu, dtype, gate)
  finally:
    _lib.set_tile_width(0)


def _emulated_slabs_match_oracle(C, T, world, cu, dtype, gate):
  g, x = make_inputs(C, T, dtype=dtype, gate=gate, seed=C + T + world)
  dy = torch.randn(C, T, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
  bounds = ts.even_bounds(T, world, align=64)
  plans = ts.plan_slabs(cu, bounds)
  sl = [slice(a, b) for a, b in zip(bounds, bounds[1:])]
  gs = [g[:, s].contiguous() for s in sl]
  xs = [x[:, s].contiguous() for s in sl]
  dys = [dy[:, s].contiguous() for s in sl]
  ys = ts.emulate_forward(gs, xs, plans)
  y = torch.cat(ys, dim=1)
  cu_t = torch.tensor(cu, dtype=torch.int64, device="cuda")
  gold_y, _ = oracle.scan_fwd(g, x, cu_t)
  assert_close_to_gold(y, gold_y, dtype, "time-sharded y")
  grads = ts.emulate_backward(dys, gs, ys, plans)
  dg = torch.cat([d[0] for d in grads], dim=1)
  dx = torch.cat([d[1] for d in grads], dim=1)
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu_t)
  assert_close_to_gold(dx, gdx, dtype, "time-sharded dx")
  assert_close_to_gold(dg, gdg, dtype, "time-sharded dg")


@pytest.mark.gpu
@pytest.mark.parametrize(("C", "T", "world", "cu"), CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gate", ["verylong", "nearone"])
def test_peer_exchange_matches_collective_path(C, T, world, cu, dtype, gate):
  """The exchange over peer memory (every rank's side emulated in this
  process: publish every rank, then fold every rank) folds exactly the
  carries and halos of the gathered-records path, bit for bit, over three
  exchanges per direction (both record slots and the consumed-before-
  overwrite check are used).  The slabs then agree with that path within the
  tolerance (a look-back composes predecessors in a timing-dependent order,
  so two launches of one scan may differ in the last bits) and both match
  the fp64 oracle."""
  from associative_scan_triton import _lib
  g, x = make_inputs(C, T, dtype=dtype, gate=gate, seed=C + T + world)
  dy = torch.randn(C, T, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
  bounds = ts.even_bounds(T, world, align=64)
  plans = ts.plan_slabs(cu, bounds)
  masks = ts.plan_masks(plans)
  sl = [slice(a, b) for a, b in zip(bounds, bounds[1:])]
  gs = [g[:, s].contiguous() for s in sl]
  xs = [x[:, s].contiguous() for s in sl]
  dys = [dy[:, s].contiguous() for s in sl]
  ref_y = ts.emulate_forward(gs, xs, plans)
  ref_grads = ts.emulate_backward(dys, gs, ref_y, plans)
  f32 = dict(dtype=torch.float32, device="cuda")
  rec_f = torch.empty(world, 2 * C, **f32)
  rec_b = torch.empty(world, 4 * C, **f32)
  zero = torch.zeros(C, **f32)
  for k in range(world):
    ts.slab_forward_aggregate(gs[k], xs[k], plans[k], out=rec_f[k].view(C, 2))
    ts.slab_backward_aggregate(dys[k], gs[k], ref_y[k], plans[k], out=rec_b[k, :2 * C].view(C, 2),
                               zero=zero)
    rec_b[k, 2 * C:3 * C].copy_(gs[k][:, 0])
    rec_b[k, 3 * C:].copy_(ref_y[k][:, -1])
  peers = ts.PeerExchange.emulated(C, world, "cuda")
  try:
    for _ in range(3):
      carries = [torch.empty(C, 2, **f32) for _ in range(world)]
      for k in range(world):
        peers[k].exchange(0, _lib.EXCHANGE_PUBLISH, masks, rec_f[k].view(C, 2), None)
      for k in range(world):
        peers[k].exchange(0, _lib.EXCHANGE_FOLD, masks, None, carries[k])
      bcar = [torch.empty(C, **f32) for _ in range(world)]
      halos = [torch.empty(C, **f32) for _ in range(world)]
      for k in range(world):
        peers[k].exchange(1, _lib.EXCHANGE_PUBLISH, masks, rec_b[k, :2 * C].view(C, 2), None,
                          gates=gs[k], states=ref_y[k])
      for k in range(world):
        peers[k].exchange(1, _lib.EXCHANGE_FOLD, masks, None, bcar[k], halo=halos[k])
      torch.cuda.synchronize()
      for k in range(world):
        assert torch.equal(carries[k], ts.fold_forward(rec_f, plans, k)), f"slab {k} carry"
        ref_c, ref_h = ts.fold_backward(rec_b, plans, k)
        assert torch.equal(bcar[k], ref_c), f"slab {k} adjoint carry"
        assert torch.equal(halos[k], ref_h), f"slab {k} halo"
    for _ in range(2):  # the whole passes through the peer exchange, twice
      ys = ts.emulate_forward(gs, xs, plans, peers=peers)
      grads = ts.emulate_backward(dys, gs, ys, plans, peers=peers)
    torch.cuda.synchronize()
  finally:
    for p in peers:
      p.close()
  _lib.check_device_error()
  for k in range(world):
    for ours, ref, what in ((ys[k], ref_y[k], "y"), (grads[k][0], ref_grads[k][0], "dg"),
                            (grads[k][1], ref_grads[k][1], "dx")):
      assert_close_to_gold(ours, ref.double().cpu().numpy(), dtype, f"slab {k} {what} vs gathered path")
  cu_t = torch.tensor(cu, dtype=torch.int64, device="cuda")
  gold_y, _ = oracle.scan_fwd(g, x, cu_t)
  y = torch.cat(ys, dim=1)
  assert_close_to_gold(y, gold_y, dtype, "peer-exchange y")
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu_t)
  assert_close_to_gold(torch.cat([d[1] for d in grads], 1), gdx, dtype, "peer-exchange dx")
  assert_close_to_gold(torch.cat([d[0] for d in grads], 1), gdg, dtype, "peer-exchange dg")


def _peer_parts_step(gs, xs, dys, plans, peers, H):
  """One forward and backward of every slab through the peer exchange with
  each row of a slab without inner boundaries scanned as H parts (the path
  TimeShardStep(exchange="peer") takes): publish every rank, then fold every
  rank, so no kernel waits for a later one."""
  from associative_scan_triton import _lib
  W, C = len(plans), gs[0].shape[0]
  masks = ts.plan_masks(plans)
  hs = [H if not p.inner_boundary else 1 for p in plans]
  f32 = dict(dtype=torch.float32, device="cuda")

  def views(k, *t):
    return [u.view(hs[k] * C, u.shape[1] // hs[k]) for u in t]

  def cu_of(k):
    p = plans[k]
    if hs[k] == 1:
      return torch.tensor(p.local_cu, dtype=torch.int64, device="cuda")
    return torch.tensor([0, p.length // hs[k]], dtype=torch.int64, device="cuda")

  aggs = [torch.empty(hs[k] * C, 2, **f32) for k in range(W)]
  carries = [torch.empty(hs[k] * C, 2, **f32) for k in range(W)]
  for k in range(W):
    gv, xv = views(k, gs[k], xs[k])
    cu = cu_of(k)
    _lib.forward_slab(gv, xv, None, None, cu, cu.numel() - 1, hs[k] * C, False, row_aggregate=aggs[k])
  for k in range(W):
    peers[k].exchange(0, _lib.EXCHANGE_PUBLISH, masks, aggs[k], None, parts=hs[k])
  for k in range(W):
    peers[k].exchange(0, _lib.EXCHANGE_FOLD, masks, aggs[k], carries[k], parts=hs[k])
  ys = []
  for k in range(W):
    y = torch.empty_like(xs[k])
    gv, xv, yv = views(k, gs[k], xs[k], y)
    cu = cu_of(k)
    _lib.forward_slab(gv, xv, yv, None, cu, cu.numel() - 1, hs[k] * C, False, row_carry=carries[k])
    ys.append(y)
  bags = [torch.empty(hs[k] * C, 2, **f32) for k in range(W)]
  bcar = [torch.empty(hs[k] * C, **f32) for k in range(W)]
  halos = [torch.empty(hs[k] * C, **f32) for k in range(W)]
  for k in range(W):
    dyv, gv, hv = views(k, dys[k], gs[k], ys[k])
    cu = cu_of(k)
    _lib.backward_slab(dyv, gv, hv, None, None, cu, cu.numel() - 1, hs[k] * C, True,
                       row_carry=torch.zeros(hs[k] * C, **f32), row_aggregate=bags[k])
  for k in range(W):
    peers[k].exchange(1, _lib.EXCHANGE_PUBLISH, masks, bags[k], None, gates=gs[k], states=ys[k],
                      parts=hs[k])
  for k in range(W):
    peers[k].exchange(1, _lib.EXCHANGE_FOLD, masks, bags[k], bcar[k], halo=halos[k], gates=gs[k],
                      states=ys[k], parts=hs[k])
  grads = []
  for k in range(W):
    dx, dg = torch.empty_like(xs[k]), torch.empty_like(xs[k])
    dyv, gv, hv, dxv, dgv = views(k, dys[k], gs[k], ys[k], dx, dg)
    cu = cu_of(k)
    _lib.backward_slab(dyv, gv, hv, dxv, dgv, cu, cu.numel() - 1, hs[k] * C, True,
                       row_carry=bcar[k], row_state_halo=halos[k])
    grads.append((dg, dx))
  return ys, grads


@pytest.mark.gpu
@pytest.mark.parametrize("H", [2, 4])
@pytest.mark.parametrize(("C", "T", "world", "cu"), [
  (8, 1 << 16, 4, [0, 1 << 16]),
  (5, 3 * 4096 * 4, 4, [0, 5000, 12288, 20000, 49152]),  # inner boundaries: those slabs keep H=1
  (3, 8192 * 8, 2, [0, 8192 * 4, 8192 * 8]),              # a slab starting a sequence
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gate", ["verylong", "nearone"])
def test_peer_exchange_row_parts_match_oracle(C, T, world, cu, H, dtype, gate):
  """Rows of a slab cut into H parts for the seeded passes: the exchange
  composes the parts' records and returns one carry (and halo) per part; the
  slabs match the fp64 oracle on the whole axis, over two steps."""
  g, x = make_inputs(C, T, dtype=dtype, gate=gate, seed=C + T + world + H)
  dy = torch.randn(C, T, generator=torch.Generator().manual_seed(4)).to("cuda", dtype)
  bounds = ts.even_bounds(T, world, align=64)
  plans = ts.plan_slabs(cu, bounds)
  sl = [slice(a, b) for a, b in zip(bounds, bounds[1:])]
  gs = [g[:, s].contiguous() for s in sl]
  xs = [x[:, s].contiguous() for s in sl]
  dys = [dy[:, s].contiguous() for s in sl]
  peers = ts.PeerExchange.emulated(C, world, "cuda")
  try:
    for _ in range(2):
      ys, grads = _peer_parts_step(gs, xs, dys, plans, peers, H)
    torch.cuda.synchronize()
  finally:
    for p in peers:
      p.close()
  from associative_scan_triton import _lib
  _lib.check_device_error()
  cu_t = torch.tensor(cu, dtype=torch.int64, device="cuda")
  gold_y, _ = oracle.scan_fwd(g, x, cu_t)
  y = torch.cat(ys, dim=1)
  assert_close_to_gold(y, gold_y, dtype, f"row parts H={H} y")
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu_t)
  assert_close_to_gold(torch.cat([d[1] for d in grads], 1), gdx, dtype, f"row parts H={H} dx")
  assert_close_to_gold(torch.cat([d[0] for d in grads], 1), gdg, dtype, f"row parts H={H} dg")


def test_row_parts_choice():
  """H: a power of two filling four waves of rows, whole 8192-column parts,
  1 for slabs with a boundary inside."""
  import unittest.mock as um
  props = um.Mock(multi_processor_count=148)
  plan = ts.SlabPlan(0, 131072, (0, 131072), False, False)
  with um.patch.object(torch.cuda, "get_device_properties", return_value=props):
    assert ts.row_parts(256, 131072, plan, "cpu") == 4      # 1024 rows >= 592
    assert ts.row_parts(1536, 131072, plan, "cpu") == 1
    assert ts.row_parts(16, 131072, plan, "cpu") == 16      # capped by whole 8192-column parts
    assert ts.row_parts(16, 8192 * 3, plan, "cpu") == 1
    inner = ts.SlabPlan(0, 131072, (0, 5, 131072), False, True)
    assert ts.row_parts(256, 131072, inner, "cpu") == 1


@pytest.mark.gpu
def test_peer_exchange_wait_gives_up():
  """A fold whose predecessor never publishes (nothing ever sets its flag)
  gives up after the bounded wait, reports ASCAN_DEV_ERR_EXCHANGE with the
  missing rank, and leaves the context usable."""
  from associative_scan_triton import _lib
  C, world = 64, 2
  _lib.clear_device_error()
  peers = ts.PeerExchange.emulated(C, world, "cuda")
  carry = torch.full((C, 2), 7.0, device="cuda")
  try:
    # rank 1's forward needs rank 0's record of exchange 0, which never comes
    with pytest.raises(_lib.ScanError, match="peer rank"):
      peers[1].exchange(0, _lib.EXCHANGE_FOLD, (0, 0), None, carry, timeout_s=0.05)
      _lib.check_device_error()
    code, _ = _lib.get_device_error()
    assert code == 0  # raising cleared it
    # the stream still works: a later publish + fold of the next exchange number
    agg = torch.rand(C, 2, device="cuda")
    peers[0].exchange(0, _lib.EXCHANGE_BOTH, (0, 0), agg, torch.empty(C, 2, device="cuda"))
    torch.cuda.synchronize()
  finally:
    for p in peers:
      p.close()
    _lib.clear_device_error()


@pytest.mark.gpu
def test_slab_aggregate_matches_definition():
  C, T = 6, 4096 * 2 + 128
  g, x = make_inputs(C, T, gate="long", seed=11)
  plan = ts.plan_slabs([0, 3000, T], [0, T])[0]
  agg = ts.slab_forward_aggregate(g, x, plan)
  want = _fwd_aggregate(g.double().cpu().numpy(), x.double().cpu().numpy(), plan)
  np.testing.assert_allclose(agg.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
  dy = torch.randn_like(x)
  h = torch.randn_like(x)
  bagg = ts.slab_backward_aggregate(dy, g, h, plan)
  bwant = _bwd_aggregate(dy.double().cpu().numpy(), g.double().cpu().numpy(), plan)
  np.testing.assert_allclose(bagg.cpu().numpy(), bwant, rtol=1e-5, atol=1e-6)


def _slab_agg_reference(g, v, cu, forward, r2l, carry):
  """fp64 restatement of a slab pass's row aggregate: the scan of the whole
  row in scan order (heads restart the value and the coefficient product with
  the head's own coefficient; the row carry enters at the row's first element
  in scan order), read at the row's last element in scan order.  Backward:
  coefficient g[t+1] (causal) or g[t-1] (reverse), 1 for the row's first
  element in scan order."""
  C, L = g.shape
  cu = [int(c) for c in cu]
  starts = {c for c in cu[:-1] if c < L}
  ends = {c - 1 for c in cu[1:] if c > 0}
  order = list(range(L - 1, -1, -1)) if r2l else list(range(L))
  heads = ends if r2l else starts
  coeff = np.ones((C, L))
  if forward:
    coeff[:] = g
  elif r2l:
    coeff[:, :-1] = g[:, 1:]
  else:
    coeff[:, 1:] = g[:, :-1]
  A, Y = np.ones(C), np.zeros(C)
  for k, t in enumerate(order):
    a, b = coeff[:, t].copy(), v[:, t].copy()
    if k == 0 and carry is not None:
      if forward:
        b, a = b + a * carry[:, 1], a * carry[:, 0]
      else:
        b, a = b + carry, np.ones(C)
    if k == 0 or t in heads:
      A, Y = a, b
    else:
      Y, A = a * Y + b, A * a
  return np.stack([A, Y], axis=1)


SLAB_AGG_CASES = [
  (6, 8320, [0, 8320]),                      # one sequence, two CTAs per row
  (6, 8320, [0, 3000, 8320]),                # an inner boundary
  (6, 8320, [0, 1, 8319, 8320]),             # one-element pieces at both ends
  (3, 300_000, [0, 300_000]),                # many CTAs per row
  (3, 300_000, [0, 77, 299_000, 300_000]),
  (1500, 1024, [0, 1024]),                   # many short rows, one CTA each
  (5, 4101, [0, 4101]),                      # rows not a whole number of vectors
]


@pytest.mark.gpu
@pytest.mark.parametrize(("C", "L", "cu"), SLAB_AGG_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_carry", [False, True])
def test_slab_aggregate_reduction_matches_definition(C, L, cu, dtype, with_carry):
  from associative_scan_triton import _lib
  g, x = make_inputs(C, L, dtype=dtype, gate="verylong", seed=C + L)
  dy = torch.randn(C, L, generator=torch.Generator().manual_seed(L)).to("cuda", dtype)
  h = torch.randn(C, L, device="cuda").to(dtype)
  cu_t = torch.tensor(cu, dtype=torch.int64, device="cuda")
  gd, xd, dyd = (t.double().cpu().numpy() for t in (g, x, dy))
  rng = np.random.default_rng(1)
  carry_f = np.stack([rng.uniform(0.5, 1.0, C), rng.standard_normal(C)], 1)
  carry_b = rng.standard_normal(C)
  for reverse in (False, True):
    agg = torch.empty(C, 2, device="cuda")
    carry = torch.tensor(carry_f, dtype=torch.float32, device="cuda") if with_carry else None
    _lib.forward_slab(g, x, None, None, cu_t, len(cu) - 1, C, reverse, row_carry=carry,
                      row_aggregate=agg)
    want = _slab_agg_reference(gd, xd, cu, True, reverse,
                               carry.double().cpu().numpy() if with_carry else None)
    np.testing.assert_allclose(agg.cpu().numpy(), want, rtol=1e-4, atol=1e-5,
                               err_msg=f"forward aggregate reverse={reverse}")
  for causal in (True, False):
    agg = torch.empty(C, 2, device="cuda")
    carry = torch.tensor(carry_b, dtype=torch.float32, device="cuda") if with_carry else None
    _lib.backward_slab(dy, g, h, None, None, cu_t, len(cu) - 1, C, causal, row_carry=carry,
                       row_aggregate=agg)
    want = _slab_agg_reference(gd, dyd, cu, False, causal,
                               carry.double().cpu().numpy() if with_carry else None)
    np.testing.assert_allclose(agg.cpu().numpy(), want, rtol=1e-4, atol=1e-5,
                               err_msg=f"backward aggregate causal={causal}")


SEEDED_CASES = [
  # rows of whole tiles, one sequence: row order, the producers inject the row I/O
  (8, 49152, [0, 49152], [0, 16384, 32768, 49152]),
  # equal sequences of whole tiles in every slab: segment order
  (8, 49152, list(range(0, 49153, 8192)), [0, 16384, 32768, 49152]),
  # the middle slab splits into two equal pieces that both continue from the
  # neighbouring slabs: segment order with carries in both directions
  (8, 49152, [0, 24576, 49152], [0, 16384, 32768, 49152]),
  # a sequence start at a slab edge and one inside a slab
  (8, 49152, [0, 16384, 20000, 49152], [0, 16384, 32768, 49152]),
  # rows that are not whole tiles: the slab kernels (row I/O in the consumers)
  (6, 15000, [0, 15000], [0, 5000, 10000, 15000]),
  (6, 15000, [0, 4999, 5000, 5001, 15000], [0, 5000, 10000, 15000]),
  # short sequences across the slab edges: flat order
  (6, 49152, list(range(0, 49152, 96)) + [49152], [0, 16384, 32768, 49152]),
]


@pytest.mark.gpu
@pytest.mark.parametrize(("C", "L", "cu", "bounds"), SEEDED_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("r2l", [False, True])
@pytest.mark.parametrize("width", [0, 32])
def test_seeded_slab_passes_match_whole_axis(C, L, cu, bounds, dtype, r2l, width):
  """Every slab's forward (alone, with the gate products, with the row
  aggregate) and backward (alone, with the row aggregate), both scan
  directions, seeded with the carry and state halo read off the fp64 oracle
  of the whole axis, equals that oracle on the slab's columns.  The time
  shard itself only runs the causal direction; the reverse forward and the
  anti-causal backward take the same seeded paths with the row's first
  element in scan order at the slab's right edge (forward) or left edge
  (backward).  Width 32 forces the 8192-element tiles wherever they exist."""
  from associative_scan_triton import _lib
  _lib.set_tile_width(width)
  try:
    _seeded_slab_passes(C, L, cu, bounds, dtype, r2l)
  finally:
    _lib.set_tile_width(0)


def _seeded_slab_passes(C, L, cu, bounds, dtype, r2l):
  from associative_scan_triton import _lib
  g, x = make_inputs(C, L, dtype=dtype, gate="long", seed=L + len(cu))
  dy = torch.randn(C, L, generator=torch.Generator().manual_seed(7)).to("cuda", dtype)
  # gates of 1 or 1 - 2^-8 (exact in every dtype): gate products over a whole
  # slab stay far from underflow, so the carried product is checked too
  gen = torch.Generator().manual_seed(11)
  gp = (1.0 - (torch.rand(C, L, generator=gen) < 0.02).float() / 256).to("cuda", dtype)
  y64, a64 = oracle.scan_fwd(g, x, cu, reverse=r2l)
  yp64, ap64 = oracle.scan_fwd(gp, x, cu, reverse=r2l)
  h = torch.from_numpy(y64).to("cuda", dtype)  # the states the backward reads
  dx64, dg64 = oracle.scan_bwd(dy, g, h, cu, causal=not r2l)
  g64, hq = g.double().cpu().numpy(), h.double().cpu().numpy()
  starts = set(cu)  # columns where a sequence starts (and the axis end)
  f32 = dict(dtype=torch.float32, device="cuda")
  for k, p in enumerate(ts.plan_slabs(cu, bounds)):
    a, b = p.t0, p.t1
    sl = slice(a, b)
    gs, xs, dys, hs = (t[:, sl].contiguous() for t in (g, x, dy, h))
    lcu = torch.tensor(p.local_cu, dtype=torch.int64, device="cuda")
    S = lcu.numel() - 1
    # forward: the state and gate product just before the row's first
    # element in scan order (column a - 1, or b for the reverse scan)
    src = b if r2l else a - 1
    linked = 0 <= src < L and (b if r2l else a) not in starts

    def fwd_carry(yy, aa):
      if linked:
        return torch.tensor(np.stack([aa[:, src], yy[:, src]], 1), **f32)
      return torch.tensor(np.stack([np.ones(C), np.zeros(C)], 1), **f32)

    ys = torch.empty_like(xs)
    _lib.forward_slab(gs, xs, ys, None, lcu, S, C, r2l, row_carry=fwd_carry(y64, a64))
    assert_close_to_gold(ys, y64[:, sl], dtype, f"slab {k} states reverse={r2l}")
    gps = gp[:, sl].contiguous()
    ys2, gos = torch.empty_like(xs), torch.empty_like(xs)
    _lib.forward_slab(gps, xs, ys2, gos, lcu, S, C, r2l, row_carry=fwd_carry(yp64, ap64))
    assert_close_to_gold(ys2, yp64[:, sl], dtype, f"slab {k} states (gate output) reverse={r2l}")
    assert_close_to_gold(gos, ap64[:, sl], dtype, f"slab {k} gate products reverse={r2l}")
    # states and the row aggregate in one pass (the slab kernels' record_row_agg)
    carry_p = fwd_carry(yp64, ap64)
    ys3, agg = torch.empty_like(xs), torch.empty(C, 2, **f32)
    _lib.forward_slab(gps, xs, ys3, None, lcu, S, C, r2l, row_carry=carry_p, row_aggregate=agg)
    assert_close_to_gold(ys3, yp64[:, sl], dtype, f"slab {k} states (with aggregate)")
    want = _slab_agg_reference(gps.double().cpu().numpy(), xs.double().cpu().numpy(), p.local_cu,
                               True, r2l, carry_p.double().cpu().numpy())
    np.testing.assert_allclose(agg.cpu().numpy(), want, rtol=1e-4, atol=1e-5,
                               err_msg=f"slab {k} forward aggregate reverse={r2l}")
    # backward: the adjoint term from the column the adjoint comes from
    # (b causal, a - 1 anti-causal) and the state neighbour on the other side
    nb = a - 1 if r2l else b
    if 0 <= nb < L and (a if r2l else b) not in starts:
      bcarry = g64[:, nb] * dx64[:, nb]
    else:
      bcarry = np.zeros(C)
    hn = b if r2l else a - 1
    halo = hq[:, hn] if 0 <= hn < L and (b if r2l else a) not in starts else np.zeros(C)
    dxs, dgs = torch.empty_like(xs), torch.empty_like(xs)
    _lib.backward_slab(dys, gs, hs, dxs, dgs, lcu, S, C, not r2l,
                       row_carry=torch.tensor(bcarry, **f32),
                       row_state_halo=torch.tensor(halo, **f32))
    assert_close_to_gold(dxs, dx64[:, sl], dtype, f"slab {k} d_tokens causal={not r2l}")
    assert_close_to_gold(dgs, dg64[:, sl], dtype, f"slab {k} d_gates causal={not r2l}")
    dxs2, dgs2, bagg = torch.empty_like(xs), torch.empty_like(xs), torch.empty(C, 2, **f32)
    _lib.backward_slab(dys, gs, hs, dxs2, dgs2, lcu, S, C, not r2l,
                       row_carry=torch.tensor(bcarry, **f32),
                       row_state_halo=torch.tensor(halo, **f32), row_aggregate=bagg)
    assert_close_to_gold(dxs2, dx64[:, sl], dtype, f"slab {k} d_tokens (with aggregate)")
    assert_close_to_gold(dgs2, dg64[:, sl], dtype, f"slab {k} d_gates (with aggregate)")
    want = _slab_agg_reference(gs.double().cpu().numpy(), dys.double().cpu().numpy(), p.local_cu,
                               False, not r2l, np.asarray(bcarry, dtype=np.float32).astype(np.float64))
    np.testing.assert_allclose(bagg.cpu().numpy(), want, rtol=1e-4, atol=1e-5,
                               err_msg=f"slab {k} backward aggregate causal={not r2l}")


@pytest.mark.gpu
@pytest.mark.parametrize(("world", "cu"), [
  (2, [0, 512]), (4, [0, 512]), (4, [0, 100, 128, 300, 512]), (8, [0, 64, 65, 448, 512]),
])
def test_device_fold_matches_host_fold(world, cu):
  """ascan_time_shard_fold against forward_carry / backward_carry /
  state_halo on the same random records, for every rank."""
  C = 37
  bounds = ts.even_bounds(512, world, align=8)
  plans = ts.plan_slabs(cu, bounds)
  gen = torch.Generator().manual_seed(world)
  fwd = [torch.stack([0.5 + 0.5 * torch.rand(C, generator=gen), torch.randn(C, generator=gen)], 1)
         for _ in range(world)]
  bwd = [torch.stack([0.5 + 0.5 * torch.rand(C, generator=gen), torch.randn(C, generator=gen)], 1)
         for _ in range(world)]
  firsts = [torch.rand(C, generator=gen) for _ in range(world)]
  lasts = [torch.randn(C, generator=gen) for _ in range(world)]
  rec_f = torch.stack([a.reshape(-1) for a in fwd]).cuda()
  rec_b = torch.stack([torch.cat([a.reshape(-1), f, l]) for a, f, l in zip(bwd, firsts, lasts)]).cuda()
  for rank in range(world):
    dev = ts.fold_forward(rec_f, plans, rank)
    host = ts.forward_carry(plans, fwd, rank)
    torch.testing.assert_close(dev.cpu(), host, rtol=1e-6, atol=1e-6)
    carry, halo = ts.fold_backward(rec_b, plans, rank)
    torch.testing.assert_close(carry.cpu(), ts.backward_carry(plans, bwd, firsts, rank),
                               rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(halo.cpu(), ts.state_halo(plans, lasts, rank), rtol=0, atol=0)


@pytest.mark.gpu
def test_time_shard_step_with_list_exchange_matches_oracle():
  """TimeShardStep (the multi-rank driver's step object) on every slab of one
  GPU, its all-gather replaced by writes into the shared buffer: forward and
  backward slabs against the fp64 oracle on the whole axis."""
  C, T, world = 8, 1 << 16, 4
  cu = [0, 10000, 1 << 14, 40000, T]
  g, x = make_inputs(C, T, gate="verylong", seed=9)
  dy = torch.randn(C, T, generator=torch.Generator().manual_seed(2)).cuda()
  bounds = ts.even_bounds(T, world, align=64)
  plans = ts.plan_slabs(cu, bounds)
  sl = [slice(a, b) for a, b in zip(bounds, bounds[1:])]
  shared = {}

  def gather_for(k):
    def gather(out, inp):  # every rank's record lands in one buffer per direction
      buf = shared.setdefault(out.shape, torch.zeros_like(out))
      buf[k].copy_(inp)
      out.copy_(buf)
    return gather

  steps = [ts.TimeShardStep((C, b - a), g.dtype, plans, k, "cuda", gather=gather_for(k))
           for k, (a, b) in enumerate(zip(bounds, bounds[1:]))]
  gs = [g[:, s].contiguous() for s in sl]
  xs = [x[:, s].contiguous() for s in sl]
  dys = [dy[:, s].contiguous() for s in sl]
  # two sweeps over the ranks: the first fills every record, the second reads them all
  for _ in range(2):
    ys = [st.forward(gk, xk) for st, gk, xk in zip(steps, gs, xs)]
  y = torch.cat(ys, 1)
  cu_t = torch.tensor(cu, dtype=torch.int64)
  gold_y, _ = oracle.scan_fwd(g, x, cu_t)
  assert_close_to_gold(y, gold_y, torch.float32, "TimeShardStep y")
  for _ in range(2):
    grads = [st.backward(dk, gk, yk) for st, dk, gk, yk in zip(steps, dys, gs, ys)]
  gdx, gdg = oracle.scan_bwd(dy, g, y, cu_t)
  assert_close_to_gold(torch.cat([d[1] for d in grads], 1), gdx, torch.float32, "TimeShardStep dx")
  assert_close_to_gold(torch.cat([d[0] for d in grads], 1), gdg, torch.float32, "TimeShardStep dg")


@pytest.mark.gpu
def test_slab_entry_points_refuse_unaligned_views():
  from associative_scan_triton import _lib
  C, L = 2, 1024
  base = torch.rand(C * L + 1, device="cuda")
  g = base[1:].view(C, L)  # 4-byte offset: not 16-byte aligned
  x = torch.rand(C, L, device="cuda")
  cu = torch.tensor([0, L], device="cuda")
  agg = torch.empty(C, 2, device="cuda")
  with pytest.raises(_lib.ScanError, match="invalid"):
    _lib.forward_slab(g, x, None, None, cu, 1, C, False, row_aggregate=agg)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_nccl_ranks_match_oracle(tmp_path, exchange):
  """One rank per GPU (2-4): the NCCL exchange, and the exchange kernel over
  NVLink peer memory, against the fp64 oracle."""
  world = min(torch.cuda.device_count(), 4)
  script = REPO / "tests" / "time_shard_ranks.py"
  cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
         "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script),
         str(tmp_path), exchange]
  env = dict(os.environ, NCCL_NVLS_ENABLE="0")
  r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
  assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
  assert (tmp_path / "ok").read_text().strip() == str(world)
