"""Collective-free partitions of a packed scan: channel blocks and sequence
shards.  CPU tests check the partitions and run them as gloo ranks on the
oracle (each rank scans its own part; the gather exists only to check the
result); the GPU test runs every sequence shard through the kernels."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from associative_scan_triton import sharding
from oracle import oracle


def test_channel_blocks_cover_rows():
  for C, world in [(1536, 8), (10, 3), (2, 4), (7, 7)]:
    blocks = [sharding.channel_block(C, world, k) for k in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == C
    assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1
  with pytest.raises(ValueError):
    sharding.channel_block(8, 2, 2)


def test_sequence_shards_are_whole_and_balanced():
  rng = np.random.default_rng(0)
  lens = rng.integers(64, 8193, size=32)  # the varlen config's length law
  cu = [0] + np.cumsum(lens).tolist()
  for world in (1, 2, 4, 8):
    shards = sharding.sequence_shards(cu, world)
    assert shards[0].s0 == 0 and shards[-1].s1 == 32
    assert all(a.s1 == b.s0 for a, b in zip(shards, shards[1:]))
    for sh in shards:
      assert sh.local_cu == tuple(v - sh.t0 for v in cu[sh.s0:sh.s1 + 1]) or sh.s0 == sh.s1
    widths = [sh.t1 - sh.t0 for sh in shards]
    assert max(widths) - min(widths) <= 2 * max(lens)  # within a couple of sequences
  few = sharding.sequence_shards([0, 5, 9], 4)
  assert sum(1 for sh in few if sh.s0 == sh.s1) == 2 and few[-1].t1 == 9


def _worker(rank, world, port, errq):
  import torch.distributed as dist
  try:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(3)
    C, lens = 6, rng.integers(1, 300, size=11)
    cu = [0] + np.cumsum(lens).tolist()
    BL = cu[-1]
    g = torch.from_numpy(rng.uniform(0.9, 1.0, size=(C, BL)).astype(np.float32))
    x = torch.from_numpy(rng.standard_normal((C, BL)).astype(np.float32))
    full, _ = oracle.scan_fwd(g, x, torch.tensor(cu))
    # channel block: this rank's rows with the full cu_seqlens
    c0, c1 = sharding.channel_block(C, world, rank)
    part, _ = oracle.scan_fwd(g[c0:c1], x[c0:c1], torch.tensor(cu))
    rows = [None] * world
    dist.all_gather_object(rows, (c0, c1, part))
    # sequence shard: this rank's columns with rebased boundaries
    sh = sharding.sequence_shards(cu, world)[rank]
    if sh.t1 > sh.t0:
      piece, _ = oracle.scan_fwd(g[:, sh.t0:sh.t1].contiguous(), x[:, sh.t0:sh.t1].contiguous(),
                                 torch.tensor(sh.local_cu))
    else:
      piece = np.zeros((C, 0))
    cols = [None] * world
    dist.all_gather_object(cols, (sh.t0, sh.t1, piece))
    if rank == 0:
      by_rows = np.concatenate([p for _, _, p in sorted(rows, key=lambda r: r[0])], axis=0)
      by_cols = np.concatenate([p for _, _, p in sorted(cols, key=lambda r: r[0])], axis=1)
      np.testing.assert_array_equal(by_rows, full)
      np.testing.assert_array_equal(by_cols, full)
    dist.destroy_process_group()
  except BaseException as e:
    errq.put(f"rank {rank}: {type(e).__name__}: {e}")
    raise


@pytest.mark.parametrize("world", [2, 3])
def test_partitions_on_gloo_ranks(world):
  import multiprocessing as mp
  ctx = mp.get_context("spawn")
  errq = ctx.Queue()
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
  procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
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


@pytest.mark.gpu
def test_sequence_shards_through_the_kernels():
  from associative_scan_triton import _lib
  from scan_testlib import assert_close_to_gold, make_inputs
  rng = np.random.default_rng(1)
  lens = rng.integers(64, 8193, size=32)
  cu = [0] + np.cumsum(lens).tolist()
  C, BL = 16, cu[-1]
  g, x = make_inputs(C, BL, gate="sigmoid", seed=5)
  gold, _ = oracle.scan_fwd(g, x, torch.tensor(cu))
  pieces = []
  for sh in sharding.sequence_shards(cu, 4):
    gs = g[:, sh.t0:sh.t1].contiguous()
    xs = x[:, sh.t0:sh.t1].contiguous()
    y = torch.empty_like(xs)
    lcu = torch.tensor(sh.local_cu, dtype=torch.int64, device="cuda")
    _lib.forward(gs, xs, y, None, lcu, len(sh.local_cu) - 1, C, False)
    pieces.append(y)
  assert_close_to_gold(torch.cat(pieces, dim=1), gold, torch.float32, "sequence shards")
