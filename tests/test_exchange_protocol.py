"""CPU model of the carry exchange over peer memory (``time_shard_exchange_kernel``
in ``csrc/ascan_exchange.cuh``), with the ranks as agents under random
interleavings.

Each rank owns a buffer with, per direction, an epoch word (exchanges it has
finished), a flag word (e + 1 once its record of exchange e is out), a
consumed word (e + 1 once it has read everything of exchange e) and two
record slots; exchange e uses slot e % 2.  One exchange of one rank, as the
kernel runs it:

1. publish: if e >= 2, wait until every other rank's consumed word is at
   least e - 1 (slot e % 2 was last read in exchange e - 2); write the record
   element by element; release the flag (e + 1);
2. fold: wait until the flag of every rank it reads is at least e + 1
   (forward: the ranks before it; backward: the ranks after it and, for the
   state halo, the one before); read their records; then set its consumed
   word and its epoch to e + 1.

Every wait gives up after a bounded number of polls and reports.  The runs
check that every record a rank read is the one of the right rank and the
right exchange, element by element (no overwrite, no torn read), over many
exchanges in both directions -- and that the model catches the protocol
without the consumed check, and ends with reports and no hang when a rank
stops taking part.
"""

from __future__ import annotations

import random

import pytest

REC = 3  # elements per record (one per step: plain stores and loads)


class Buf:
  def __init__(self):
    self.epoch = [0, 0]
    self.flag = [0, 0]
    self.consumed = [0, 0]
    self.ring = [[[None] * REC for _ in range(2)] for _ in range(2)]  # [dir][slot][elem]


def reads(rank, world, d):
  """The ranks whose records this rank's fold reads (backward with the halo)."""
  if d == 0:
    return [j for j in range(rank)]
  return [j for j in range(rank + 1, world)] + ([rank - 1] if rank > 0 else [])


def rank_agent(rank, world, bufs, steps, limit, log, reports, check_consumed=True,
               stop_at=None, dirs=(0, 1)):
  own = bufs[rank]
  for s in range(steps):
    for d in dirs:
      if stop_at == (s, d):
        return  # this rank stops taking part
      e = own.epoch[d]
      # publish
      if check_consumed and e >= 2:
        for j in range(world):
          if j == rank:
            continue
          polls = 0
          while bufs[j].consumed[d] < e - 1:
            if polls >= limit:
              reports.append((rank, "consumed", j, d, e))
              break
            polls += 1
            yield
      slot = own.ring[d][e % 2]
      for i in range(REC):
        slot[i] = (rank, e, i)
        yield
      own.flag[d] = e + 1
      yield
      # fold: every wait first, then every read
      for j in reads(rank, world, d):
        polls = 0
        while bufs[j].flag[d] < e + 1:
          if polls >= limit:
            reports.append((rank, "flag", j, d, e))
            break
          polls += 1
          yield
      got = {}
      for j in reads(rank, world, d):
        vals = []
        for i in range(REC):
          vals.append(bufs[j].ring[d][e % 2][i])
          yield
        got[j] = vals
      log.append((rank, d, e, got))
      own.consumed[d] = e + 1
      own.epoch[d] = e + 1
      yield


def run(world, steps, rng, limit=100_000, check_consumed=True, stop=None, bias=None,
        dirs=(0, 1)):
  """All ranks' agents in one random interleaving; ``bias``: per-rank weights
  (a slow rank gets picked less often); ``dirs``: the directions of one step
  (a training step exchanges forward then backward; inference only forward)."""
  bufs = [Buf() for _ in range(world)]
  log, reports = [], []
  agents = {r: rank_agent(r, world, bufs, steps, limit, log, reports, check_consumed,
                          stop[1] if stop and stop[0] == r else None, dirs)
            for r in range(world)}
  weights = bias or [1.0] * world
  n = 0
  while agents:
    ranks = list(agents)
    r = rng.choices(ranks, weights=[weights[k] for k in ranks])[0]
    try:
      next(agents[r])
    except StopIteration:
      del agents[r]
    n += 1
    assert n < 20_000_000
  return log, reports


def records_ok(log):
  return all(vals == [(j, e, i) for i in range(REC)]
             for _, _, e, got in log for j, vals in got.items())


@pytest.mark.parametrize("world", [2, 3, 5, 8])
@pytest.mark.parametrize("dirs", [(0, 1), (0,), (1,)])
def test_every_read_is_the_right_record(world, dirs):
  rng = random.Random(world * 10 + len(dirs))
  for trial in range(20):
    bias = [rng.choice([0.2, 1.0, 1.0, 3.0]) for _ in range(world)]
    log, reports = run(world, steps=6, rng=rng, bias=bias, dirs=dirs)
    assert not reports
    assert len(log) == world * 6 * len(dirs)
    assert records_ok(log)


def test_without_the_consumed_check_a_slot_is_overwritten():
  """The planted mistake: publishing into slot e % 2 without waiting for the
  peers to consume exchange e - 2 lets a fast rank overwrite a record a slow
  rank has not read yet.  With forward-only exchanges nothing else holds
  rank 0 back (its fold reads nobody), and the model finds the overwrite.
  (Alternating directions, as a training step does, happen to couple the
  ranks tightly enough on their own; the check keeps any sequence safe.)"""
  rng = random.Random(11)
  bad = 0
  for trial in range(60):
    log, _ = run(3, steps=6, rng=rng, check_consumed=False, bias=[3.0, 0.1, 0.1], dirs=(0,))
    bad += not records_ok(log)
  assert bad > 0


def test_a_rank_that_stops_ends_the_others_with_reports():
  """A rank that stops after some exchanges (it raised, or its process
  ended): the waits that depend on it give up after their limit and report;
  every other rank finishes all its steps -- no hang."""
  rng = random.Random(5)
  for trial in range(20):
    world = 4
    stop = (rng.randrange(world), (rng.randrange(1, 4), rng.randrange(2)))
    log, reports = run(world, steps=5, rng=rng, limit=300, stop=stop)
    # the waits on the stopped rank give up (others may give up in turn on a
    # rank that was itself waiting out its limit)
    assert any(rep[2] == stop[0] for rep in reports)
    for r in range(world):  # every other rank ran all its exchanges
      if r != stop[0]:
        assert sum(1 for x in log if x[0] == r) == 5 * 2
