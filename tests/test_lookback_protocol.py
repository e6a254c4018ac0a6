"""CPU model of the tile hand-off protocol of the persistent scan kernels.

The model restates, per tile of one row in scan order, what the kernels do
with the tile's status slot (``publish`` / ``read_status`` in
``csrc/ascan_device.cuh``) and with its carry-in (``warp_tile_prefix`` in
``csrc/ascan_tma.cuh``, ``lookback_warp`` in ``csrc/ascan_device.cuh``):

* the scan-first warp finds the tile's carry-in: given with the tile (a time
  slab's row carry, or the predecessor's inclusive record fetched by the
  producer) or by looking back over the predecessors' slots -- an inclusive
  record ends the walk, an aggregate is composed and the walk goes on, and
  nothing before ticket 0 counts as the empty prefix;
* the scan-last warp publishes the tile's status: inclusive at once when the
  tile holds a sequence head, needs no carry, or has its carry-in already;
  otherwise its aggregate first and, once the carry-in is known, the
  inclusive record;
* every wait is bounded; a wait that gives up aborts the launch, and every
  other wait then returns at once.

Tiles are agents whose steps run in random interleavings, with at most
``ctas`` tiles in flight and tickets taken in order, as in the persistent
kernels.  Values are pairs (a, b) of the map h -> a h + b composed modulo a
prime, so every grouping gives the same exact result and a wrong prefix can
never pass as rounding.  Each run is checked against the sequential scan of
the row: every tile's final record and every carry-in a tile used.
"""

from __future__ import annotations

import random

import pytest

MOD = (1 << 61) - 1
IDENT = (1, 0)
AGGREGATE, INCLUSIVE = 1, 2


def compose(x, y):
  """x, then y: the scan's combine (gate product, state)."""
  return (x[0] * y[0] % MOD, (y[0] * x[1] + y[1]) % MOD)


class Row:
  """One row of ``n`` tiles of ``e`` elements with sequence heads at random
  places; ``carry``: a time slab's row carry, which the producer turns into
  tile 0's known carry-in (the row's first element then stops being a head)."""

  def __init__(self, rng, n, e, head_p, carry=None):
    self.n = n
    self.elems = [[(rng.randrange(1, MOD), rng.randrange(MOD)) for _ in range(e)]
                  for _ in range(n)]
    self.heads = [[rng.random() < head_p for _ in range(e)] for _ in range(n)]
    self.heads[0][0] = carry is None  # the row starts a sequence unless it is carried
    self.carry = carry
    # sequential scan: the prefix entering each tile and the inclusive value at its end
    state = carry if carry is not None else IDENT
    self.excl, self.incl = [], []
    for t in range(n):
      self.excl.append(state)
      for (a, b), h in zip(self.elems[t], self.heads[t]):
        state = (a, b) if h else compose(state, (a, b))
      self.incl.append(state)
    # the tile totals the consumers compose (from the tile's last head, if any)
    self.tot, self.has_head = [], []
    for t in range(n):
      acc, hh = IDENT, False
      for (a, b), h in zip(self.elems[t], self.heads[t]):
        if h:
          acc, hh = (a, b), True
        else:
          acc = compose(acc, (a, b))
      self.tot.append(acc)
      self.has_head.append(hh)


class Launch:
  """Shared state of one launch: status slots, the carry-in hand-off slots,
  the abort word and what each tile used."""

  def __init__(self, row, rule, limit, prefetch):
    self.row, self.rule, self.limit, self.prefetch = row, rule, limit, prefetch
    self.status = [None] * row.n
    self.te_slot = [None] * row.n
    self.te_used = [None] * row.n
    self.aborted = False
    self.gave_up = []

  def lookback(self, t):
    """The scan-first warp's walk over the predecessors (one slot per step)."""
    acc, d, polls = IDENT, 1, 0
    while True:
      q = t - d
      if q < 0:  # nothing precedes ticket 0: the empty prefix
        return compose(IDENT, acc)
      s = self.status[q]
      if s is None:
        if self.aborted or polls >= self.limit:
          self.aborted = True
          self.gave_up.append(t)
          return compose(IDENT, acc)  # unpublished records count as empty
        polls += 1
        yield
        continue
      if s[0] == INCLUSIVE:
        return compose(s[1], acc)
      acc = compose(s[1], acc)
      d += 1
      yield

  def tile_agents(self, t, drop=False, delay=0):
    """The two warps of tile t that take part in the hand-off, as generators."""
    row = self.row
    te_known, te_val = False, None
    if t == 0 and row.carry is not None:
      te_known, te_val = True, row.carry  # the row carry, injected by the producer
    elif self.prefetch and t > 0 and self.status[t - 1] is not None \
        and self.status[t - 1][0] == INCLUSIVE:
      te_known, te_val = True, self.status[t - 1][1]  # fetched with the tile
    first_is_head = row.heads[t][0]
    need = not first_is_head and (t > 0 or te_known)

    def scan_first():
      if not need or drop:
        return
      if te_known:
        te = te_val
      else:
        te = yield from self.lookback(t)
      self.te_slot[t] = te
      self.te_used[t] = te
      yield

    def scan_last():
      if drop:
        return
      for _ in range(delay):
        yield
      tot = row.tot[t]
      if row.has_head[t] or not need:
        self.status[t] = (INCLUSIVE, tot)
        yield
        return
      if te_known and self.rule == "inclusive-when-known":
        self.status[t] = (INCLUSIVE, compose(te_val, tot))
        yield
        return
      self.status[t] = (AGGREGATE, tot)
      yield
      polls = 0
      while self.te_slot[t] is None:
        if self.aborted or polls >= self.limit:
          self.aborted = True
          self.gave_up.append(t)
          return
        polls += 1
        yield
      self.status[t] = (INCLUSIVE, compose(self.te_slot[t], tot))
      yield

    return [scan_first(), scan_last()]


def run_launch(row, rng, ctas, rule="inclusive-when-known", limit=10_000, prefetch=False,
               drop=None, delay=None):
  """Random interleaving of all tiles' steps; returns the launch and the
  number of steps taken (every run ends: all waits are bounded)."""
  L = Launch(row, rule, limit, prefetch)
  next_ticket, active, steps = 0, [], 0
  while next_ticket < row.n or active:
    while next_ticket < row.n and len(active) < ctas:
      t = next_ticket
      next_ticket += 1
      agents = L.tile_agents(t, drop=(t == drop), delay=(delay[1] if delay and delay[0] == t
                                                          else 0))
      active.append([t, agents])
    k = rng.randrange(len(active))
    t, agents = active[k]
    j = rng.randrange(len(agents))
    try:
      next(agents[j])
    except StopIteration:
      agents.pop(j)
    if not agents:
      active.pop(k)
    steps += 1
    assert steps < 10_000_000
  return L


def check(L):
  row = L.row
  for t in range(row.n):
    assert L.status[t] is not None and L.status[t][0] == INCLUSIVE, f"tile {t}: {L.status[t]}"
    assert L.status[t][1] == row.incl[t], f"tile {t}: wrong inclusive record"
    if L.te_used[t] is not None:
      assert L.te_used[t] == row.excl[t], f"tile {t}: wrong carry-in"


@pytest.mark.parametrize("carried", [False, True])
@pytest.mark.parametrize("prefetch", [False, True])
@pytest.mark.parametrize("head_p", [0.0, 0.05, 0.3])
def test_protocol_gives_the_sequential_prefixes(carried, prefetch, head_p):
  """Every interleaving ends with the sequential scan's records: rows with no
  head (one long sequence), few and many heads, with and without a row carry,
  with and without the producer's fetch of the predecessor's record."""
  rng = random.Random(hash((carried, prefetch, head_p)) & 0xffff)
  for trial in range(150):
    carry = (rng.randrange(1, MOD), rng.randrange(MOD)) if carried else None
    row = Row(rng, n=rng.randrange(1, 24), e=4, head_p=head_p, carry=carry)
    L = run_launch(row, rng, ctas=rng.randrange(1, 9), prefetch=prefetch)
    assert not L.gave_up
    check(L)


def test_aggregate_first_with_a_known_carry_loses_it():
  """The rule the kernels had before: a tile whose carry-in came with it still
  published its aggregate first.  A successor that read that aggregate
  composed it with the empty prefix before ticket 0 and lost the row carry;
  the model finds such interleavings, so the test above would catch the
  rule if it came back."""
  rng = random.Random(7)
  wrong = 0
  for trial in range(300):
    carry = (rng.randrange(2, MOD), rng.randrange(1, MOD))
    row = Row(rng, n=6, e=4, head_p=0.0, carry=carry)
    L = run_launch(row, rng, ctas=4, rule="aggregate-first")
    try:
      check(L)
    except AssertionError:
      wrong += 1
  assert wrong > 0
  rng = random.Random(7)
  for trial in range(300):
    carry = (rng.randrange(2, MOD), rng.randrange(1, MOD))
    row = Row(rng, n=6, e=4, head_p=0.0, carry=carry)
    check(run_launch(row, rng, ctas=4))


def test_late_publisher_is_waited_for():
  """A tile that publishes late (within the wait limit) only delays its
  successors; every record still comes out right."""
  rng = random.Random(3)
  for trial in range(100):
    row = Row(rng, n=10, e=4, head_p=0.05)
    L = run_launch(row, rng, ctas=5, limit=5_000, delay=(rng.randrange(10), 500))
    assert not L.gave_up
    check(L)


def test_dropped_publisher_ends_the_launch_with_an_error():
  """A tile that never publishes (its warps gone): the waits behind it give
  up after their limit, the launch is aborted (later waits return at once),
  every agent finishes -- no hang -- and the give-up is reported."""
  rng = random.Random(5)
  for trial in range(50):
    row = Row(rng, n=12, e=4, head_p=0.0)
    drop = rng.randrange(0, 11)
    L = run_launch(row, rng, ctas=4, limit=200, drop=drop)
    assert L.aborted and L.gave_up
    assert all(t > drop for t in L.gave_up)
    for t in range(drop):  # the tiles before the dropped one are unaffected
      assert L.status[t] == (INCLUSIVE, row.incl[t])
