"""Partitioning a packed ``[C, BL]`` scan across ranks without any collective.

The recurrence couples elements only along a row and only inside one
sequence, so two cuts need no exchange at all (one process per GPU, each
calling the ordinary ops on its part):

* channel blocks -- rank ``k`` owns rows ``[c0, c1)`` with the full
  ``cu_seqlens`` (the reference's packed layout keeps rows contiguous);
* sequence shards -- rank ``k`` owns whole sequences ``[s0, s1)`` of every
  row, i.e. columns ``[cu[s0], cu[s1])``, with ``cu_seqlens`` rebased to that
  column range; sequences are assigned greedily in order so that every rank's
  column count is close to ``BL / W``.

The third cut, a time shard of one long sequence, needs one exchange of
per-row carries and lives in :mod:`associative_scan_triton.time_shard`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

__all__ = ["channel_block", "SequenceShard", "sequence_shards"]


def channel_block(num_channels: int, world: int, rank: int) -> tuple[int, int]:
  """Rows ``[c0, c1)`` of rank ``rank``: contiguous, sizes differing by at most one."""
  if world <= 0 or not 0 <= rank < world:
    raise ValueError(f"rank {rank} of {world}")
  base, extra = divmod(num_channels, world)
  c0 = rank * base + min(rank, extra)
  return c0, c0 + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class SequenceShard:
  """Whole sequences ``[s0, s1)`` = columns ``[t0, t1)`` of every row."""
  s0: int
  s1: int
  t0: int
  t1: int
  local_cu: tuple[int, ...]  # cu_seqlens rebased to the shard: (0, ..., t1 - t0)


def sequence_shards(cu_seqlens: Sequence[int], world: int) -> list[SequenceShard]:
  """Split the sequences of ``cu_seqlens`` (host integers, ``cu[0] = 0``) into
  ``world`` contiguous groups of whole sequences with near-equal column
  counts.  A rank may get no sequence when there are fewer sequences than
  ranks (an empty shard: ``t0 == t1``)."""
  cu = [int(v) for v in cu_seqlens]
  if world <= 0 or not cu or cu[0] != 0 or any(b < a for a, b in zip(cu, cu[1:])):
    raise ValueError("cu_seqlens must start at 0 and be non-decreasing; world must be positive")
  S, total = len(cu) - 1, cu[-1]
  shards = []
  s = 0
  for k in range(world):
    s0 = s
    if k == world - 1:
      s = S
    else:
      target = total * (k + 1) / world  # cumulative column count this rank should reach
      while s < S and abs(cu[s + 1] - target) <= abs(cu[s] - target):
        s += 1
    t0, t1 = cu[s0], cu[s]
    shards.append(SequenceShard(s0, s, t0, t1, tuple(v - t0 for v in cu[s0:s + 1]) or (0,)))
  return shards
