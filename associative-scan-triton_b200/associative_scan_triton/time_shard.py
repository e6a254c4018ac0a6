"""Time-sharded causal scan: one long sequence axis split across GPUs.

The reference runs every row of ``[C, BL]`` inside one Triton program per
sequence (``src/associative_scan_triton/_kernels.py:84-168``), so a sequence
can never outgrow one device.  Here rank ``k`` of ``W`` holds columns
``[t_k, t_{k+1})`` of every row -- its *slab*, a ``[C, L_k]`` tensor -- and
the recurrence crosses slab edges by reduce-then-scan:

forward (``h[t] = g[t] h[t-1] + x[t]``)
  1. aggregate pass: each rank scans its slab from a zero state without
     writing outputs and keeps, per row, the gate product ``P`` and the state
     ``Y`` at its last column (``ascan_forward_slab`` with ``tokens_out=NULL``);
  2. exchange: one all-gather of ``[C, 2]`` floats per rank (NCCL over
     NVLink);
  3. each rank folds the records of the ranks before it into its carry
     ``(product, state)`` (:func:`forward_carry`);
  4. seeded pass: the slab's forward with that carry entering each row's
     first column (``ascan_forward_slab`` with ``row_carry``).
  Traffic: 2 reads in pass 1, 2 reads + 1 write in pass 2 (5 element
  transfers against 3 for a single-device scan).

backward (``dh[t] = dy[t] + g[t+1] dh[t+1]``, ``dg[t] = dh[t] h[t-1]``)
  mirrored from the last rank to the first; the exchange also carries each
  slab's first gate column and last state column, the neighbours that the
  adjacent slabs' edge elements need (:func:`backward_carry`).

Sequence boundaries come from the global ``cu_seqlens`` (shared by every
channel, as in the reference's packed layout); :func:`plan_slabs` rebases them
to each slab and records whether the slab's first piece continues a sequence
from the previous slab and whether a boundary lies inside it.  The carry
folds need only those flags and the exchanged per-row records, so they are
the same code for the multi-process driver (:func:`scan_causal_time_sharded`,
:class:`ScanCausalTimeShard`), for single-process emulation of all slabs on
one GPU (:func:`emulate_forward`, :func:`emulate_backward`) and for the CPU
protocol tests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch

from . import _lib

__all__ = [
  "SlabPlan", "plan_slabs", "even_bounds", "forward_carry", "backward_carry",
  "slab_forward_aggregate", "slab_forward", "slab_backward_aggregate", "slab_backward",
  "emulate_forward", "emulate_backward", "scan_causal_time_sharded", "ScanCausalTimeShard",
]


@dataclass(frozen=True)
class SlabPlan:
  """Geometry of one slab ``[t0, t1)`` of the global sequence axis."""
  t0: int
  t1: int
  local_cu: tuple[int, ...]  # boundaries inside the slab, rebased: (0, ..., t1 - t0)
  starts_new: bool           # a sequence starts at t0 (the carry into the slab is ignored)
  inner_boundary: bool       # a sequence boundary lies strictly inside (t0, t1)

  @property
  def length(self) -> int:
    return self.t1 - self.t0

  @property
  def last_piece_continues(self) -> bool:
    """The slab's last piece is the continuation of a sequence from before t0."""
    return not self.starts_new and not self.inner_boundary


def even_bounds(total: int, world: int, align: int = 32) -> list[int]:
  """Slab edges splitting ``total`` columns into ``world`` near-equal slabs,
  every edge a multiple of ``align`` columns (16-byte aligned rows for every
  dtype when ``align`` is a multiple of 8)."""
  if world <= 0 or total < world * align:
    raise ValueError(f"cannot split {total} columns into {world} slabs of >= {align}")
  units = total // align
  edges = [align * ((units * k) // world) for k in range(world)] + [total]
  return edges


def plan_slabs(cu_seqlens: Sequence[int], bounds: Sequence[int]) -> list[SlabPlan]:
  """Rebase the global ``cu_seqlens`` (host integers, ``cu[0] = 0``,
  ``cu[-1] = bounds[-1]``) to the slabs ``[bounds[k], bounds[k+1])``."""
  cu = [int(v) for v in cu_seqlens]
  if not cu or cu[0] != 0 or cu[-1] != bounds[-1] or bounds[0] != 0:
    raise ValueError("cu_seqlens must start at 0 and end at the last slab edge")
  if any(b < a for a, b in zip(cu, cu[1:])):
    raise ValueError("cu_seqlens must be non-decreasing")
  edges = sorted(set(cu))
  plans = []
  for t0, t1 in zip(bounds, bounds[1:]):
    if t1 <= t0:
      raise ValueError(f"empty slab [{t0}, {t1})")
    inner = [v - t0 for v in edges if t0 < v < t1]
    plans.append(SlabPlan(t0, t1, tuple([0] + inner + [t1 - t0]), t0 in edges, bool(inner)))
  return plans


# ---------------------------------------------------------------------------
# carry folds (device tensors of one row each; no kernels, no communication)
# ---------------------------------------------------------------------------

def forward_carry(plans: Sequence[SlabPlan], aggregates: Sequence[torch.Tensor],
                  rank: int) -> torch.Tensor:
  """Carry ``[C, 2]`` = (gate product since the sequence start, state) that
  enters slab ``rank``, folded from the aggregates ``[C, 2]`` = (P, Y) of the
  slabs before it (each scanned from a zero state)."""
  ref = aggregates[0]
  prod = torch.ones(ref.shape[0], dtype=ref.dtype, device=ref.device)
  state = torch.zeros_like(prod)
  for j in range(rank):
    P, Y = aggregates[j][:, 0], aggregates[j][:, 1]
    if plans[j].last_piece_continues:
      state = P * state + Y
      prod = P * prod
    else:  # the last piece of slab j starts inside it (or at its first column)
      state = Y.clone()
      prod = P.clone()
  if plans[rank].starts_new:
    prod.fill_(1.0)
    state.zero_()
  return torch.stack([prod, state], dim=1).contiguous()


def backward_carry(plans: Sequence[SlabPlan], aggregates: Sequence[torch.Tensor],
                   first_gates: Sequence[torch.Tensor], rank: int) -> torch.Tensor:
  """Additive adjoint term ``[C]`` for the last column of slab ``rank``:
  ``g[t1] * dh[t1]`` from the slab after it when the sequence goes on across
  the edge, else 0.  ``aggregates[j]`` = (Q, D): coefficient product and
  adjoint at slab j's first column from a zero carry; ``first_gates[j]`` =
  slab j's first gate column."""
  ref = aggregates[0]
  carry = torch.zeros(ref.shape[0], dtype=ref.dtype, device=ref.device)
  for j in range(len(plans) - 1, rank, -1):
    Q, D = aggregates[j][:, 0], aggregates[j][:, 1]
    dh_first = D + Q * carry if not plans[j].inner_boundary else D.clone()
    carry = first_gates[j] * dh_first if not plans[j].starts_new else torch.zeros_like(D)
  return carry.contiguous()


def state_halo(plans: Sequence[SlabPlan], last_states: Sequence[torch.Tensor],
               rank: int) -> torch.Tensor:
  """``h[t0 - 1]`` per row for slab ``rank`` (0 where a sequence starts at t0)."""
  ref = last_states[0]
  if rank == 0 or plans[rank].starts_new:
    return torch.zeros(ref.shape[0], dtype=torch.float32, device=ref.device)
  return last_states[rank - 1].float().contiguous()


# ---------------------------------------------------------------------------
# per-slab passes (one GPU, one slab)
# ---------------------------------------------------------------------------

_CU_CACHE: dict[tuple, torch.Tensor] = {}


def _cu_tensor(plan: SlabPlan, device) -> torch.Tensor:
  """The slab's rebased boundaries on the device, uploaded once per plan (a
  fresh upload from pageable memory would synchronise every pass)."""
  key = (plan.local_cu, str(torch.device(device)))
  t = _CU_CACHE.get(key)
  if t is None:
    if len(_CU_CACHE) > 256:
      _CU_CACHE.clear()
    t = torch.tensor(plan.local_cu, dtype=torch.int64, device=device)
    _CU_CACHE[key] = t
  return t


def slab_forward_aggregate(gates: torch.Tensor, tokens: torch.Tensor,
                           plan: SlabPlan) -> torch.Tensor:
  """Pass 1 of the forward: (P, Y) ``[C, 2]`` of the slab from a zero state."""
  C = gates.shape[0]
  agg = torch.empty(C, 2, dtype=torch.float32, device=gates.device)
  cu = _cu_tensor(plan, gates.device)
  _lib.forward_slab(gates, tokens, None, None, cu, cu.numel() - 1, C, False,
                    row_aggregate=agg)
  return agg


def slab_forward(gates: torch.Tensor, tokens: torch.Tensor, plan: SlabPlan,
                 carry: torch.Tensor, out: torch.Tensor | None = None,
                 gates_out: torch.Tensor | None = None) -> torch.Tensor:
  """Pass 2 of the forward: the slab's states with ``carry`` [C, 2] entering."""
  C = gates.shape[0]
  y = torch.empty_like(tokens) if out is None else out
  cu = _cu_tensor(plan, gates.device)
  _lib.forward_slab(gates, tokens, y, gates_out, cu, cu.numel() - 1, C, False,
                    row_carry=carry)
  return y


def slab_backward_aggregate(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                            plan: SlabPlan) -> torch.Tensor:
  """Pass 1 of the backward: (Q, D) ``[C, 2]`` at the slab's first column from
  a zero carry at its last column."""
  C = gates.shape[0]
  agg = torch.empty(C, 2, dtype=torch.float32, device=gates.device)
  zero = torch.zeros(C, dtype=torch.float32, device=gates.device)
  cu = _cu_tensor(plan, gates.device)
  _lib.backward_slab(grad, gates, states, None, None, cu, cu.numel() - 1, C, True,
                     row_carry=zero, row_aggregate=agg)
  return agg


def slab_backward(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                  plan: SlabPlan, carry: torch.Tensor,
                  halo: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
  """Pass 2 of the backward: (d_gates, d_tokens) of the slab."""
  C = gates.shape[0]
  dx = torch.empty_like(grad)
  dg = torch.empty_like(gates)
  cu = _cu_tensor(plan, gates.device)
  _lib.backward_slab(grad, gates, states, dx, dg, cu, cu.numel() - 1, C, True,
                     row_carry=carry, row_state_halo=halo)
  return dg, dx


# ---------------------------------------------------------------------------
# single-process emulation: every slab on the current device, exchange = list
# ---------------------------------------------------------------------------

def emulate_forward(gates: Sequence[torch.Tensor], tokens: Sequence[torch.Tensor],
                    plans: Sequence[SlabPlan]) -> list[torch.Tensor]:
  """The time-sharded forward of all slabs in one process (same passes and
  folds as the distributed driver; the exchange is a Python list)."""
  aggs = [slab_forward_aggregate(g, x, p) for g, x, p in zip(gates, tokens, plans)]
  return [slab_forward(g, x, p, forward_carry(plans, aggs, k))
          for k, (g, x, p) in enumerate(zip(gates, tokens, plans))]


def emulate_backward(grads: Sequence[torch.Tensor], gates: Sequence[torch.Tensor],
                     states: Sequence[torch.Tensor],
                     plans: Sequence[SlabPlan]) -> list[tuple[torch.Tensor, torch.Tensor]]:
  """The time-sharded backward of all slabs in one process."""
  aggs = [slab_backward_aggregate(dy, g, h, p) for dy, g, h, p in zip(grads, gates, states, plans)]
  firsts = [g[:, 0].float().contiguous() for g in gates]
  lasts = [h[:, -1].float().contiguous() for h in states]
  return [slab_backward(dy, g, h, p, backward_carry(plans, aggs, firsts, k),
                        state_halo(plans, lasts, k))
          for k, (dy, g, h, p) in enumerate(zip(grads, gates, states, plans))]


# ---------------------------------------------------------------------------
# multi-process driver (one rank per GPU, torch.distributed)
# ---------------------------------------------------------------------------

def _all_gather(t: torch.Tensor, group=None) -> list[torch.Tensor]:
  """One all-gather of a small per-row record (NCCL on CUDA tensors, gloo on
  CPU tensors); returns every rank's tensor, rank order."""
  import torch.distributed as dist
  world = dist.get_world_size(group)
  t = t.contiguous()
  out = [torch.empty_like(t) for _ in range(world)]
  dist.all_gather(out, t, group=group)
  return out


def _rank_plans(cu_seqlens, bounds) -> list[SlabPlan]:
  cu = cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else list(cu_seqlens)
  return plan_slabs(cu, bounds)


def time_sharded_forward(gates: torch.Tensor, tokens: torch.Tensor, plans: Sequence[SlabPlan],
                         rank: int, gather: Callable[[torch.Tensor], list[torch.Tensor]]):
  """Forward of this rank's slab: aggregate, exchange, seeded scan."""
  agg = slab_forward_aggregate(gates, tokens, plans[rank])
  aggs = gather(agg)
  return slab_forward(gates, tokens, plans[rank], forward_carry(plans, aggs, rank))


def time_sharded_backward(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                          plans: Sequence[SlabPlan], rank: int,
                          gather: Callable[[torch.Tensor], list[torch.Tensor]]):
  """Backward of this rank's slab: aggregate, one exchange of
  (Q, D, first gate, last state) per row, seeded fused backward."""
  agg = slab_backward_aggregate(grad, gates, states, plans[rank])
  packed = torch.cat([agg, gates[:, :1].float(), states[:, -1:].float()], dim=1)
  recs = gather(packed)
  aggs = [r[:, :2].contiguous() for r in recs]
  firsts = [r[:, 2].contiguous() for r in recs]
  lasts = [r[:, 3].contiguous() for r in recs]
  return slab_backward(grad, gates, states, plans[rank],
                       backward_carry(plans, aggs, firsts, rank),
                       state_halo(plans, lasts, rank))


class ScanCausalTimeShard(torch.autograd.Function):
  """Autograd over one rank's slab; every rank of ``group`` calls it with its
  own slab, the same ``cu_seqlens`` (global, host integers) and ``bounds``."""

  @staticmethod
  def forward(ctx, gates, tokens, cu_seqlens, bounds, group):
    import torch.distributed as dist
    plans = _rank_plans(cu_seqlens, bounds)
    rank = dist.get_rank(group)
    gather = lambda t: _all_gather(t, group)  # noqa: E731
    out = time_sharded_forward(gates, tokens, plans, rank, gather)
    ctx.save_for_backward(out, gates)
    ctx.plans, ctx.rank, ctx.group = plans, rank, group
    return out

  @staticmethod
  def backward(ctx, grad):
    out, gates = ctx.saved_tensors
    gather = lambda t: _all_gather(t, ctx.group)  # noqa: E731
    dg, dx = time_sharded_backward(grad.contiguous(), gates, out, ctx.plans, ctx.rank, gather)
    return dg, dx, None, None, None


def scan_causal_time_sharded(gates: torch.Tensor, tokens: torch.Tensor, args: dict) -> torch.Tensor:
  """``scan_causal`` for a time-sharded sequence axis.

  ``gates``, ``tokens``: this rank's slab ``[C, t1 - t0]`` (contiguous, CUDA,
  16-byte aligned).  ``args``: ``{"cu_seqlens": global boundaries (host ints
  or a tensor), "bounds": slab edges (one per rank, plus the total),
  "group": process group or None}``.  The last rank's slab ends the axis."""
  return ScanCausalTimeShard.apply(gates, tokens, args["cu_seqlens"], list(args["bounds"]),
                                   args.get("group"))
