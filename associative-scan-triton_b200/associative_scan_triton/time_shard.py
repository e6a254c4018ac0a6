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
     NVLink) into a preallocated ``[W, 2C]`` buffer;
  3. each rank folds the records of the ranks before it into its carry
     ``(product, state)`` with one small kernel (``ascan_time_shard_fold``;
     :func:`forward_carry` is the same fold on the host);
  4. seeded pass: the slab's forward with that carry entering each row's
     first column (``ascan_forward_slab`` with ``row_carry``).
  Pass 1 is a row reduction over the slab's last sequence piece (no scan, no
  stores).  Traffic: 2 reads in pass 1, 2 reads + 1 write in pass 2 (5
  element transfers against 3 for a single-device scan).

backward (``dh[t] = dy[t] + g[t+1] dh[t+1]``, ``dg[t] = dh[t] h[t-1]``)
  mirrored from the last rank to the first; the exchange also carries each
  slab's first gate column and last state column, the neighbours that the
  adjacent slabs' edge elements need (:func:`backward_carry`).

Sequence boundaries come from the global ``cu_seqlens`` (shared by every
channel, as in the reference's packed layout); :func:`plan_slabs` rebases them
to each slab and records whether the slab's first piece continues a sequence
from the previous slab and whether a boundary lies inside it.  The carry
folds need only those flags and the exchanged per-row records, so they are
the same code for the multi-process driver (:class:`TimeShardStep`,
:func:`scan_causal_time_sharded`, :class:`ScanCausalTimeShard`), for
single-process emulation of all slabs on one GPU (:func:`emulate_forward`,
:func:`emulate_backward`) and, restated on the host
(:func:`forward_carry`, :func:`backward_carry`, :func:`state_halo`), for the
CPU protocol tests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch

from . import _lib

__all__ = [
  "SlabPlan", "plan_slabs", "even_bounds", "forward_carry", "backward_carry",
  "slab_forward_aggregate", "slab_forward", "slab_backward_aggregate", "slab_backward",
  "emulate_forward", "emulate_backward", "plan_masks", "fold_forward", "fold_backward",
  "TimeShardStep", "scan_causal_time_sharded", "ScanCausalTimeShard", "PeerExchange", "row_parts",
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


def plan_masks(plans: Sequence[SlabPlan]) -> tuple[int, int]:
  """(starts_new, inner_boundary) bit masks over the slabs (at most 32)."""
  if len(plans) > 32:
    raise ValueError("at most 32 slabs")
  starts = sum(1 << j for j, p in enumerate(plans) if p.starts_new)
  inner = sum(1 << j for j, p in enumerate(plans) if p.inner_boundary)
  return starts, inner


def fold_forward(records: torch.Tensor, plans: Sequence[SlabPlan], rank: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
  """:func:`forward_carry` on the device: ``records`` ``[W, >= 2C]`` float32
  holds every slab's (P, Y) row aggregate interleaved in its first 2C floats."""
  C = records.shape[1] // 2 if out is None else out.shape[0]
  carry = torch.empty(C, 2, dtype=torch.float32, device=records.device) if out is None else out
  starts, inner = plan_masks(plans)
  _lib.time_shard_fold(records, len(plans), rank, C, starts, inner, 0, carry)
  return carry


def fold_backward(records: torch.Tensor, plans: Sequence[SlabPlan], rank: int,
                  carry_out: torch.Tensor | None = None,
                  halo_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
  """:func:`backward_carry` and :func:`state_halo` on the device: record j of
  ``records`` ``[W, 4C]`` is slab j's (Q, D) aggregate (2C floats), first gate
  column (C) and last state column (C)."""
  C = records.shape[1] // 4
  dev = records.device
  carry = torch.empty(C, dtype=torch.float32, device=dev) if carry_out is None else carry_out
  halo = torch.empty(C, dtype=torch.float32, device=dev) if halo_out is None else halo_out
  starts, inner = plan_masks(plans)
  _lib.time_shard_fold(records, len(plans), rank, C, starts, inner, 1, carry, halo)
  return carry, halo


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
                           plan: SlabPlan, out: torch.Tensor | None = None) -> torch.Tensor:
  """Pass 1 of the forward: (P, Y) ``[C, 2]`` of the slab from a zero state."""
  C = gates.shape[0]
  agg = torch.empty(C, 2, dtype=torch.float32, device=gates.device) if out is None else out
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
                            plan: SlabPlan, out: torch.Tensor | None = None,
                            zero: torch.Tensor | None = None) -> torch.Tensor:
  """Pass 1 of the backward: (Q, D) ``[C, 2]`` at the slab's first column from
  a zero carry at its last column."""
  C = gates.shape[0]
  agg = torch.empty(C, 2, dtype=torch.float32, device=gates.device) if out is None else out
  if zero is None:
    zero = torch.zeros(C, dtype=torch.float32, device=gates.device)
  cu = _cu_tensor(plan, gates.device)
  _lib.backward_slab(grad, gates, states, None, None, cu, cu.numel() - 1, C, True,
                     row_carry=zero, row_aggregate=agg)
  return agg


def slab_backward(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                  plan: SlabPlan, carry: torch.Tensor, halo: torch.Tensor,
                  d_gates: torch.Tensor | None = None,
                  d_tokens: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
  """Pass 2 of the backward: (d_gates, d_tokens) of the slab."""
  C = gates.shape[0]
  dx = torch.empty_like(grad) if d_tokens is None else d_tokens
  dg = torch.empty_like(gates) if d_gates is None else d_gates
  cu = _cu_tensor(plan, gates.device)
  _lib.backward_slab(grad, gates, states, dx, dg, cu, cu.numel() - 1, C, True,
                     row_carry=carry, row_state_halo=halo)
  return dg, dx


# ---------------------------------------------------------------------------
# the exchange over peer memory (no collective)
# ---------------------------------------------------------------------------

class PeerExchange:
  """One rank's side of the carry exchange over peer memory
  (``ascan_time_shard_exchange``): its exchange buffer, the other ranks'
  buffers mapped into this process through CUDA IPC, and a device table of
  all of them.  :meth:`exchange` publishes this rank's record, waits for the
  records its slab depends on and folds them into the carry in one kernel --
  the all-gather and the fold of the collective path in one launch, with the
  backward record's edge columns read straight from the slab's tensors.

  :meth:`connect` is collective over a process group (one rank per GPU);
  :meth:`emulated` builds every rank's side in one process on one device,
  for tests (publish every rank, then fold every rank)."""

  def __init__(self, num_channels: int, world: int, rank: int, device, own: int,
               addresses: Sequence[int], mapped: Sequence[int] = ()):
    self.C, self.world, self.rank = int(num_channels), int(world), int(rank)
    self.device = torch.device(device)
    self.own = int(own)
    self.mapped = list(mapped)  # peers' buffers this process mapped (closed on close())
    self.table = torch.tensor([int(a) for a in addresses], dtype=torch.int64, device=self.device)
    self._open = True

  @classmethod
  def connect(cls, num_channels: int, device, group=None) -> "PeerExchange":
    """Every rank of ``group`` creates its buffer; the IPC handles go round
    with one ``all_gather_object`` and every rank maps the others' buffers.

    When a step fails, the error propagates after this rank has unmapped the
    buffers it already mapped; its own buffer is freed only if its handle
    never left the process (once the handles went round, another rank may
    hold a mapping of it, and it stays allocated until the process ends)."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    device = torch.device(device)
    own = _lib.exchange_create(num_channels, device)
    shared = False
    mapped: list[int] = []
    try:
      handle = _lib.exchange_export(own)
      handles: list = [None] * world
      shared = True  # from here on, other ranks may map the buffer
      dist.all_gather_object(handles, handle, group=group)
      addresses = []
      for j, h in enumerate(handles):
        if j == rank:
          addresses.append(own)
        else:
          peer = _lib.exchange_import(h, device)
          mapped.append(peer)
          addresses.append(peer)
    except BaseException:
      for peer in mapped:
        try:
          _lib.exchange_close(peer)
        except Exception:  # keep the original error
          pass
      if not shared:
        try:
          _lib.exchange_destroy(own)
        except Exception:
          pass
      raise
    return cls(num_channels, world, rank, device, own, addresses, mapped)

  @classmethod
  def emulated(cls, num_channels: int, world: int, device) -> list["PeerExchange"]:
    """All ``world`` ranks' sides in this process on ``device``."""
    bufs = [_lib.exchange_create(num_channels, device) for _ in range(world)]
    return [cls(num_channels, world, k, device, bufs[k], bufs) for k in range(world)]

  def exchange(self, direction: int, mode: int, masks: tuple[int, int],
               aggregate: torch.Tensor | None, carry: torch.Tensor | None,
               halo: torch.Tensor | None = None, gates: torch.Tensor | None = None,
               states: torch.Tensor | None = None, timeout_s: float = 2.0,
               parts: int = 1) -> None:
    """One exchange of ``direction`` (0 forward, 1 backward); ``mode``
    ``_lib.EXCHANGE_PUBLISH``, ``_lib.EXCHANGE_FOLD`` or ``_lib.EXCHANGE_BOTH``;
    ``parts`` > 1: the slab's rows were scanned as that many parts each
    (:func:`row_parts`), one aggregate and one carry per part."""
    starts, inner = masks
    _lib.time_shard_exchange(self.own, self.table, self.world, self.rank, self.C, aggregate,
                             starts, inner, direction, mode, carry, halo, gates=gates,
                             states=states, timeout_s=timeout_s, parts=parts)

  def close(self, barrier: Callable[[], None] | None = None) -> None:
    """Unmaps the peers' buffers, waits at ``barrier`` (every rank must have
    unmapped this rank's buffer before it is freed) and frees this rank's."""
    if not self._open:
      return
    self._open = False
    torch.cuda.synchronize(self.device)
    for peer in self.mapped:
      _lib.exchange_close(peer)
    if barrier is not None:
      barrier()
    _lib.exchange_destroy(self.own)


def row_parts(num_channels: int, length: int, plan: SlabPlan, device,
              waves: int = 4, tile: int = 8192) -> int:
  """How many parts H to cut each row of a slab into for the peer exchange:
  the smallest power of two with H * C rows filling ``waves`` waves of the
  persistent kernels (one CTA per SM), so that in the seeded passes' tile
  order a tile's predecessor is several waves older; 1 when the slab has a
  sequence boundary inside or its parts would not be whole ``tile``s."""
  if plan.inner_boundary:
    return 1
  sms = torch.cuda.get_device_properties(torch.device(device)).multi_processor_count
  H = 1
  while H * num_channels < waves * sms and length % (2 * H * tile) == 0:
    H *= 2
  return H


# ---------------------------------------------------------------------------
# single-process emulation: every slab on the current device, exchange = list
# ---------------------------------------------------------------------------

def emulate_forward(gates: Sequence[torch.Tensor], tokens: Sequence[torch.Tensor],
                    plans: Sequence[SlabPlan],
                    peers: Sequence[PeerExchange] | None = None) -> list[torch.Tensor]:
  """The time-sharded forward of all slabs in one process: the same passes
  and device fold as the distributed driver; the exchange is writing every
  slab's record into one ``[W, 2C]`` buffer, or, with ``peers``
  (:meth:`PeerExchange.emulated`), the peer-memory exchange kernel: every
  rank publishes, then every rank folds."""
  C, W = gates[0].shape[0], len(plans)
  records = torch.empty(W, 2 * C, dtype=torch.float32, device=gates[0].device)
  for k, (g, x, p) in enumerate(zip(gates, tokens, plans)):
    slab_forward_aggregate(g, x, p, out=records[k].view(C, 2))
  if peers is None:
    carries = [fold_forward(records, plans, k) for k in range(W)]
  else:
    masks = plan_masks(plans)
    carries = [torch.empty(C, 2, dtype=torch.float32, device=gates[0].device) for _ in range(W)]
    for k in range(W):
      peers[k].exchange(0, _lib.EXCHANGE_PUBLISH, masks, records[k].view(C, 2), None)
    for k in range(W):
      peers[k].exchange(0, _lib.EXCHANGE_FOLD, masks, None, carries[k])
  return [slab_forward(g, x, p, carries[k])
          for k, (g, x, p) in enumerate(zip(gates, tokens, plans))]


def emulate_backward(grads: Sequence[torch.Tensor], gates: Sequence[torch.Tensor],
                     states: Sequence[torch.Tensor], plans: Sequence[SlabPlan],
                     peers: Sequence[PeerExchange] | None = None
                     ) -> list[tuple[torch.Tensor, torch.Tensor]]:
  """The time-sharded backward of all slabs in one process (``peers``: as in
  :func:`emulate_forward`)."""
  C, W = gates[0].shape[0], len(plans)
  device = gates[0].device
  records = torch.empty(W, 4 * C, dtype=torch.float32, device=device)
  zero = torch.zeros(C, dtype=torch.float32, device=device)
  for k, (dy, g, h, p) in enumerate(zip(grads, gates, states, plans)):
    slab_backward_aggregate(dy, g, h, p, out=records[k, :2 * C].view(C, 2), zero=zero)
    if peers is None:
      records[k, 2 * C:3 * C].copy_(g[:, 0])
      records[k, 3 * C:].copy_(h[:, -1])
  if peers is None:
    folds = [fold_backward(records, plans, k) for k in range(W)]
  else:
    masks = plan_masks(plans)
    folds = [(torch.empty(C, dtype=torch.float32, device=device),
              torch.empty(C, dtype=torch.float32, device=device)) for _ in range(W)]
    for k in range(W):
      peers[k].exchange(1, _lib.EXCHANGE_PUBLISH, masks, records[k, :2 * C].view(C, 2), None,
                        gates=gates[k], states=states[k])
    for k in range(W):
      peers[k].exchange(1, _lib.EXCHANGE_FOLD, masks, None, folds[k][0], halo=folds[k][1])
  return [slab_backward(dy, g, h, p, folds[k][0], folds[k][1])
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


class TimeShardStep:
  """One rank's slab of a time-sharded causal scan, forward and backward,
  with every buffer allocated once: the records, their all-gather targets,
  the carries and (unless the caller passes its own) the outputs.

  forward:  row reduction -> all-gather of [2C] floats -> device fold ->
            seeded forward slab pass;
  backward: row reduction + first gate / last state columns -> all-gather
            of [4C] floats -> device fold -> seeded fused backward slab pass.
  Six kernels and two collectives per fwd+bwd, no host synchronisation, so a
  step can be captured in a CUDA graph.  ``gather(out, inp)`` defaults to
  ``torch.distributed.all_gather_into_tensor`` on ``group``.

  ``exchange="peer"`` (every rank on one node, one GPU each) replaces each
  direction's all-gather and fold -- and the backward's two column copies --
  by one :class:`PeerExchange` kernel over NVLink peer memory: three kernels
  per direction, no collective.  Call :meth:`close` (collective) before the
  process group goes away."""

  def __init__(self, shape, dtype, plans: Sequence[SlabPlan], rank: int, device,
               group=None, gather: Callable[[torch.Tensor, torch.Tensor], None] | None = None,
               allocate_outputs: bool = True, exchange: str = "nccl",
               timeout_s: float = 2.0):
    C, L = (int(v) for v in shape)
    self.C, self.L, self.rank, self.world = C, L, rank, len(plans)
    self.plans, self.plan = list(plans), plans[rank]
    if self.plan.length != L:
      raise ValueError(f"slab {rank} has {self.plan.length} columns, tensors have {L}")
    device = torch.device(device)
    self.cu = _cu_tensor(self.plan, device)
    self.num_seq = self.cu.numel() - 1
    f32 = dict(dtype=torch.float32, device=device)
    self.rec_f = torch.empty(2 * C, **f32)
    self.all_f = torch.empty(self.world, 2 * C, **f32)
    self.rec_b = torch.empty(4 * C, **f32)
    self.all_b = torch.empty(self.world, 4 * C, **f32)
    self.carry_f = torch.empty(C, 2, **f32)
    self.carry_b = torch.empty(C, **f32)
    self.halo = torch.empty(C, **f32)
    self.zero = torch.zeros(C, **f32)
    self.masks = plan_masks(plans)
    self.y = self.dx = self.dg = None
    if allocate_outputs:
      self.y = torch.empty(C, L, dtype=dtype, device=device)
      self.dx = torch.empty(C, L, dtype=dtype, device=device)
      self.dg = torch.empty(C, L, dtype=dtype, device=device)
    if exchange not in ("nccl", "peer"):
      raise ValueError(f"exchange must be 'nccl' or 'peer', got {exchange!r}")
    self.exchange_kind, self.timeout_s, self.group = exchange, float(timeout_s), group
    self.peer = PeerExchange.connect(C, device, group) if exchange == "peer" else None
    # peer exchange: every row scanned as H parts (one aggregate and one carry
    # per part), so that the seeded passes see H times more rows
    self.parts = row_parts(C, L, self.plan, device) if self.peer is not None else 1
    H = self.parts
    if H > 1:
      self.cu_parts = torch.tensor([0, L // H], dtype=torch.int64, device=device)
      self.agg_f = torch.empty(H * C, 2, **f32)
      self.agg_b = torch.empty(H * C, 2, **f32)
      self.carry_f = torch.empty(H * C, 2, **f32)
      self.carry_b = torch.empty(H * C, **f32)
      self.halo = torch.empty(H * C, **f32)
      self.zero = torch.zeros(H * C, **f32)
    if gather is None:
      import torch.distributed as dist

      def gather(out, inp):
        dist.all_gather_into_tensor(out, inp, group=group)
    self._gather = gather

  def close(self) -> None:
    """Releases the peer exchange (collective over the group); a no-op for
    the NCCL exchange."""
    if self.peer is not None:
      import torch.distributed as dist
      self.peer.close(barrier=lambda: dist.barrier(group=self.group))
      self.peer = None

  @staticmethod
  def _mark(marks):
    if marks is not None:
      ev = torch.cuda.Event(enable_timing=True)
      ev.record()
      marks.append(ev)

  def forward(self, gates: torch.Tensor, tokens: torch.Tensor,
              out: torch.Tensor | None = None, marks: list | None = None) -> torch.Tensor:
    """``marks``: if a list, a timing event is recorded after each phase
    (aggregate, exchange, fold, seeded pass)."""
    C, cu, S = self.C, self.cu, self.num_seq
    y = self.y if out is None else out
    if y is None:
      y = torch.empty_like(tokens)
    if self.parts > 1:
      return self._forward_parts(gates, tokens, y, marks)
    _lib.forward_slab(gates, tokens, None, None, cu, S, C, False,
                      row_aggregate=self.rec_f.view(C, 2))
    self._mark(marks)
    if self.peer is not None:  # exchange and fold in one kernel
      self.peer.exchange(0, _lib.EXCHANGE_BOTH, self.masks, self.rec_f.view(C, 2), self.carry_f,
                         timeout_s=self.timeout_s)
      self._mark(marks)
    else:
      self._gather(self.all_f, self.rec_f)
      self._mark(marks)
      starts, inner = self.masks
      _lib.time_shard_fold(self.all_f, self.world, self.rank, C, starts, inner, 0, self.carry_f)
    self._mark(marks)
    _lib.forward_slab(gates, tokens, y, None, cu, S, C, False, row_carry=self.carry_f)
    self._mark(marks)
    return y

  def backward(self, grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
               d_gates: torch.Tensor | None = None, d_tokens: torch.Tensor | None = None,
               marks: list | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``marks``: as in :meth:`forward` (aggregate + edge columns, exchange,
    fold, seeded pass)."""
    C, cu, S = self.C, self.cu, self.num_seq
    dg = self.dg if d_gates is None else d_gates
    dx = self.dx if d_tokens is None else d_tokens
    if dg is None:
      dg = torch.empty_like(gates)
    if dx is None:
      dx = torch.empty_like(grad)
    if self.parts > 1:
      return self._backward_parts(grad, gates, states, dg, dx, marks)
    _lib.backward_slab(grad, gates, states, None, None, cu, S, C, True, row_carry=self.zero,
                       row_aggregate=self.rec_b[:2 * C].view(C, 2))
    if self.peer is not None:  # edge columns, exchange and fold in one kernel
      self._mark(marks)
      self.peer.exchange(1, _lib.EXCHANGE_BOTH, self.masks, self.rec_b[:2 * C].view(C, 2),
                         self.carry_b, halo=self.halo, gates=gates, states=states,
                         timeout_s=self.timeout_s)
      self._mark(marks)
    else:
      self.rec_b[2 * C:3 * C].copy_(gates[:, 0])
      self.rec_b[3 * C:].copy_(states[:, -1])
      self._mark(marks)
      self._gather(self.all_b, self.rec_b)
      self._mark(marks)
      starts, inner = self.masks
      _lib.time_shard_fold(self.all_b, self.world, self.rank, C, starts, inner, 1, self.carry_b,
                           self.halo)
    self._mark(marks)
    _lib.backward_slab(grad, gates, states, dx, dg, cu, S, C, True, row_carry=self.carry_b,
                       row_state_halo=self.halo)
    self._mark(marks)
    return dg, dx


  def _views(self, *ts):
    Cv, Lv = self.parts * self.C, self.L // self.parts
    return [t.view(Cv, Lv) for t in ts]

  def _forward_parts(self, gates, tokens, y, marks):
    """Forward with every row cut into ``parts`` rows of L / parts columns
    (the slab has no sequence boundary inside): the same three passes on the
    [parts * C, L / parts] view; the exchange composes the parts' records and
    hands back one carry per part."""
    Cv = self.parts * self.C
    gv, xv, yv = self._views(gates, tokens, y)
    _lib.forward_slab(gv, xv, None, None, self.cu_parts, 1, Cv, False, row_aggregate=self.agg_f)
    self._mark(marks)
    self.peer.exchange(0, _lib.EXCHANGE_BOTH, self.masks, self.agg_f, self.carry_f,
                       timeout_s=self.timeout_s, parts=self.parts)
    self._mark(marks)
    self._mark(marks)
    _lib.forward_slab(gv, xv, yv, None, self.cu_parts, 1, Cv, False, row_carry=self.carry_f)
    self._mark(marks)
    return y

  def _backward_parts(self, grad, gates, states, dg, dx, marks):
    """Backward on the [parts * C, L / parts] view (see :meth:`_forward_parts`)."""
    Cv = self.parts * self.C
    dyv, gv, hv, dgv, dxv = self._views(grad, gates, states, dg, dx)
    _lib.backward_slab(dyv, gv, hv, None, None, self.cu_parts, 1, Cv, True, row_carry=self.zero,
                       row_aggregate=self.agg_b)
    self._mark(marks)
    self.peer.exchange(1, _lib.EXCHANGE_BOTH, self.masks, self.agg_b, self.carry_b,
                       halo=self.halo, gates=gates, states=states, timeout_s=self.timeout_s,
                       parts=self.parts)
    self._mark(marks)
    self._mark(marks)
    _lib.backward_slab(dyv, gv, hv, dxv, dgv, self.cu_parts, 1, Cv, True, row_carry=self.carry_b,
                       row_state_halo=self.halo)
    self._mark(marks)
    return dg, dx


def time_sharded_forward(gates: torch.Tensor, tokens: torch.Tensor, plans: Sequence[SlabPlan],
                         rank: int, gather: Callable[[torch.Tensor], list[torch.Tensor]]):
  """Forward of this rank's slab with a list-returning gather (host folds):
  aggregate, exchange, seeded scan."""
  agg = slab_forward_aggregate(gates, tokens, plans[rank])
  aggs = gather(agg)
  return slab_forward(gates, tokens, plans[rank], forward_carry(plans, aggs, rank))


def time_sharded_backward(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                          plans: Sequence[SlabPlan], rank: int,
                          gather: Callable[[torch.Tensor], list[torch.Tensor]]):
  """Backward of this rank's slab with a list-returning gather (host folds):
  aggregate, one exchange of (Q, D, first gate, last state) per row, seeded
  fused backward."""
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
    step = TimeShardStep(gates.shape, gates.dtype, plans, rank, gates.device, group=group,
                         allocate_outputs=False)
    out = step.forward(gates, tokens)
    ctx.save_for_backward(out, gates)
    ctx.step = step
    return out

  @staticmethod
  def backward(ctx, grad):
    out, gates = ctx.saved_tensors
    dg, dx = ctx.step.backward(grad.contiguous(), gates, out)
    return dg, dx, None, None, None


def scan_causal_time_sharded(gates: torch.Tensor, tokens: torch.Tensor, args: dict) -> torch.Tensor:
  """``scan_causal`` for a time-sharded sequence axis.

  ``gates``, ``tokens``: this rank's slab ``[C, t1 - t0]`` (contiguous, CUDA,
  16-byte aligned).  ``args``: ``{"cu_seqlens": global boundaries (host ints
  or a tensor), "bounds": slab edges (one per rank, plus the total),
  "group": process group or None}``.  The last rank's slab ends the axis."""
  return ScanCausalTimeShard.apply(gates, tokens, args["cu_seqlens"], list(args["bounds"]),
                                   args.get("group"))
