"""One rank of the multi-GPU time-shard test (launched by
torch.distributed.run from tests/test_time_shard.py::test_nccl_ranks_match_oracle).

Every rank builds the same seeded global problem and keeps its slab.  Mode
``nccl`` runs ``scan_causal_time_sharded`` forward and backward (one exchange
each over NCCL); mode ``peer`` runs three forward+backward steps of
``TimeShardStep(exchange="peer")`` (the exchange kernel over NVLink peer
memory) and checks that every step gives the same result (within fp32
reassociation).  The slabs are
gathered on rank 0, which checks them against the fp64 oracle on the whole
axis and writes ``<out_dir>/ok``.
"""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
for p in (str(REPO), str(REPO / "associative-scan-triton_b200"), str(HERE)):
  if p not in sys.path:
    sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from associative_scan_triton import time_shard as ts  # noqa: E402


def main() -> int:
  out_dir = Path(sys.argv[1])
  mode = sys.argv[2] if len(sys.argv) > 2 else "nccl"
  rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
  local = int(os.environ.get("LOCAL_RANK", rank))
  torch.cuda.set_device(local)
  dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                          device_id=torch.device("cuda", local))
  C, T = 16, 1 << 18
  cu = [0, 70000, 1 << 17, 200001, T]  # one boundary on a slab edge for world 2 and 4
  gen = torch.Generator().manual_seed(5)
  # gates of 1 or 1 - 2^-8: the gate product over the whole axis stays near
  # 0.13, so every slab's carry reaches the end of the axis
  g = (1.0 - (torch.rand(C, T, generator=gen) < 0.002).float() / 256).cuda()
  x = torch.randn(C, T, generator=gen).cuda()
  dy = torch.randn(C, T, generator=gen).cuda()
  bounds = ts.even_bounds(T, world, align=64)
  t0, t1 = bounds[rank], bounds[rank + 1]
  if mode == "peer":
    plans = ts.plan_slabs(cu, bounds)
    step = ts.TimeShardStep((C, t1 - t0), torch.float32, plans, rank, "cuda", exchange="peer",
                            timeout_s=10.0)
    gs, xs = g[:, t0:t1].contiguous(), x[:, t0:t1].contiguous()
    dys = dy[:, t0:t1].contiguous()
    runs = []
    for _ in range(3):
      y = step.forward(gs, xs).clone()
      dg, dx = step.backward(dys, gs, y)
      runs.append((y, dx.clone(), dg.clone()))
    torch.cuda.synchronize()
    from associative_scan_triton import _lib
    _lib.check_device_error()
    # every step the same result (within fp32 reassociation: a look-back
    # composes predecessors in a timing-dependent order)
    for r in runs[1:]:
      for a, b in zip(r, runs[0]):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5 * float(b.abs().max()))
    step.close()
    pieces = list(runs[-1])
  else:
    gs = g[:, t0:t1].contiguous().requires_grad_(True)
    xs = x[:, t0:t1].contiguous().requires_grad_(True)
    y = ts.scan_causal_time_sharded(gs, xs, {"cu_seqlens": cu, "bounds": bounds, "group": None})
    y.backward(dy[:, t0:t1].contiguous())
    pieces = [y.detach(), xs.grad, gs.grad]
  gathered = []
  for piece in pieces:  # slabs may differ in length: pad to the longest
    width = max(b - a for a, b in zip(bounds, bounds[1:]))
    pad = torch.zeros(C, width, device=piece.device)
    pad[:, : piece.shape[1]] = piece
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    gathered.append(torch.cat([b[:, : bounds[k + 1] - bounds[k]] for k, b in enumerate(bufs)], 1))
  dist.barrier()
  dist.destroy_process_group()
  if rank == 0:
    from oracle import oracle
    from scan_testlib import assert_close_to_gold
    cu_t = torch.tensor(cu, dtype=torch.int64)
    gold_y, _ = oracle.scan_fwd(g, x, cu_t)
    assert_close_to_gold(gathered[0], gold_y, torch.float32, f"{mode} time-shard y")
    gdx, gdg = oracle.scan_bwd(dy, g, gathered[0], cu_t)
    assert_close_to_gold(gathered[1], gdx, torch.float32, f"{mode} time-shard dx")
    assert_close_to_gold(gathered[2], gdg, torch.float32, f"{mode} time-shard dg")
    (out_dir / "ok").write_text(str(world))
  return 0


if __name__ == "__main__":
  sys.exit(main())
