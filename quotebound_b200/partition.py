"""(batch x value-head group) partitioner for 1/2/4/8 GPUs of one box, one process per GPU.

The recurrence has no exchange between sequences or between value heads, so the work splits with no
data-path collective.  A group is the Hv/Hk value heads that read one key head, so dq and dk (summed
over the group, src/delta_grad.cpp:194-198) stay on one GPU.  The batch is split first (whole head
sets per GPU); only when there are fewer batch rows than GPUs are key-head groups split as well.

The one collective: the gate parameters A_log and dt_bias are shared by every batch row, so when
the batch is split their per-GPU gradient sums are added with one all-reduce of [dA_log | ddt_bias]
(2 * Hv float32).  Every rank writes its own heads' sums into a zeroed [2 * Hv] buffer, so one
all-reduce over all ranks gives the total whatever the split.
"""
from __future__ import annotations

import dataclasses

import torch


@dataclasses.dataclass(frozen=True)
class Shard:
    rank: int
    b0: int
    b1: int
    hk0: int
    hk1: int
    hv0: int
    hv1: int


def plan(B: int, Hk: int, Hv: int, world: int) -> list[Shard]:
    """The shard of every rank.  Raises ValueError when the shape does not split evenly."""
    if world < 1 or Hv % Hk:
        raise ValueError(f"partition: bad world {world} or heads (Hk {Hk}, Hv {Hv})")
    r = Hv // Hk
    shards = []
    if B % world == 0:
        per = B // world
        for w in range(world):
            shards.append(Shard(w, w * per, (w + 1) * per, 0, Hk, 0, Hv))
        return shards
    if world % B == 0 and Hk % (world // B) == 0:
        split = world // B
        per = Hk // split
        for w in range(world):
            b, j = divmod(w, split)
            shards.append(Shard(w, b, b + 1, j * per, (j + 1) * per, j * per * r, (j + 1) * per * r))
        return shards
    raise ValueError(f"partition: B={B}, Hk={Hk} do not split evenly over {world} GPUs")


def needs_allreduce(shards: list[Shard]) -> bool:
    """True when two ranks hold the same value head (then the gate-parameter gradients must be summed)."""
    owners = {}
    for s in shards:
        for h in range(s.hv0, s.hv1):
            owners[h] = owners.get(h, 0) + 1
    return any(c > 1 for c in owners.values())


def reduce_gate_grads(dA_log: torch.Tensor, ddt_bias: torch.Tensor, shard: Shard, Hv: int, group=None):
    """Sum this rank's [hv0, hv1) head sums with every other rank's: returns full [Hv] dA_log, ddt_bias."""
    buf = torch.zeros(2 * Hv, dtype=torch.float32, device=dA_log.device)
    buf[shard.hv0:shard.hv1] = dA_log
    buf[Hv + shard.hv0:Hv + shard.hv1] = ddt_bias
    if torch.distributed.is_initialized():
        torch.distributed.all_reduce(buf, group=group)
    return buf[:Hv], buf[Hv:]
