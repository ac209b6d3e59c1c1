"""Multi-GPU utterance scheduler (one engine per GPU, no collective on the data path).

Utterances of a box-wide request are independent (the reference serves one
sequence per TTSTransformer, src/tts_transformer.h:171-195), so the work
shards by utterance.  Cost of an utterance ~ prefill positions + frames to
generate; utterances are assigned longest-processing-time first to the least
loaded rank (LPT, a 4/3-approximation of the optimal makespan).  Each rank then
runs its share on its own GPU; only the final codes are gathered, through the
host (the process group is used for the plan broadcast and the gather).
"""
from __future__ import annotations

import dataclasses
import heapq
from typing import Callable, Sequence


@dataclasses.dataclass
class Utterance:
    uid: int
    prefill: int          # talker prefill positions
    frames: int           # frames to generate (max_len)
    payload: object = None

    @property
    def cost(self) -> int:
        return self.prefill + self.frames


def lpt_partition(utts: Sequence[Utterance], n_ranks: int) -> list[list[Utterance]]:
    """Longest-processing-time-first assignment; deterministic (ties by uid, rank)."""
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    heap = [(0, r) for r in range(n_ranks)]
    out: list[list[Utterance]] = [[] for _ in range(n_ranks)]
    for u in sorted(utts, key=lambda u: (-u.cost, u.uid)):
        load, r = heapq.heappop(heap)
        out[r].append(u)
        heapq.heappush(heap, (load + u.cost, r))
    return out


def makespan(parts: list[list[Utterance]]) -> int:
    return max((sum(u.cost for u in p) for p in parts), default=0)


def run_sharded(utts: Sequence[Utterance], run_one: Callable[[Utterance], object], rank: int, world: int,
                group=None) -> dict[int, object] | None:
    """Run this rank's LPT share with `run_one`; gather {uid: result} on rank 0.

    Every rank computes the same plan from the same list, so nothing but the
    results crosses ranks.  With world == 1 no process group is needed.
    """
    parts = lpt_partition(utts, world)
    mine = {u.uid: run_one(u) for u in parts[rank]}
    if world == 1:
        return mine
    import torch.distributed as dist
    gathered = [None] * world if rank == 0 else None
    dist.gather_object(mine, gathered, dst=0, group=group)
    if rank != 0:
        return None
    merged: dict[int, object] = {}
    for d in gathered:
        merged.update(d)
    return merged
