"""Request sharding across GPUs (one process per GPU), host side only.

The decode path does not shard: every GPU holds a full weight replica and its
own paged KV pool, and serves a disjoint subset of the requests.  This module
is the host logic around that:

- partition(): assign requests to ranks, balancing the KV bytes each rank
  streams per step (longest request first onto the least loaded rank;
  deterministic, so every rank computes the same assignment without talking);
- ShardedRunner: run a per-rank serve function over the rank's share, then
  exchange outcomes on the host (torch.distributed object collectives, gloo or
  nccl -- never on the data path).  A rank whose serve function fails with
  DeviceError (the engine's QTB_E_DEVICE: a bounded wait expired or a device
  check failed) reports it; its requests are re-queued and partitioned over
  the surviving ranks, which serve them in the next round.  A rank leaves only
  between rounds, with none of its kernels in flight.

The reference serves batches on one host (qwen_tts.c:2389-2740,
qwen_tts_batch.h); this is the multi-GPU counterpart of its admission loop.
"""
from __future__ import annotations

import dataclasses
from typing import Callable, Dict, List, Sequence


class DeviceError(RuntimeError):
    """The engine reported QTB_E_DEVICE for this rank's work."""


@dataclasses.dataclass(frozen=True)
class Request:
    rid: int           # request id (unique)
    kv_len: int        # positions already in the KV cache (prompt / prefix)
    n_frames: int      # frames to decode


def request_cost(r: Request) -> int:
    """KV positions streamed over the request's decode (the dominant bytes at
    large batch: every step reads the whole cache)."""
    return r.n_frames * (r.kv_len + (r.n_frames + 1) // 2)


def partition(requests: Sequence[Request], ranks: Sequence[int]) -> Dict[int, List[Request]]:
    """Greedy longest-processing-time assignment of requests to `ranks`,
    ties broken by request id and rank order (identical on every process)."""
    out: Dict[int, List[Request]] = {r: [] for r in ranks}
    if not ranks:
        raise ValueError("no rank left to serve the requests")
    load = {r: 0 for r in ranks}
    for req in sorted(requests, key=lambda q: (-request_cost(q), q.rid)):
        dst = min(ranks, key=lambda r: (load[r], list(ranks).index(r)))
        out[dst].append(req)
        load[dst] += request_cost(req)
    for r in ranks:
        out[r].sort(key=lambda q: q.rid)
    return out


class ShardedRunner:
    """Serve a request set over the ranks of a process group.

    serve(rank, requests) -> {rid: result} runs on every rank for its share;
    it may raise DeviceError.  run() returns the union of all results on
    every rank (results must be picklable)."""

    def __init__(self, dist, group=None, max_rounds: int = 4):
        self.dist = dist
        self.group = group
        self.max_rounds = max_rounds

    def run(self, requests: Sequence[Request], serve: Callable[[int, List[Request]], Dict[int, object]]):
        dist = self.dist
        rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        alive = list(range(world))
        pending = list(requests)
        results: Dict[int, object] = {}
        self.failed: List[int] = []
        for _ in range(self.max_rounds):
            if not pending:
                break
            share = partition(pending, alive)
            mine = share.get(rank, [])
            ok, got = True, {}
            if rank in alive and mine:
                try:
                    got = serve(rank, mine)
                except DeviceError:
                    ok, got = False, {}
            outcomes = [None] * world
            dist.all_gather_object(outcomes, (rank, ok, got), group=self.group)
            newly_failed = []
            for r, ok_r, got_r in outcomes:
                if r in alive and not ok_r:
                    newly_failed.append(r)
                results.update(got_r)
            for r in newly_failed:
                alive.remove(r)
                self.failed.append(r)
            pending = [q for q in pending if q.rid not in results]
        if pending:
            raise RuntimeError(f"{len(pending)} requests unserved after {self.max_rounds} rounds "
                               f"(ranks left: {alive})")
        return results
