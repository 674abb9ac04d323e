"""Multi-GPU request sharding and the answer gather.

Requests share nothing and the model fits on every GPU, so the data-parallel split is by
request: one process per GPU, each with its own model, workspace and prefix pool. The only
collective is after the forwards: every rank's fixed-size answer records are all-gathered
(NCCL over NVLink on GPUs, gloo on CPU), so rank 0 (or every rank) holds all answers in
request order. Nothing runs inside the forward.

Balancing follows the reference's longest-processing-time planning for training steps
(src/strands_decider/distributed.py:134-196, `_best_cuts` / `plan_step`): requests are
sorted by token cost (state + all questions) and each goes to the least-loaded rank.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import torch

PROB_SLOTS = 8            # probabilities carried per answer record (kmax <= 8)
REC = 4 + PROB_SLOTS      # question id, argmax, confidence, score, probs...
PAD_ID = 2 ** 31 - 1      # question id of a padding record (sorts after every real one)


def request_cost(r: dict) -> int:
    """Tokens a request forwards through the prefix-cache path."""
    return len(r["state"]) + sum(len(q) for q in r["questions"])


def plan_shards(costs: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of request indices to `world` ranks.

    Deterministic: ties break by request index, then by rank. Each rank's list is sorted."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(s) for s in shards]


def shard_loads(costs: list[int], shards: list[list[int]]) -> list[int]:
    return [sum(costs[i] for i in s) for s in shards]


@dataclass
class AnswerRecords:
    """Answers of one rank as fixed-size int32 records, one row per question: column 0 the
    question id and column 1 the argmax as integers, columns 2.. the fp32 bit patterns of
    the confidence, the score and the probabilities (`as_floats` reads them back). Integer
    ids stay exact up to 2^31 - 2 (fp32 would collide past 2^24)."""

    rows: torch.Tensor   # [n, REC] int32

    @classmethod
    def pack(cls, qids, argmax, confidence, score, probs) -> AnswerRecords:
        dev = probs.device
        if isinstance(qids, torch.Tensor):
            if qids.dtype not in (torch.int32, torch.int64):
                raise TypeError("question ids must be an integer tensor")
            q = qids.to(device=dev, dtype=torch.int32)
        else:
            qids = list(qids)
            if qids and not 0 <= min(qids) <= max(qids) < PAD_ID:
                raise ValueError(f"question ids must lie in [0, {PAD_ID})")
            q = torch.as_tensor(qids, dtype=torch.int32, device=dev)
        n = int(q.numel())
        f = torch.zeros(n, REC, dtype=torch.float32, device=dev)
        f[:, 2] = confidence.float()
        f[:, 3] = score.float()
        k = min(probs.shape[1], PROB_SLOTS)
        f[:, 4:4 + k] = probs[:, :k].float()
        rows = f.view(torch.int32)
        rows[:, 0] = q
        rows[:, 1] = argmax.to(torch.int32)
        return cls(rows)

    @staticmethod
    def as_floats(rows: torch.Tensor) -> torch.Tensor:
        """[n, REC] float32: ids and argmax as values, the rest as stored."""
        f = rows.view(torch.float32).clone()
        f[:, 0] = rows[:, 0].float()
        f[:, 1] = rows[:, 1].float()
        return f


def gather_answers(local: AnswerRecords, capacity: int, total: int | None = None, group=None) -> torch.Tensor:
    """All-gather every rank's records with ONE collective; returns int32 [n, REC] sorted by
    question id.

    Every rank pads its records to `capacity` rows (the most any rank holds, which the shard
    plan gives every rank without a collective; padding rows carry id PAD_ID) and issues the
    same single all-gather. The result is sorted on the device, padding last, and cut to
    `total` rows when the caller knows the real count (no host synchronisation); with
    total=None the padding rows are dropped, which reads the count back to the host."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n, dev = local.rows.shape[0], local.rows.device
    if n > capacity:
        raise ValueError(f"{n} answer records exceed the gather capacity of {capacity}")
    padded = torch.full((capacity, REC), 0, dtype=torch.int32, device=dev)
    padded[:, 0] = PAD_ID
    padded[:n] = local.rows
    if dev.type == "cuda":
        out = torch.empty(world * capacity, REC, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(out, padded, group=group)
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
        out = torch.cat(parts)
    out = out[torch.argsort(out[:, 0], stable=True)]
    if total is not None:
        return out[:total]
    return out[out[:, 0] != PAD_ID]
