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
    """Answers of one rank as fixed-size fp32 records (one row per question)."""

    rows: torch.Tensor   # [n, REC]

    @classmethod
    def pack(cls, qids, argmax, confidence, score, probs) -> AnswerRecords:
        n = len(qids)
        rows = torch.zeros(n, REC, dtype=torch.float32, device=probs.device)
        rows[:, 0] = torch.as_tensor(qids, dtype=torch.float32, device=probs.device)
        rows[:, 1] = argmax.float()
        rows[:, 2] = confidence.float()
        rows[:, 3] = score.float()
        k = min(probs.shape[1], PROB_SLOTS)
        rows[:, 4:4 + k] = probs[:, :k].float()
        return cls(rows)


def gather_answers(local: AnswerRecords, group=None) -> torch.Tensor:
    """All-gather every rank's records; returns [total, REC] sorted by question id.

    Counts differ per rank, so the counts go first (one small collective) and the records
    are padded to the largest count (id -1 marks padding). Every rank issues the same two
    collectives in the same order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = local.rows.device
    n = torch.tensor([local.rows.shape[0]], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    mx = int(max(int(c) for c in counts))
    padded = torch.full((mx, REC), -1.0, dtype=torch.float32, device=dev)
    padded[: local.rows.shape[0]] = local.rows
    out = torch.empty(world * mx, REC, dtype=torch.float32, device=dev)
    if dev.type == "cuda":
        dist.all_gather_into_tensor(out, padded, group=group)
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
        out = torch.cat(parts)
    out = out[out[:, 0] >= 0]
    return out[torch.argsort(out[:, 0])]
