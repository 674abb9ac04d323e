"""Request sharding (LPT) and the answer all-gather, on CPU gloo ranks (world size 2 and 3).

The device forward is replaced by a deterministic host function of the request so the
collective logic runs without a GPU; the GPU path uses the same functions with NCCL.
Failure detection: a rank that dies before the gather makes the survivors' collective fail
within the process-group timeout (no GPU is involved)."""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from strands_decider_b200 import config, dispatch
from strands_decider_b200.synth import request_batch


def test_plan_shards_covers_every_request_once_and_balances():
    w = config.Workload("varlen", 64, (64, 2048), 32, 48, seed=3)
    reqs = request_batch(w, 1000, 0, 64)
    costs = [dispatch.request_cost(r) for r in reqs]
    for world in (1, 2, 3, 4, 8):
        shards = dispatch.plan_shards(costs, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(reqs)))
        loads = dispatch.shard_loads(costs, shards)
        # LPT bound: max load <= (4/3 - 1/(3m)) * optimum; check against the mean + largest item
        assert max(loads) <= sum(costs) / world + max(costs)
    assert dispatch.plan_shards(costs, 4) == dispatch.plan_shards(costs, 4)   # deterministic


def test_plan_shards_uniform_is_round_robin_like():
    shards = dispatch.plan_shards([10] * 8, 4)
    assert [len(s) for s in shards] == [2, 2, 2, 2]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fake_answers(req_ids: list[int], q_per_req: int) -> dispatch.AnswerRecords:
    qids = [r * q_per_req + q for r in req_ids for q in range(q_per_req)]
    n = len(qids)
    g = torch.Generator().manual_seed(0)
    probs = torch.rand(n, 3, generator=g)
    probs = probs / probs.sum(1, keepdim=True)
    # deterministic by question id so the gathered result can be checked
    probs = torch.stack([torch.tensor([(q % 7) / 10, (q % 5) / 10, 0.3]) for q in qids]) if n else probs
    return dispatch.AnswerRecords.pack(qids, probs.argmax(1), probs.max(1).values, torch.tensor(
        [float(q) for q in qids]), probs)


def _worker(rank: int, world: int, port: int, q: mp.Queue, fail_rank: int) -> None:
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        reqs = request_batch(config.Workload("t", 10, (5, 40), 3, 4, seed=1), 100, 0, 10)
        shards = dispatch.plan_shards([dispatch.request_cost(r) for r in reqs], world)
        if rank == fail_rank:
            raise RuntimeError("rank failed before the gather")
        rec = _fake_answers(shards[rank], 3)
        # every rank knows every shard, so the gather capacity needs no collective
        capacity = 3 * max(len(s) for s in shards)
        out = dispatch.gather_answers(rec, capacity, total=3 * len(reqs))
        dropped = dispatch.gather_answers(rec, capacity)      # padding dropped via the host
        assert torch.equal(out, dropped)
        q.put((rank, "ok", out.tolist()))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-300:]}"))


def _run(world: int, fail_rank: int = -1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world", [2, 3])
def test_gather_answers_over_gloo(world):
    res = _run(world)
    want = _fake_answers(list(range(10)), 3).rows
    for rank in range(world):
        status, payload = res[rank]
        assert status == "ok", payload
        got = torch.tensor(payload, dtype=torch.int32)
        assert got.shape == want.shape
        assert torch.equal(got, want)
        f = dispatch.AnswerRecords.as_floats(got)
        assert torch.equal(f[:, 0], torch.arange(30, dtype=torch.float32))


def test_answer_records_keep_large_question_ids_exact():
    """Ids past 2^24 (where fp32 collides) survive packing, and padding ids are refused."""
    ids = [2 ** 24 + 1, 2 ** 24, 2 ** 31 - 2]
    probs = torch.tensor([[0.2, 0.8], [0.6, 0.4], [0.5, 0.5]])
    rec = dispatch.AnswerRecords.pack(ids, probs.argmax(1), probs.max(1).values, torch.zeros(3), probs)
    assert rec.rows.dtype == torch.int32 and rec.rows[:, 0].tolist() == ids
    assert torch.equal(dispatch.AnswerRecords.as_floats(rec.rows)[:, 4:6], probs)
    with pytest.raises(ValueError):
        dispatch.AnswerRecords.pack([dispatch.PAD_ID], probs[:1].argmax(1), probs[:1, 0], torch.zeros(1), probs[:1])


def test_dead_rank_is_detected_by_the_survivors():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "error" and "failed before the gather" in res[1][1]
    # the survivor's collective ends with an error (timeout / connection closed), not a hang
    assert res[0][0] == "error"
