"""Continuous batching of requests (engine.RequestBatcher), on the host with a stand-in engine:
requests submitted from many threads share engine calls, each future gets its own result,
limits are respected and an engine error reaches every request of its batch."""

from __future__ import annotations

import threading
import time

import pytest
import torch

from strands_decider_b200.engine import RequestBatcher


class _Engine:
    def __init__(self, fail_on=None, delay=0.0):
        self._lock = threading.Lock()
        self.calls: list[int] = []
        self.fail_on, self.delay = fail_on, delay

    def _slot_probs_many(self, items):
        time.sleep(self.delay)
        self.calls.append(len(items))
        if self.fail_on is not None and any(it["state_text"] == self.fail_on for it in items):
            raise ValueError("engine failure")
        return [(torch.full((len(it["question_texts"]), 2), float(len(it["state_text"]))), len(it["state_text"]))
                for it in items]


def _submit_all(b, texts):
    futs = [None] * len(texts)

    def go(i):
        futs[i] = b.submit(texts[i], ["q"] * (1 + i % 3), [2] * (1 + i % 3), ["choice"] * (1 + i % 3))

    ts = [threading.Thread(target=go, args=(i,)) for i in range(len(texts))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return futs


def test_concurrent_requests_share_engine_calls_and_get_their_own_answers():
    eng = _Engine(delay=0.01)
    b = RequestBatcher(eng, max_requests=16, window_ms=50)
    texts = ["x" * (i + 1) for i in range(24)]
    futs = _submit_all(b, texts)
    for i, f in enumerate(futs):
        probs, ntok = f.result(timeout=10)
        assert ntok == i + 1 and probs.shape == (1 + i % 3, 2) and float(probs[0, 0]) == i + 1
    assert sum(eng.calls) == 24 and len(eng.calls) < 24 and max(eng.calls) <= 16
    b.close()


def test_token_budget_starts_a_new_batch():
    eng = _Engine()
    b = RequestBatcher(eng, max_requests=64, max_tokens=60, window_ms=50)
    futs = _submit_all(b, ["y" * 50] * 6)   # about 27 estimated tokens each: two fit per batch
    for f in futs:
        f.result(timeout=10)
    assert sum(eng.calls) == 6 and max(eng.calls) <= 2
    b.close()


def test_engine_errors_fail_every_request_of_the_batch():
    eng = _Engine(fail_on="bad")
    b = RequestBatcher(eng, max_requests=8, window_ms=100)
    futs = _submit_all(b, ["ok1", "bad", "ok2"])
    errors = [f.exception(timeout=10) for f in futs]
    assert all(isinstance(e, ValueError) for e in errors if e is not None)
    assert any(e is not None for e in errors)
    b.close()
    with pytest.raises(RuntimeError):
        b.submit("late", ["q"], [2], ["choice"])
