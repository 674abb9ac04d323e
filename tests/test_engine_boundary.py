"""The engine boundary on the host (no GPU): the B200 engine class is the reference's own
`SystemOneEngine` with the two device methods overridden, and the device loader refuses
before loading anything when no B200 is usable (the infer.py:516-519 convention, tested by
the reference in tests/test_devices.py:56-64)."""

from __future__ import annotations

import pytest
import torch

from tests.conftest import require_reference


def test_engine_class_inherits_the_reference_host_logic():
    infer = require_reference()
    from strands_decider_b200.engine import B200SlotProbs, reference_engine_class

    cls = reference_engine_class()
    assert issubclass(cls, infer.SystemOneEngine) and issubclass(cls, B200SlotProbs)
    assert cls is reference_engine_class()   # built once
    # the host logic is the reference's, not restated here
    for name in ("_fit", "_temperatures", "_option_idx", "_pad"):
        assert getattr(cls, name) is getattr(infer.SystemOneEngine, name), name
    assert cls._slot_probs_batched is B200SlotProbs._slot_probs_batched
    assert cls._slot_probs_shared_prefix is B200SlotProbs._slot_probs_shared_prefix


def test_load_engine_refuses_without_a_b200(monkeypatch, tmp_path):
    require_reference()
    from strands_decider_b200 import engine

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="b200"):
        engine.load_engine(str(tmp_path))
    with pytest.raises(ValueError, match="device"):
        engine.load_engine(str(tmp_path), device="cuda")
