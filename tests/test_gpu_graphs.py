"""CUDA graphs in the runtime: every DecisionModel forward replays a graph captured once per
shape bucket, with the batch padded up to the bucket by dummy sequences.

* A batch that is already a bucket (no padding) gives the same bits from a graph replay as
  from eager launches of the same kernels (the batch is sized so that no GEMM splits K, whose
  atomic partial sums are the one source of run-to-run differences).
* Padded batches (the prefix path, ragged states and questions) answer as the eager path
  within 1e-4 with the same argmax, and the padding reads and writes no cached state. (A padded
  batch has more rows, which can change how a small GEMM splits K and so the order of its fp32
  partial sums: differences of a few 1e-5 in a probability, as between two eager runs of
  batches of different sizes.)
* Batches that fall in the same bucket share one graph.
"""

from __future__ import annotations

import pytest
import torch

from strands_decider_b200 import config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    from strands_decider_b200 import _lib
    from strands_decider_b200.weights import DeviceWeights

    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    _lib.load()
    w = DeviceWeights.synthetic(config.TINY, seed=4, latent_device="cpu")
    yield w
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _models(w, **kw):
    from strands_decider_b200.runtime import DecisionModel

    return (DecisionModel(w, graphs=True, **kw), DecisionModel(w, graphs=False, **kw))


def test_graph_replay_equals_eager_bit_for_bit(tiny):
    from strands_decider_b200.runtime import ForwardBucket

    g = torch.Generator().manual_seed(1)
    V = config.TINY.vocab
    rows = [torch.randint(0, V, (128,), generator=g).tolist() for _ in range(64)]
    b = ForwardBucket.for_batch(8192, [128] * 64, 64, 4, False, False, False)
    assert (b.tokens, b.seqs, b.rows) == (8192, 64, 64)      # no padding
    mg, me = _models(tiny, max_tokens=8192, pool_slots=2, pool_kv_tokens=256)
    opt = [[11, 12, 13, 14]] * 64
    args = (opt, [4] * 64, [1, 2] * 32, [1.0, 0.7] * 32)
    eager = me.score_prompts(rows, *args).cpu()
    first = mg.score_prompts(rows, *args).cpu()        # captures
    again = mg.score_prompts(rows, *args).cpu()        # replays
    for got in (first, again):
        assert torch.equal(got.probs, eager.probs)
        assert torch.equal(got.argmax, eager.argmax)
        assert torch.equal(got.confidence, eager.confidence) and torch.equal(got.score, eager.score)
    assert len(mg._graphs) == 1


def test_padded_buckets_answer_as_eager_and_leave_the_pool_alone(tiny):
    mg, me = _models(tiny, max_tokens=4096, pool_slots=8, pool_kv_tokens=2048)
    g = torch.Generator().manual_seed(2)
    V = config.TINY.vocab
    reqs = []
    for slen, qlens in [(70, [9, 1, 40]), (3, [5]), (130, [64, 17]), (1, [2, 31, 7, 8])]:
        reqs.append({"state": torch.randint(0, V, (slen,), generator=g).tolist(),
                     "questions": [torch.randint(0, V, (n,), generator=g).tolist() for n in qlens],
                     "kinds": [1] * len(qlens), "n_opts": [3] * len(qlens), "opt_ids": [[11, 12, 13]] * len(qlens)})
    got = mg.score_requests(reqs, ordinal_smoothing=0.1).cpu()
    want = me.score_requests(reqs, ordinal_smoothing=0.1).cpu()
    assert (got.probs - want.probs).abs().max().item() < 1e-4
    assert torch.equal(got.argmax, want.argmax)
    assert (got.confidence - want.confidence).abs().max().item() < 1e-4
    # the dummies saved nothing: the pools of both models hold the same states
    for a, b in ((mg.gdn_state, me.gdn_state), (mg.conv_hist, me.conv_hist)):
        assert (a[:, :4] - b[:, :4]).abs().max().item() < 1e-4
        assert a[:, 4:].abs().max().item() == 0.0
    assert torch.equal(mg.slot_len.cpu(), me.slot_len.cpu())
    # appends through graphs, then questions, still equal the eager path
    more = [torch.randint(0, V, (n,), generator=g).tolist() for n in (5, 1, 9, 2)]
    for m in (mg, me):
        m.prefill_states([r["state"] for r in reqs], [0, 1, 2, 3], reserve=32)
        m.append_states(more, [0, 1, 2, 3])
    qs = [r["questions"][0] for r in reqs]
    a = mg.score_suffixes(qs, [0, 1, 2, 3], [[11, 12]] * 4, [2] * 4, [0] * 4, [1.0] * 4).cpu()
    b = me.score_suffixes(qs, [0, 1, 2, 3], [[11, 12]] * 4, [2] * 4, [0] * 4, [1.0] * 4).cpu()
    assert (a.probs - b.probs).abs().max().item() < 1e-4


def test_batches_in_one_bucket_share_a_graph(tiny):
    mg, me = _models(tiny, max_tokens=2048, pool_slots=2, pool_kv_tokens=256)
    g = torch.Generator().manual_seed(3)
    V = config.TINY.vocab
    for lens in ((100, 120), (90, 125), (111, 111)):   # 220-222 tokens, longest 111-125: one bucket
        rows = [torch.randint(0, V, (n,), generator=g).tolist() for n in lens]
        got = mg.score_prompts(rows, [[11, 12, 13]] * 2, [3, 3], [1, 1], [1.0, 1.0]).cpu()
        want = me.score_prompts(rows, [[11, 12, 13]] * 2, [3, 3], [1, 1], [1.0, 1.0]).cpu()
        assert (got.probs - want.probs).abs().max().item() < 1e-4
    assert len(mg._graphs) == 1
