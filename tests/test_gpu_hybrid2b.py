"""Parity at the headline shapes: the 2B-shape NVFP4 decider (hidden 2048, 24 layers at 3:1
GDN : attention, GDN 16 heads x 128, attention 8q / 2kv x 256, FFN 6144, vocab 248320 tied) on
the B200, against the CPU oracle run on the same weights (the device's packed bytes read back
and dequantised by oracle.quant, the device's embedding table).

* The hybrid-2B workload's requests (a 512-token state, then a 3-way choice, a yes/no noul and
  a 3-level score, each a 32-token suffix): 8 requests through the prefix path in one batch,
  replayed from the runtime's CUDA graphs; the oracle checks 3 of them. Two configurations:
  the library defaults (the 4096-token state forward on dequantised weight copies with e4m3
  low planes and CTA-pair GEMMs, the 768-token question forward on streamed packed tiles with
  two bf16 planes), and every GEMM on the dequantised path with e4m3 low planes, as the
  benchmark's 65536-token batches run them.
* The prefix-cache workload's shapes: states of 64, 1000 and 2048 tokens, 32 questions of 48
  tokens each with 2 to 5 options.

Bar (option probabilities within 2e-3 absolute of the reference, same choice): every
probability within 2e-3 of the oracle's; the argmax equal wherever the oracle's two largest
probabilities differ by more than twice the largest error seen (a closer pair is a tie at this
precision), and such near-ties are rare (at most 2 of the rows).
"""

from __future__ import annotations

import os

import pytest
import torch

from oracle import head as OH
from oracle import synth as osynth
from oracle import torso as OT
from strands_decider_b200 import config

pytestmark = pytest.mark.gpu

TOL = 2e-3


@pytest.fixture(scope="module")
def hybrid2b():
    from strands_decider_b200 import _lib
    from strands_decider_b200.weights import DeviceWeights

    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    _lib.load()
    torch.set_num_threads(os.cpu_count() or 1)
    spec = config.HYBRID_2B
    w = DeviceWeights.synthetic(spec, seed=0, device="cuda", latent_device="cuda", keep_logical=True)
    W = osynth.device_logical_weights(w, seed=0)
    yield spec, w, W
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _oracle(spec, W, reqs) -> torch.Tensor:
    """Each request's state once into an explicit cache, then every question against it."""
    cfg = osynth.torso_config(spec)
    pooled, opt, nopt = [], [], []
    with torch.inference_mode():
        for r in reqs:
            _, cache = OT.forward_sequence(cfg, W, torch.tensor(r["state"]), keep_cache=True)
            for qi, q in enumerate(r["questions"]):
                hid, _ = OT.forward_sequence(cfg, W, torch.tensor(q), cache=cache)
                pooled.append(hid[-1])
                opt.append(r["opt_ids"][qi])
                nopt.append(r["n_opts"][qi])
    K = max(nopt)
    opt_t = torch.tensor([o + [0] * (K - len(o)) for o in opt])
    return OH.decide(torch.stack(pooled), W["embed"], opt_t, torch.tensor(nopt), torch.ones(len(nopt)))


def _check(got: torch.Tensor, want: torch.Tensor, n_opts: list[int]) -> float:
    got = got[:, : want.shape[1]]
    err = (got - want).abs().max().item()
    assert err < TOL, f"max |dp| {err:.2e} against the oracle"
    ties = 0
    for i, n in enumerate(n_opts):
        top2 = want[i, :n].topk(2).values
        if float(top2[0] - top2[1]) > 2 * err:
            assert int(got[i, :n].argmax()) == int(want[i, :n].argmax()), i
        else:
            ties += 1
    assert ties <= 2, f"{ties} near-tied rows"
    return err


@pytest.mark.parametrize("dequant_min_tokens", [0, 1])
def test_hybrid2b_workload_matches_oracle(hybrid2b, dequant_min_tokens):
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.synth import request_batch

    spec, w, W = hybrid2b
    reqs = request_batch(config.HYBRID_2B_WORKLOAD, spec.vocab, 0, 8)
    m = DecisionModel(w, max_tokens=4096, pool_slots=8, pool_kv_tokens=4096, dequant_min_tokens=dequant_min_tokens,
                      lo_plane="e4m3", graphs=True)
    got = m.score_requests(reqs).cpu()
    got2 = m.score_requests(reqs).cpu()      # the second call replays the captured graphs
    assert len(m._graphs) == 2
    assert (got.probs - got2.probs).abs().max().item() < 1e-6
    pick = [0, 3, 7]                          # the oracle's share: first, middle and last of the batch
    want = _oracle(spec, W, [reqs[i] for i in pick])
    rows = [3 * i + q for i in pick for q in range(3)]
    _check(got.probs[rows], want, [reqs[i]["n_opts"][q] for i in pick for q in range(3)])
    m.close()


def test_prefix_cache_workload_shapes_match_oracle(hybrid2b):
    """States of 64, 1000 and 2048 tokens, each with 32 questions of 48 tokens, 2-5 options."""
    from strands_decider_b200.runtime import DecisionModel

    spec, w, W = hybrid2b
    wl = config.PREFIX_CACHE_WORKLOAD
    g = torch.Generator().manual_seed(17)
    reqs = []
    for slen in (64, 1000, 2048):
        qs = [torch.randint(0, spec.vocab, (wl.question_len,), generator=g).tolist() for _ in range(wl.n_questions)]
        nopt = torch.randint(2, 6, (wl.n_questions,), generator=g).tolist()
        reqs.append({"state": torch.randint(0, spec.vocab, (slen,), generator=g).tolist(), "questions": qs,
                     "kinds": [1] * wl.n_questions, "n_opts": nopt,
                     "opt_ids": [[11 + j for j in range(k)] for k in nopt]})
    m = DecisionModel(w, max_tokens=4608, pool_slots=4, pool_kv_tokens=4096, lo_plane="e4m3")
    got = m.score_requests(reqs).cpu()
    want = _oracle(spec, W, reqs)
    _check(got.probs, want, [k for r in reqs for k in r["n_opts"]])
    m.close()
