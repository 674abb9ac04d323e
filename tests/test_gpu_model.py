"""Whole-torso parity on the B200: the native prefill + fused decision head against the
reference's own outputs (golden fixtures) and the CPU oracle.

Tolerance (BASELINE correctness bar): option probabilities within 2e-3 absolute of the
reference, identical argmax; packed weights bit-exact to the CPU quantiser."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import head as OH
from oracle import synth as osynth
from oracle import torso as OT
from strands_decider_b200 import config
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

PROB_TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    from strands_decider_b200 import _lib

    _lib.load()
    yield
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _model(spec, seed, fmt=None, max_tokens=4096, slots=16, dequant_min_tokens=0, lo_plane="e4m3"):
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.weights import DeviceWeights

    spec = spec.with_format(fmt) if fmt else spec
    w = DeviceWeights.synthetic(spec, seed=seed, latent_device="cpu", keep_logical=True)
    return DecisionModel(w, max_tokens=max_tokens, pool_slots=slots, pool_kv_tokens=max_tokens,
                         dequant_min_tokens=dequant_min_tokens, lo_plane=lo_plane)


def _logical_digest(model):
    from strands_decider_b200.weights import packed_to_numpy

    return osynth.packed_digest({k: packed_to_numpy(v) for k, v in model.w.logical.items()})


def test_reduced_decider_matches_reference_golden():
    """4 x 256 ids on the reduced int4 decider (the reference's CPU-runnable config)."""
    g = np.load(os.path.join(GOLDEN, "reduced_1024_int4.npz"))
    m = _model(config.REDUCED_1024, seed=0)
    assert _logical_digest(m) == str(g["packed_digest"]), "device quantisation differs from the CPU quantiser"
    rows = g["ids"].tolist()
    out = m.score_prompts(rows, [[11, 12, 13]] * 4, [3] * 4, ["choice"] * 4, [1.0] * 4).cpu()
    want = g["probs"]
    assert np.abs(out.probs.numpy() - want).max() < PROB_TOL, (out.probs, want)
    assert np.array_equal(out.argmax.numpy(), want.argmax(1))


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_dequantised_weight_path_matches_the_streamed_path(fmt):
    """Large batches run every GEMM on a bf16 copy of its weight dequantised once per call;
    forcing that path at the golden prompts' 1024 tokens gives the same probabilities as
    the default (packed tiles unpacked inside the GEMM) and the reference."""
    g = np.load(os.path.join(GOLDEN, "reduced_1024_int4.npz"))
    spec = config.REDUCED_1024.with_format(fmt)
    rows = g["ids"].tolist()
    outs = []
    for dq in (-1, 1):
        m = _model(spec, seed=0, dequant_min_tokens=dq, lo_plane="bf16")
        outs.append(m.score_prompts(rows, [[11, 12, 13]] * 4, [3] * 4, ["choice"] * 4, [1.0] * 4).cpu())
        del m
    # the dequantised bf16 weights equal the GEMM's own unpack bit for bit; what differs is
    # run-to-run order of the split-K atomic sums in the small GEMMs (about 1e-7 relative)
    assert np.abs(outs[0].probs.numpy() - outs[1].probs.numpy()).max() < 1e-4
    if fmt == "int4":
        assert np.abs(outs[1].probs.numpy() - g["probs"]).max() < PROB_TOL


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_tiny_ragged_matches_reference_golden(fmt):
    """Ragged prompts, mixed option counts, kinds and temperatures on the tiny spec."""
    g = np.load(os.path.join(GOLDEN, f"tiny_{fmt}_ragged.npz"))
    m = _model(config.TINY, seed=1, fmt=fmt)
    assert _logical_digest(m) == str(g["packed_digest"])
    s0, s1 = g["state0"].tolist(), g["state1"].tolist()
    rows = [s0 + g["q0"].tolist(), s0 + g["q1"].tolist(), s1 + g["q2"].tolist(), s1 + g["q3"].tolist()]
    nopt = g["n_opts"].tolist()
    opt = [g["opt_ids"][i, :n].tolist() for i, n in enumerate(nopt)]
    kinds = ["choice", "noul", "score", "choice"]
    out = m.score_prompts(rows, opt, nopt, kinds, g["temps"].tolist()).cpu()
    want = g["probs"]
    assert np.abs(out.probs.numpy() - want[:, : out.probs.shape[1]]).max() < PROB_TOL
    for i, n in enumerate(nopt):
        assert int(out.argmax[i]) == int(want[i, :n].argmax())
    # derived answer numbers against the reference formulas on the reference's probabilities
    ref = OH.device_style_outputs(torch.from_numpy(want), [0 if k == "noul" else 1 if k == "choice" else 2
                                                           for k in kinds], nopt)
    assert torch.allclose(out.confidence, ref["confidence"], atol=5e-3)
    assert torch.allclose(out.score, ref["score"], atol=5e-3)
    if fmt == "int4":  # hidden states at every position, after the final norm
        hid = g["hidden"]
        resid = m.residual(sum(map(len, rows))).cpu()
        off = 0
        for i, r in enumerate(rows):
            x = resid[off:off + len(r)]
            normed = OT.rms_norm_1p(x, m.w.final_norm.cpu(), 1e-6)
            ref_h = torch.from_numpy(hid[i, : len(r)])
            rel = ((normed - ref_h).norm(dim=1) / ref_h.norm(dim=1)).max().item()
            assert rel < 2e-2, (i, rel)
            off += len(r)


def test_prefix_cache_equals_full_prompt_on_device():
    """The shared-prefix path (state once into a pool slot, suffixes read it in place)
    equals the full-prompt path (tests/test_prefix_cache.py:43-64 of the reference),
    including states shorter than the conv width and suffixes crossing chunk bounds."""
    m = _model(config.TINY, seed=1, fmt="int4")
    g = torch.Generator().manual_seed(3)
    V = config.TINY.vocab
    reqs = []
    for slen, qlens in [(70, [9, 1, 40]), (2, [3, 5]), (33, [64]), (1, [2, 31])]:
        st = torch.randint(0, V, (slen,), generator=g).tolist()
        qs = [torch.randint(0, V, (n,), generator=g).tolist() for n in qlens]
        reqs.append({"state": st, "questions": qs, "kinds": [1] * len(qs), "n_opts": [3] * len(qs),
                     "opt_ids": [[11, 12, 13]] * len(qs)})
    cached = m.score_requests(reqs).cpu()
    rows = [r["state"] + q for r in reqs for q in r["questions"]]
    n = len(rows)
    full = m.score_prompts(rows, [[11, 12, 13]] * n, [3] * n, [1] * n, [1.0] * n).cpu()
    assert torch.abs(cached.probs - full.probs).max().item() < 1e-3
    assert torch.equal(cached.argmax, full.argmax)


def test_prefix_cache_equals_full_prompt_with_many_sequences():
    """The same equivalence with 40 requests (80 suffixes): the GDN layers then run one CTA
    per (sequence, head) instead of the clusters a few sequences use."""
    m = _model(config.TINY, seed=2, fmt="nvfp4", max_tokens=8192, slots=40)
    g = torch.Generator().manual_seed(5)
    V = config.TINY.vocab
    reqs = []
    for _ in range(40):
        slen = int(torch.randint(1, 90, (1,), generator=g))
        st = torch.randint(0, V, (slen,), generator=g).tolist()
        qs = [torch.randint(0, V, (int(n),), generator=g).tolist() for n in torch.randint(1, 40, (2,), generator=g)]
        reqs.append({"state": st, "questions": qs, "kinds": [1, 2], "n_opts": [3, 3], "opt_ids": [[11, 12, 13]] * 2})
    cached = m.score_requests(reqs).cpu()
    rows = [r["state"] + q for r in reqs for q in r["questions"]]
    n = len(rows)
    full = m.score_prompts(rows, [[11, 12, 13]] * n, [3] * n, [1, 2] * (n // 2), [1.0] * n).cpu()
    assert torch.abs(cached.probs - full.probs).max().item() < 1e-3
    assert torch.equal(cached.argmax, full.argmax)


def test_prefix_cache_equals_full_prompt_at_large_batch():
    """Prefix ≡ full prompt with 400 requests (about 40 000 tokens per forward), where the GDN
    prep kernel runs its large-batch form (8 tokens per warp), reading conv history from the
    pool."""
    m = _model(config.TINY, seed=2, fmt="int4", max_tokens=81920, slots=400)
    g = torch.Generator().manual_seed(8)
    V = config.TINY.vocab
    reqs = []
    for _ in range(400):
        st = torch.randint(0, V, (int(torch.randint(1, 160, (1,), generator=g)),), generator=g).tolist()
        q = torch.randint(0, V, (int(torch.randint(70, 110, (1,), generator=g)),), generator=g).tolist()
        reqs.append({"state": st, "questions": [q], "kinds": [1], "n_opts": [3], "opt_ids": [[11, 12, 13]]})
    cached = m.score_requests(reqs).cpu()
    rows = [r["state"] + r["questions"][0] for r in reqs]
    full = m.score_prompts(rows, [[11, 12, 13]] * 400, [3] * 400, [1] * 400, [1.0] * 400).cpu()
    assert torch.abs(cached.probs - full.probs).max().item() < 1e-3
    assert (cached.argmax == full.argmax).float().mean().item() > 0.99


def test_oracle_prefix_path_matches_device_prefix_path():
    """Same requests through the oracle's explicit cache and the device pool."""
    m = _model(config.TINY, seed=1, fmt="nvfp4")
    W = osynth.logical_weights(config.TINY, seed=1, fmt="nvfp4")
    cfg = osynth.torso_config(config.TINY)
    g = torch.Generator().manual_seed(4)
    V = config.TINY.vocab
    st = torch.randint(0, V, (90,), generator=g)
    qs = [torch.randint(0, V, (n,), generator=g) for n in (12, 40)]
    _, cache = OT.forward_sequence(cfg, W, st, keep_cache=True)
    pooled = torch.stack([OT.forward_sequence(cfg, W, q, cache=cache)[0][-1] for q in qs])
    want = OH.decide(pooled, W["embed"], torch.tensor([[11, 12, 13, 14]] * 2), torch.tensor([4, 4]),
                     torch.tensor([1.0, 1.0]))
    got = m.score_requests([{"state": st.tolist(), "questions": [q.tolist() for q in qs], "kinds": [1, 1],
                             "n_opts": [4, 4], "opt_ids": [[11, 12, 13, 14]] * 2}]).cpu()
    assert torch.abs(got.probs - want).max().item() < PROB_TOL


@pytest.mark.parametrize("case", ["slot", "slot_mlp", "pointer"])
def test_trained_readouts_match_reference_golden(case):
    """SlotHead / PointerHead on the device (b200_model_set_readout, head_decide_kernel) against
    the reference's heads on the tiny int4 torso (tests/golden/tiny_int4_readouts.npz), on the
    full-prompt path and on the shared-prefix path."""
    from strands_decider_b200 import synth
    from strands_decider_b200.readout import DeviceReadout
    from tests.golden.make_golden import READOUT_CASES, readout_case_inputs

    g = np.load(os.path.join(GOLDEN, "tiny_int4_readouts.npz"))
    spec = config.TINY
    m = _model(spec, seed=1, fmt="int4")
    rows, opt_idx, nopt, temps = readout_case_inputs(spec)
    name, out, mlp = next(c for c in READOUT_CASES if c[0] == case)
    kind = "pointer" if case == "pointer" else "slot"
    m.set_readout(DeviceReadout(kind, synth.readout_params(kind, spec.hidden, out, mlp, seed=11), spec.hidden))
    opt_pos = opt_idx.tolist() if kind == "pointer" else None
    full = m.score_prompts(rows, None, nopt, [1] * 3, temps, opt_pos=opt_pos).cpu()
    want = g[f"probs_{case}"][:, : full.probs.shape[1]]
    assert np.abs(full.probs.numpy() - want).max() < PROB_TOL
    assert np.array_equal(full.argmax.numpy(), want.argmax(1))
    # the same questions as suffixes of a cached state (positions then count from the suffix;
    # every option line lies in the suffix)
    cut = 5
    states = [r[:cut] for r in rows]
    sufs = [r[cut:] for r in rows]
    m.prefill_states(states, [0, 1, 2])
    spos = [[p - cut if p >= 0 else -1 for p in ps] for ps in opt_idx.tolist()] if kind == "pointer" else None
    cached = m.score_suffixes(sufs, [0, 1, 2], None, nopt, [1] * 3, temps, opt_pos=spos).cpu()
    assert np.abs(cached.probs.numpy() - full.probs.numpy()).max() < 1e-3
    m.set_readout(None)


def test_readout_argument_checks():
    from strands_decider_b200 import synth
    from strands_decider_b200.readout import DeviceReadout

    spec = config.TINY
    m = _model(spec, seed=1, fmt="int4")
    m.set_readout(DeviceReadout("pointer", synth.readout_params("pointer", spec.hidden, 32, seed=2), spec.hidden))
    with pytest.raises(ValueError, match="opt_pos"):
        m.score_prompts([[1, 2, 3, 4]], None, [2], [1], [1.0])
    with pytest.raises(ValueError, match="outside"):
        m.score_prompts([[1, 2, 3, 4]], None, [2], [1], [1.0], opt_pos=[[1, 4]])
    m.set_readout(DeviceReadout("slot", synth.readout_params("slot", spec.hidden, 4, seed=2), spec.hidden))
    with pytest.raises(ValueError, match="at most"):
        m.score_prompts([[1, 2, 3, 4]], None, [5], [1], [1.0])
    with pytest.raises(ValueError, match="lacks"):
        DeviceReadout("slot", {"norm.weight": torch.ones(spec.hidden)}, spec.hidden)


@pytest.mark.parametrize("fmt", ["int4", "ternary"])
def test_appended_states_equal_full_prompts(fmt):
    """Growing cached states in place (append_states: GDN state, conv history and keys /
    values continued and saved back into the same slot), by a multi-token chunk and then one
    token at a time, then scoring questions against them, equals the full prompts."""
    m = _model(config.TINY, seed=1, fmt=fmt, slots=4)
    g = torch.Generator().manual_seed(6)
    V = config.TINY.vocab
    r = lambda n: torch.randint(0, V, (n,), generator=g).tolist()  # noqa: E731
    states = [r(50), r(3), r(1)]
    chunks = [r(37), r(70), r(2)]
    singles = [[r(1) for _ in range(3)] for _ in range(3)]
    qs = [r(9), r(33), r(5)]
    m.prefill_states(states, [0, 1, 2], reserve=120)
    m.append_states(chunks, [0, 1, 2])
    for step in range(3):
        m.append_states([singles[i][step] for i in range(3)], [0, 1, 2])
    opt = [[11, 12, 13]] * 3
    cached = m.score_suffixes(qs, [0, 1, 2], opt, [3] * 3, [1] * 3, [1.0] * 3).cpu()
    rows = [states[i] + chunks[i] + sum(singles[i], []) + qs[i] for i in range(3)]
    full = m.score_prompts(rows, opt, [3] * 3, [1] * 3, [1.0] * 3).cpu()
    assert torch.abs(cached.probs - full.probs).max().item() < 1e-3
    assert torch.equal(cached.argmax, full.argmax)
    with pytest.raises(ValueError, match="room"):
        m.append_states([r(130)], [2])
