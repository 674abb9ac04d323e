"""The CPU oracle, pinned against outputs of the reference itself (tests/golden/*.npz,
made by tests/golden/make_golden.py from transformers' Qwen3.5 torso and strands-decider's
own readout functions)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import head as H
from oracle import quant as Q
from oracle import synth as osynth
from oracle import torso as T
from strands_decider_b200 import config
from tests.conftest import GOLDEN
from tests.golden.make_golden import CHUNK_SEQS, chunk_rule_inputs


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


# ----------------------------------------------------------------------------- chunk rule


@pytest.mark.parametrize("seq", CHUNK_SEQS)
def test_chunk_rule_matches_reference_with_initial_state(seq):
    """The restated chunk rule against transformers' own (TF:234-311), correlated keys,
    non-zero initial state; tolerance as tests/test_mps_kernels.py:62-73."""
    g = _load("chunk_rule.npz")
    x, state = chunk_rule_inputs(seq)
    o, s = T.chunk_gated_delta_rule(x["query"], x["key"], x["value"], x["g"], x["beta"],
                                    initial_state=state)
    torch.testing.assert_close(o, torch.from_numpy(g[f"s{seq}_out"]), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(s, torch.from_numpy(g[f"s{seq}_state"]), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("seq", CHUNK_SEQS)
def test_recurrent_rule_matches_reference_with_initial_state(seq):
    """The restated token-by-token rule against transformers' own (TF:314-353), the form of
    single-token appends: correlated keys, non-zero initial state."""
    g = _load("recurrent_rule.npz")
    x, state = chunk_rule_inputs(seq)
    o, s = T.recurrent_gated_delta_rule(x["query"], x["key"], x["value"], x["g"], x["beta"], state)
    torch.testing.assert_close(o, torch.from_numpy(g[f"s{seq}_out"]), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(s, torch.from_numpy(g[f"s{seq}_state"]), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("seq", [1, 64, 130])
def test_chunk_rule_equals_token_recurrence(seq):
    x, state = chunk_rule_inputs(seq)
    o1, s1 = T.chunk_gated_delta_rule(x["query"], x["key"], x["value"], x["g"], x["beta"], state)
    o2, s2 = T.recurrent_gated_delta_rule(x["query"], x["key"], x["value"], x["g"], x["beta"], state)
    torch.testing.assert_close(o1, o2, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(s1, s2, rtol=1e-3, atol=1e-3)


# ----------------------------------------------------------------------------- torso + head


def _oracle_probs(spec, W, rows, opt, nopt, temps):
    cfg = osynth.torso_config(spec)
    pooled = []
    for r in rows:
        hid, _ = T.forward_sequence(cfg, W, torch.tensor(r))
        pooled.append(hid[-1])
    pooled = torch.stack(pooled)
    opt_t = torch.tensor([o + [0] * (max(map(len, opt)) - len(o)) for o in opt])
    return H.decide(pooled, W["embed"], opt_t, torch.tensor(nopt), torch.tensor(temps)), pooled


@pytest.mark.slow
def test_reduced_decider_matches_reference():
    """4 x 256 ids on the reduced int4 decider: probabilities and pooled states."""
    g = _load("reduced_1024_int4.npz")
    spec = config.REDUCED_1024
    packed = dict(osynth.quantized_linears(spec, seed=0))
    assert osynth.packed_digest(packed) == str(g["packed_digest"])
    W = osynth.logical_weights(spec, seed=0, packed=packed)
    rows = g["ids"].astype(np.int64).tolist()
    opt = g["opt_ids"].tolist()
    probs, pooled = _oracle_probs(spec, W, rows, opt, [3] * 4, [1.0] * 4)
    np.testing.assert_allclose(pooled.numpy(), g["pooled"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(probs.numpy(), g["probs"], atol=1e-5)


def _tiny_case(fmt):
    g = _load(f"tiny_{fmt}_ragged.npz")
    s0, s1 = g["state0"].tolist(), g["state1"].tolist()
    rows = [s0 + g["q0"].tolist(), s0 + g["q1"].tolist(), s1 + g["q2"].tolist(), s1 + g["q3"].tolist()]
    nopt = g["n_opts"].tolist()
    opt = [g["opt_ids"][i, :n].tolist() for i, n in enumerate(nopt)]
    return g, rows, opt, nopt, g["temps"].tolist()


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_tiny_ragged_matches_reference(fmt):
    """Ragged, right-padded prompts with mixed option counts and temperatures."""
    g, rows, opt, nopt, temps = _tiny_case(fmt)
    spec = config.TINY
    packed = dict(osynth.quantized_linears(spec, seed=1, fmt=fmt))
    assert osynth.packed_digest(packed) == str(g["packed_digest"])
    W = osynth.logical_weights(spec, seed=1, fmt=fmt, packed=packed)
    probs, pooled = _oracle_probs(spec, W, rows, opt, nopt, temps)
    np.testing.assert_allclose(probs.numpy(), g["probs"][:, : probs.shape[1]], atol=1e-5)
    np.testing.assert_allclose(pooled.numpy(), g["pooled"], rtol=1e-4, atol=1e-4)
    if fmt == "int4":  # every real position of every prompt
        cfg = osynth.torso_config(spec)
        for i, r in enumerate(rows):
            hid, _ = T.forward_sequence(cfg, W, torch.tensor(r))
            np.testing.assert_allclose(hid.numpy(), g["hidden"][i, : len(r)], rtol=1e-4, atol=1e-4)


def test_oracle_at_the_2b_shapes_matches_reference():
    """hidden 2048, GDN 16 heads, attention 8q/2kv x head_dim 256 with partial RoPE, FFN 6144 and
    the 248320-row tied embedding (4 layers, bf16 weights): final hidden states and option
    probabilities, including option rows at the end of the vocabulary."""
    from tests.golden.make_golden import PIN_OPTS, hybrid2b_pin_spec, hybrid2b_pin_weights

    g = _load("hybrid2b_shapes_bf16.npz")
    spec = hybrid2b_pin_spec()
    ids = g["ids"].astype(np.int64).tolist()
    W = hybrid2b_pin_weights(spec, rows=ids + [o for opts in PIN_OPTS for o in opts])
    cfg = osynth.torso_config(spec)
    hid, _ = T.forward_sequence(cfg, W, torch.tensor(ids))
    np.testing.assert_allclose(hid[-3:].numpy(), g["hidden_tail"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(hid[-1].numpy(), g["pooled"], rtol=1e-4, atol=1e-4)
    for i, opts in enumerate(PIN_OPTS):
        p = H.decide(hid[-1:], W["embed"], torch.tensor([opts]), torch.tensor([len(opts)]),
                     torch.tensor([[1.0, 0.8][i]]))
        np.testing.assert_allclose(p[0].numpy(), g["probs"][i, : len(opts)], atol=1e-5)


def test_prefix_cache_continuation_equals_full_prompt():
    """The property tests/test_prefix_cache.py:43-64 asserts for the reference: a suffix
    forwarded against a cached state equals the full prompt, at every suffix position.
    Covers a prefix shorter than the conv width and suffixes crossing chunk boundaries."""
    spec = config.TINY
    W = osynth.logical_weights(spec, seed=1, fmt="int4")
    cfg = osynth.torso_config(spec)
    g = torch.Generator().manual_seed(5)
    for plen, slen in [(2, 3), (70, 9), (64, 64), (1, 1), (100, 80)]:
        pre = torch.randint(0, spec.vocab, (plen,), generator=g)
        suf = torch.randint(0, spec.vocab, (slen,), generator=g)
        _, cache = T.forward_sequence(cfg, W, pre, keep_cache=True)
        cont, _ = T.forward_sequence(cfg, W, suf, cache=cache)
        full, _ = T.forward_sequence(cfg, W, torch.cat([pre, suf]))
        torch.testing.assert_close(cont, full[plen:], rtol=1e-4, atol=1e-4)


# ----------------------------------------------------------------------------- answer math


def test_answer_formulas_match_reference():
    g = _load("answer_formulas.npz")
    for i, n in enumerate(g["n"]):
        p = g["probs"][i, :n].tolist()
        assert H.derive_confidence(p) == pytest.approx(g["confidence"][i], abs=1e-12)
        assert H.derive_score_confidence(p) == pytest.approx(g["score_confidence"][i], abs=1e-12)
        assert H.derive_score_confidence(p, 0.1) == pytest.approx(g["score_confidence_s01"][i], abs=1e-12)


def test_masked_log_softmax_semantics():
    """tests/test_core.py:197-213 of the reference."""
    lp = H.masked_log_softmax(torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0]]), torch.tensor([3]))
    p = lp.exp()
    assert p[0, :3].sum().item() == pytest.approx(1.0, abs=1e-5)
    assert p[0, 3:].sum().item() == 0.0
    assert p.argmax().item() == 2
    lp = H.masked_log_softmax(torch.zeros(2, 4), torch.tensor([2, 4])).exp()
    assert lp[0, 0].item() == pytest.approx(0.5) and lp[1, 0].item() == pytest.approx(0.25)


# ----------------------------------------------------------------------------- formats


def test_bf16_and_e4m3_match_torch_conversions():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 1, 300)])
    x = np.clip(x, -448, 448)
    grid = Q.e4m3_decode(np.arange(0, 127, dtype=np.uint8))
    x = np.concatenate([x, ((grid[1:] + grid[:-1]) / 2).astype(np.float32), grid])
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(Q.e4m3_encode(x), want)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(Q.f32_to_bf16_bits(x), want)


def test_e2m1_rounding_is_nearest_even():
    v = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.2501, 7.0, -1.75, -0.1], np.float32)
    got = Q.e2m1_decode(Q.e2m1_encode(v))
    assert got.tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 0.5, 6.0, -2.0, 0.0]


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_quantise_roundtrip_properties(fmt):
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    w[3] = 0.0                                   # an all-zero row / group
    parts = Q.quantize(fmt, w)
    d = Q.dequantize(fmt, parts)
    assert d.dtype == np.float32 and d.shape == w.shape
    assert np.all(d[3] == 0)
    assert np.array_equal(Q.bf16_round(d), d)   # dequantised values are bf16 values
    # quantising the dequantised tensor again is (nearly) idempotent for int4
    if fmt == "int4":
        d2 = Q.dequantize(fmt, Q.quantize(fmt, d))
        rel = np.abs(d2 - d).max() / np.abs(d).max()
        assert rel < 0.02
    err = np.abs(d - w).mean() / np.abs(w).mean()
    assert err < {"int4": 0.15, "nvfp4": 0.12, "ternary": 0.6}[fmt]


def test_nvfp4_table_dequantiser_equals_the_elementwise_definition():
    """The table-driven NVFP4 dequantiser (used for whole 2B-shape models) returns the same
    bits as the definition applied element by element, including zero blocks and every
    (scale byte, code) pair that occurs."""
    rng = np.random.default_rng(7)
    for amp in (0.02, 3.0):
        w = (rng.standard_normal((96, 1024)) * amp).astype(np.float32)
        w[5, :16] = 0.0
        w[7, 16:32] *= 1e-4                      # tiny blocks: small scale bytes
        p = Q.quantize("nvfp4", w)
        a = Q.dequantize("nvfp4", p)
        b = Q.dequantize_nvfp4_elementwise(p["data"], p["scales"], float(np.asarray(p["global_scale"]).reshape(-1)[0]))
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_int4_nibble_order():
    q = np.array([[1, -1, 7, -8, 0, 2, 3, -3] * 16], dtype=np.int64)
    packed = (np.bitwise_or.reduce((q.reshape(1, -1, 8) & 0xF).astype(np.uint32)
                                   << (np.arange(8, dtype=np.uint32) * 4), axis=2)).view(np.int32)
    assert np.array_equal(Q.unpack_int4(packed), q)
    assert packed.view(np.uint32)[0, 0] == 0xD32087F1


@pytest.mark.parametrize("case", ["slot", "slot_mlp", "pointer"])
def test_trained_readouts_match_reference(case):
    """SlotHead (one linear, and Linear-GELU-Linear) and PointerHead with gather_options
    (modeling.py:99-190) over the tiny int4 torso's final hidden states."""
    from strands_decider_b200 import synth
    from tests.golden.make_golden import READOUT_CASES, readout_case_inputs

    g = _load("tiny_int4_readouts.npz")
    spec = config.TINY
    W = osynth.logical_weights(spec, seed=1, fmt="int4")
    cfg = osynth.torso_config(spec)
    rows, opt_idx, nopt, temps = readout_case_inputs(spec)
    name, out, mlp = next(c for c in READOUT_CASES if c[0] == case)
    kind = "pointer" if case == "pointer" else "slot"
    Hd = synth.readout_params(kind, spec.hidden, out, mlp, seed=11)
    with torch.inference_mode():
        hid = [T.forward_sequence(cfg, W, torch.tensor(r))[0] for r in rows]
        pooled = torch.stack([h[-1] for h in hid])
        if kind == "pointer":
            opts = torch.stack([h[torch.from_numpy(opt_idx[i]).long().clamp_min(0)] for i, h in enumerate(hid)])
            logits = H.pointer_head(pooled, opts, Hd)
        else:
            logits = H.slot_head(pooled, Hd)
        probs = H.decide_from_logits(logits, torch.tensor(nopt), torch.tensor(temps))
    np.testing.assert_allclose(probs.numpy(), g[f"probs_{case}"], atol=2e-5)
