"""The `--device b200` engine's two overrides and the checkpoint-style weight loader, on the GPU.

* `_slot_probs_batched` (infer.py:253-279) and `_slot_probs_shared_prefix` (infer.py:281-337)
  through the engine built on the reference's own `SystemOneEngine` (reference_engine_class),
  with a word-level tokenizer (the fixture pattern of the reference's
  tests/test_mlx_engine.py:56-67): both paths agree with each other, return the reference's
  contract (probs [n, K] float32 with zeros past n_slots, the input-token count) and match
  the oracle's full-prompt probabilities within 2e-3. `_fit`, `_temperatures` and
  `_option_idx` are the reference's, inherited. These tests need the reference package
  importable (tests/conftest.py says where it is looked for) and skip without it.
* `DeviceWeights.from_state_dict` on a transformers-named state dict packs the same bytes
  as the synthetic loader from the same latents.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

WORDS = ("the a of to and in is it that for on with as was at by this be are from or an policy "
         "library book renew renewal loan due date fine days week member card return overdue "
         "item hold request staff desk online account limit late fee paid cookbook friday "
         "leave failed my can i what which how many should we answer question options yes no "
         "score low mid high choose one best rate urgency team billing support sales").split()


def _tokenizer():
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {w: i for i, w in enumerate(["<pad>", "<eos>", "<unk>", *[str(k) for k in range(1, 25)],
                                         *sorted(set(WORDS))])}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    return PreTrainedTokenizerFast(tokenizer_object=tok, pad_token="<pad>", eos_token="<eos>", unk_token="<unk>")


def _text(g: torch.Generator, n: int) -> str:
    return " ".join(WORDS[int(i)] for i in torch.randint(0, len(WORDS), (n,), generator=g))


def _engine(max_length=256, slots=2):
    from tests.conftest import require_reference

    infer = require_reference()
    from strands_decider.modeling import StrandsDeciderConfig

    from strands_decider_b200 import config
    from strands_decider_b200.engine import Readout, reference_engine_class
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.weights import DeviceWeights

    spec = config.TINY
    w = DeviceWeights.synthetic(spec, seed=3, latent_device="cpu")
    rt = DecisionModel(w, max_tokens=2048, pool_slots=slots, pool_kv_tokens=1024)
    tok = _tokenizer()
    dc = StrandsDeciderConfig(max_length=max_length, head_type="option_token", use_lora=False,
                              temperature_by_kind={"score": 1.5})
    eng = reference_engine_class()(rt, Readout(dc, tok), infer.EngineConfig(device="b200", max_batch=8))
    return spec, eng, tok


def _oracle_probs(spec, rows, opt_rows, n_slots, temps):
    from oracle import head as OH
    from oracle import synth as osynth
    from oracle import torso as OT

    W = osynth.logical_weights(spec, seed=3)
    cfg = osynth.torso_config(spec)
    pooled = torch.stack([OT.forward_sequence(cfg, W, torch.tensor(r))[0][-1] for r in rows])
    K = max(n_slots)
    opt = torch.tensor([o + [0] * (K - len(o)) for o in opt_rows])
    return OH.decide(pooled, W["embed"], opt, torch.tensor(n_slots), torch.tensor(temps))


def test_engine_batched_and_shared_prefix_paths_match_each_other_and_the_oracle():
    spec, eng, tok = _engine()
    g = torch.Generator().manual_seed(0)
    state = _text(g, 60)
    questions = [_text(g, 9), _text(g, 14), _text(g, 5)]
    n_slots, kinds = [3, 2, 5], ["choice", "noul", "score"]
    pb, nb = eng._slot_probs_batched(state, questions, n_slots, kinds)
    pp, npfx = eng._slot_probs_shared_prefix(state, questions, n_slots, kinds)
    assert pb.dtype == torch.float32 and pb.shape == (3, 5) and pb.device.type == "cpu"
    for i, n in enumerate(n_slots):
        assert torch.all(pb[i, n:] == 0) and torch.all(pp[i, n:] == 0)
        assert abs(float(pb[i, :n].sum()) - 1.0) < 1e-5
    assert (pb - pp).abs().max().item() < 2e-4
    s, q = eng._fit(state, questions)
    assert nb == sum(len(s) + len(x) for x in q) and npfx == len(s) + sum(len(x) for x in q)
    rows = [s + x for x in q]
    opt_rows = eng._option_rows(n_slots)
    assert opt_rows[2] == [tok.convert_tokens_to_ids(str(k)) for k in range(1, 6)]
    want = _oracle_probs(spec, rows, opt_rows, n_slots, [1.0, 1.0, 1.5])
    assert (pb - want).abs().max().item() < 2e-3
    assert torch.equal(pb.argmax(1), want.argmax(1))


def test_engine_front_truncates_long_questions_like_the_reference():
    spec, eng, tok = _engine(max_length=40)
    g = torch.Generator().manual_seed(1)
    state, questions = _text(g, 80), [_text(g, 50), _text(g, 6)]
    s, q = eng._fit(state, questions)
    reserve = min(50, max(1, int(40 * 0.75)))
    assert len(q[0]) == reserve and len(q[1]) == 6 and len(s) <= 40 - reserve
    full = tok(questions[0], add_special_tokens=False)["input_ids"]
    assert q[0] == full[-reserve:]
    p, _ = eng._slot_probs_shared_prefix(state, questions, [4, 2], ["choice", "noul"])
    assert p.shape == (2, 4)


def test_engine_rejects_more_options_than_single_token_numbers():
    spec, eng, tok = _engine()
    with pytest.raises(ValueError):
        eng._slot_probs_batched("the policy", ["which one"], [30], ["choice"])


def test_state_dict_loader_packs_the_same_bytes_as_the_synthetic_loader():
    from strands_decider_b200 import config, synth
    from strands_decider_b200.weights import DeviceWeights

    for fmt in ("int4", "nvfp4", "ternary"):
        spec = config.TINY.with_format(fmt)
        a = DeviceWeights.synthetic(spec, seed=5, latent_device="cpu")
        sd = {"model.embed_tokens.weight": synth.embedding(spec, 5).float(),
              "model.norm.weight": synth.final_norm(spec, 5)}
        for li in range(spec.n_layers):
            for name, t in synth.linear_latents(spec, li, 5, "cpu"):
                sd["model." + name] = t
            for k, v in synth.small_params(spec, li, 5).items():
                sd["model." + k] = v[:, None, :] if k.endswith("conv1d.weight") else v   # nn.Conv1d shape
        b = DeviceWeights.from_state_dict(spec, sd)
        assert torch.equal(a.embed, b.embed) and torch.equal(a.final_norm, b.final_norm)
        for la, lb in zip(a.layers, b.layers, strict=True):
            for key in ("mix_in", "mix_out", "down", "gate_up"):
                for (na, ta), (nb_, tb) in zip(la[key].parts(), lb[key].parts(), strict=True):
                    assert na == nb_ and torch.equal(ta, tb), (fmt, key, na)
            for key in la:
                if isinstance(la[key], torch.Tensor):
                    assert torch.equal(la[key], lb[key]), key


def test_state_dict_loader_rejects_missing_and_misshapen_tensors():
    from strands_decider_b200 import config
    from strands_decider_b200.weights import DeviceWeights

    spec = config.TINY
    with pytest.raises(ValueError, match="lacks"):
        DeviceWeights.from_state_dict(spec, {"embed_tokens.weight": torch.zeros(spec.vocab, spec.hidden)})
    from strands_decider_b200 import synth

    sd = {"embed_tokens.weight": synth.embedding(spec, 0).float(), "norm.weight": synth.final_norm(spec, 0)}
    for li in range(spec.n_layers):
        sd.update({n: t for n, t in synth.linear_latents(spec, li, 0, "cpu")})
        sd.update(synth.small_params(spec, li, 0))
    sd["layers.0.mlp.down_proj.weight"] = sd["layers.0.mlp.down_proj.weight"][:, :-128]
    with pytest.raises(ValueError, match="shape"):
        DeviceWeights.from_state_dict(spec, sd)


class _Rendered:
    """The two fields of the reference's RenderedQuestion a pointer readout reads."""

    def __init__(self, text, option_spans, n_slots, kind):
        self.text, self.option_spans, self.n_slots, self.kind = text, option_spans, n_slots, kind


def test_engine_pointer_head_paths_match_each_other_and_the_oracle():
    """head_type "pointer": option positions come from the fitted questions' token offsets
    (infer.py:221-237) on both paths, and the device head matches the oracle's PointerHead."""
    from oracle import head as OH
    from oracle import synth as osynth
    from oracle import torso as OT
    from strands_decider_b200 import synth
    from strands_decider_b200.readout import DeviceReadout

    spec, eng, tok = _engine()
    eng.model.config.head_type = "pointer"
    params = synth.readout_params("pointer", spec.hidden, 64, seed=4)
    eng._rt.set_readout(DeviceReadout("pointer", params, spec.hidden))
    g = torch.Generator().manual_seed(5)
    state = _text(g, 40)
    rendered, texts = [], []
    for n in (3, 4):
        lines = [_text(g, 3) for _ in range(n)]
        head = _text(g, 6)
        text, spans = head, []
        for ln in lines:
            text += " " + ln
            spans.append((len(text) - len(ln), len(text)))
        text += " answer"
        texts.append(text)
        rendered.append(_Rendered(text, spans, n, "choice"))
    pb, _ = eng._slot_probs_batched(state, texts, [3, 4], ["choice"] * 2, rendered=rendered)
    pp, _ = eng._slot_probs_shared_prefix(state, texts, [3, 4], ["choice"] * 2, rendered=rendered)
    assert (pb - pp).abs().max().item() < 2e-4
    s, q = eng._fit(state, texts)
    pos = eng._option_idx(rendered, 0).tolist()
    W = osynth.logical_weights(spec, seed=3)
    cfg = osynth.torso_config(spec)
    hid = [OT.forward_sequence(cfg, W, torch.tensor(s + x))[0] for x in q]
    pooled = torch.stack([h[-1] for h in hid])
    opts = torch.stack([h[torch.tensor([len(s) + p if p >= 0 else 0 for p in ps])] for h, ps in zip(hid, pos)])
    logits = OH.pointer_head(pooled, opts, params)
    want = OH.decide_from_logits(logits, torch.tensor([3, 4]), torch.tensor([1.0, 1.0]))
    assert (pb - want).abs().max().item() < 2e-3
    eng._rt.set_readout(None)


def test_many_requests_in_two_launches_match_one_at_a_time():
    """_slot_probs_many (every state in one prefill, every question in one suffix forward) and
    the RequestBatcher fed from several threads give each request what its own
    _slot_probs_shared_prefix gives."""
    import threading

    from strands_decider_b200.engine import RequestBatcher

    spec, eng, tok = _engine(slots=8)
    g = torch.Generator().manual_seed(11)
    items = []
    for i in range(5):
        nq = 1 + i % 3
        items.append({"state_text": _text(g, 20 + 9 * i), "question_texts": [_text(g, 4 + j) for j in range(nq)],
                      "n_slots": [2 + (i + j) % 3 for j in range(nq)], "kinds": ["choice"] * nq})
    want = [eng._slot_probs_shared_prefix(it["state_text"], it["question_texts"], it["n_slots"], it["kinds"])
            for it in items]
    got = eng._slot_probs_many(items)
    for (pw, nw), (pg, ng) in zip(want, got, strict=True):
        assert ng == nw and pg.shape == pw.shape
        assert (pg - pw).abs().max().item() < 2e-4
    b = RequestBatcher(eng, max_requests=4, window_ms=20)
    futs = [None] * len(items)

    def go(i):
        it = items[i]
        futs[i] = b.submit(it["state_text"], it["question_texts"], it["n_slots"], it["kinds"])

    ts = [threading.Thread(target=go, args=(i,)) for i in range(len(items))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for (pw, nw), f in zip(want, futs, strict=True):
        pg, ng = f.result(timeout=60)
        assert ng == nw and (pg - pw).abs().max().item() < 2e-4
    b.close()
