"""The B200 engine inside the reference's own `SystemOneEngine.evaluate`, against the
reference's CPU engine on the same checkpoint (the device-parity pattern of the reference's
tests/test_mlx_engine.py:112-128).

A tiny random-weight Qwen3.5 text model (3 Gated-DeltaNet layers and one attention layer,
with shapes the B200 kernels take) is saved as the base checkpoint in bf16, and a decider
checkpoint is saved on it by the reference's `StrandsDeciderModel.save_pretrained`, with a
slot head or a pointer head. The reference loads it with `strands_decider.infer.load_engine`
(device "cpu": the torso upcast to fp32); this repository loads it with
`strands_decider_b200.engine.load_engine` (bf16 weights, so both sides hold the same
values). Each request goes through `evaluate` on both: the answers' probabilities must agree
within 2e-3 (they are rounded to 4 places), the choices must match, and so must `usage`.

The reference's CPU engine runs whole prompts (use_prefix_cache=False): under the installed
transformers its shared-prefix path drops the cached GDN state, so it is not an oracle. The
B200 engine is checked on both of its paths against it. The reference runs in a child process
that sees no GPU, as on a CPU host: with a GPU visible, transformers hands the Gated-DeltaNet
scan of a CPU torso to flash-linear-attention's GPU kernels, which refuse CPU tensors. Needs
the reference package (tests/conftest.py says where it is looked for); skipped without it.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest
import torch

from tests.conftest import require_reference

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _requests():
    from strands_decider.schema import ChoiceQuestion, NoulQuestion, ScoreQuestion, SystemOneRequest

    qs = {
        "desk": ChoiceQuestion(instructions="Which desk should take this message?",
                               criteria={"lending": "loans, renewals and holds", "accounts": "fees and blocked cards",
                                         "events": "talks and room bookings"}),
        "overdue": NoulQuestion(instructions="Is an item already overdue?"),
        "tone": ScoreQuestion(instructions="How upset does the member sound?", criteria=["calm", "tense", "upset"]),
        "topic": ChoiceQuestion(instructions="What is the message mainly about?",
                                criteria={"loan": "borrowing or renewing", "fee": "money owed", "room": "a booking",
                                          "card": "a member card", "other": "something else"}),
    }
    policy = ("Members may borrow ten items at a time for three weeks. A loan renews twice unless "
              "someone else holds the item. Cards with more than five dollars of fees are blocked. ")
    return [
        SystemOneRequest(state="A member asks to extend a loan on a travel guide.", questions={"desk": qs["desk"]}),
        SystemOneRequest(state=policy * 4 + "My card was blocked at the desk and the book is late. I am upset!",
                         questions=qs),
        SystemOneRequest(state=policy + "Can we book the small room for a talk on Friday?",
                         questions={"topic": qs["topic"], "overdue": qs["overdue"]}),
    ]


def _tokenizer(requests):
    from strands_decider.prompting import render_question, render_state
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    texts = [render_state(r.state) for r in requests]
    texts += [render_question(q).text for r in requests for q in r.questions.values()]
    words = {w for t in texts for w, _ in pre_tokenizers.Whitespace().pre_tokenize_str(t)}
    vocab = {w: i for i, w in enumerate(["<pad>", "<eos>", "<unk>", *sorted(words)])}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    return PreTrainedTokenizerFast(tokenizer_object=tok, pad_token="<pad>", eos_token="<eos>", unk_token="<unk>")


def _checkpoint(root, head_type: str) -> str:
    import transformers
    from strands_decider.modeling import StrandsDeciderConfig, StrandsDeciderModel

    tok = _tokenizer(_requests())
    base = os.path.join(root, "base")
    if not os.path.isdir(base):
        torch.manual_seed(0)
        cfg = transformers.Qwen3_5TextConfig(
            vocab_size=len(tok), hidden_size=256, intermediate_size=512, num_hidden_layers=4,
            num_attention_heads=4, num_key_value_heads=2, head_dim=64, linear_num_key_heads=2,
            linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128,
            layer_types=["linear_attention"] * 3 + ["full_attention"], tie_word_embeddings=True,
            initializer_range=0.05)
        transformers.Qwen3_5ForCausalLM(cfg).to(torch.bfloat16).save_pretrained(base)
    torch.manual_seed(1)
    dc = StrandsDeciderConfig(base_model=base, head_type=head_type, pointer_dim=64, max_length=512, use_lora=False,
                              temperature_by_kind={"score": 1.3})
    torso = transformers.Qwen3_5ForCausalLM.from_pretrained(base).model
    path = os.path.join(root, f"ckpt_{head_type}")
    StrandsDeciderModel(dc, torso, tok).save_pretrained(path)
    return path


@pytest.fixture(scope="module", params=["slot", "pointer"])
def checkpoint(request, tmp_path_factory):
    require_reference()
    return _checkpoint(str(tmp_path_factory.mktemp("ref_engine")), request.param)


def _numbers(response) -> dict:
    out = {}
    for name, a in response.answers.items():
        if a.type == "noul":
            out[name] = ([a.noul], None)
        else:
            out[name] = (list(a.probabilities.values()), getattr(a, "choice", None))
    return out


def _reference_cpu_answers(checkpoint: str) -> dict:
    """The reference CPU engine's answers and usage for every request, whole-prompt path, plus
    the usage its shared-prefix path reports, from a child process with no GPU visible."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "tests.test_gpu_reference_engine", checkpoint], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def _cpu_main(checkpoint: str) -> None:
    from tests.conftest import require_reference as _ensure_path  # noqa: F401  (puts the reference on sys.path)
    from strands_decider.infer import load_engine as load_reference

    whole = load_reference(checkpoint, device="cpu", use_prefix_cache=False)
    shared = load_reference(checkpoint, device="cpu", use_prefix_cache=True)
    out = {"answers": [], "usage_whole": [], "usage_shared": []}
    for request in _requests():
        resp = whole.evaluate(request)
        out["answers"].append(_numbers(resp))
        out["usage_whole"].append(resp.usage.model_dump())
        out["usage_shared"].append(shared.evaluate(request).usage.model_dump())
    print(json.dumps(out))


@pytest.fixture(scope="module")
def reference_answers(checkpoint):
    return _reference_cpu_answers(checkpoint)


@pytest.mark.parametrize("prefix", [False, True])
def test_b200_engine_answers_as_the_reference_cpu_engine(checkpoint, reference_answers, prefix):
    from strands_decider_b200 import _lib
    from strands_decider_b200.engine import load_engine

    b200 = load_engine(checkpoint, weight_format="bf16", use_prefix_cache=prefix, max_tokens=4096, pool_slots=4)
    assert "SystemOneEngine" in [c.__name__ for c in type(b200).__mro__]
    for i, request in enumerate(_requests()):
        got = b200.evaluate(request)
        # the token count depends only on the path taken, not on its numerics
        assert got.usage.model_dump() == reference_answers["usage_shared" if prefix else "usage_whole"][i]
        w, g = reference_answers["answers"][i], _numbers(got)
        assert w.keys() == g.keys()
        for name in w:
            assert g[name][0] == pytest.approx(w[name][0], abs=TOL), (name, g[name], w[name])
            assert g[name][1] == w[name][1], name
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def test_b200_engine_refuses_like_the_reference(checkpoint):
    """The reference's own checks run unchanged: too many options for a slot head's num_slots
    (infer.py:352-360) is a ValueError before anything reaches the device."""
    from strands_decider.schema import ChoiceQuestion, SystemOneRequest

    from strands_decider_b200.engine import load_engine

    b200 = load_engine(checkpoint, weight_format="bf16", max_tokens=2048, pool_slots=2)
    if b200.model.config.head_type != "slot":
        pytest.skip("the option-count limit applies to slot heads")
    many = ChoiceQuestion(instructions="pick",
                          criteria={f"o{i}": f"option {i}" for i in range(b200.model.config.num_slots + 1)})
    with pytest.raises(ValueError, match="slots"):
        b200.evaluate(SystemOneRequest(state="a loan", questions={"q": many}))


if __name__ == "__main__":   # the reference CPU engine's side, run by _reference_cpu_answers
    _cpu_main(sys.argv[1])
