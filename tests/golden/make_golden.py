"""Generate the golden fixtures by running the reference itself.

Run where the reference and transformers are importable, naming the reference by its
checkout root (the directory holding `src/strands_decider`) or by a directory that holds the
installed `strands_decider` package, as the first argument or in STRANDS_DECIDER_SRC:

    python tests/golden/make_golden.py <reference checkout> [--readouts-only | ...]

What runs is the reference's own code, unmodified:
  * the torso: transformers' `Qwen3_5ForCausalLM(cfg).model` (the module strands-decider
    loads, `src/strands_decider/modeling.py:293-303`), fp32 on CPU, with the synthetic
    weights after quantise -> dequantise (oracle.quant) copied into its parameters;
  * the readout: strands-decider's `pool_last_token`, `apply_temperature` and
    `masked_log_softmax` (`modeling.py:193-238`) over the tied embedding rows of the
    option tokens (`frozen_slot_log_probs`, `modeling.py:412-438`), on the full-prompt
    path (`infer.py:253-279`), right-padded as `SystemOneEngine._pad` does;
  * the answer formulas `derive_confidence` / `derive_score_confidence` (`schema.py`);
  * transformers' `torch_chunk_gated_delta_rule` with an initial state (`TF:234-311`);
  * the trained readouts `SlotHead` / `PointerHead` with `gather_options`
    (`modeling.py:99-190`) on the tiny torso's hidden states (`--readouts-only` regenerates
    just that fixture);
  * transformers' token-by-token `torch_recurrent_gated_delta_rule` (`TF:314-353`) on the
    chunk-rule inputs, the form single-token appends take (`--recurrent-only` regenerates just
    that fixture);
  * the torso at the 2B shapes (head_dim 256, vocab 248320; 4 layers) on one prompt
    (`--hybrid2b-only` regenerates just that fixture).

The fixtures are small .npz files committed beside this script; the tests read only
them (the reference is not present where the GPU tests run).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root


CHUNK_SEQS = (1, 63, 64, 65, 200)


def chunk_rule_inputs(seq: int, heads: int = 2, dim: int = 64):
    """Seeded inputs of one chunk-rule case (shapes [seq, heads, dim]); correlated keys."""
    gg = torch.Generator().manual_seed(seq)
    r = lambda *s: torch.randn(*s, generator=gg)  # noqa: E731
    shared = 2.0 * r(1, heads, dim)
    x = dict(query=r(seq, heads, dim), key=r(seq, heads, dim) + shared, value=r(seq, heads, dim),
             g=-torch.rand(seq, heads, generator=gg) * 0.1,
             beta=0.5 + 0.5 * torch.rand(seq, heads, generator=gg))
    return x, r(heads, dim, dim)


def build_reference_torso(spec, W):
    import transformers

    cfg = transformers.Qwen3_5TextConfig(
        vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.inter,
        num_hidden_layers=spec.n_layers, num_attention_heads=spec.attn_heads,
        num_key_value_heads=spec.attn_kv_heads, head_dim=spec.head_dim,
        linear_num_key_heads=spec.gdn_heads, linear_num_value_heads=spec.gdn_heads,
        linear_key_head_dim=spec.gdn_dk, linear_value_head_dim=spec.gdn_dv,
        linear_conv_kernel_dim=spec.conv_width, layer_types=list(spec.layer_types),
        rms_norm_eps=spec.eps, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": spec.rope_theta,
                         "partial_rotary_factor": spec.partial_rotary})
    torso = transformers.Qwen3_5ForCausalLM(cfg).model.float().eval()
    sd = {"embed_tokens.weight": W["embed"], "norm.weight": W["final_norm"]}
    for li, L in enumerate(W["layers"]):
        p = f"layers.{li}."
        sd[p + "input_layernorm.weight"] = L["input_norm"]
        sd[p + "post_attention_layernorm.weight"] = L["post_norm"]
        sd[p + "mlp.gate_proj.weight"] = L["mlp"]["gate"]
        sd[p + "mlp.up_proj.weight"] = L["mlp"]["up"]
        sd[p + "mlp.down_proj.weight"] = L["mlp"]["down"]
        if "gdn" in L:
            G, q = L["gdn"], p + "linear_attn."
            sd[q + "in_proj_qkv.weight"] = G["qkv"]
            sd[q + "in_proj_z.weight"] = G["z"]
            sd[q + "in_proj_b.weight"] = G["b"]
            sd[q + "in_proj_a.weight"] = G["a"]
            sd[q + "out_proj.weight"] = G["out"]
            sd[q + "conv1d.weight"] = G["conv_w"][:, None, :]
            sd[q + "A_log"] = G["A_log"]
            sd[q + "dt_bias"] = G["dt_bias"]
            sd[q + "norm.weight"] = G["norm_w"]
        else:
            A, q = L["attn"], p + "self_attn."
            for k in ("q", "k", "v", "o"):
                sd[q + f"{k}_proj.weight"] = A[k]
            sd[q + "q_norm.weight"] = A["q_norm"]
            sd[q + "k_norm.weight"] = A["k_norm"]
    missing, unexpected = torso.load_state_dict(sd, strict=False)
    missing = [m for m in missing if "rotary" not in m]
    assert not missing and not unexpected, (missing, unexpected)
    return torso


def reference_probs(torso, rows, opt_ids, n_opts, temps, pad_id=0):
    """Full-prompt path: right-pad, forward, pool, option rows, temperature, masked softmax."""
    from strands_decider.modeling import apply_temperature, masked_log_softmax, pool_last_token

    width = max(len(r) for r in rows)
    ids = torch.tensor([r + [pad_id] * (width - len(r)) for r in rows])
    mask = torch.tensor([[1] * len(r) + [0] * (width - len(r)) for r in rows])
    with torch.inference_mode():
        hidden = torso(input_ids=ids, attention_mask=mask, return_dict=True).last_hidden_state
        pooled = pool_last_token(hidden, mask).to(torch.float32)
        table = torso.get_input_embeddings().weight
        kmax = max(len(o) for o in opt_ids)
        logits = torch.full((len(rows), kmax), -1e4)
        for i, o in enumerate(opt_ids):
            logits[i, : len(o)] = pooled[i] @ table[o].to(torch.float32).t()
        logits = apply_temperature(logits, torch.tensor(temps, dtype=torch.float32))
        lp = masked_log_softmax(logits, torch.tensor(n_opts))
    return lp.exp().numpy(), pooled.numpy(), hidden.numpy(), mask.numpy()


# The 2B shapes (hidden 2048, GDN 16 heads x 128, attention 8q/2kv x 256 with partial RoPE,
# FFN 6144, vocab 248320 tied) in a 4-layer torso [GDN x3, attention], bf16 weights: pins the
# oracle at head_dim 256 and the full vocabulary. The layers are the 2B model's own; 24 of them
# only repeat these four.
PIN_BLOCK_ROWS = 4096
PIN_OPTS = ([11, 12, 13], [248300, 248310, 248319, 5])


def hybrid2b_pin_spec():
    import dataclasses

    from strands_decider_b200 import config

    return dataclasses.replace(config.HYBRID_2B, name="hybrid-2b-shapes-4-layers",
                               layer_types=config.hybrid_pattern(4), weight_format="bf16")


def hybrid2b_pin_inputs(spec):
    g = torch.Generator().manual_seed(22)
    return torch.randint(0, spec.vocab, (160,), generator=g).tolist()


def hybrid2b_pin_weights(spec, rows=None):
    """The pin's weights in oracle.torso's nested form: linears and small parameters from the
    seeded synthetic generators (seed 2) rounded to bf16; the tied embedding N(0, 0.02) in
    blocks of PIN_BLOCK_ROWS rows, each block from its own generator, rounded to bf16. With
    `rows`, only the blocks holding those rows are generated (the others stay zero), which is
    all a forward over those ids and option rows reads."""
    from oracle import synth as osynth

    W = osynth.logical_weights(spec, seed=2, fmt="bf16")
    emb = torch.zeros(spec.vocab, spec.hidden)
    blocks = range((spec.vocab + PIN_BLOCK_ROWS - 1) // PIN_BLOCK_ROWS)
    if rows is not None:
        blocks = sorted({int(r) // PIN_BLOCK_ROWS for r in rows})
    for b in blocks:
        g = torch.Generator().manual_seed(1000 + b)
        lo, hi = b * PIN_BLOCK_ROWS, min(spec.vocab, (b + 1) * PIN_BLOCK_ROWS)
        emb[lo:hi] = (torch.randn(hi - lo, spec.hidden, generator=g) * 0.02).to(torch.bfloat16).float()
    W["embed"] = emb
    return W


def make_hybrid2b_pin():
    """The reference torso at the 2B shapes (4 layers) on one 160-token prompt, read out over two
    option sets (one reaching the last vocabulary rows)."""
    spec = hybrid2b_pin_spec()
    W = hybrid2b_pin_weights(spec)
    torso = build_reference_torso(spec, W)
    ids = hybrid2b_pin_inputs(spec)
    probs, pooled, hidden, _ = reference_probs(torso, [ids, ids], [list(o) for o in PIN_OPTS],
                                               [len(o) for o in PIN_OPTS], [1.0, 0.8])
    np.savez_compressed(os.path.join(HERE, "hybrid2b_shapes_bf16.npz"), ids=np.array(ids, np.int32),
                        probs=probs.astype(np.float32), pooled=pooled[0].astype(np.float32),
                        hidden_tail=hidden[0, -3:].astype(np.float32))
    print("hybrid-2b shapes pin", probs)


READOUT_CASES = (("slot", 24, 0), ("slot_mlp", 24, 64), ("pointer", 64, 0))


def readout_case_inputs(spec):
    """The tiny readout case: 3 prompts, option-line end positions (-1 pads), option counts,
    temperatures; regenerated from seeds by the generator and by the tests alike."""
    g = torch.Generator().manual_seed(7)
    lens = (61, 38, 90)
    rows = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in lens]
    nopt = [3, 5, 4]
    opt_idx = np.full((3, 5), -1, np.int32)
    for i, (n, k) in enumerate(zip(lens, nopt, strict=True)):
        # option lines end at increasing positions in the last 30 tokens, before <answer>
        opt_idx[i, :k] = sorted(torch.randperm(28, generator=g)[:k].add(n - 30).tolist())
    return rows, opt_idx, nopt, [1.0, 0.8, 1.3]


def make_readouts() -> None:
    """5. trained readouts (SlotHead with and without its GELU layer, PointerHead) of the
    reference on the tiny int4 torso's final hidden states."""
    from strands_decider.modeling import (PointerHead, SlotHead, apply_temperature, gather_options,
                                          masked_log_softmax, pool_last_token)

    from oracle import synth as osynth
    from strands_decider_b200 import config, synth

    spec = config.TINY
    W = osynth.logical_weights(spec, seed=1, fmt="int4")
    torso = build_reference_torso(spec, W)
    rows, opt_idx, nopt, temps = readout_case_inputs(spec)
    width = max(len(r) for r in rows)
    ids = torch.tensor([r + [0] * (width - len(r)) for r in rows])
    mask = torch.tensor([[1] * len(r) + [0] * (width - len(r)) for r in rows])
    out = {}
    with torch.inference_mode():
        hidden = torso(input_ids=ids, attention_mask=mask, return_dict=True).last_hidden_state
        pooled = pool_last_token(hidden, mask).to(torch.float32)
        options = gather_options(hidden, torch.from_numpy(opt_idx).long()).to(torch.float32)
        for name, out_dim, mlp in READOUT_CASES:
            kind = "pointer" if name == "pointer" else "slot"
            head = (PointerHead(spec.hidden, dim=out_dim) if kind == "pointer"
                    else SlotHead(spec.hidden, out_dim, hidden=mlp)).eval()
            head.load_state_dict(synth.readout_params(kind, spec.hidden, out_dim, mlp, seed=11))
            logits = head(pooled, options) if kind == "pointer" else head(pooled)
            lp = masked_log_softmax(apply_temperature(logits, torch.tensor(temps)), torch.tensor(nopt))
            out[f"probs_{name}"] = lp.exp().numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tiny_int4_readouts.npz"), **out)
    print("readouts", {k: v.shape for k, v in out.items()})


def make_recurrent_rule() -> None:
    """transformers' recurrent rule (TF:314-353) on the chunk-rule inputs, with an initial state."""
    import transformers.models.qwen3_5.modeling_qwen3_5 as q35

    out = {}
    for seq in CHUNK_SEQS:
        x, state = chunk_rule_inputs(seq)
        o, s = q35.torch_recurrent_gated_delta_rule(**{k: v[None] for k, v in x.items()},
                                                    initial_state=state[None], output_final_state=True,
                                                    use_qk_l2norm_in_kernel=True)
        out[f"s{seq}_out"] = o[0].numpy()
        out[f"s{seq}_state"] = s[0].numpy()
    np.savez_compressed(os.path.join(HERE, "recurrent_rule.npz"), **out)
    print("recurrent rule", sorted(out))


def reference_import_path(root: str) -> str:
    """The directory to put on sys.path for `import strands_decider`: root/src for a
    checkout, root itself for an installed copy."""
    src = os.path.join(root, "src")
    path = src if os.path.isdir(os.path.join(src, "strands_decider")) else root
    if not os.path.isdir(os.path.join(path, "strands_decider")):
        raise SystemExit(f"no strands_decider package under {root!r}")
    return path


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_import_path(reference_root))
    if "--readouts-only" in sys.argv:
        make_readouts()
        return
    if "--recurrent-only" in sys.argv:
        make_recurrent_rule()
        return
    if "--hybrid2b-only" in sys.argv:
        make_hybrid2b_pin()
        return
    import transformers.models.qwen3_5.modeling_qwen3_5 as q35
    from strands_decider.schema import derive_confidence, derive_score_confidence

    from oracle import synth as osynth
    from strands_decider_b200 import config

    torch.manual_seed(0)
    torch.set_num_threads(os.cpu_count() or 1)

    # 1. the reduced CPU decider: 4 prompts x 256 ids, 3 single-token options, at the last position
    spec = config.REDUCED_1024
    packed = dict(osynth.quantized_linears(spec, seed=0))
    W = osynth.logical_weights(spec, seed=0, packed=packed)
    torso = build_reference_torso(spec, W)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, spec.vocab, (4, 256), generator=g)
    rows = ids.tolist()
    opt = [[11, 12, 13]] * 4
    probs, pooled, _, _ = reference_probs(torso, rows, opt, [3] * 4, [1.0] * 4)
    np.savez_compressed(os.path.join(HERE, "reduced_1024_int4.npz"), ids=ids.numpy().astype(np.int32),
                        opt_ids=np.array(opt, dtype=np.int32), probs=probs.astype(np.float32),
                        pooled=pooled.astype(np.float32),
                        packed_digest=np.array(osynth.packed_digest(packed)))
    print("reduced_1024 probs", probs)

    # 2. ragged prompts with padding, mixed kinds and temperatures, state+question prompts,
    #    on the tiny spec (every hidden state kept, so the torso is pinned position by position)
    spec = config.TINY
    for fmt in ("int4", "nvfp4", "ternary"):
        packed = dict(osynth.quantized_linears(spec, seed=1, fmt=fmt))
        W = osynth.logical_weights(spec, seed=1, fmt=fmt, packed=packed)
        torso = build_reference_torso(spec, W)
        g = torch.Generator().manual_seed(1)
        states = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (70, 5)]
        qs = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (9, 1, 33, 64)]
        rows = [states[0] + qs[0], states[0] + qs[1], states[1] + qs[2], states[1] + qs[3]]
        opt = [[11, 12, 13], [11, 12], [11, 12, 13, 14, 15], [11, 12, 13, 14]]
        nopt = [3, 2, 5, 4]
        temps = [1.0, 0.7, 1.6, 2.5]
        probs, pooled, hidden, mask = reference_probs(torso, rows, opt, nopt, temps)
        np.savez_compressed(
            os.path.join(HERE, f"tiny_{fmt}_ragged.npz"),
            state0=np.array(states[0], np.int32), state1=np.array(states[1], np.int32),
            q0=np.array(qs[0], np.int32), q1=np.array(qs[1], np.int32),
            q2=np.array(qs[2], np.int32), q3=np.array(qs[3], np.int32),
            opt_ids=np.array([o + [0] * (5 - len(o)) for o in opt], np.int32),
            n_opts=np.array(nopt, np.int32), temps=np.array(temps, np.float32),
            probs=probs.astype(np.float32), pooled=pooled.astype(np.float32),
            hidden=hidden.astype(np.float32) if fmt == "int4" else np.zeros(0, np.float32),
            mask=mask.astype(np.int32),
            packed_digest=np.array(osynth.packed_digest(packed)))
        print(fmt, "tiny probs", probs)

    # 3. the chunk rule with an initial state and correlated keys (tests/test_mps_kernels.py:23-35);
    #    inputs are regenerated from their seeds by chunk_rule_inputs, only outputs are stored
    out = {}
    for seq in CHUNK_SEQS:
        x, state = chunk_rule_inputs(seq)
        o, s = q35.torch_chunk_gated_delta_rule(**{k: v[None] for k, v in x.items()},
                                                initial_state=state[None], output_final_state=True,
                                                use_qk_l2norm_in_kernel=True)
        out[f"s{seq}_out"] = o[0].numpy()
        out[f"s{seq}_state"] = s[0].numpy()
    np.savez_compressed(os.path.join(HERE, "chunk_rule.npz"), **out)
    make_recurrent_rule()

    # 4. answer formulas
    dists = [[1 / 3, 1 / 3, 1 / 3], [1.0, 0.0, 0.0], [0.88, 0.12, 0.0], [0.7, 0.2, 0.1],
             [0.0, 0.5, 0.5, 0.0, 0.0], [0.2] * 5, [0.5, 0.0, 0.0, 0.0, 0.5], [0.3, 0.7],
             [0.05, 0.9, 0.05], [0.1, 0.2, 0.3, 0.4]]
    conf = [derive_confidence(d) for d in dists]
    sconf = [derive_score_confidence(d) for d in dists]
    sconf_s = [derive_score_confidence(d, ordinal_smoothing=0.1) for d in dists]
    flat = np.zeros((len(dists), 5), np.float64)
    for i, d in enumerate(dists):
        flat[i, : len(d)] = d
    np.savez_compressed(os.path.join(HERE, "answer_formulas.npz"), probs=flat,
                        n=np.array([len(d) for d in dists]), confidence=np.array(conf),
                        score_confidence=np.array(sconf), score_confidence_s01=np.array(sconf_s))
    make_readouts()
    make_hybrid2b_pin()
    print("done")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("--") else os.environ.get(
        "STRANDS_DECIDER_SRC")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout or install dir> [--...-only] "
                         "(or set STRANDS_DECIDER_SRC)")
    main(root)
