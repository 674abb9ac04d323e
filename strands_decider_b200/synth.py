"""Seeded synthetic decider weights and request batches (random-init, no checkpoint).

Every tensor has its own generator seeded from (seed, tensor name), so any tensor can be
regenerated alone, in any order, on the same device type. Distributions:
  linears and the tied embedding   N(0, 0.02)
  RMSNorm (1 + w) weights           w ~ N(0, 0.1)
  gated RMSNorm weight              1 + N(0, 0.1)
  depthwise conv weight             U(-0.5, 0.5)   (nn.Conv1d's default bound for width 4)
  A_log                             log U(0.01, 1)
  dt_bias                           1              (transformers' init, TF:805)
The embedding is rounded to bf16, the precision it is stored in on the device.
"""

from __future__ import annotations

import zlib
from collections.abc import Iterator

import torch

from .config import ATTN, GDN, ModelSpec, Workload

STD = 0.02


def _gen(seed: int, name: str, device: str) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 63))
    return g


def randn(seed: int, name: str, shape, device: str = "cpu", std: float = STD) -> torch.Tensor:
    return torch.randn(*shape, generator=_gen(seed, name, device), device=device) * std


def rand(seed: int, name: str, shape, lo: float, hi: float, device: str = "cpu") -> torch.Tensor:
    return torch.rand(*shape, generator=_gen(seed, name, device), device=device) * (hi - lo) + lo


def small_params(spec: ModelSpec, li: int, seed: int, device: str = "cpu") -> dict[str, torch.Tensor]:
    """Layer li's non-linear parameters, fp32, reference names."""
    p = f"layers.{li}."
    H = spec.hidden
    out = {p + "input_layernorm.weight": randn(seed, p + "input_layernorm.weight", (H,), device, 0.1),
           p + "post_attention_layernorm.weight": randn(seed, p + "post_attention_layernorm.weight",
                                                        (H,), device, 0.1)}
    if spec.layer_types[li] == GDN:
        q = p + "linear_attn."
        out[q + "conv1d.weight"] = rand(seed, q + "conv1d.weight", (spec.conv_dim, spec.conv_width),
                                        -0.5, 0.5, device)
        out[q + "A_log"] = torch.log(rand(seed, q + "A_log", (spec.gdn_heads,), 0.01, 1.0, device))
        out[q + "dt_bias"] = torch.ones(spec.gdn_heads, device=device)
        out[q + "norm.weight"] = 1.0 + randn(seed, q + "norm.weight", (spec.gdn_dv,), device, 0.1)
    else:
        q = p + "self_attn."
        out[q + "q_norm.weight"] = randn(seed, q + "q_norm.weight", (spec.head_dim,), device, 0.1)
        out[q + "k_norm.weight"] = randn(seed, q + "k_norm.weight", (spec.head_dim,), device, 0.1)
    return out


def linear_latents(spec: ModelSpec, li: int, seed: int, device: str = "cpu"
                   ) -> Iterator[tuple[str, torch.Tensor]]:
    """Layer li's linear weights [out, in] fp32 N(0, 0.02), reference names."""
    for name, n_out, n_in in spec.logical_linears(li):
        full = f"layers.{li}.{name}.weight"
        yield full, randn(seed, full, (n_out, n_in), device)


def embedding(spec: ModelSpec, seed: int, device: str = "cpu") -> torch.Tensor:
    """Tied embedding table [vocab, hidden] as bf16."""
    return randn(seed, "embed_tokens.weight", (spec.vocab, spec.hidden), device).to(torch.bfloat16)


def final_norm(spec: ModelSpec, seed: int, device: str = "cpu") -> torch.Tensor:
    return randn(seed, "norm.weight", (spec.hidden,), device, 0.1)


def layer_kind(spec: ModelSpec, li: int) -> str:
    return "gdn" if spec.layer_types[li] == GDN else "attn" if spec.layer_types[li] == ATTN else "?"


# ----------------------------------------------------------------------------- requests


def request_batch(w: Workload, vocab: int, first: int = 0, count: int | None = None):
    """Deterministic synthetic requests first .. first+count-1 of workload w.

    Returns a list of dicts {state: [ids], questions: [[ids]], kinds: [...], n_opts: [...],
    opt_ids: [[ids]]}. Option ids are the fixed single-token ids 11..15 (the digit tokens
    "1".."5" stand-ins); token ids are uniform in [0, vocab)."""
    count = w.n_requests - first if count is None else count
    out = []
    for r in range(first, first + count):
        g = torch.Generator().manual_seed(w.seed * 7919 + r)
        lo, hi = w.state_len
        s_len = lo if lo == hi else int(torch.randint(lo, hi + 1, (1,), generator=g))
        state = torch.randint(0, vocab, (s_len,), generator=g).tolist()
        qs, kinds, nopts = [], [], []
        for qi in range(w.n_questions):
            qs.append(torch.randint(0, vocab, (w.question_len,), generator=g).tolist())
            kinds.append(w.kinds[qi % len(w.kinds)])
            if w.option_range is not None:
                lo_o, hi_o = w.option_range
                nopts.append(int(torch.randint(lo_o, hi_o + 1, (1,), generator=g)))
            else:
                nopts.append(w.options[qi % len(w.options)])
        out.append({"state": state, "questions": qs, "kinds": kinds, "n_opts": nopts,
                    "opt_ids": [[11 + j for j in range(k)] for k in nopts]})
    return out


# ----------------------------------------------------------------------------- readouts


def readout_params(kind: str, hidden: int, out: int, mlp_hidden: int = 0, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded weights of a trained readout under the reference's parameter names
    (SlotHead / PointerHead, src/strands_decider/modeling.py:99-158): LayerNorm weight 1 +
    N(0, 0.1) and bias N(0, 0.1); linear weights N(0, in^-1/2), biases N(0, 0.02).
    kind "slot" (out = num_slots, optional GELU layer of mlp_hidden) or "pointer" (out = dim)."""
    def n(name, shape, std):
        return randn(seed, f"readout.{name}", shape, "cpu", std)

    W = {"norm.weight": 1.0 + n("norm.weight", (hidden,), 0.1), "norm.bias": n("norm.bias", (hidden,), 0.1)}
    if kind == "pointer":
        for p in ("q", "k"):
            W[f"{p}.weight"] = n(f"{p}.weight", (out, hidden), hidden ** -0.5)
            W[f"{p}.bias"] = n(f"{p}.bias", (out,), 0.02)
    elif mlp_hidden > 0:
        W["proj.0.weight"] = n("proj.0.weight", (mlp_hidden, hidden), hidden ** -0.5)
        W["proj.0.bias"] = n("proj.0.bias", (mlp_hidden,), 0.02)
        W["proj.2.weight"] = n("proj.2.weight", (out, mlp_hidden), mlp_hidden ** -0.5)
        W["proj.2.bias"] = n("proj.2.bias", (out,), 0.02)
    else:
        W["proj.weight"] = n("proj.weight", (out, hidden), hidden ** -0.5)
        W["proj.bias"] = n("proj.bias", (out,), 0.02)
    return W
