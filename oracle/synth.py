"""Oracle-side weights: the seeded latent tensors, quantised by oracle.quant, dequantised,
and arranged as the reference's modules hold them.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Quantisation is per logical tensor (one reference `nn.Linear`). For NVFP4 that fixes the
per-tensor fp32 scale to the logical tensor's own amax, whatever fusion the device uses.
"""

from __future__ import annotations

import numpy as np
import torch

from strands_decider_b200 import synth
from strands_decider_b200.config import GDN, ModelSpec

from . import quant as Q
from .torso import TorsoConfig


def torso_config(spec: ModelSpec) -> TorsoConfig:
    return TorsoConfig(vocab=spec.vocab, hidden=spec.hidden, inter=spec.inter,
                       layer_types=spec.layer_types, gdn_heads=spec.gdn_heads, gdn_dk=spec.gdn_dk,
                       gdn_dv=spec.gdn_dv, conv_width=spec.conv_width, attn_heads=spec.attn_heads,
                       attn_kv_heads=spec.attn_kv_heads, head_dim=spec.head_dim,
                       rope_theta=spec.rope_theta, partial_rotary=spec.partial_rotary, eps=spec.eps)


def quantized_linears(spec: ModelSpec, seed: int, fmt: str | None = None):
    """Yield (name, packed parts dict) for every logical linear, quantised on the CPU."""
    fmt = fmt or spec.weight_format
    for li in range(spec.n_layers):
        for name, w in synth.linear_latents(spec, li, seed, "cpu"):
            yield name, Q.quantize(fmt, w.numpy())


def logical_weights(spec: ModelSpec, seed: int, fmt: str | None = None,
                    packed: dict | None = None, embed: torch.Tensor | None = None) -> dict:
    """fp32 weights in the nested form oracle.torso expects.

    `packed` (name -> parts) may supply already-quantised tensors (for instance read back
    from the device); otherwise they are quantised here from the seeded latents. `embed`
    may supply the tied embedding table (for instance the device's), else it is regenerated
    from the seed."""
    fmt = fmt or spec.weight_format
    deq = {}
    src = packed.items() if packed is not None else quantized_linears(spec, seed, fmt)
    for name, parts in src:
        deq[name] = torch.from_numpy(Q.dequantize(fmt, parts).copy())
    W = {"embed": (embed if embed is not None else synth.embedding(spec, seed)).float(),
         "final_norm": synth.final_norm(spec, seed),
         "layers": []}
    for li in range(spec.n_layers):
        p = f"layers.{li}."
        sp = synth.small_params(spec, li, seed)
        L = {"input_norm": sp[p + "input_layernorm.weight"],
             "post_norm": sp[p + "post_attention_layernorm.weight"],
             "mlp": {"gate": deq[p + "mlp.gate_proj.weight"], "up": deq[p + "mlp.up_proj.weight"],
                     "down": deq[p + "mlp.down_proj.weight"]}}
        if spec.layer_types[li] == GDN:
            q = p + "linear_attn."
            L["gdn"] = {"qkv": deq[q + "in_proj_qkv.weight"], "z": deq[q + "in_proj_z.weight"],
                        "b": deq[q + "in_proj_b.weight"], "a": deq[q + "in_proj_a.weight"],
                        "out": deq[q + "out_proj.weight"], "conv_w": sp[q + "conv1d.weight"],
                        "A_log": sp[q + "A_log"], "dt_bias": sp[q + "dt_bias"],
                        "norm_w": sp[q + "norm.weight"]}
        else:
            q = p + "self_attn."
            L["attn"] = {"q": deq[q + "q_proj.weight"], "k": deq[q + "k_proj.weight"],
                         "v": deq[q + "v_proj.weight"], "o": deq[q + "o_proj.weight"],
                         "q_norm": sp[q + "q_norm.weight"], "k_norm": sp[q + "k_norm.weight"]}
        W["layers"].append(L)
    return W


def packed_digest(parts_by_name) -> str:
    """A sha256 over the packed bytes of every logical linear, in name order."""
    import hashlib

    h = hashlib.sha256()
    for name in sorted(parts_by_name):
        h.update(name.encode())
        for key in sorted(parts_by_name[name]):
            h.update(key.encode())
            h.update(np.ascontiguousarray(parts_by_name[name][key]).tobytes())
    return h.hexdigest()


def device_logical_weights(dw, seed: int) -> dict:
    """The oracle's fp32 weights for a device model built with keep_logical=True: every
    logical linear's packed bytes read back from the GPU and dequantised here by oracle.quant
    (the device's own dequantiser is not used), the tied embedding table copied from the GPU
    (it may have been generated there), and the small parameters regenerated from the seed."""
    from strands_decider_b200.weights import packed_to_numpy

    if not dw.logical:
        raise ValueError("the device weights were built without keep_logical=True")
    packed = {name: packed_to_numpy(pw) for name, pw in dw.logical.items()}
    return logical_weights(dw.spec, seed, fmt=dw.spec.weight_format, packed=packed, embed=dw.embed.cpu())
