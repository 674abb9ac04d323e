"""Loading a strands-decider checkpoint onto the B200 backend.

A checkpoint directory (src/strands_decider/modeling.py:490-606) holds

  strands_decider_config.json (or the legacy hobson_config.json)  the decider config
  head.safetensors or slot_head.pt                                 the trained readout
  lora/ adapter_config.json + adapter_model.safetensors            the LoRA adapter (use_lora)
  tokenizer files

and names its base model, a Qwen3.5 checkpoint loaded through Qwen3_5ForCausalLM's text
tower (modeling.py:279-308). Here the base weights come from a local directory (or an
in-memory state dict): there is no download. `load_decider` merges the adapter into the
base linears in fp32 (W + scaling * B A, peft's LoRA merge), quantises every linear on the
GPU into the chosen packed format (`DeviceWeights.from_state_dict`) and copies the head
(`DeviceReadout`).
"""

from __future__ import annotations

import glob
import json
import os
import re
from dataclasses import dataclass, field, fields
from typing import Any

import torch

from .config import ModelSpec

CONFIG_NAMES = ("strands_decider_config.json", "hobson_config.json")
_PREFIXES = ("base_model.model.", "model.language_model.", "language_model.model.", "language_model.", "model.")


def read_tensors(path: str) -> dict[str, torch.Tensor]:
    """All tensors of a safetensors file, a directory of safetensors shards, or a torch
    state-dict file (loaded with weights_only=True), on the CPU."""
    if os.path.isdir(path):
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"{path}: no .safetensors files")
        out: dict[str, torch.Tensor] = {}
        for f in files:
            out.update(read_tensors(f))
        return out
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file

        return dict(load_file(path))
    return dict(torch.load(path, map_location="cpu", weights_only=True))


def torso_state(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Keys as the text torso names them (`layers.N...`, `embed_tokens.weight`,
    `norm.weight`); the multimodal / causal-LM / peft wrappers' prefixes are dropped, as are
    tensors outside the text torso (vision tower, a separate lm_head)."""
    out = {}
    for k, v in sd.items():
        if k.startswith(("visual.", "model.visual.", "lm_head.", "mtp.")):
            continue
        for p in _PREFIXES:
            if k.startswith(p):
                k = k[len(p):]
                break
        if k.startswith(("layers.", "embed_tokens.", "norm.")):
            out[k] = v
    return out


def merge_lora(sd: dict[str, torch.Tensor], adapter_dir: str) -> dict[str, torch.Tensor]:
    """W + scaling * (B @ A) for every adapted linear (peft's merge_and_unload for LoRA):
    scaling = lora_alpha / r, or lora_alpha / sqrt(r) with use_rslora. Returns a new dict with
    fp32 merged weights. Only plain linear LoRA is merged: options that change the arithmetic
    without adding tensors (fan_in_fan_out, per-module rank or alpha patterns, DoRA) and any
    adapter tensor other than lora_A / lora_B weight pairs (DoRA magnitudes, LoRA biases,
    embedding LoRA, saved modules) are refused, as the reference's MLX merge refuses them
    (mlx_engine.py:74-118); so is an adapted weight missing from the base."""
    cfg = json.load(open(os.path.join(adapter_dir, "adapter_config.json"), encoding="utf-8"))
    r, alpha = int(cfg["r"]), float(cfg["lora_alpha"])
    unsupported = [k for k in ("fan_in_fan_out", "rank_pattern", "alpha_pattern", "use_dora") if cfg.get(k)]
    if unsupported:
        raise ValueError(f"{adapter_dir}: cannot merge an adapter with {unsupported}")
    scaling = alpha / (r ** 0.5 if cfg.get("use_rslora") else r)
    raw = {re.sub(r"\.lora_([AB])(\.default)?\.weight$", r".lora_\1.weight", k): v
           for k, v in read_tensors(adapter_dir).items()}
    other = sorted(k for k in raw if not k.endswith((".lora_A.weight", ".lora_B.weight")))
    if other:
        raise ValueError(f"{adapter_dir}: only lora_A / lora_B weight pairs merge; cannot merge "
                         f"{other[:3]}{' ...' if len(other) > 3 else ''}")
    ad = torso_state(raw)
    out = dict(sd)
    for ka in [k for k in ad if k.endswith(".lora_A.weight")]:
        base = ka[: -len(".lora_A.weight")]
        kb = base + ".lora_B.weight"
        kw = base + ".weight"
        if kb not in ad:
            raise ValueError(f"adapter has {ka} without {kb}")
        if kw not in out:
            raise ValueError(f"adapter targets {kw}, which the base model lacks")
        a, b = ad[ka].float(), ad[kb].float()
        out[kw] = out[kw].float() + scaling * (b @ a)
    return out


@dataclass
class CheckpointConfig:
    """The fields of a checkpoint's decider config file (strands_decider_config.json, the
    format of modeling.py:43-97) that the loader reads; every other field is kept in `extra`."""

    base_model: str = ""
    head_type: str = "slot"
    num_slots: int = 24
    pointer_dim: int = 256
    head_hidden: int = 0
    max_length: int = 3072
    temperature: float = 1.0
    temperature_by_kind: dict[str, float] = field(default_factory=dict)
    ordinal_smoothing: float = 0.0
    extra: dict[str, Any] = field(default_factory=dict)


def decider_config(checkpoint_dir: str) -> CheckpointConfig:
    """The checkpoint's config file, read into a CheckpointConfig."""
    path = next((os.path.join(checkpoint_dir, n) for n in CONFIG_NAMES
                 if os.path.exists(os.path.join(checkpoint_dir, n))), None)
    if path is None:
        raise FileNotFoundError(f"{checkpoint_dir}: no {' or '.join(CONFIG_NAMES)}")
    raw = json.load(open(path, encoding="utf-8"))
    known = {f.name for f in fields(CheckpointConfig)} - {"extra"}
    return CheckpointConfig(**{k: v for k, v in raw.items() if k in known},
                         extra={k: v for k, v in raw.items() if k not in known})


def head_state(checkpoint_dir: str) -> dict[str, torch.Tensor]:
    """head.safetensors or slot_head.pt; a directory with both is refused (modeling.py:586-606)."""
    st, pt = os.path.join(checkpoint_dir, "head.safetensors"), os.path.join(checkpoint_dir, "slot_head.pt")
    if os.path.exists(st) and os.path.exists(pt):
        raise ValueError(f"{checkpoint_dir}: holds both head.safetensors and slot_head.pt. Keep only one.")
    if os.path.exists(st):
        return read_tensors(st)
    if os.path.exists(pt):
        return read_tensors(pt)
    raise FileNotFoundError(f"{checkpoint_dir}: no head.safetensors or slot_head.pt")


def load_decider(checkpoint_dir: str, base, weight_format: str = "nvfp4", device: str = "cuda",
                 hf_config=None):
    """(DeviceWeights, DeviceReadout or None, CheckpointConfig, ModelSpec) for a checkpoint.

    base: the base model's weights, a directory of safetensors shards (with its config.json)
    or a state dict; hf_config: its transformers text config when `base` is a state dict.
    With use_lora the checkpoint's lora/ adapter is merged first. The readout is None when
    the config's head_type is "option_token"."""
    from .readout import DeviceReadout
    from .weights import DeviceWeights

    cfg = decider_config(checkpoint_dir)
    if isinstance(base, str):
        sd = read_tensors(base)
        if hf_config is None:
            import transformers

            hf_config = transformers.AutoConfig.from_pretrained(base)
            hf_config = hf_config.get_text_config() if hasattr(hf_config, "get_text_config") else hf_config
    else:
        sd = dict(base)
        if hf_config is None:
            raise ValueError("hf_config is needed when the base weights are a state dict")
    sd = torso_state(sd)
    lora = os.path.join(checkpoint_dir, "lora")
    if cfg.extra.get("use_lora", True) and os.path.isdir(lora):
        sd = merge_lora(sd, lora)
    elif cfg.extra.get("use_lora", False):
        raise FileNotFoundError(f"{lora}: missing, but the config sets use_lora")
    spec = ModelSpec.from_hf_config(hf_config, weight_format=weight_format)
    weights = DeviceWeights.from_state_dict(spec, sd, device=device)
    readout = None
    if cfg.head_type in ("slot", "pointer"):
        readout = DeviceReadout(cfg.head_type, head_state(checkpoint_dir), spec.hidden, device=device)
    return weights, readout, cfg, spec
