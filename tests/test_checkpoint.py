"""Checkpoint loading (src/strands_decider/modeling.py:490-606 format): decider config, head
file, LoRA merge and the base model's key prefixes. CPU, on synthetic files; the GPU test
at the end quantises a whole synthetic checkpoint."""

from __future__ import annotations

import json
import os

import pytest
import torch

from strands_decider_b200 import checkpoint as ck
from strands_decider_b200 import config, synth


def _base_state(spec, seed=0, prefix="model.language_model."):
    sd = {prefix + "embed_tokens.weight": synth.embedding(spec, seed).float(),
          prefix + "norm.weight": synth.final_norm(spec, seed), "lm_head.weight": torch.zeros(3, 3),
          "model.visual.patch.weight": torch.zeros(2)}
    for li in range(spec.n_layers):
        for name, t in synth.linear_latents(spec, li, seed, "cpu"):
            sd[prefix + name] = t
        for k, v in synth.small_params(spec, li, seed).items():
            sd[prefix + k] = v[:, None, :] if k.endswith("conv1d.weight") else v
    return sd


def _write_adapter(path, spec, r=4, alpha=8.0, rslora=False):
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    g = torch.Generator().manual_seed(9)
    ad = {}
    targets = [("layers.0.mlp.gate_proj", spec.inter, spec.hidden), ("layers.3.self_attn.q_proj",
                                                                      spec.attn_q_rows, spec.hidden)]
    for name, n_out, n_in in targets:
        ad[f"base_model.model.{name}.lora_A.weight"] = torch.randn(r, n_in, generator=g) * 0.05
        ad[f"base_model.model.{name}.lora_B.weight"] = torch.randn(n_out, r, generator=g) * 0.05
    save_file(ad, os.path.join(path, "adapter_model.safetensors"))
    json.dump({"r": r, "lora_alpha": alpha, "use_rslora": rslora, "target_modules": ["q_proj", "gate_proj"]},
              open(os.path.join(path, "adapter_config.json"), "w"))
    return ad, targets


def test_torso_state_strips_wrapper_prefixes_and_other_towers():
    sd = ck.torso_state(_base_state(config.TINY))
    assert "embed_tokens.weight" in sd and "norm.weight" in sd and "layers.0.mlp.gate_proj.weight" in sd
    assert not any(k.startswith(("lm_head", "model.visual", "visual")) for k in sd)
    assert all(k.startswith(("layers.", "embed_tokens.", "norm.")) for k in sd)


@pytest.mark.parametrize("rslora", [False, True])
def test_lora_merge_is_w_plus_scaled_b_a(tmp_path, rslora):
    spec = config.TINY
    sd = ck.torso_state(_base_state(spec))
    ad, targets = _write_adapter(str(tmp_path / "lora"), spec, rslora=rslora)
    merged = ck.merge_lora(sd, str(tmp_path / "lora"))
    scale = 8.0 / (4 ** 0.5 if rslora else 4)
    for name, _, _ in targets:
        a = ad[f"base_model.model.{name}.lora_A.weight"]
        b = ad[f"base_model.model.{name}.lora_B.weight"]
        torch.testing.assert_close(merged[name + ".weight"], sd[name + ".weight"] + scale * (b @ a))
    untouched = "layers.1.mlp.down_proj.weight"
    assert torch.equal(merged[untouched], sd[untouched])


def test_lora_merge_refuses_targets_missing_from_the_base(tmp_path):
    spec = config.TINY
    sd = ck.torso_state(_base_state(spec))
    _write_adapter(str(tmp_path / "lora"), spec)
    del sd["layers.0.mlp.gate_proj.weight"]
    with pytest.raises(ValueError, match="lacks"):
        ck.merge_lora(sd, str(tmp_path / "lora"))


def test_config_and_head_files(tmp_path):
    from safetensors.torch import save_file

    d = tmp_path / "ckpt"
    d.mkdir()
    with pytest.raises(FileNotFoundError):
        ck.decider_config(str(d))
    json.dump({"head_type": "pointer", "pointer_dim": 32, "max_length": 2048, "use_lora": True, "lora_r": 16,
               "temperature_by_kind": {"score": 1.4}}, open(d / "hobson_config.json", "w"))
    cfg = ck.decider_config(str(d))
    assert cfg.head_type == "pointer" and cfg.pointer_dim == 32 and cfg.max_length == 2048
    assert cfg.temperature_by_kind == {"score": 1.4} and cfg.extra["lora_r"] == 16
    params = synth.readout_params("pointer", 64, 32, seed=1)
    save_file(params, str(d / "head.safetensors"))
    torch.save(params, str(d / "slot_head.pt"))
    with pytest.raises(ValueError, match="both"):
        ck.head_state(str(d))
    os.remove(d / "slot_head.pt")
    got = ck.head_state(str(d))
    assert set(got) == set(params) and all(torch.equal(got[k], params[k]) for k in params)


@pytest.mark.gpu
def test_load_decider_quantises_the_merged_checkpoint(tmp_path):
    from safetensors.torch import save_file

    from strands_decider_b200.weights import DeviceWeights
    from tests.test_config import _hf_config

    spec = config.TINY.with_format("nvfp4")
    base = tmp_path / "base"
    base.mkdir()
    sd = _base_state(spec)
    keys = sorted(sd)
    save_file({k: sd[k].contiguous() for k in keys[: len(keys) // 2]}, str(base / "model-00001-of-00002.safetensors"))
    save_file({k: sd[k].contiguous() for k in keys[len(keys) // 2:]}, str(base / "model-00002-of-00002.safetensors"))
    _hf_config(spec).save_pretrained(str(base))
    ck_dir = tmp_path / "ckpt"
    _write_adapter(str(ck_dir / "lora"), spec)
    json.dump({"head_type": "slot", "num_slots": 24, "use_lora": True},
              open(ck_dir / "strands_decider_config.json", "w"))
    save_file(synth.readout_params("slot", spec.hidden, 24, seed=3), str(ck_dir / "head.safetensors"))
    weights, readout, cfg, got_spec = ck.load_decider(str(ck_dir), str(base), weight_format="nvfp4")
    assert got_spec.hidden == spec.hidden and got_spec.layer_types == spec.layer_types
    want = DeviceWeights.from_state_dict(got_spec, ck.merge_lora(ck.torso_state(sd), str(ck_dir / "lora")))
    for la, lb in zip(weights.layers, want.layers, strict=True):
        for key in ("mix_in", "mix_out", "gate_up", "down"):
            for (na, ta), (nb, tb) in zip(la[key].parts(), lb[key].parts(), strict=True):
                assert na == nb and torch.equal(ta, tb), key
    assert readout is not None and readout.kind == "slot" and readout.out == 24 and cfg.head_type == "slot"


@pytest.mark.parametrize("bad", ["rank_pattern", "alpha_pattern", "use_dora", "fan_in_fan_out", "magnitude"])
def test_lora_merge_refuses_what_it_cannot_merge(tmp_path, bad):
    """Adapter options that change the arithmetic without adding tensors, and adapter tensors
    other than lora_A / lora_B pairs (here a DoRA magnitude vector), are refused."""
    from safetensors.torch import load_file, save_file

    spec = config.TINY
    sd = ck.torso_state(_base_state(spec))
    path = tmp_path / "lora"
    _write_adapter(str(path), spec)
    cfg = json.load(open(path / "adapter_config.json"))
    if bad == "magnitude":
        ad = load_file(str(path / "adapter_model.safetensors"))
        ad["base_model.model.layers.0.mlp.gate_proj.lora_magnitude_vector"] = torch.ones(spec.inter)
        save_file(ad, str(path / "adapter_model.safetensors"))
    else:
        cfg[bad] = {"gate_proj": 8} if bad.endswith("pattern") else True
        json.dump(cfg, open(path / "adapter_config.json", "w"))
    with pytest.raises(ValueError, match="cannot merge"):
        ck.merge_lora(sd, str(path))
