"""Packed device weights: quantise each logical linear on the GPU, then fuse.

Each reference `nn.Linear` is quantised on its own (so NVFP4's per-tensor scale is the
logical tensor's), by `b200_quantize`, bit-exact to the CPU definitions. The device then
keeps the fused layouts the kernels read (see config.py): row concatenation, padding to
a multiple of 256 rows, and the gate/up interleave in blocks of 64 rows.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib, synth
from .config import GDN, ROW_PAD, SWIGLU_BLOCK, ModelSpec


@dataclass
class PackedWeight:
    fmt: str
    n: int
    k: int
    data: torch.Tensor
    scales: torch.Tensor | None = None
    row_scale: torch.Tensor | None = None
    tiles: torch.Tensor | None = None        # the GEMM's streaming copy (b200_tile_weights)
    tile_scales: torch.Tensor | None = None

    def _base(self) -> _lib.QWeight:
        return _lib.QWeight(_lib.FMT[self.fmt], self.n, self.k, _lib.ptr(self.data),
                            _lib.ptr(self.scales) if self.scales is not None else None,
                            _lib.ptr(self.row_scale) if self.row_scale is not None else None, None, None)

    def ensure_tiles(self) -> None:
        """Build the per-(256-row tile, 64-column stage) streaming copy the GEMM reads."""
        if self.fmt == "bf16" or self.tiles is not None or self.n % 256 != 0:
            return
        tb, sb = C.c_size_t(), C.c_size_t()
        _lib.check(_lib.load().b200_tile_bytes(_lib.FMT[self.fmt], self.n, self.k, C.byref(tb), C.byref(sb)))
        self.tiles = torch.empty(tb.value, dtype=torch.uint8, device=self.data.device)
        self.tile_scales = torch.empty(max(sb.value, 16), dtype=torch.uint8, device=self.data.device)
        base = self._base()
        _lib.call("b200_tile_weights", C.byref(base), _lib.ptr(self.tiles), _lib.ptr(self.tile_scales),
                  _lib.stream_ptr())

    def qweight(self) -> _lib.QWeight:
        self.ensure_tiles()
        q = self._base()
        q.tiles = _lib.ptr(self.tiles) if self.tiles is not None else None
        q.tile_scales = _lib.ptr(self.tile_scales) if self.tile_scales is not None else None
        return q

    def parts(self) -> list[tuple[str, torch.Tensor]]:
        out = [("data", self.data)]
        if self.scales is not None:
            out.append(("scales", self.scales))
        if self.row_scale is not None:
            out.append(("row_scale", self.row_scale))
        return out

    def rows(self, idx: torch.Tensor, n: int) -> PackedWeight:
        def sel(t):
            return None if t is None else t.index_select(0, idx)
        return PackedWeight(self.fmt, n, self.k, sel(self.data), sel(self.scales), sel(self.row_scale))

    def nbytes(self) -> int:
        """Bytes of the canonical packed weight (the streaming copy duplicates them)."""
        return sum(t.numel() * t.element_size() for _, t in self.parts())


def quantize(fmt: str, w: torch.Tensor, stream: torch.cuda.Stream | None = None) -> PackedWeight:
    """fp32 CUDA tensor [n, k] (one logical linear) -> packed device weight."""
    assert w.is_cuda and w.dtype == torch.float32 and w.dim() == 2
    w = w.contiguous()
    n, k = w.shape
    dev = w.device
    if fmt == "bf16":
        return PackedWeight("bf16", n, k, w.to(torch.bfloat16))
    if fmt == "int4":
        data = torch.empty(n, k // 8, dtype=torch.int32, device=dev)
        scales = torch.empty(n, k // 128, dtype=torch.int16, device=dev)
        row_scale = None
    elif fmt == "nvfp4":
        data = torch.empty(n, k // 2, dtype=torch.uint8, device=dev)
        scales = torch.empty(n, k // 16, dtype=torch.uint8, device=dev)
        row_scale = torch.empty(n, dtype=torch.float32, device=dev)
    elif fmt == "ternary":
        data = torch.empty(n, k // 4, dtype=torch.uint8, device=dev)
        scales = torch.empty(n, dtype=torch.int16, device=dev)
        row_scale = None
    else:
        raise ValueError(f"unknown weight format {fmt!r}")
    _lib.call("b200_quantize", _lib.FMT[fmt], _lib.ptr(w), n, k, _lib.ptr(data), _lib.ptr(scales),
              _lib.ptr(row_scale) if row_scale is not None else None, _lib.stream_ptr(stream))
    return PackedWeight(fmt, n, k, data, scales, row_scale)


def concat_rows(parts: list[PackedWeight], pad_to: int = ROW_PAD) -> PackedWeight:
    """Stack logical weights row-wise and pad with zero rows to a multiple of pad_to."""
    fmt, k = parts[0].fmt, parts[0].k
    assert all(p.fmt == fmt and p.k == k for p in parts)
    n = sum(p.n for p in parts)
    npad = (n + pad_to - 1) // pad_to * pad_to

    def cat(name, fill=0):
        ts = [getattr(p, name) for p in parts]
        if ts[0] is None:
            return None
        t = torch.cat(ts, 0)
        if npad > n:
            t = torch.cat([t, torch.full((npad - n, *t.shape[1:]), fill, dtype=t.dtype, device=t.device)], 0)
        return t.contiguous()
    return PackedWeight(fmt, npad, k, cat("data"), cat("scales"), cat("row_scale", 1))


def interleave_gate_up(gate: PackedWeight, up: PackedWeight) -> PackedWeight:
    """Rows [gate 64j..64j+63, up 64j..64j+63] for each block j (the SwiGLU epilogue layout)."""
    inter = gate.n
    assert up.n == inter and inter % SWIGLU_BLOCK == 0
    both = concat_rows([gate, up], pad_to=1)
    j = torch.arange(inter // SWIGLU_BLOCK, device=gate.data.device)
    i = torch.arange(SWIGLU_BLOCK, device=gate.data.device)
    g_idx = (j[:, None] * SWIGLU_BLOCK + i[None, :])
    idx = torch.stack([g_idx, g_idx + inter], 1).reshape(-1)
    out = both.rows(idx, 2 * inter)
    return concat_rows([out])  # pad to ROW_PAD


class DeviceWeights:
    """All weights of one model on one GPU, in the fused device layouts."""

    def __init__(self, spec: ModelSpec):
        self.spec = spec
        self.layers: list[dict] = []
        self.embed: torch.Tensor | None = None
        self.final_norm: torch.Tensor | None = None
        self.logical: dict[str, PackedWeight] = {}   # kept only when keep_logical=True

    @classmethod
    def synthetic(cls, spec: ModelSpec, seed: int = 0, device: str = "cuda", latent_device: str | None = None,
                  keep_logical: bool = False) -> DeviceWeights:
        """Seeded random-init weights (synth.py), quantised on the GPU into spec.weight_format.

        latent_device "cpu" regenerates exactly the tensors the CPU oracle uses; "cuda" is
        faster for the 2B shape (different random streams, same distributions)."""
        if latent_device is None:
            latent_device = "cpu" if spec.linear_params() < 400_000_000 else "cuda"

        def layer(li):
            return synth.linear_latents(spec, li, seed, latent_device), synth.small_params(spec, li, seed)

        return cls._assemble(spec, synth.embedding(spec, seed, latent_device), synth.final_norm(spec, seed, "cpu"),
                             layer, device, keep_logical)

    @classmethod
    def from_state_dict(cls, spec: ModelSpec, sd: dict[str, torch.Tensor], device: str = "cuda",
                        keep_logical: bool = False) -> DeviceWeights:
        """Quantise a Qwen3.5 text-model state dict (transformers' names, as
        `Qwen3_5ForCausalLM(cfg).model.state_dict()` has them; the torso strands-decider loads,
        src/strands_decider/modeling.py:293-303) into spec.weight_format on the GPU.

        The linears may be fp32, bf16 or fp16; each is quantised from its fp32 value. The
        depthwise conv weight may be [C, 1, W] (nn.Conv1d) or [C, W]. The embedding is
        stored as bf16 (the tied output rows of the decision head read it too)."""
        sd = {k.removeprefix("model."): v for k, v in sd.items()}
        need = ["embed_tokens.weight", "norm.weight"]
        for li in range(spec.n_layers):
            need += [f"layers.{li}.{n}.weight" for n, _, _ in spec.logical_linears(li)]
        missing = [k for k in need if k not in sd]
        if missing:
            raise ValueError(f"state dict lacks {len(missing)} tensors, e.g. {missing[:3]}")

        def layer(li):
            p = f"layers.{li}."
            lin = [(f"{p}{n}.weight", sd[f"{p}{n}.weight"].float()) for n, _, _ in spec.logical_linears(li)]
            for name, w in lin:
                n_out, n_in = next((o, i) for n, o, i in spec.logical_linears(li) if name.endswith(n + ".weight"))
                if tuple(w.shape) != (n_out, n_in):
                    raise ValueError(f"{name}: shape {tuple(w.shape)} != {(n_out, n_in)}")
            small = {}
            for k, v in sd.items():
                if k.startswith(p) and not any(k == nm for nm, _ in lin):
                    v = v.float()
                    if k.endswith("conv1d.weight") and v.dim() == 3:
                        v = v[:, 0, :]
                    small[k] = v
            return iter(lin), small

        return cls._assemble(spec, sd["embed_tokens.weight"].to(torch.bfloat16), sd["norm.weight"].float(), layer,
                             device, keep_logical)

    @classmethod
    def _assemble(cls, spec: ModelSpec, embed: torch.Tensor, final_norm: torch.Tensor, layer, device: str,
                  keep_logical: bool) -> DeviceWeights:
        """Quantise every logical linear of every layer and build the fused layouts.
        layer(li) -> (iterator of (full name, [out, in] tensor), {full name: small tensor})."""
        self = cls(spec)
        fmt = spec.weight_format
        self.embed = embed.to(device).contiguous()
        self.final_norm = final_norm.to(device).contiguous()
        for li in range(spec.n_layers):
            q = {}
            lin, small = layer(li)
            for name, w in lin:
                pw = quantize(fmt, w.to(device).contiguous())
                del w
                q[name.split(".", 2)[2].rsplit(".", 1)[0]] = pw   # e.g. "linear_attn.in_proj_qkv"
                if keep_logical:
                    self.logical[name] = pw
            sp = {k.split(".", 2)[2]: v.to(device).contiguous() for k, v in small.items()}
            L = {"kind": spec.layer_types[li], "input_norm": sp["input_layernorm.weight"],
                 "post_norm": sp["post_attention_layernorm.weight"],
                 "gate_up": interleave_gate_up(q["mlp.gate_proj"], q["mlp.up_proj"]),
                 "down": concat_rows([q["mlp.down_proj"]])}
            if spec.layer_types[li] == GDN:
                L["mix_in"] = concat_rows([q["linear_attn.in_proj_qkv"], q["linear_attn.in_proj_z"],
                                           q["linear_attn.in_proj_b"], q["linear_attn.in_proj_a"]])
                L["mix_out"] = concat_rows([q["linear_attn.out_proj"]])
                L["conv_w"] = sp["linear_attn.conv1d.weight"]
                L["a_log"] = sp["linear_attn.A_log"]
                L["dt_bias"] = sp["linear_attn.dt_bias"]
                L["norm_w"] = sp["linear_attn.norm.weight"]
            else:
                L["mix_in"] = concat_rows([q["self_attn.q_proj"], q["self_attn.k_proj"], q["self_attn.v_proj"]])
                L["mix_out"] = concat_rows([q["self_attn.o_proj"]])
                L["q_norm"] = sp["self_attn.q_norm.weight"]
                L["k_norm"] = sp["self_attn.k_norm.weight"]
            self.layers.append(L)
        for L in self.layers:
            for key in ("mix_in", "mix_out", "gate_up", "down"):
                L[key].ensure_tiles()
        torch.cuda.synchronize()
        return self

    def nbytes(self) -> int:
        n = self.embed.numel() * 2
        for L in self.layers:
            for key in ("mix_in", "mix_out", "gate_up", "down"):
                n += L[key].nbytes()
        return n

    def layer_struct(self, li: int) -> _lib.LayerWeights:
        L = self.layers[li]
        s = self.spec
        lw = _lib.LayerWeights()
        lw.input_norm = _lib.ptr(L["input_norm"])
        lw.post_norm = _lib.ptr(L["post_norm"])
        lw.mix_in = L["mix_in"].qweight()
        lw.mix_out = L["mix_out"].qweight()
        lw.gate_up = L["gate_up"].qweight()
        lw.down = L["down"].qweight()
        if L["kind"] == GDN:
            lw.gdn = _lib.GdnParams(s.gdn_heads, s.gdn_dk, s.gdn_dv, s.conv_width, s.eps, _lib.ptr(L["conv_w"]),
                                    _lib.ptr(L["a_log"]), _lib.ptr(L["dt_bias"]), _lib.ptr(L["norm_w"]))
        else:
            lw.q_norm = _lib.ptr(L["q_norm"])
            lw.k_norm = _lib.ptr(L["k_norm"])
        return lw


def packed_to_numpy(pw: PackedWeight) -> dict:
    """Device packed weight -> the dict oracle.quant expects (CPU numpy, unsigned views)."""
    import numpy as np

    if pw.fmt == "bf16":
        out = {"data": pw.data.view(torch.int16).cpu().numpy().view(np.uint16)}
    else:
        out = {"data": pw.data.cpu().numpy()}
    if pw.scales is not None:
        s = pw.scales.cpu().numpy()
        out["scales"] = s.view(np.uint16) if s.dtype == np.int16 else s
    if pw.row_scale is not None:
        out["global_scale"] = pw.row_scale[:1].cpu().numpy()
    return out


_ = C  # ctypes structures are built in _lib
