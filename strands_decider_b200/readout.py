"""Trained readouts on the device: the reference's SlotHead and PointerHead.

Checkpoints whose `head_type` is "slot" or "pointer" answer through a small trained head on
the torso's final hidden state instead of the option-token logits
(src/strands_decider/modeling.py:99-190, `build_head`): a LayerNorm, then

  slot     Linear(hidden -> num_slots), or Linear -> GELU -> Linear with `head_hidden` > 0
  pointer  logits[k] = k(LN(h at option k's last token)) . q(LN(h at <answer>)) / sqrt(dim)

`DeviceReadout` holds the head's fp32 weights (the reference keeps its head in fp32 too,
modeling.py:161-180) on the GPU in nn.Linear layout and describes them to the C ABI
(`b200_readout`); `DecisionModel.set_readout` makes the model's decision head use it.
"""

from __future__ import annotations

import torch

from . import _lib

KINDS = {"slot": _lib.HEAD_SLOT, "pointer": _lib.HEAD_POINTER}


class DeviceReadout:
    def __init__(self, kind: str, params: dict[str, torch.Tensor], hidden: int, ln_eps: float = 1e-5,
                 device: str | torch.device = "cuda"):
        """params: the head's state dict under the reference's names (`norm.*`, then `proj.*`,
        or `proj.0.*` / `proj.2.*`, or `q.*` / `k.*`)."""
        if kind not in KINDS:
            raise ValueError(f"unknown readout kind {kind!r}; expected 'slot' or 'pointer'")
        self.kind, self.hidden, self.ln_eps = kind, hidden, float(ln_eps)
        p = {k.removeprefix("head."): v.detach().to(device=device, dtype=torch.float32).contiguous()
             for k, v in params.items()}
        need = ["norm.weight", "norm.bias"]
        if kind == "pointer":
            need += ["q.weight", "q.bias", "k.weight", "k.bias"]
        elif "proj.0.weight" in p:
            need += ["proj.0.weight", "proj.0.bias", "proj.2.weight", "proj.2.bias"]
        else:
            need += ["proj.weight", "proj.bias"]
        missing = [k for k in need if k not in p]
        if missing:
            raise ValueError(f"{kind} head state lacks {missing}")
        if p["norm.weight"].shape != (hidden,) or p["norm.bias"].shape != (hidden,):
            raise ValueError("head LayerNorm does not match the torso's hidden size")
        self.p = p
        if kind == "pointer":
            self.w1, self.b1, self.w2, self.b2 = p["q.weight"], p["q.bias"], p["k.weight"], p["k.bias"]
            self.out, self.mlp_hidden = self.w1.shape[0], 0
            if self.w2.shape != self.w1.shape or self.w1.shape[1] != hidden:
                raise ValueError("pointer head q / k must both be [dim, hidden]")
        elif "proj.0.weight" in p:
            self.w1, self.b1, self.w2, self.b2 = p["proj.0.weight"], p["proj.0.bias"], p["proj.2.weight"], p["proj.2.bias"]
            self.mlp_hidden, self.out = self.w1.shape[0], self.w2.shape[0]
            if self.w1.shape[1] != hidden or self.w2.shape[1] != self.mlp_hidden:
                raise ValueError("slot head layers do not chain")
        else:
            self.w1, self.b1, self.w2, self.b2 = p["proj.weight"], p["proj.bias"], None, None
            self.out, self.mlp_hidden = self.w1.shape[0], 0
            if self.w1.shape[1] != hidden:
                raise ValueError("slot head projection does not match the torso's hidden size")

    @classmethod
    def from_module(cls, head: torch.nn.Module, kind: str, hidden: int,
                    device: str | torch.device = "cuda") -> DeviceReadout:
        """From the reference's `model.head` (SlotHead or PointerHead), LayerNorm eps included."""
        eps = getattr(getattr(head, "norm", None), "eps", 1e-5)
        return cls(kind, dict(head.state_dict()), hidden, eps, device)

    def struct(self) -> _lib.Readout:
        r = _lib.Readout()
        r.kind, r.hidden, r.out, r.mlp_hidden, r.ln_eps = KINDS[self.kind], self.hidden, self.out, self.mlp_hidden, \
            self.ln_eps
        r.ln_w, r.ln_b = _lib.ptr(self.p["norm.weight"]), _lib.ptr(self.p["norm.bias"])
        r.w1, r.b1 = _lib.ptr(self.w1), _lib.ptr(self.b1)
        r.w2 = _lib.ptr(self.w2) if self.w2 is not None else None
        r.b2 = _lib.ptr(self.b2) if self.b2 is not None else None
        return r
