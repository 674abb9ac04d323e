"""The option-token decision head and the answer read-back, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows strands-decider:
  pool_last_token          src/strands_decider/modeling.py:193-207
  option-token readout     src/strands_decider/modeling.py:412-438 (tied table rows,
                           `pooled @ rows.T`, padded with MASK_VALUE)
  apply_temperature        src/strands_decider/modeling.py:224-238
  masked_log_softmax       src/strands_decider/modeling.py:210-221
  _to_answer               src/strands_decider/infer.py:444-472
  read_noul / read_score   src/strands_decider/prompting.py:153-187
  derive_confidence        src/strands_decider/schema.py:185-198
  derive_score_confidence  src/strands_decider/schema.py:141-182
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

MASK_VALUE = -1e4  # modeling.py:39

KIND_NOUL, KIND_CHOICE, KIND_SCORE = 0, 1, 2


def option_logits(pooled: torch.Tensor, table: torch.Tensor, opt_ids: torch.Tensor,
                  n_opts: torch.Tensor) -> torch.Tensor:
    """pooled [B, H] fp32, opt_ids [B, K] -> logits [B, K]; slots past n_opts hold MASK_VALUE
    (modeling.py:433-437)."""
    rows = table[opt_ids.clamp_min(0)].float()               # [B, K, H]
    logits = torch.einsum("bh,bkh->bk", pooled.float(), rows)
    k = logits.shape[1]
    valid = torch.arange(k)[None, :] < n_opts[:, None]
    return logits.masked_fill(~valid, MASK_VALUE)


def apply_temperature(logits: torch.Tensor, temperature: torch.Tensor) -> torch.Tensor:
    """modeling.py:233-235 (per-row tensor)."""
    t = temperature.to(logits.dtype).clamp_min(1e-6)
    return logits / t.view(-1, 1)


def masked_log_softmax(logits: torch.Tensor, n_slots: torch.Tensor) -> torch.Tensor:
    """modeling.py:210-221."""
    k = logits.size(-1)
    valid = torch.arange(k).unsqueeze(0) < n_slots.unsqueeze(1)
    masked = logits.masked_fill(~valid, MASK_VALUE)
    lp = F.log_softmax(masked.float(), dim=-1)
    return lp.masked_fill(~valid, float("-inf"))


def decide(pooled, table, opt_ids, n_opts, temperature):
    """-> probs [B, K] (masked entries 0), as `log_probs.exp()` (infer.py:279, 337)."""
    logits = option_logits(pooled, table, opt_ids, n_opts)
    return masked_log_softmax(apply_temperature(logits, temperature), n_opts).exp()


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """nn.LayerNorm over the last dim (biased variance), fp32."""
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * w + b


def slot_head(pooled: torch.Tensor, H: dict, eps: float = 1e-5) -> torch.Tensor:
    """SlotHead.forward (modeling.py:120-121): [B, hidden] -> [B, num_slots]. H holds
    `norm.weight/bias` and `proj.weight/bias` (one linear) or `proj.0.*`, `proj.2.*` (the
    Linear -> GELU -> Linear variant, modeling.py:110-116); eval mode, dropout is identity."""
    h = layer_norm(pooled, H["norm.weight"], H["norm.bias"], eps)
    if "proj.weight" in H:
        return h @ H["proj.weight"].T + H["proj.bias"]
    h = torch.nn.functional.gelu(h @ H["proj.0.weight"].T + H["proj.0.bias"])
    return h @ H["proj.2.weight"].T + H["proj.2.bias"]


def pointer_head(decide_h: torch.Tensor, options: torch.Tensor, H: dict, eps: float = 1e-5) -> torch.Tensor:
    """PointerHead.forward (modeling.py:154-158): decide [B, hidden], options [B, K, hidden]
    -> logits [B, K] = k(LN(options)) . q(LN(decide)) * dim^-1/2."""
    q = layer_norm(decide_h, H["norm.weight"], H["norm.bias"], eps) @ H["q.weight"].T + H["q.bias"]
    o = layer_norm(options, H["norm.weight"], H["norm.bias"], eps) @ H["k.weight"].T + H["k.bias"]
    return (o @ q.unsqueeze(-1)).squeeze(-1) * q.shape[-1] ** -0.5


def gather_options(hidden: torch.Tensor, opt_idx: torch.Tensor) -> torch.Tensor:
    """modeling.py:183-190: hidden [B, L, d] + opt_idx [B, K] (-1 pads) -> [B, K, d]."""
    idx = opt_idx.clamp_min(0).unsqueeze(-1).expand(-1, -1, hidden.size(-1))
    return hidden.gather(1, idx)


def decide_from_logits(logits: torch.Tensor, n_opts: torch.Tensor, temperature: torch.Tensor) -> torch.Tensor:
    """apply_temperature -> masked_log_softmax -> exp (modeling.py:463-468)."""
    return masked_log_softmax(apply_temperature(logits, temperature), n_opts).exp()


def derive_confidence(p: list[float]) -> float:
    """schema.py:185-198."""
    n = len(p)
    if n <= 1:
        return 1.0
    return float(max(0.0, min(1.0, (n * max(p) - 1.0) / (n - 1.0))))


def derive_score_confidence(p: list[float], ordinal_smoothing: float = 0.0) -> float:
    """schema.py:141-182."""
    n = len(p)
    if n <= 1:
        return 1.0
    total = sum(p)
    if total <= 0:
        return 0.0
    p = [x / total for x in p]
    mean = sum(i * pi for i, pi in enumerate(p))
    var = sum(pi * (i - mean) ** 2 for i, pi in enumerate(p))
    sigma = var ** 0.5
    sigma_max = (n - 1) / 2.0
    floor = ordinal_smoothing ** 0.5 if ordinal_smoothing > 0 else 0.0
    if sigma_max <= floor:
        return 1.0 if sigma <= floor else 0.0
    return float(max(0.0, min(1.0, (sigma_max - sigma) / (sigma_max - floor))))


def readback(kind: int, probs: list[float], ordinal_smoothing: float = 0.0) -> dict:
    """The numbers `_to_answer` derives (infer.py:444-472), before rounding, for slots in
    rendered order 0..n-1 with the identity option order (noul slot 1 = "true",
    prompting.py:27, 153-156; score level i at slot i, prompting.py:178-187)."""
    if kind == KIND_NOUL:
        return {"noul": float(probs[1])}
    if kind == KIND_CHOICE:
        best = max(range(len(probs)), key=lambda i: probs[i])
        return {"choice": best, "confidence": derive_confidence(list(probs))}
    score = sum(i * p for i, p in enumerate(probs))
    return {"score": float(score),
            "confidence": derive_score_confidence(list(probs), ordinal_smoothing)}


def device_style_outputs(probs: torch.Tensor, kinds: list[int], n_opts: list[int],
                         ordinal_smoothing: float = 0.0) -> dict[str, torch.Tensor]:
    """The per-row (argmax, confidence, score) triple the fused device head writes, from
    the same read-back rules: confidence is `derive_confidence` for choice rows,
    `derive_score_confidence` for score rows and P(true) for noul rows' score field."""
    B = probs.shape[0]
    arg = torch.zeros(B, dtype=torch.int32)
    conf = torch.zeros(B)
    score = torch.zeros(B)
    for i in range(B):
        p = probs[i, : n_opts[i]].tolist()
        arg[i] = max(range(len(p)), key=lambda j: p[j])
        if kinds[i] == KIND_NOUL:
            conf[i] = abs(2 * p[1] - 1) if len(p) > 1 else 1.0
            score[i] = p[1] if len(p) > 1 else 0.0
        elif kinds[i] == KIND_CHOICE:
            conf[i] = derive_confidence(p)
            score[i] = float(arg[i])
        else:
            conf[i] = derive_score_confidence(p, ordinal_smoothing)
            score[i] = sum(j * pj for j, pj in enumerate(p))
    return {"argmax": arg, "confidence": conf, "score": score}


def round4(x: float) -> float:
    return round(x, 4) if math.isfinite(x) else x
