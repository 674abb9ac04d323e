"""torch fp32 CPU restatement of the Qwen3.5 hybrid torso, with an explicit prefix cache.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The arithmetic the reference runs lives in transformers 5.5,
`transformers/models/qwen3_5/modeling_qwen3_5.py` (cited `TF:line`; the reference pins
`transformers>=5.15,<6`, and the cited functions are unchanged in form between the two).
strands-decider calls it through `StrandsDeciderModel.encode` (`src/strands_decider/
modeling.py:342-356`). This module restates it one sequence at a time, in fp32, with the
cache made explicit:

  * a GDN layer's cache is the last 3 pre-convolution inputs (`TF:462-464`; the reference
    keeps 4, of which a width-4 causal conv reads 3) and the recurrent state S[h, dk, dv]
    (`TF:522-524`);
  * an attention layer's cache is the post-norm, post-RoPE keys and the values
    (`TF:670-671`).

A continuation with a cache is computed exactly as the same tokens appended to the
prefix: the chunk rule starts from the cached state (`TF:285-289` with
`initial_state`), the conv reads the cached inputs, and attention reads the cached
keys. (transformers 5.5 itself passes `initial_state=None` for a multi-token
continuation, `TF:498-508`, which is why the reference's own prefix-cache test fails
in this container; the restatement keeps the state, as the reference intends,
`src/strands_decider/infer.py:1-19`.)
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

# ----------------------------------------------------------------------------- config


@dataclass(frozen=True)
class TorsoConfig:
    vocab: int
    hidden: int
    inter: int
    layer_types: tuple[str, ...]          # "linear_attention" | "full_attention"
    gdn_heads: int                        # linear_num_key_heads == linear_num_value_heads
    gdn_dk: int = 128
    gdn_dv: int = 128
    conv_width: int = 4
    attn_heads: int = 8
    attn_kv_heads: int = 2
    head_dim: int = 128
    rope_theta: float = 1e7
    partial_rotary: float = 0.25
    eps: float = 1e-6

    @property
    def key_dim(self) -> int:
        return self.gdn_heads * self.gdn_dk

    @property
    def value_dim(self) -> int:
        return self.gdn_heads * self.gdn_dv

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)


# ----------------------------------------------------------------------------- helpers


def rms_norm_1p(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3_5RMSNorm: x * rsqrt(mean(x^2) + eps) * (1 + w), in fp32 (TF:711-728)."""
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * (1.0 + w.float())


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3_5RMSNormGated: RMSNorm(x) * w * silu(z), weight NOT offset by 1 (TF:175-190)."""
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return (w * y) * F.silu(z.float())


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """TF:228-231."""
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def rope_inv_freq(cfg: TorsoConfig) -> torch.Tensor:
    """Qwen3_5TextRotaryEmbedding.compute_default_rope_parameters (TF:124-135)."""
    dim = cfg.rope_dim
    return 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))


def rope_cos_sin(cfg: TorsoConfig, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [T, rope_dim] for text positions (TF:139-155; the interleaved mRoPE of
    TF:157-172 is the identity when the three position streams are equal, as for text)."""
    inv = rope_inv_freq(cfg)
    freqs = (inv[:, None].float() @ positions[None, :].float()).transpose(0, 1)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """TF:536-540."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, heads, hd]; partial rotary on the first rope_dim dims (TF:544-579)."""
    rd = cos.shape[-1]
    c, s = cos[:, None, :], sin[:, None, :]
    xr, xp = x[..., :rd], x[..., rd:]
    return torch.cat([xr * c + rotate_half(xr) * s, xp], dim=-1)


# ----------------------------------------------------------------------------- GDN chunk rule


def chunk_gated_delta_rule(q, k, v, g, beta, initial_state=None, chunk_size: int = 64,
                           use_qk_l2norm: bool = True):
    """Restatement of `torch_chunk_gated_delta_rule` (TF:234-311) for one sequence.

    q, k [T, H, dk], v [T, H, dv], g, beta [T, H] -> (o [T, H, dv], final state [H, dk, dv]).
    Same steps: l2norm (TF:246-248), q * dk^-1/2 (TF:262-263), per-chunk cumulative decay
    (TF:275-276), the UT system solved by forward substitution (TF:277-282), w/u
    (TF:283-284), and the inter-chunk recurrence (TF:294-305).
    """
    if use_qk_l2norm:
        q = l2norm(q)
        k = l2norm(k)
    q, k, v, beta, g = [x.transpose(0, 1).contiguous().float() for x in (q, k, v, beta, g)]
    H, T, dk = k.shape
    dv = v.shape[-1]
    pad = (chunk_size - T % chunk_size) % chunk_size
    q = F.pad(q, (0, 0, 0, pad))
    k = F.pad(k, (0, 0, 0, pad))
    v = F.pad(v, (0, 0, 0, pad))
    beta = F.pad(beta, (0, pad))
    g = F.pad(g, (0, pad))
    total = T + pad
    q = q * (1 / (dk ** 0.5))
    v_beta = v * beta[..., None]
    k_beta = k * beta[..., None]
    q, k, v, k_beta, v_beta = [x.reshape(H, -1, chunk_size, x.shape[-1]) for x in (q, k, v, k_beta, v_beta)]
    g = g.reshape(H, -1, chunk_size)
    mask_incl = torch.triu(torch.ones(chunk_size, chunk_size, dtype=torch.bool), diagonal=0)
    g = g.cumsum(dim=-1)
    decay = ((g[..., :, None] - g[..., None, :]).tril().exp().float()).tril()
    attn = -((k_beta @ k.transpose(-1, -2)) * decay).masked_fill(mask_incl, 0)
    for i in range(1, chunk_size):
        row = attn[..., i, :i].clone()
        sub = attn[..., :i, :i].clone()
        attn[..., i, :i] = row + (row[..., None] * sub).sum(-2)
    attn = attn + torch.eye(chunk_size)
    value = attn @ v_beta
    k_cumdecay = attn @ (k_beta * g.exp()[..., None])
    state = torch.zeros(H, dk, dv) if initial_state is None else initial_state.float().clone()
    out = torch.zeros_like(value)
    mask_strict = torch.triu(torch.ones(chunk_size, chunk_size, dtype=torch.bool), diagonal=1)
    for i in range(total // chunk_size):
        q_i, k_i, v_i = q[:, i], k[:, i], value[:, i]
        a = (q_i @ k_i.transpose(-1, -2) * decay[:, i]).masked_fill_(mask_strict, 0)
        v_new = v_i - k_cumdecay[:, i] @ state
        out[:, i] = (q_i * g[:, i, :, None].exp()) @ state + a @ v_new
        state = state * g[:, i, -1, None, None].exp() + (
            k_i * (g[:, i, -1, None] - g[:, i]).exp()[..., None]).transpose(-1, -2) @ v_new
    out = out.reshape(H, -1, dv)[:, :T]
    return out.transpose(0, 1).contiguous(), state


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, use_qk_l2norm: bool = True):
    """Token-by-token restatement of `torch_recurrent_gated_delta_rule` (TF:314-353).

    A second, independent statement of the same recurrence, used to cross-check the chunked
    form (the chunk rule must agree with it for any chunking)."""
    if use_qk_l2norm:
        q = l2norm(q)
        k = l2norm(k)
    T, H, dk = k.shape
    dv = v.shape[-1]
    q = q.float() * (1 / dk ** 0.5)
    state = torch.zeros(H, dk, dv) if initial_state is None else initial_state.float().clone()
    out = torch.zeros(T, H, dv)
    for t in range(T):
        state = state * g[t].float().exp()[:, None, None]
        kv_mem = (state * k[t].float()[:, :, None]).sum(dim=-2)
        delta = (v[t].float() - kv_mem) * beta[t].float()[:, None]
        state = state + k[t].float()[:, :, None] * delta[:, None, :]
        out[t] = (state * q[t][:, :, None]).sum(dim=-2)
    return out, state


# ----------------------------------------------------------------------------- cache


@dataclass
class SeqCache:
    """Everything a continuation of one sequence needs (all fp32)."""

    length: int = 0
    conv: dict[int, torch.Tensor] = field(default_factory=dict)   # layer -> [3, conv_dim]
    state: dict[int, torch.Tensor] = field(default_factory=dict)  # layer -> [H, dk, dv]
    k: dict[int, torch.Tensor] = field(default_factory=dict)      # layer -> [P, kvh, hd]
    v: dict[int, torch.Tensor] = field(default_factory=dict)


# ----------------------------------------------------------------------------- layers


def gdn_layer(cfg: TorsoConfig, L: dict, h: torch.Tensor, li: int, cache: SeqCache | None,
              out_cache: SeqCache | None) -> torch.Tensor:
    """Qwen3_5GatedDeltaNet.forward (TF:422-533) for one sequence h [T, hidden]."""
    T = h.shape[0]
    W = L["gdn"]
    mixed = h @ W["qkv"].T                                   # TF:442
    z = (h @ W["z"].T).reshape(T, cfg.gdn_heads, cfg.gdn_dv)  # TF:445-446
    b = h @ W["b"].T                                         # TF:448
    a = h @ W["a"].T                                         # TF:449
    kw = cfg.conv_width
    hist = (cache.conv[li] if cache is not None and li in cache.conv
            else torch.zeros(kw - 1, cfg.conv_dim))
    xin = torch.cat([hist, mixed], dim=0)                    # [kw-1+T, C]
    conv = torch.zeros(T, cfg.conv_dim)
    for j in range(kw):                                      # TF:474 (conv1d, padding kw-1)
        conv = conv + xin[j:j + T] * W["conv_w"][:, j]
    conv = F.silu(conv)
    if out_cache is not None:
        out_cache.conv[li] = xin[-(kw - 1):].clone()
    q, k, v = torch.split(conv, [cfg.key_dim, cfg.key_dim, cfg.value_dim], dim=-1)  # TF:477-485
    q = q.reshape(T, cfg.gdn_heads, cfg.gdn_dk)
    k = k.reshape(T, cfg.gdn_heads, cfg.gdn_dk)
    v = v.reshape(T, cfg.gdn_heads, cfg.gdn_dv)
    beta = b.sigmoid()                                       # TF:491
    g = -W["A_log"].float().exp() * F.softplus(a.float() + W["dt_bias"])  # TF:493
    init = cache.state.get(li) if cache is not None else None
    o, state = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=init)  # TF:498-508
    if out_cache is not None:
        out_cache.state[li] = state
    o = gated_rms_norm(o.reshape(-1, cfg.gdn_dv), z.reshape(-1, cfg.gdn_dv), W["norm_w"], cfg.eps)
    return o.reshape(T, -1) @ W["out"].T                     # TF:527-532


def attn_layer(cfg: TorsoConfig, L: dict, h: torch.Tensor, li: int, pos0: int,
               cache: SeqCache | None, out_cache: SeqCache | None) -> torch.Tensor:
    """Qwen3_5Attention.forward (TF:647-692) + eager attention (TF:594-617), one sequence."""
    T = h.shape[0]
    W = L["attn"]
    hd = cfg.head_dim
    qg = (h @ W["q"].T).view(T, cfg.attn_heads, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:]                     # TF:658-661
    gate = gate.reshape(T, -1)
    q = rms_norm_1p(q, W["q_norm"], cfg.eps)                 # TF:663
    k = rms_norm_1p((h @ W["k"].T).view(T, cfg.attn_kv_heads, hd), W["k_norm"], cfg.eps)  # TF:664
    v = (h @ W["v"].T).view(T, cfg.attn_kv_heads, hd)        # TF:665
    pos = torch.arange(pos0, pos0 + T)
    cos, sin = rope_cos_sin(cfg, pos)
    q = apply_rope(q, cos, sin)                              # TF:667-668
    k = apply_rope(k, cos, sin)
    if cache is not None and li in cache.k:
        k_all = torch.cat([cache.k[li], k], dim=0)           # TF:670-671
        v_all = torch.cat([cache.v[li], v], dim=0)
    else:
        k_all, v_all = k, v
    if out_cache is not None:
        out_cache.k[li] = k_all.clone()
        out_cache.v[li] = v_all.clone()
    rep = cfg.attn_heads // cfg.attn_kv_heads
    kr = k_all.repeat_interleave(rep, dim=1)                 # repeat_kv, TF:582-591
    vr = v_all.repeat_interleave(rep, dim=1)
    S = k_all.shape[0]
    scores = torch.einsum("thd,shd->hts", q, kr) * hd ** -0.5
    qpos = torch.arange(pos0, pos0 + T)[:, None]
    kpos = torch.arange(0, S)[None, :]
    scores = scores.masked_fill((kpos > qpos)[None], float("-inf"))
    p = torch.softmax(scores.float(), dim=-1)
    o = torch.einsum("hts,shd->thd", p, vr).reshape(T, -1)
    o = o * torch.sigmoid(gate)                              # TF:689
    return o @ W["o"].T                                      # TF:691


def mlp(L: dict, h: torch.Tensor) -> torch.Tensor:
    """Qwen3_5MLP (TF:706-708)."""
    M = L["mlp"]
    return (F.silu(h @ M["gate"].T) * (h @ M["up"].T)) @ M["down"].T


def forward_sequence(cfg: TorsoConfig, W: dict, ids: torch.Tensor, cache: SeqCache | None = None,
                     keep_cache: bool = False) -> tuple[torch.Tensor, SeqCache | None]:
    """Qwen3_5TextModel.forward (TF:1227-1290) for one sequence of ids [T] (int64).

    Returns the final-normed hidden states [T, hidden] and, with keep_cache, the cache a
    continuation needs.
    """
    pos0 = cache.length if cache is not None else 0
    out_cache = SeqCache(length=pos0 + ids.numel()) if keep_cache else None
    x = W["embed"][ids].float()                              # TF:1241
    for li, lt in enumerate(cfg.layer_types):                # TF:1272-1283
        L = W["layers"][li]
        h = rms_norm_1p(x, L["input_norm"], cfg.eps)         # TF:755
        if lt == "linear_attention":
            x = x + gdn_layer(cfg, L, h, li, cache, out_cache)
        else:
            x = x + attn_layer(cfg, L, h, li, pos0, cache, out_cache)
        h = rms_norm_1p(x, L["post_norm"], cfg.eps)          # TF:779
        x = x + mlp(L, h)
    return rms_norm_1p(x, W["final_norm"], cfg.eps), out_cache  # TF:1285
