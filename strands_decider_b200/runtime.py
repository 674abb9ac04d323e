"""The device-side decision runtime: one model context, workspace and prefix pool per GPU.

`DecisionModel` wraps `b200_model_forward` (the whole torso prefill plus the fused
decision head, in native code) with the two paths of the reference engine:

  full prompts   `score_prompts`  - each (state + question) row forwarded whole, as
                 `SystemOneEngine._slot_probs_batched` (infer.py:253-279)
  prefix cache   `score_requests` - each state forwarded once into a prefix-pool slot,
                 then every question suffix forwarded against its state's slot, as
                 `_slot_probs_shared_prefix` (infer.py:281-337), with no cache copies

Batches are ragged and packed (no padding tokens are computed).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .config import ATTN, GDN, ModelSpec
from .weights import DeviceWeights

KIND = {"noul": 0, "choice": 1, "score": 2}


def rope_tables(spec: ModelSpec, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_positions, rope_dim/2] fp32, computed exactly as the reference computes
    them on the CPU (TF:124-135 inverse frequencies, TF:144-153 position products)."""
    dim = spec.rope_dim
    inv = 1.0 / (spec.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))
    pos = torch.arange(spec.max_positions, dtype=torch.float32)
    freqs = (inv[:, None].float() @ pos[None, :].float()).transpose(0, 1)
    return freqs.cos().contiguous().to(device), freqs.sin().contiguous().to(device)


@dataclass
class Decisions:
    """Per-row outputs of the fused head (device tensors)."""

    probs: torch.Tensor       # [rows, kmax] fp32, masked slots 0
    argmax: torch.Tensor      # [rows] int32
    confidence: torch.Tensor  # [rows] fp32
    score: torch.Tensor       # [rows] fp32

    def cpu(self) -> Decisions:
        return Decisions(self.probs.cpu(), self.argmax.cpu(), self.confidence.cpu(), self.score.cpu())


class DecisionModel:
    def __init__(self, weights: DeviceWeights, max_tokens: int = 8192, pool_slots: int = 64,
                 pool_kv_tokens: int | None = None, device: str | torch.device = "cuda",
                 dequant_min_tokens: int = 0, lo_plane: str = "e4m3"):
        """dequant_min_tokens: batches of at least this many tokens run each GEMM on a bf16 copy
        of its weight dequantised once per call (0 = the library default, 4096; < 0 = never).
        lo_plane: the low activation plane of those GEMMs, "bf16" (two bf16 planes, about 16
        significant bits) or "e4m3" (e4m3 low plane against an e4m3 weight copy: 3/4 of the
        tensor work, about 12 significant bits in the low term)."""
        if lo_plane not in ("bf16", "e4m3"):
            raise ValueError(f"lo_plane must be 'bf16' or 'e4m3', not {lo_plane!r}")
        _lib.load()
        self.w = weights
        self.spec = s = weights.spec
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        cfg = _lib.ModelConfig()
        cfg.vocab, cfg.hidden, cfg.inter, cfg.n_layers = s.vocab, s.hidden, s.inter, s.n_layers
        for i, lt in enumerate(s.layer_types):
            cfg.layer_kind[i] = _lib.LAYER_GDN if lt == GDN else _lib.LAYER_ATTN
        cfg.gdn_heads, cfg.gdn_dk, cfg.gdn_dv, cfg.conv_width = s.gdn_heads, s.gdn_dk, s.gdn_dv, s.conv_width
        cfg.attn_heads, cfg.attn_kv_heads, cfg.head_dim = s.attn_heads, s.attn_kv_heads, s.head_dim
        cfg.rope_dim, cfg.max_pos, cfg.eps = s.rope_dim, s.max_positions, s.eps
        cfg.weight_format = _lib.FMT[s.weight_format]
        cfg.dequant_min_tokens = dequant_min_tokens
        cfg.lo_format = _lib.LO_E4M3 if lo_plane == "e4m3" else _lib.LO_BF16
        self.lo_plane = lo_plane
        self._cfg = cfg
        h = C.c_void_p()
        _lib.check(_lib.load().b200_model_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self._layer_structs = []
        for li in range(s.n_layers):
            lw = weights.layer_struct(li)
            self._layer_structs.append(lw)
            _lib.check(_lib.load().b200_model_set_layer(h, li, C.byref(lw)))
        self.rope_cos, self.rope_sin = rope_tables(s, self.device)
        _lib.check(_lib.load().b200_model_set_globals(h, _lib.ptr(weights.embed), _lib.ptr(weights.final_norm),
                                                      _lib.ptr(self.rope_cos), _lib.ptr(self.rope_sin)))
        nbytes = C.c_size_t(0)
        _lib.check(_lib.load().b200_model_workspace_bytes(h, max_tokens, C.byref(nbytes)))
        self.workspace = torch.empty(int(nbytes.value), dtype=torch.uint8, device=self.device)
        self._alloc_pool(pool_slots, pool_kv_tokens or pool_slots * 512)
        self.readout = None

    # ------------------------------------------------------------------ pool
    def _alloc_pool(self, slots: int, kv_tokens: int) -> None:
        s, dev = self.spec, self.device
        n_gdn = sum(1 for t in s.layer_types if t == GDN)
        n_attn = sum(1 for t in s.layer_types if t == ATTN)
        self.pool_slots, self.kv_capacity = slots, kv_tokens
        self.gdn_state = torch.zeros(max(n_gdn, 1), slots, s.gdn_heads, s.gdn_dk, s.gdn_dv, device=dev)
        self.conv_hist = torch.zeros(max(n_gdn, 1), slots, s.conv_width - 1, s.conv_dim, device=dev)
        self.k_cache = torch.zeros(max(n_attn, 1), kv_tokens, s.attn_kv_heads, s.head_dim, dtype=torch.bfloat16,
                                   device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.slot_len = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.slot_kv = torch.zeros(slots, dtype=torch.int32, device=dev)
        self._pool = _lib.PrefixPool(slots, kv_tokens, _lib.ptr(self.slot_len), _lib.ptr(self.slot_kv),
                                     _lib.ptr(self.gdn_state), _lib.ptr(self.conv_hist), _lib.ptr(self.k_cache),
                                     _lib.ptr(self.v_cache))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().b200_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ raw forward
    def forward(self, ids: torch.Tensor, cu: torch.Tensor, prefix_slot: torch.Tensor | None = None,
                save_slot: torch.Tensor | None = None, decide: dict | None = None, max_len: int = 0,
                stream: torch.cuda.Stream | None = None) -> Decisions | None:
        """ids int32 [T], cu int32 [B+1] on the device; decide: dict of device tensors
        (last_tok, opt_ids [R, kmax], n_opts, kinds, temps) -> Decisions."""
        T = int(ids.numel())
        B = int(cu.numel()) - 1
        if T > self.max_tokens:
            raise ValueError(f"batch of {T} tokens exceeds max_tokens={self.max_tokens}")
        seqs = _lib.Seqs(B, T, max_len or T, _lib.ptr(cu), _lib.ptr(prefix_slot), _lib.ptr(save_slot))
        dec = None
        out = None
        if decide is not None:
            R, kmax = decide["opt_ids"].shape
            out = Decisions(torch.empty(R, kmax, device=self.device), torch.empty(R, dtype=torch.int32,
                            device=self.device), torch.empty(R, device=self.device), torch.empty(R, device=self.device))
            dec = _lib.DecideArgs(R, kmax, _lib.ptr(decide["last_tok"]), _lib.ptr(decide["opt_ids"]),
                                  _lib.ptr(decide["n_opts"]), _lib.ptr(decide["kinds"]), _lib.ptr(decide["temps"]),
                                  float(decide.get("ordinal_smoothing", 0.0)), _lib.ptr(out.probs),
                                  _lib.ptr(out.argmax), _lib.ptr(out.confidence), _lib.ptr(out.score),
                                  _lib.ptr(decide["opt_tok"]) if decide.get("opt_tok") is not None else None)
        _lib.check(_lib.load().b200_model_forward(
            self._h, _lib.ptr(ids), C.byref(seqs), C.byref(self._pool), C.byref(dec) if dec is not None else None,
            _lib.ptr(self.workspace), self.workspace.numel(), _lib.stream_ptr(stream)))
        return out

    def residual(self, n_tokens: int) -> torch.Tensor:
        """The fp32 residual stream [T, hidden] the last forward left at the workspace start."""
        return self.workspace[: n_tokens * self.spec.hidden * 4].view(torch.float32).view(n_tokens, self.spec.hidden)

    # ------------------------------------------------------------------ packing helpers
    def _dev(self, x, dtype=torch.int32) -> torch.Tensor:
        return torch.as_tensor(x, dtype=dtype).to(self.device, non_blocking=True)

    @staticmethod
    def _pack(rows: list[list[int]]) -> tuple[list[int], list[int]]:
        cu = [0]
        flat: list[int] = []
        for r in rows:
            if not r:
                raise ValueError("every sequence must have at least one token")
            flat.extend(r)
            cu.append(len(flat))
        return flat, cu

    def _decide_dict(self, last_tok, opt_ids, n_opts, kinds, temps, ordinal_smoothing=0.0, opt_pos=None,
                     cu=None) -> dict:
        """Device decide arguments. With the option-token readout, opt_ids are each row's option
        token ids (<= 16). With a trained readout (set_readout) opt_ids are unused; a pointer
        head needs opt_pos: per row, the positions of its options' last tokens within the row's
        own sequence (row i is tokens cu[i] .. cu[i+1] - 1 of the batch)."""
        d = {"last_tok": self._dev(last_tok), "n_opts": self._dev(n_opts),
             "kinds": self._dev([KIND.get(k, k) if isinstance(k, str) else int(k) for k in kinds]),
             "temps": self._dev(temps, torch.float32), "ordinal_smoothing": ordinal_smoothing}
        if self.readout is None:
            kmax = max(max(len(o) for o in opt_ids), 1)
            if kmax > 16:
                raise ValueError("the option-token head reads at most 16 options")
            d["opt_ids"] = self._dev([list(o) + [0] * (kmax - len(o)) for o in opt_ids])
            return d
        kmax = max(max(n_opts), 1)
        if kmax > 32 or (self.readout.kind == "slot" and kmax > self.readout.out):
            raise ValueError(f"question has {kmax} options; this readout scores at most "
                             f"{32 if self.readout.kind == 'pointer' else min(32, self.readout.out)}")
        d["opt_ids"] = torch.zeros(len(n_opts), kmax, dtype=torch.int32, device=self.device)
        if self.readout.kind == "pointer":
            if opt_pos is None:
                raise ValueError("a pointer readout needs the option token positions (opt_pos)")
            rows = []
            for i, ps in enumerate(opt_pos):
                if len(ps) < n_opts[i]:
                    raise ValueError(f"row {i}: {n_opts[i]} options but {len(ps)} option positions")
                n_i = cu[i + 1] - cu[i]
                if any(not 0 <= int(p) < n_i for p in ps[: n_opts[i]]):
                    raise ValueError(f"row {i}: an option position lies outside the forwarded sequence "
                                     f"of {n_i} tokens (with a cached state, positions count from the suffix)")
                rows.append([cu[i] + int(p) if int(p) >= 0 else -1 for p in ps[:kmax]]
                            + [-1] * (kmax - min(len(ps), kmax)))
            d["opt_tok"] = self._dev(rows)
        return d

    def set_readout(self, readout) -> None:
        """Use a trained readout (readout.DeviceReadout) for the decision head; None returns to
        the option-token logits. The readout's weights must stay alive while it is set."""
        if readout is not None and readout.hidden != self.spec.hidden:
            raise ValueError("readout hidden size does not match the model")
        r = readout.struct() if readout is not None else None
        _lib.check(_lib.load().b200_model_set_readout(self._h, C.byref(r) if r is not None else None))
        self.readout = readout

    # ------------------------------------------------------------------ the two reference paths
    def score_prompts(self, rows: list[list[int]], opt_ids, n_opts, kinds, temps, ordinal_smoothing=0.0,
                      stream=None, opt_pos=None) -> Decisions:
        """Full-prompt path: every row is a whole (state + question) prompt."""
        flat, cu = self._pack(rows)
        d = self._decide_dict([c - 1 for c in cu[1:]], opt_ids, n_opts, kinds, temps, ordinal_smoothing, opt_pos,
                              cu)
        return self.forward(self._dev(flat), self._dev(cu), decide=d, max_len=max(map(len, rows)), stream=stream)

    def prefill_states(self, states: list[list[int]], slots: list[int], stream=None, reserve: int = 0) -> None:
        """Forward each state once and keep its cache in the given pool slots. The pool is laid
        out afresh for these slots (other slots are dropped); `reserve` tokens of key/value room
        are left after each state for append_states."""
        if max(slots) >= self.pool_slots or min(slots) < 0 or len(set(slots)) != len(slots):
            raise ValueError("pool slots must be distinct and in range")
        flat, cu = self._pack(states)
        kv = torch.zeros(self.pool_slots, dtype=torch.int32)
        self._slot_room = [0] * self.pool_slots
        self._slot_len = [-1] * self.pool_slots
        off = 0
        for s, st in zip(slots, states):
            kv[s] = off
            self._slot_room[s] = len(st) + reserve
            self._slot_len[s] = len(st)
            off += len(st) + reserve
        if off > self.kv_capacity:
            raise ValueError("states (with their reserve) exceed the pool's KV capacity")
        self.slot_kv.copy_(kv.to(self.device, non_blocking=True))
        self.forward(self._dev(flat), self._dev(cu), save_slot=self._dev(slots), max_len=max(map(len, states)),
                     stream=stream)

    def append_states(self, tokens: list[list[int]], slots: list[int], stream=None) -> None:
        """Grow cached states in place: forward tokens[i] as the continuation of slot slots[i]
        and save the continued GDN state, conv history and keys / values back into that slot
        (one token at a time is the decode-time update: a batch of single tokens runs the GDN
        layers through the token-by-token recurrent kernel, longer ones through the chunk
        kernel). The slot must have been prefilled with enough `reserve` for the grown length."""
        room = getattr(self, "_slot_room", None)
        if room is None:
            raise ValueError("append_states needs slots laid out by prefill_states")
        if len(set(slots)) != len(slots):
            raise ValueError("pool slots must be distinct")
        for s, t in zip(slots, tokens, strict=True):
            if not 0 <= s < self.pool_slots or self._slot_len[s] < 0:
                raise ValueError(f"slot {s} holds no state")
            if self._slot_len[s] + len(t) > room[s]:
                raise ValueError(f"slot {s}: {self._slot_len[s]} + {len(t)} tokens exceed its room of {room[s]}")
        flat, cu = self._pack(tokens)
        sl = self._dev(slots)
        self.forward(self._dev(flat), self._dev(cu), prefix_slot=sl, save_slot=sl, max_len=max(map(len, tokens)),
                     stream=stream)
        for s, t in zip(slots, tokens):
            self._slot_len[s] += len(t)

    def score_suffixes(self, suffixes: list[list[int]], slots: list[int], opt_ids, n_opts, kinds, temps,
                       ordinal_smoothing=0.0, stream=None, opt_pos=None) -> Decisions:
        """Forward question suffixes against their states' pool slots and decide (opt_pos, for a
        pointer readout, are positions within each suffix)."""
        flat, cu = self._pack(suffixes)
        d = self._decide_dict([c - 1 for c in cu[1:]], opt_ids, n_opts, kinds, temps, ordinal_smoothing, opt_pos,
                              cu)
        return self.forward(self._dev(flat), self._dev(cu), prefix_slot=self._dev(slots), decide=d,
                            max_len=max(map(len, suffixes)), stream=stream)

    def score_requests(self, requests: list[dict], temps_by_kind: dict | None = None,
                       ordinal_smoothing: float = 0.0, stream=None) -> Decisions:
        """Requests {state, questions, kinds, n_opts, opt_ids}: the prefix-cache path."""
        temps_by_kind = temps_by_kind or {}
        slots = list(range(len(requests)))
        self.prefill_states([r["state"] for r in requests], slots, stream=stream)
        suf, sl, opt, nopt, kinds, temps = [], [], [], [], [], []
        for s, r in zip(slots, requests):
            for qi, q in enumerate(r["questions"]):
                suf.append(q)
                sl.append(s)
                opt.append(r["opt_ids"][qi])
                nopt.append(r["n_opts"][qi])
                kinds.append(r["kinds"][qi])
                temps.append(float(temps_by_kind.get(r["kinds"][qi], 1.0)))
        return self.score_suffixes(suf, sl, opt, nopt, kinds, temps, ordinal_smoothing, stream=stream)
