"""The device-side decision runtime: one model context, workspace and prefix pool per GPU.

`DecisionModel` wraps `b200_model_forward` (the whole torso prefill plus the fused
decision head, in native code) with the two paths of the reference engine:

  full prompts   `score_prompts`  - each (state + question) row forwarded whole, as
                 `SystemOneEngine._slot_probs_batched` (infer.py:253-279)
  prefix cache   `score_requests` - each state forwarded once into a prefix-pool slot,
                 then every question suffix forwarded against its state's slot, as
                 `_slot_probs_shared_prefix` (infer.py:281-337), with no cache copies

Batches are ragged and packed. With `graphs=True` (the default) every forward replays a CUDA
graph captured once per shape bucket (`ForwardBucket`): the batch is padded up to the bucket
with dummy sequences that read and save no cached state and whose answers are dropped, its
inputs go to the device in one copy, and the ~400 launches of the 2B torso replay as one
graph launch. `graphs=False` launches the same kernels eagerly.
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


def round_bucket(n: int, min_step: int, per_octave: int) -> int:
    """n rounded up to a multiple of a step that grows with n: the largest power of two that
    is at most n / per_octave, and at least min_step (so padding is under 1 / per_octave)."""
    if n <= 0:
        return 0
    step = max(min_step, 1 << max(0, n.bit_length() - 1 - (per_octave.bit_length() - 1)))
    return -(-n // step) * step


@dataclass(frozen=True)
class ForwardBucket:
    """The shape of one captured forward: tokens, sequences, the length bound, decision rows
    and options per row, and which of the prefix / save slot arrays and the pointer-readout
    option positions it passes."""

    tokens: int
    seqs: int
    max_len: int
    rows: int
    kmax: int
    prefix: bool
    save: bool
    opt_tok: bool

    @staticmethod
    def for_batch(n_tokens: int, lens: list[int], rows: int, kmax: int, prefix: bool, save: bool,
                  opt_tok: bool) -> ForwardBucket:
        """The bucket a batch pads up to. Padding tokens go to dummy sequences (at least one
        token each, none longer than the bucket's max_len), so a bucket with more tokens than
        the batch also has more sequences."""
        B = len(lens)
        T_b = round_bucket(n_tokens, 16, 8)
        B_b = round_bucket(B, 1, 4)
        if T_b > n_tokens and B_b == B:
            B_b = round_bucket(B + 1, 1, 4)
        if T_b - n_tokens < B_b - B:                 # every dummy needs a token
            T_b = round_bucket(n_tokens + (B_b - B), 16, 8)
        pad, dummies = T_b - n_tokens, B_b - B
        longest = max(max(lens), -(-pad // dummies) if dummies else 0)
        R_b = round_bucket(rows, 1, 4) if rows else 0
        K_b = next(k for k in (2, 4, 8, 16, 32) if k >= kmax) if rows else 0
        return ForwardBucket(T_b, B_b, round_bucket(longest, 64, 4), R_b, K_b, prefix, save, opt_tok)


class _Graph:
    """One captured forward of a bucket: its static device inputs (one int32 buffer, filled by
    one host-to-device copy per call from a pinned host buffer), the graph, and its outputs."""

    def __init__(self, model: DecisionModel, b: ForwardBucket):
        self.b = b
        T, B, R, K = b.tokens, b.seqs, b.rows, b.kmax
        sizes = [("ids", T), ("cu", B + 1), ("prefix_slot", B), ("save_slot", B), ("last_tok", R),
                 ("opt_ids", R * K), ("n_opts", R), ("kinds", R), ("temps", R), ("opt_tok", R * K)]
        self.off, n = {}, 0
        for name, k in sizes:
            self.off[name] = (n, k)
            n += k
        self.host = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        self.dev = torch.zeros(n, dtype=torch.int32, device=model.device)
        self.graph = None
        self.out: Decisions | None = None
        self.ordinal_smoothing = 0.0
        self.copied: torch.cuda.Event | None = None   # the last host-to-device copy of `host`

    def view(self, t: torch.Tensor, name: str) -> torch.Tensor:
        o, k = self.off[name]
        return t[o:o + k]

    def fill(self, flat: list[int], cu: list[int], prefix: list[int] | None, save: list[int] | None,
             dec: dict | None) -> None:
        """Pack one batch (padded with dummies) into the pinned host buffer (after the previous
        call's copy out of it has finished)."""
        if self.copied is not None:
            self.copied.synchronize()
        b = self.b
        T, B = len(flat), len(cu) - 1
        h = self.host
        ids = self.view(h, "ids")
        ids[:T] = torch.as_tensor(flat, dtype=torch.int32)
        ids[T:] = 0
        # dummies: the padding tokens spread over B_b - B sequences, as evenly as possible
        d = b.seqs - B
        pad = b.tokens - T
        ends = cu + [T + (pad * (i + 1)) // d for i in range(d)] if d else list(cu)
        self.view(h, "cu")[:] = torch.as_tensor(ends, dtype=torch.int32)
        for name, vals in (("prefix_slot", prefix), ("save_slot", save)):
            v = self.view(h, name)
            v[:] = -1
            if vals is not None:
                v[:B] = torch.as_tensor(vals, dtype=torch.int32)
        if b.rows:
            R, K = len(dec["last_tok"]), b.kmax
            self.view(h, "last_tok")[:] = b.tokens - 1
            self.view(h, "last_tok")[:R] = torch.as_tensor(dec["last_tok"], dtype=torch.int32)
            oi = self.view(h, "opt_ids").view(b.rows, K)
            oi.zero_()
            src = dec["opt_ids"]
            oi[:R, : src.shape[1]] = src
            self.view(h, "n_opts")[:] = 1
            self.view(h, "n_opts")[:R] = torch.as_tensor(dec["n_opts"], dtype=torch.int32)
            self.view(h, "kinds")[:] = 0
            self.view(h, "kinds")[:R] = torch.as_tensor(dec["kinds"], dtype=torch.int32)
            tv = self.view(h, "temps").view(torch.float32)
            tv[:] = 1.0
            tv[:R] = torch.as_tensor(dec["temps"], dtype=torch.float32)
            ot = self.view(h, "opt_tok").view(b.rows, K)
            ot.fill_(-1)
            ot[:, 0] = b.tokens - 1
            if dec.get("opt_tok") is not None:
                ot[:R, :] = -1
                ot[:R, : dec["opt_tok"].shape[1]] = dec["opt_tok"]

    def launch(self, model: DecisionModel, stream=None, slots: bool = True) -> Decisions | None:
        """The forward on the device buffers (eager); the graph records exactly this. With
        slots=False the prefix / save slot arrays are left out (no cached state is read or
        written)."""
        b, d = self.b, self.dev
        dec = None
        if b.rows:
            dec = {"last_tok": self.view(d, "last_tok"), "opt_ids": self.view(d, "opt_ids").view(b.rows, b.kmax),
                   "n_opts": self.view(d, "n_opts"), "kinds": self.view(d, "kinds"),
                   "temps": self.view(d, "temps").view(torch.float32),
                   "ordinal_smoothing": self.ordinal_smoothing,
                   "opt_tok": self.view(d, "opt_tok").view(b.rows, b.kmax) if b.opt_tok else None}
        return model.forward(self.view(d, "ids"), self.view(d, "cu"),
                             self.view(d, "prefix_slot") if b.prefix and slots else None,
                             self.view(d, "save_slot") if b.save and slots else None, dec, max_len=b.max_len,
                             stream=stream)


class DecisionModel:
    def __init__(self, weights: DeviceWeights, max_tokens: int = 8192, pool_slots: int = 64,
                 pool_kv_tokens: int | None = None, device: str | torch.device = "cuda",
                 dequant_min_tokens: int = 0, lo_plane: str = "e4m3", graphs: bool = True):
        """dequant_min_tokens: batches of at least this many tokens run each GEMM on a bf16 copy
        of its weight dequantised once per call (0 = the library default, 4096; < 0 = never).
        lo_plane: the low activation plane of those GEMMs, "bf16" (two bf16 planes, about 16
        significant bits) or "e4m3" (e4m3 low plane against an e4m3 weight copy: 3/4 of the
        tensor work, about 12 significant bits in the low term).
        graphs: replay one CUDA graph per shape bucket (captured on first use) instead of
        launching every kernel from the host."""
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
        self.use_graphs = graphs
        self.max_graphs = 64          # captured buckets kept (oldest dropped first)
        self._graphs: dict = {}

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

    def _decide_host(self, last_tok, opt_ids, n_opts, kinds, temps, ordinal_smoothing=0.0, opt_pos=None,
                     cu=None) -> dict:
        """Decide arguments as CPU tensors. With the option-token readout, opt_ids are each row's
        option token ids (<= 16). With a trained readout (set_readout) opt_ids are unused; a
        pointer head needs opt_pos: per row, the positions of its options' last tokens within
        the row's own sequence (row i is tokens cu[i] .. cu[i+1] - 1 of the batch)."""
        I = torch.int32
        d = {"last_tok": torch.as_tensor(last_tok, dtype=I), "n_opts": torch.as_tensor(n_opts, dtype=I),
             "kinds": torch.as_tensor([KIND.get(k, k) if isinstance(k, str) else int(k) for k in kinds], dtype=I),
             "temps": torch.as_tensor(temps, dtype=torch.float32), "ordinal_smoothing": float(ordinal_smoothing),
             "opt_tok": None}
        if self.readout is None:
            kmax = max(max(len(o) for o in opt_ids), 1)
            if kmax > 16:
                raise ValueError("the option-token head reads at most 16 options")
            d["opt_ids"] = torch.as_tensor([list(o) + [0] * (kmax - len(o)) for o in opt_ids], dtype=I)
            return d
        kmax = max(max(n_opts), 1)
        if kmax > 32 or (self.readout.kind == "slot" and kmax > self.readout.out):
            raise ValueError(f"question has {kmax} options; this readout scores at most "
                             f"{32 if self.readout.kind == 'pointer' else min(32, self.readout.out)}")
        d["opt_ids"] = torch.zeros(len(n_opts), kmax, dtype=I)
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
            d["opt_tok"] = torch.as_tensor(rows, dtype=I)
        return d

    def set_readout(self, readout) -> None:
        """Use a trained readout (readout.DeviceReadout) for the decision head; None returns to
        the option-token logits. The readout's weights must stay alive while it is set. Graphs
        captured with the previous readout are dropped."""
        if readout is not None and readout.hidden != self.spec.hidden:
            raise ValueError("readout hidden size does not match the model")
        r = readout.struct() if readout is not None else None
        _lib.check(_lib.load().b200_model_set_readout(self._h, C.byref(r) if r is not None else None))
        self.readout = readout
        self._graphs.clear()

    # ------------------------------------------------------------------ one forward: graph or eager
    def _run(self, flat: list[int], cu: list[int], prefix: list[int] | None, save: list[int] | None,
             dec: dict | None, stream=None) -> Decisions | None:
        """One b200_model_forward over a packed batch given on the host: a graph replay of its
        bucket (captured on first use) when graphs are on, else eager launches. Returns the
        decisions of the real rows (device tensors; with graphs they are the graph's output
        buffers, valid until the next call in the same bucket)."""
        lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
        n_rows = len(dec["last_tok"]) if dec is not None else 0
        kmax = int(dec["opt_ids"].shape[1]) if dec is not None else 0
        b = None
        if self.use_graphs and not torch.cuda.is_current_stream_capturing():
            b = ForwardBucket.for_batch(len(flat), lens, n_rows, kmax, prefix is not None, save is not None,
                                        dec is not None and dec.get("opt_tok") is not None)
            if b.tokens > self.max_tokens:
                b = None
        if b is None:
            ddev = None
            if dec is not None:
                ddev = {k: (v.to(self.device, non_blocking=True) if isinstance(v, torch.Tensor) else v)
                        for k, v in dec.items()}
            return self.forward(self._dev(flat), self._dev(cu), self._dev(prefix) if prefix is not None else None,
                                self._dev(save) if save is not None else None, ddev, max_len=max(lens), stream=stream)
        key = (b, dec["ordinal_smoothing"] if dec is not None else 0.0)
        g = self._graphs.get(key)
        if g is None:
            if len(self._graphs) >= self.max_graphs:       # drop the oldest capture
                torch.cuda.synchronize(self.device)        # none of its replays still running
                self._graphs.pop(next(iter(self._graphs)))
            g = self._graphs[key] = _Graph(self, b)
            g.ordinal_smoothing = key[1]
        g.fill(flat, cu, prefix, save, dec)
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.stream(st):
            g.dev.copy_(g.host, non_blocking=True)
            if g.copied is None:
                g.copied = torch.cuda.Event()
            g.copied.record(st)
            if g.graph is None:
                self._capture(g, st)
            g.graph.replay()
            if not b.rows:
                return None
            o = g.out   # the graph's own output buffers: the caller gets copies
            return Decisions(o.probs[:n_rows, :kmax].clone(), o.argmax[:n_rows].clone(),
                             o.confidence[:n_rows].clone(), o.score[:n_rows].clone())

    def _capture(self, g: _Graph, st) -> None:
        """Capture g's forward. A warm-up launch on the same inputs with the slot arrays left out
        (it reads and saves no cached state) runs the library's one-time set-up outside the
        capture."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(st)
        with torch.cuda.stream(side):
            g.launch(self, stream=side, slots=False)
        st.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):   # captures on a side stream, after a device synchronisation
            g.out = g.launch(self, stream=torch.cuda.current_stream(self.device))
        g.graph = graph

    def _dev(self, x, dtype=torch.int32) -> torch.Tensor:
        return torch.as_tensor(x, dtype=dtype).to(self.device, non_blocking=True)

    # ------------------------------------------------------------------ the two reference paths
    def score_prompts(self, rows: list[list[int]], opt_ids, n_opts, kinds, temps, ordinal_smoothing=0.0,
                      stream=None, opt_pos=None) -> Decisions:
        """Full-prompt path: every row is a whole (state + question) prompt."""
        flat, cu = self._pack(rows)
        d = self._decide_host([c - 1 for c in cu[1:]], opt_ids, n_opts, kinds, temps, ordinal_smoothing, opt_pos, cu)
        return self._run(flat, cu, None, None, d, stream=stream)

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
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.stream(st):
            self.slot_kv.copy_(kv.pin_memory(), non_blocking=True)
        self._run(flat, cu, None, list(slots), None, stream=st)

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
        self._run(flat, cu, list(slots), list(slots), None, stream=stream)
        for s, t in zip(slots, tokens):
            self._slot_len[s] += len(t)

    def score_suffixes(self, suffixes: list[list[int]], slots: list[int], opt_ids, n_opts, kinds, temps,
                       ordinal_smoothing=0.0, stream=None, opt_pos=None) -> Decisions:
        """Forward question suffixes against their states' pool slots and decide (opt_pos, for a
        pointer readout, are positions within each suffix)."""
        flat, cu = self._pack(suffixes)
        d = self._decide_host([c - 1 for c in cu[1:]], opt_ids, n_opts, kinds, temps, ordinal_smoothing, opt_pos, cu)
        return self._run(flat, cu, list(slots), None, d, stream=stream)

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
