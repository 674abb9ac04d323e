"""The `--device b200` engine: the reference's engine API with the prefill on B200.

strands-decider's device plugins override exactly two methods of `SystemOneEngine`
(src/strands_decider/infer.py:127-411): `_slot_probs_batched` (infer.py:253-279) and
`_slot_probs_shared_prefix` (infer.py:281-337); `MLXEngine` is the precedent
(src/strands_decider/mlx_engine.py:121-205). `B200SlotProbs` is that pair, running the
torso prefill, the prefix-state cache and the decision head on the GPU through the native
runtime (runtime.DecisionModel -> libstrands_b200.so).

Everything else is the reference's own code, inherited: `reference_engine_class()` returns
`class B200Engine(B200SlotProbs, SystemOneEngine)`, so `evaluate` (rendering, the
`num_slots` refusal, chunking by `max_batch`, the `UnforkableCache` fallback, the answer
read-back), `_fit`, `_temperatures`, `_option_idx` and `_pad` are strands-decider's. The
engine therefore needs the `strands_decider` package importable; `load_engine` builds one
from a checkpoint directory, as `strands_decider.infer.load_engine` does for the torch
devices (infer.py:476-496).

Contract of both methods (infer.py:253-337): return (probs [n, K] float32 on the CPU with
entries past each row's n_slots equal to 0, input-token count). The readout is the
checkpoint's trained head ("slot" / "pointer", modeling.py:99-180) or, with head_type
"option_token", the frozen torso's option-number distribution (`frozen_slot_log_probs`,
modeling.py:412-438): slot k is the tied-embedding row of the token "k+1".
"""

from __future__ import annotations

import threading
from typing import Any

import torch

from .runtime import KIND, DecisionModel


class Readout:
    """What the engine reads from StrandsDeciderModel besides the torso (as mlx_engine's
    _Readout): the decider config (strands_decider.modeling.StrandsDeciderConfig), the
    tokenizer, and the trained head module if any (the device head is built from it)."""

    def __init__(self, config: Any, tokenizer: Any, head: Any = None):
        self.config = config
        self.tokenizer = tokenizer
        self.head = head


def option_token_ids(tokenizer: Any, num_slots: int) -> list[int]:
    """slot k -> the single token of "k+1" (modeling.py:359-373); stops at the first slot
    whose number is not one token."""
    out = []
    for k in range(num_slots):
        ids = tokenizer.encode(str(k + 1), add_special_tokens=False)
        if len(ids) != 1:
            break
        out.append(int(ids[0]))
    return out


class B200SlotProbs:
    """The two device overrides. Expects the SystemOneEngine attributes: `cfg`, `model`
    (with `.config`), `tok`, `_fit`, `_temperatures`, plus `_rt` (a DecisionModel)."""

    _rt: DecisionModel

    def _option_rows(self, n_slots: list[int]) -> list[list[int]]:
        ids = getattr(self, "_opt_ids", None)
        if ids is None:
            ids = self._opt_ids = option_token_ids(self.tok, self.model.config.num_slots)
        for n in n_slots:
            if n > len(ids):
                raise ValueError(
                    f"question has {n} options but the option-token readout has {len(ids)} single-token "
                    f"option numbers; split the question")
        return [ids[:n] for n in n_slots]

    def _head_type(self) -> str:
        """The checkpoint's readout: "slot" / "pointer" (a trained head, modeling.py:161-180) or
        "option_token" (the torso's own option-number logits)."""
        ht = getattr(self.model.config, "head_type", "option_token")
        if ht in ("slot", "pointer") and self._rt.readout is None:
            head = getattr(self.model, "head", None)
            if head is None:
                raise RuntimeError(f"head_type {ht!r} needs the trained head's weights: call "
                                   "DecisionModel.set_readout(DeviceReadout(...)) first")
            from .readout import DeviceReadout

            self._rt.set_readout(DeviceReadout.from_module(head, ht, self._rt.spec.hidden, self._rt.device))
        return ht

    def _readout_args(self, rendered: Any, n_slots: list[int], base: int) -> dict:
        """opt_ids for the option-token readout, opt_pos for a pointer head, nothing for a slot head."""
        ht = self._head_type()
        if ht == "pointer":
            if rendered is None:
                raise ValueError("a pointer head needs the rendered questions (option spans)")
            return {"opt_ids": None, "opt_pos": self._option_idx(rendered, base).tolist()}
        if ht == "slot":
            return {"opt_ids": None}
        return {"opt_ids": self._option_rows(n_slots)}

    def _temps(self, kinds: list[str]) -> list[float]:
        t = self._temperatures(kinds)
        return [float(x) for x in (t.tolist() if isinstance(t, torch.Tensor) else t)]

    def _slot_probs_batched(self, state_text: str, question_texts: list[str], n_slots: list[int], kinds: list[str],
                            rendered: Any = None) -> tuple[torch.Tensor, int]:
        """infer.py:253-279 on the device: every (state + question) forwarded whole."""
        s, q = self._fit(state_text, question_texts)
        rows = [s + qi for qi in q]
        ra = self._readout_args(rendered, n_slots, len(s))   # full prompts: options sit after the state
        dec = self._rt.score_prompts(rows, ra["opt_ids"], n_slots, kinds, self._temps(kinds),
                                     getattr(self.model.config, "ordinal_smoothing", 0.0), opt_pos=ra.get("opt_pos"))
        return dec.probs.float().cpu(), sum(len(r) for r in rows)

    def _slot_probs_shared_prefix(self, state_text: str, question_texts: list[str], n_slots: list[int],
                                  kinds: list[str], rendered: Any = None) -> tuple[torch.Tensor, int]:
        """infer.py:281-337 on the device: the state once into a pool slot, every suffix
        against it in place (no `_expand_cache` copies)."""
        s, q = self._fit(state_text, question_texts)
        ra = self._readout_args(rendered, n_slots, 0)         # suffix-relative positions
        self._rt.prefill_states([s], [0])
        dec = self._rt.score_suffixes(q, [0] * len(q), ra["opt_ids"], n_slots, kinds, self._temps(kinds),
                                      getattr(self.model.config, "ordinal_smoothing", 0.0), opt_pos=ra.get("opt_pos"))
        return dec.probs.float().cpu(), len(s) + sum(len(x) for x in q)


    def _slot_probs_many(self, items: list[dict]) -> list[tuple[torch.Tensor, int]]:
        """Several requests' `_slot_probs_shared_prefix` in two launches: every state into its
        own pool slot in one prefill, then every request's questions against their slots in
        one suffix forward. items: dicts with state_text, question_texts, n_slots, kinds and
        optionally rendered. Returns each request's (probs [n, K], input-token count)."""
        states, sufs, slots, n_all, kinds_all, temps_all, opt_ids, opt_pos = [], [], [], [], [], [], [], []
        spans = []
        ht = self._head_type()
        for i, it in enumerate(items):
            s, q = self._fit(it["state_text"], it["question_texts"])   # also keeps this request's offsets
            ra = self._readout_args(it.get("rendered"), it["n_slots"], 0)
            states.append(s)
            spans.append((len(sufs), len(q), len(s) + sum(len(x) for x in q)))
            sufs.extend(q)
            slots.extend([i] * len(q))
            n_all.extend(it["n_slots"])
            kinds_all.extend(it["kinds"])
            temps_all.extend(self._temps(it["kinds"]))
            if ht == "option_token":
                opt_ids.extend(ra["opt_ids"])
            if ht == "pointer":
                opt_pos.extend(ra["opt_pos"])
        if len(items) > self._rt.pool_slots:
            raise ValueError(f"{len(items)} requests exceed the pool's {self._rt.pool_slots} slots")
        self._rt.prefill_states(states, list(range(len(items))))
        dec = self._rt.score_suffixes(sufs, slots, opt_ids or None, n_all, kinds_all, temps_all,
                                      getattr(self.model.config, "ordinal_smoothing", 0.0),
                                      opt_pos=opt_pos or None)
        probs = dec.probs.float().cpu()
        out = []
        for (start, n, ntok), it in zip(spans, items, strict=True):
            k = max(it["n_slots"])
            out.append((probs[start:start + n, :k].contiguous(), ntok))
        return out


class RequestBatcher:
    """Continuous batching for a serving process: requests submitted from many threads (the
    HTTP server's workers) are collected for up to `window_ms` (or until `max_requests` or
    `max_tokens` are pending) and answered by one shared prefill through
    `engine._slot_probs_many`, instead of one request at a time (the reference serves one
    request per engine call, server.py:124-125). `submit` returns a Future of
    (probs [n, K], input-token count); an engine error fails every request of its batch."""

    def __init__(self, engine: Any, max_requests: int = 32, max_tokens: int = 65536, window_ms: float = 2.0):
        import queue

        self.engine, self.max_tokens = engine, max_tokens
        rt = getattr(engine, "_rt", None)   # one pool slot per request of a batch
        self.max_requests = min(max_requests, rt.pool_slots) if rt is not None else max_requests
        self.window = window_ms / 1e3
        self._q: queue.Queue = queue.Queue()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="b200-batcher", daemon=True)
        self._thread.start()

    def submit(self, state_text: str, question_texts: list[str], n_slots: list[int], kinds: list[str],
               rendered: Any = None):
        from concurrent.futures import Future

        if self._stop.is_set():
            raise RuntimeError("the batcher is closed")
        fut: Future = Future()
        est = (len(state_text) + sum(len(q) for q in question_texts)) // 2 + 1   # rough token estimate
        self._q.put(({"state_text": state_text, "question_texts": question_texts, "n_slots": n_slots,
                      "kinds": kinds, "rendered": rendered}, est, fut))
        return fut

    def close(self) -> None:
        self._stop.set()
        self._q.put(None)
        self._thread.join(timeout=10)

    def _run(self) -> None:
        import queue
        import time

        carry = None
        while not self._stop.is_set():
            first = carry or self._q.get()
            carry = None
            if first is None:
                break
            batch, tokens = [first], first[1]
            deadline = time.monotonic() + self.window
            while len(batch) < self.max_requests:
                left = deadline - time.monotonic()
                if left <= 0:
                    break
                try:
                    nxt = self._q.get(timeout=left)
                except queue.Empty:
                    break
                if nxt is None:
                    self._stop.set()
                    break
                if tokens + nxt[1] > self.max_tokens:
                    carry = nxt   # starts the next batch
                    break
                batch.append(nxt)
                tokens += nxt[1]
            try:
                with self.engine._lock:
                    results = self.engine._slot_probs_many([b[0] for b in batch])
            except Exception as e:   # every request of the batch sees the engine's error
                for b in batch:
                    b[2].set_exception(e)
                continue
            for b, r in zip(batch, results, strict=True):
                b[2].set_result(r)


_ENGINE_CLASS = None


def reference_engine_class():
    """`class B200Engine(B200SlotProbs, strands_decider.infer.SystemOneEngine)`, built once
    on the installed reference (raises ImportError when `strands_decider` is not importable).

    `B200Engine(runtime, readout, config)`: runtime a DecisionModel, readout a `Readout`
    (config, tokenizer), config the reference's `EngineConfig` (its `device` is "b200")."""
    global _ENGINE_CLASS
    if _ENGINE_CLASS is not None:
        return _ENGINE_CLASS
    from strands_decider.infer import SystemOneEngine

    class B200Engine(B200SlotProbs, SystemOneEngine):
        def __init__(self, runtime: DecisionModel, readout: Any, config: Any):
            # Not SystemOneEngine.__init__: that moves a torch torso to a torch device
            # (mlx_engine.py:124-137 does the same). These are the attributes the inherited
            # helpers read; `device` is where their small index and temperature tensors live.
            self.cfg = config
            self.model = readout
            self.tok = readout.tokenizer
            self.device = "cpu"
            self._rt = runtime
            # one evaluation at a time: `_fit` leaves the request's option offsets on the
            # engine for `_option_idx` (mlx_engine.py:134-141)
            self._lock = threading.Lock()

        def evaluate(self, request):
            with self._lock:
                return super().evaluate(request)

    _ENGINE_CLASS = B200Engine
    return B200Engine


def load_engine(checkpoint: str, *, device: str = "b200", use_prefix_cache: bool = True, base: Any = None,
                weight_format: str = "nvfp4", max_tokens: int = 16384, pool_slots: int = 64,
                pool_kv_tokens: int | None = None, lo_plane: str = "e4m3"):
    """The `--device b200` branch of strands_decider.infer.load_engine (infer.py:476-496):
    an engine for a checkpoint directory, with the torso quantised into `weight_format` on the
    GPU. `base` is the base model (a directory of safetensors shards with its config.json, or
    a state dict); None reads the checkpoint config's `base_model`, which must then be a local
    directory (nothing is downloaded). Refuses before loading anything when no B200 is usable.
    The decider config and the tokenizer are read by the reference's own code
    (StrandsDeciderConfig.from_json, AutoTokenizer with its pad fallback, modeling.py:556-567)."""
    if device != "b200":
        raise ValueError(f"this loader serves device 'b200', not {device!r}")
    require_b200()
    from strands_decider.infer import EngineConfig
    from strands_decider.modeling import StrandsDeciderConfig, config_path
    from transformers import AutoTokenizer

    from . import checkpoint as ck

    cfg = StrandsDeciderConfig.from_json(config_path(checkpoint))
    tok = AutoTokenizer.from_pretrained(checkpoint)
    if tok.pad_token is None:
        tok.pad_token = tok.eos_token
    weights, readout, _, _ = ck.load_decider(checkpoint, base if base is not None else cfg.base_model,
                                             weight_format=weight_format)
    rt = DecisionModel(weights, max_tokens=max_tokens, pool_slots=pool_slots, pool_kv_tokens=pool_kv_tokens,
                       lo_plane=lo_plane)
    if readout is not None:
        rt.set_readout(readout)          # the runtime keeps the readout (and its weights) alive
    return reference_engine_class()(rt, Readout(cfg, tok), EngineConfig(device="b200",
                                                                        use_prefix_cache=use_prefix_cache))


def b200_available() -> bool:
    """True when a CUDA device of compute capability 10.x is visible and the library loads."""
    if not torch.cuda.is_available():
        return False
    if torch.cuda.get_device_capability(0)[0] != 10:
        return False
    try:
        from . import _lib

        _lib.load()
    except Exception:
        return False
    return True


def require_b200() -> None:
    """The device-registration check (infer.py:516-519 convention): refuse before loading."""
    if not b200_available():
        raise RuntimeError("device 'b200' needs an NVIDIA B200 (sm_100a) and the built library: "
                           "python -m strands_decider_b200.build")

