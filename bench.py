"""Decisions/s of the batched scoring prefill on B200 (the hybrid-2B NVFP4 workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload nvfp4|prefix|ternary-batch|latency]

Workload (one GPU): the 2B-shape hybrid decider (hidden 2048, 24 layers at 3:1
GDN:attention, GDN 16 heads x 128, attention 8q/2kv x 256, FFN 6144, vocab 248320 tied)
with NVFP4 weights; 1024 requests of 512 uniform-random tokens, each with 3 questions
(3-way choice, yes/no noul, 3-level score) of 32 tokens. A step is one batch of
--requests-per-step requests through the prefix-cache path: every state is forwarded once
into a pool slot, then all question suffixes are forwarded against their slots and decided
by the fused head. Data are synthetic (seeded), weights random-init.

Other workloads: `prefix` (512 requests with states of U[64, 2048] tokens, 32 questions of
48 tokens, 2-5 options), `ternary-batch` (4096 single-question 96-token requests as full
prompts, ternary weights) and `latency` (p50 / p99 of one 96-token request, CUDA-graphed).
On one GPU the default line also carries a summary of each of them (`prefix_cache` and
`ternary_batch`: 3 timed steps in a child process, with their own CPU baseline and parity;
`latency`) and of the int4 GEMM microbench (`c2_gemm`); `--no-extras` leaves them out.

Steps replay one CUDA graph per batch. Under torchrun (N > 1) the requests are sharded
longest-processing-time first (weak scaling, no collective in the forward) and every step's
answer records are all-gathered over NCCL.
"""

from __future__ import annotations

import argparse
import ctypes as C
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from strands_decider_b200 import _lib, config  # noqa: E402
from strands_decider_b200 import weights as WT  # noqa: E402

METRIC = "decisions/sec per B200 and per 8xB200 box; p50 single-request latency (ms)"
UNIT = "decisions/s"


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        # nvidia-smi numbers GPUs physically; CUDA_VISIBLE_DEVICES may renumber them for torch,
        # so the device is named by its UUID
        self.index = str(index)
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(index).uuid)
        except Exception:
            pass
        self.rows: list[list[str]] = []
        self.proc = None
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[0]) for r in self.rows if len(r) >= 7 and r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if len(r) >= 7 and r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 7 for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline


def _oracle_weights(spec: config.ModelSpec) -> dict:
    from strands_decider_b200 import synth

    W = {"embed": synth.embedding(spec, 0).float(), "final_norm": synth.final_norm(spec, 0), "layers": []}
    for li in range(spec.n_layers):
        lat = {n.split(".", 2)[2].rsplit(".", 1)[0]: t for n, t in synth.linear_latents(spec, li, 0)}
        sp = {k.split(".", 2)[2]: v for k, v in synth.small_params(spec, li, 0).items()}
        L = {"input_norm": sp["input_layernorm.weight"], "post_norm": sp["post_attention_layernorm.weight"],
             "mlp": {"gate": lat["mlp.gate_proj"], "up": lat["mlp.up_proj"], "down": lat["mlp.down_proj"]}}
        if spec.layer_types[li] == config.GDN:
            L["gdn"] = {"qkv": lat["linear_attn.in_proj_qkv"], "z": lat["linear_attn.in_proj_z"],
                        "b": lat["linear_attn.in_proj_b"], "a": lat["linear_attn.in_proj_a"],
                        "out": lat["linear_attn.out_proj"], "conv_w": sp["linear_attn.conv1d.weight"],
                        "A_log": sp["linear_attn.A_log"], "dt_bias": sp["linear_attn.dt_bias"],
                        "norm_w": sp["linear_attn.norm.weight"]}
        else:
            L["attn"] = {"q": lat["self_attn.q_proj"], "k": lat["self_attn.k_proj"], "v": lat["self_attn.v_proj"],
                         "o": lat["self_attn.o_proj"], "q_norm": sp["self_attn.q_norm.weight"],
                         "k_norm": sp["self_attn.k_norm.weight"]}
        W["layers"].append(L)
    return W


def cpu_baseline(spec: config.ModelSpec, wl: config.Workload, n_requests: int = 1, n_questions: int | None = None,
                 full_prompt: bool = False, W: dict | None = None) -> dict:
    """The CPU oracle (a restatement of the reference's torso and readout) on a bounded
    sample of the same workload: the first n_requests requests (their first n_questions
    questions) through the prefix-cache path (state once, then each question against the
    state's cache) or, with full_prompt, each question as one full prompt; fp32 on all
    host threads. W: the oracle's weights (for a parity check, the device's own weights
    dequantised by the oracle); by default fp32 tensors of the same shapes (the per-token
    arithmetic does not depend on their values). The returned dict carries the sample's
    probabilities under "_probs" (rows in request, question order)."""
    from oracle import head as OH
    from oracle import synth as osynth
    from oracle import torso as OT
    from strands_decider_b200 import synth

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = osynth.torso_config(spec)
    W = W if W is not None else _oracle_weights(spec)
    probs = []
    reqs = synth.request_batch(wl, spec.vocab, 0, n_requests)
    decisions = 0
    tokens = 0
    t0 = time.perf_counter()
    with torch.inference_mode():
        for r in reqs:
            qs = r["questions"][: n_questions or len(r["questions"])]
            cache = None
            if not full_prompt:
                _, cache = OT.forward_sequence(cfg, W, torch.tensor(r["state"]), keep_cache=True)
                tokens += len(r["state"])
            for qi, q in enumerate(qs):
                ids = q if cache is not None else r["state"] + q
                hid, _ = OT.forward_sequence(cfg, W, torch.tensor(ids), cache=cache)
                tokens += len(ids)
                n = r["n_opts"][qi]
                probs.append(OH.decide(hid[-1:], W["embed"], torch.tensor([r["opt_ids"][qi]]), torch.tensor([n]),
                                       torch.tensor([1.0]))[0])
                decisions += 1
    dt = time.perf_counter() - t0
    path = "full prompts" if full_prompt else "prefix-cache path"
    return {"value": decisions / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n_requests} request(s) of {wl.name}, {decisions} decisions, {tokens} tokens, {path}, "
                      f"fp32 torch on {cores} threads, {dt:.1f} s", "_probs": probs}


def parity_check(gpu_probs: torch.Tensor, cpu_probs: list[torch.Tensor], n_opts: list[int]) -> dict:
    """The timed graphs' answers for the CPU sample's questions against the oracle's:
    the largest probability difference and whether every choice (argmax) agrees."""
    d, agree = 0.0, True
    for i, (want, n) in enumerate(zip(cpu_probs, n_opts, strict=True)):
        got = gpu_probs[i, :n].double()
        d = max(d, float((got - want[:n].double()).abs().max()))
        agree = agree and int(got.argmax()) == int(want[:n].argmax())
    return {"max_dp": d, "argmax_equal": agree, "questions": len(cpu_probs), "tolerance": 2e-3,
            "oracle": "fp32 CPU oracle on the device's weights (packed bytes read back, dequantised by oracle.quant)"}


# ----------------------------------------------------------------------------- GPU arm


def _store_split(rows: int, tokens: int, n_sm: int = 148) -> bool:
    """Whether the in-projection's store GEMM splits K (and so first zeroes its output), as
    gemm.cu decides: 128-column tiles when two 256-column tiles per SM or fewer, then a K split
    when two tiles per SM or fewer."""
    mt = (tokens + 127) // 128
    bn = 128 if 2 * (rows // 256) * mt <= n_sm else 256
    return 2 * (rows // bn) * mt <= n_sm


def launches_per_forward(spec: config.ModelSpec, decide: bool, tokens: int = 0, saves: bool = False,
                         lo_plane: str = "e4m3") -> int:
    """Kernels one b200_model_forward launches: embed; per layer 2 norms, 4 GEMMs and the
    mixer's 2 kernels, plus a zeroing kernel before a split-K in-projection (batches of 129 to
    4095 tokens; up to 128 tokens on packed weights the norm before it clears the output);
    forwards of >= 4096 tokens also dequantise each of the 4 weights per layer once (bf16
    weights too with the e4m3 low plane); the slot-length update when states are saved; the head."""
    big = tokens >= 4096
    folded = tokens <= 128 and spec.weight_format != "bf16"
    dq = 4 if big and (spec.weight_format != "bf16" or lo_plane == "e4m3") else 0
    n = 1 + (1 if decide else 0) + (1 if saves else 0)
    for lt in spec.layer_types:
        rows = spec.gdn_in_rows_padded if lt == config.GDN else -(-spec.attn_qkv_rows // 256) * 256
        n += 2 + 4 + 2 + dq + (0 if big or folded or not _store_split(rows, tokens) else 1)
    return n


class Batch:
    """One step's inputs, resident on the device (or in pinned host memory for e2e).

    Prefix-cache form: every state is forwarded once into its pool slot, then every question
    suffix against its state's slot. Full-prompt form (prefix=False): each question is
    forwarded as state + question in one sequence."""

    def __init__(self, reqs: list[dict], device, pinned: bool = False, kmax: int = 3, prefix: bool = True):
        flat_s, cu_s, flat_q, cu_q = [], [0], [], [0]
        slots, qslots, opt, nopt, kinds, qids = [], [], [], [], [], []
        for i, r in enumerate(reqs):
            if prefix:
                flat_s += r["state"]
                cu_s.append(len(flat_s))
                slots.append(i)
            for qi, q in enumerate(r["questions"]):
                flat_q += q if prefix else r["state"] + q
                cu_q.append(len(flat_q))
                qslots.append(i)
                opt.append(r["opt_ids"][qi] + [0] * (kmax - len(r["opt_ids"][qi])))
                nopt.append(r["n_opts"][qi])
                kinds.append(r["kinds"][qi])
                qids.append(r["id"] * len(r["questions"]) + qi)
        self.prefix = prefix
        self.n_state_tokens, self.n_suffix_tokens = len(flat_s), len(flat_q)
        self.max_state = max(len(r["state"]) for r in reqs) if prefix else 0
        self.max_q = max(cu_q[j + 1] - cu_q[j] for j in range(len(cu_q) - 1))
        I = torch.int32
        host = {"q_ids": torch.tensor(flat_q, dtype=I), "q_cu": torch.tensor(cu_q, dtype=I),
                "last_tok": torch.tensor([c - 1 for c in cu_q[1:]], dtype=I),
                "opt_ids": torch.tensor(opt, dtype=I), "n_opts": torch.tensor(nopt, dtype=I),
                "kinds": torch.tensor(kinds, dtype=I), "temps": torch.ones(len(nopt), dtype=torch.float32),
                "qid": torch.tensor(qids, dtype=I)}
        if prefix:
            host.update({"s_ids": torch.tensor(flat_s, dtype=I), "s_cu": torch.tensor(cu_s, dtype=I),
                         "s_slot": torch.tensor(slots, dtype=I), "slot_kv": torch.tensor(cu_s[:-1], dtype=I),
                         "q_slot": torch.tensor(qslots, dtype=I)})
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in host.values())
        if pinned:
            self.host = {k: v.pin_memory() for k, v in host.items()}
            self.dev = {k: torch.empty_like(v, device=device) for k, v in host.items()}
            for k in host:
                self.dev[k].copy_(self.host[k])
        else:
            self.host = None
            self.dev = {k: v.to(device) for k, v in host.items()}
        self.n_decisions = len(nopt)
        self.tokens = self.n_state_tokens + self.n_suffix_tokens

    def upload(self) -> None:
        """The step's host-to-device copies (pinned host memory, current stream)."""
        for k, v in self.host.items():
            self.dev[k].copy_(v, non_blocking=True)


def run_step(model, b: Batch, stream) -> object:
    """One pass of the hot path over one batch, ending in the fused decision head."""
    d = b.dev
    dec = {"last_tok": d["last_tok"], "opt_ids": d["opt_ids"], "n_opts": d["n_opts"], "kinds": d["kinds"],
           "temps": d["temps"]}
    if not b.prefix:
        return model.forward(d["q_ids"], d["q_cu"], decide=dec, max_len=b.max_q, stream=stream)
    model.slot_kv[: d["slot_kv"].numel()].copy_(d["slot_kv"], non_blocking=True)
    model.forward(d["s_ids"], d["s_cu"], save_slot=d["s_slot"], max_len=b.max_state, stream=stream)
    return model.forward(d["q_ids"], d["q_cu"], prefix_slot=d["q_slot"], decide=dec, max_len=b.max_q, stream=stream)


class StepGraph:
    """run_step for one batch captured as a CUDA graph: the ~200-400 launches of the
    native layer loop replay as one graph launch on the batch's device inputs."""

    def __init__(self, model, b: Batch):
        self.b = b
        self.g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            run_step(model, b, s)          # one eager pass outside the capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(self.g):
            self.out = run_step(model, b, torch.cuda.current_stream())

    def replay(self):
        self.g.replay()
        return self.out


def records(dec, b: Batch):
    from strands_decider_b200 import dispatch

    return dispatch.AnswerRecords.pack(b.dev["qid"], dec.argmax, dec.confidence, dec.score, dec.probs)


def gemm_roofline(model, tokens: int, pk: dict, reps: int = 20) -> dict:
    """Time the dominant kernel (the gate/up projection GEMM with its SwiGLU epilogue, the
    largest GEMM of every layer) alone with CUDA events at a state-prefill batch's M, in the
    form the forward runs it: for batches of >= 4096 tokens the packed weight is first
    dequantised once into a bf16 [N, K] buffer (timed separately) and the GEMM streams that.

    achieved = algorithmic FLOPs (2 M N K) / GEMM time. The activations enter as two bf16
    planes (hi + lo, fp32-level precision), so the tensor pipe executes 2x the algorithmic
    FLOPs; frac is against the measured bf16 peak and is therefore bounded by 0.5. With e4m3 low
    planes (lo_plane "e4m3") the low plane runs as e4m3 MMAs at twice the rate: 1.5x the
    algorithmic FLOPs in bf16-MMA terms, so frac is bounded by 2/3."""
    import ctypes as C

    from strands_decider_b200 import _lib

    s = model.spec
    pw = model.w.layers[0]["gate_up"]
    xp = torch.randn(2, tokens, s.hidden, device="cuda").to(torch.bfloat16)
    out = torch.empty(2, tokens, s.inter, dtype=torch.bfloat16, device="cuda")
    o = _lib.LinearOut(_lib.EP_SWIGLU, 2 * s.inter, _lib.ptr(out), s.inter, tokens * s.inter)
    qw = pw.qweight()
    st = torch.cuda.current_stream()
    lo8 = tokens >= 4096 and getattr(model, "lo_plane", "bf16") == "e4m3"
    dequant = lo8 or (tokens >= 4096 and s.weight_format != "bf16")
    if dequant:
        wdq = torch.empty(pw.n, pw.k, dtype=torch.bfloat16, device="cuda")
        wdq8 = torch.empty(pw.n, pw.k, dtype=torch.uint8, device="cuda")
        qb = _lib.QWeight()
        qb.format, qb.n, qb.k, qb.data = _lib.FMT["bf16"], pw.n, pw.k, _lib.ptr(wdq)

        def unpack():
            if lo8:
                _lib.call("b200_dequantize_lo8", C.byref(qw), _lib.ptr(wdq), _lib.ptr(wdq8), st.cuda_stream)
            else:
                _lib.call("b200_dequantize", C.byref(qw), _lib.ptr(wdq), st.cuda_stream)
    gw = qb if dequant else qw
    if lo8:
        o.lo_format = _lib.LO_E4M3
        xl8 = torch.zeros(tokens, s.hidden, dtype=torch.uint8, device="cuda")

    def launch():
        if lo8:
            _lib.call("b200_linear_lo8", _lib.ptr(xp[0]), _lib.ptr(xl8), tokens, s.hidden, s.hidden, _lib.ptr(wdq),
                      _lib.ptr(wdq8), pw.n, C.byref(o), st.cuda_stream)
        else:
            _lib.call("b200_linear", _lib.ptr(xp[0]), _lib.ptr(xp[1]), tokens, s.hidden, s.hidden, C.byref(gw),
                      C.byref(o), st.cuda_stream)

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    dq_ms = timed(unpack) if dequant else None
    ms = timed(launch)
    flops = 2.0 * tokens * (2 * s.inter) * s.hidden
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        # the weight copies once, the token-proportional rest (activations, outputs) per token
        tj = json.load(open(tp))
        per_tok = tj.get("gate_up_dram_bytes_per_token")
        if per_tok:
            traffic = round(tj.get("gate_up_weight_bytes", 0) + per_tok * tokens)
    wname = "bf16 (dequantised once per call)" if dequant else s.weight_format
    planes = "lo8" if lo8 else "split"
    n_sm = torch.cuda.get_device_properties(0).multi_processor_count
    pair = dequant and (2 * s.inter // 256) * ((tokens + 255) // 256) >= n_sm // 2
    kname = (f"gemm_pair_kernel<swiglu,{planes}> (CTA pairs, 256x256 tiles, weights {wname})" if pair
             else f"gemm_tc_kernel<256,{wname},swiglu,{planes}>")
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": traffic,
            "kernel": f"{kname} M={tokens} N={2 * s.inter} K={s.hidden}",
            "ms_per_launch": round(ms, 4), "dequant_ms_per_launch": round(dq_ms, 4) if dq_ms else None,
            "mma_flops_per_algorithmic_flop": 1.5 if lo8 else 2,
            "peak_src": pk["src"] + " bf16 burst (tcgen05 kind::f16)"}


# ----------------------------------------------------------------------------- single-kernel cases
# `bench.py --case gemm|gdn|attention`: seeded synthetic operands on cuda:0, a few warm-up
# launches, the CUDA-event time per launch, then ONE more launch between cudaProfilerStart and
# cudaProfilerStop, so a profiler started with capture off (`ncu --profile-from-start off`)
# records exactly that launch. Shapes: a linear of the 2B decider (default the gate/up
# projection, N = 2 x 6144, K = 2048), the GDN token mixer (16 heads x 128) over `seqs`
# sequences of `len` tokens, the gated attention layer (8 query / 2 kv heads x 256).

def _case_time(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _case_profiled(fn) -> None:
    torch.cuda.cudart().cudaProfilerStart()
    fn()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    if _lib.read_fault():
        raise RuntimeError("a kernel recorded a fault")


def gemm_case(m: int, fmt: str, ep: str, n: int = 2 * 6144, k: int = 2048, planes: str = "split"):
    """b200_linear with x as two bf16 planes [2, m, k] and a packed [n, k] weight; with planes
    "lo8", b200_linear_lo8 on the weight's two copies (b200_dequantize_lo8) and an e4m3 low
    plane, as large batches run it with lo_plane "e4m3"."""
    g = torch.Generator(device="cuda").manual_seed(0)
    if ep == "swiglu":
        gate = WT.quantize(fmt, torch.randn(n // 2, k, device="cuda", generator=g) * 0.02)
        up = WT.quantize(fmt, torch.randn(n // 2, k, device="cuda", generator=g) * 0.02)
        pw = WT.interleave_gate_up(gate, up)
    else:
        pw = WT.concat_rows([WT.quantize(fmt, torch.randn(n, k, device="cuda", generator=g) * 0.02)])
    pw.ensure_tiles()
    xp = torch.randn(2, m, k, device="cuda", generator=g).to(torch.bfloat16)
    if ep == "swiglu":
        out = torch.empty(2, m, n // 2, dtype=torch.bfloat16, device="cuda")
        o = _lib.LinearOut(_lib.EP_SWIGLU, n, _lib.ptr(out), n // 2, m * (n // 2))
    else:
        out = torch.zeros(m, n, device="cuda")
        o = _lib.LinearOut(_lib.EP_STORE if ep == "store" else _lib.EP_RESID_ADD, n, _lib.ptr(out), n, 0)
    qw = pw.qweight()
    keep = (pw, xp, out)
    if planes == "lo8":
        whi = torch.empty(pw.n, k, dtype=torch.bfloat16, device="cuda")
        wlo8 = torch.empty(pw.n, k, dtype=torch.uint8, device="cuda")
        _lib.call("b200_dequantize_lo8", C.byref(qw), _lib.ptr(whi), _lib.ptr(wlo8), _lib.stream_ptr())
        xl8 = torch.randint(0, 0x38, (m, k), dtype=torch.uint8, device="cuda", generator=g)  # e4m3 below 1.0
        o.lo_format = _lib.LO_E4M3
        keep = (pw, xp, out, whi, wlo8, xl8)

        def launch_lo8():
            _lib.call("b200_linear_lo8", _lib.ptr(keep[1][0]), _lib.ptr(keep[5]), m, k, k, _lib.ptr(keep[3]),
                      _lib.ptr(keep[4]), pw.n, C.byref(o), _lib.stream_ptr())

        return launch_lo8, 2.0 * m * n * k

    def launch():
        _lib.call("b200_linear", _lib.ptr(keep[1][0]), _lib.ptr(keep[1][1]) if planes == "split" else None, m, k, k,
                  C.byref(qw), C.byref(o), _lib.stream_ptr())

    return launch, 2.0 * m * n * k


GDN_ENTRY = {"auto": "b200_gdn_mixer", "chunked": "b200_gdn_mixer_chunked", "recurrent": "b200_gdn_mixer_recurrent"}


def gdn_case(seqs: int, length: int, heads: int = 16, scan: str = "auto", prefix: str = ""):
    """b200_gdn_mixer (prep + scan kernels) over `seqs` sequences of `length` tokens; `scan`
    forces the chunked or the recurrent kernel. prefix "read": every sequence starts from its own
    pool slot's state and conv history (a question against a cached state); "append": it also
    saves the continued ones back into the slot."""
    g = torch.Generator(device="cuda").manual_seed(0)
    ld = 3 * heads * 128 + heads * 128 + 2 * heads
    T = seqs * length
    mix = torch.randn(T, ld, device="cuda", generator=g)
    out = torch.empty(2, T, heads * 128, dtype=torch.bfloat16, device="cuda")
    conv_w = torch.rand(3 * heads * 128, 4, device="cuda", generator=g) - 0.5
    a_log = torch.log(torch.rand(heads, device="cuda", generator=g) * 0.99 + 0.01)
    dt = torch.ones(heads, device="cuda")
    nw = torch.ones(128, device="cuda")
    p = _lib.GdnParams(heads, 128, 128, 4, 1e-6, _lib.ptr(conv_w), _lib.ptr(a_log), _lib.ptr(dt), _lib.ptr(nw))
    cu = torch.arange(0, T + 1, length, dtype=torch.int32, device="cuda")
    scratch = torch.empty(_lib.load().b200_gdn_scratch_floats(heads, T), device="cuda")
    keep = [mix, out, conv_w, a_log, dt, nw, cu, scratch]
    pool = None
    if prefix:
        slots = torch.arange(seqs, dtype=torch.int32, device="cuda")
        state = 0.05 * torch.randn(seqs, heads, 128, 128, device="cuda", generator=g)
        hist = torch.randn(seqs, 3, 3 * heads * 128, device="cuda", generator=g)
        slot_len = torch.zeros(seqs, dtype=torch.int32, device="cuda")
        keep += [slots, state, hist, slot_len]
        pool = C.byref(_lib.PrefixPool(seqs, 0, _lib.ptr(slot_len), _lib.ptr(slot_len), _lib.ptr(state),
                                       _lib.ptr(hist), None, None))
        s = _lib.Seqs(seqs, T, length, _lib.ptr(cu), _lib.ptr(slots), _lib.ptr(slots) if prefix == "append" else None)
    else:
        s = _lib.Seqs(seqs, T, length, _lib.ptr(cu), None, None)

    def launch():
        _lib.call(GDN_ENTRY[scan], C.byref(p), C.byref(s), _lib.ptr(keep[0]), ld, _lib.ptr(keep[1]),
                  T * heads * 128, pool, 0, _lib.ptr(keep[7]), _lib.stream_ptr())

    return launch, None


def attention_case(seqs: int, length: int):
    """b200_attention (prep + flash kernels), 8 query / 2 kv heads x 256, causal, no prefix."""
    from strands_decider_b200.runtime import rope_tables

    nq, nkv, hd = 8, 2, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    T = seqs * length
    cols = 2 * nq * hd + 2 * nkv * hd
    qkv = torch.randn(T, cols, device="cuda", generator=g)
    qn = 0.1 * torch.randn(hd, device="cuda", generator=g)
    kn = 0.1 * torch.randn(hd, device="cuda", generator=g)
    cos, sin = rope_tables(config.HYBRID_2B, "cuda")
    cu = torch.arange(0, T + 1, length, dtype=torch.int32, device="cuda")
    out = torch.empty(2, T, nq * hd, dtype=torch.bfloat16, device="cuda")
    qb = torch.empty(T, nq, hd, dtype=torch.bfloat16, device="cuda")
    kb = torch.empty(T, nkv, hd, dtype=torch.bfloat16, device="cuda")
    vb = torch.empty_like(kb)
    p = _lib.AttnParams(nq, nkv, hd, hd // 4, cos.shape[0], 1e-6, _lib.ptr(qn), _lib.ptr(kn), _lib.ptr(cos),
                        _lib.ptr(sin))
    s = _lib.Seqs(seqs, T, length, _lib.ptr(cu), None, None)
    keep = (qkv, qn, kn, cos, sin, cu, out, qb, kb, vb)

    def launch():
        _lib.call("b200_attention", C.byref(p), C.byref(s), _lib.ptr(keep[0]), cols, _lib.ptr(keep[7]),
                  _lib.ptr(keep[8]), _lib.ptr(keep[9]), _lib.ptr(keep[6]), T * nq * hd, None, 0, _lib.stream_ptr())

    # causal QK^T and PV: 4 * hd * heads FLOPs per (query, key) pair, length (length + 1) / 2 pairs
    return launch, 4.0 * hd * nq * seqs * length * (length + 1) / 2



def small_kernels_case(tokens: int = 8192, rows: int = 384):
    """One launch each of the kernels outside the GEMM / mixer / attention, at the 2B shapes:
    the embedding gather (tokens ids of the 248320 x 2048 bf16 table), RMSNorm into two bf16
    planes and into the e4m3 low-plane form (tokens x 2048 fp32), the option-token decision head
    and the pointer-head readout (rows questions over a tokens x 2048 residual), and the weight
    dequantiser and NVFP4 quantiser on the 12288 x 2048 gate/up weight."""
    from strands_decider_b200 import synth
    from strands_decider_b200.readout import DeviceReadout

    spec = config.HYBRID_2B
    H = spec.hidden
    g = torch.Generator(device="cuda").manual_seed(0)
    table = (torch.randn(spec.vocab, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids = torch.randint(0, spec.vocab, (tokens,), device="cuda", dtype=torch.int32, generator=g)
    x = torch.empty(tokens, H, device="cuda")
    w_norm = 0.1 * torch.randn(H, device="cuda", generator=g)
    planes = torch.empty(2, tokens, H, dtype=torch.bfloat16, device="cuda")
    last = torch.randint(0, tokens, (rows,), device="cuda", dtype=torch.int32, generator=g)
    opt = torch.arange(11, 14, device="cuda", dtype=torch.int32).repeat(rows, 1).contiguous()
    nopt = torch.full((rows,), 3, device="cuda", dtype=torch.int32)
    kinds = torch.arange(rows, device="cuda", dtype=torch.int32) % 3
    temps = torch.ones(rows, device="cuda")
    outs = [torch.empty(rows, 3, device="cuda"), torch.empty(rows, dtype=torch.int32, device="cuda"),
            torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")]
    opt_tok = torch.randint(0, tokens, (rows, 3), device="cuda", dtype=torch.int32, generator=g)
    dec = _lib.DecideArgs(rows, 3, _lib.ptr(last), _lib.ptr(opt), _lib.ptr(nopt), _lib.ptr(kinds), _lib.ptr(temps),
                          0.0, *[_lib.ptr(t) for t in outs], None)
    dec_ptr = _lib.DecideArgs(rows, 3, _lib.ptr(last), _lib.ptr(opt), _lib.ptr(nopt), _lib.ptr(kinds), _lib.ptr(temps),
                              0.0, *[_lib.ptr(t) for t in outs], _lib.ptr(opt_tok))
    head = DeviceReadout("pointer", synth.readout_params("pointer", H, 256, seed=1), H)
    hs = head.struct()
    wlat = torch.randn(2 * spec.inter, H, device="cuda", generator=g) * 0.02
    pw = WT.quantize("nvfp4", wlat)
    qw = pw.qweight()
    wbf = torch.empty(2 * spec.inter, H, dtype=torch.bfloat16, device="cuda")
    qd = torch.empty_like(pw.data)
    qs = torch.empty_like(pw.scales)
    qr = torch.empty_like(pw.row_scale)
    keep = (table, ids, x, w_norm, planes, last, opt, nopt, kinds, temps, outs, opt_tok, head, pw, wbf, qd, qs, qr)
    st = _lib.stream_ptr()

    def launch():
        k = keep
        _lib.call("b200_embed", _lib.ptr(k[1]), tokens, _lib.ptr(k[0]), H, _lib.ptr(k[2]), st)
        _lib.call("b200_rmsnorm", _lib.ptr(k[2]), tokens, H, _lib.ptr(k[3]), 1e-6, _lib.ptr(k[4]), tokens * H, st)
        _lib.call("b200_rmsnorm_lo8", _lib.ptr(k[2]), tokens, H, _lib.ptr(k[3]), 1e-6, _lib.ptr(k[4]), tokens * H, st)
        _lib.call("b200_decide", _lib.ptr(k[2]), H, _lib.ptr(k[3]), 1e-6, _lib.ptr(k[0]), C.byref(dec), st)
        _lib.call("b200_decide_readout", _lib.ptr(k[2]), H, _lib.ptr(k[3]), 1e-6, C.byref(hs), C.byref(dec_ptr), tokens,
                  st)
        _lib.call("b200_dequantize", C.byref(qw), _lib.ptr(k[14]), st)
        _lib.call("b200_quantize", _lib.FMT["nvfp4"], _lib.ptr(wlat), 2 * spec.inter, H, _lib.ptr(k[15]),
                  _lib.ptr(k[16]), _lib.ptr(k[17]), st)

    return launch, None


def run_case(args) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("--case needs a CUDA device")
    _lib.load()
    if args.case == "small":
        launch, flops = small_kernels_case()
        label = "embed, rmsnorm (bf16 / e4m3 low plane), decide, pointer readout, dequantise, quantise (2B shapes)"
    elif args.case == "gemm":
        launch, flops = gemm_case(args.m, args.fmt, args.ep, args.n, args.k, args.planes)
        label = f"gemm {args.fmt} {args.ep} {args.planes} M={args.m} N={args.n} K={args.k}"
    elif args.case == "gdn":
        launch, flops = gdn_case(args.seqs, args.len, scan=args.scan, prefix=args.prefix)
        label = (f"gdn {args.seqs} x {args.len} tokens, 16 heads (prep + {args.scan} scan"
                 f"{', prefix ' + args.prefix if args.prefix else ''})")
    else:
        launch, flops = attention_case(args.seqs, args.len)
        label = f"attention {args.seqs} x {args.len} tokens (prep + flash kernels)"
    ms = _case_time(launch, args.reps)
    rate = f", {flops / ms / 1e9:.1f} TFLOP/s algorithmic" if flops else ""
    print(f"{label}: {ms * 1e3:.1f} us per call{rate}", flush=True)
    _case_profiled(launch)


# ----------------------------------------------------------------------------- int4 GEMM microbench
C2_SHAPES = [(m, n) for n in (6144, 2048) for m in (1, 16, 256, 4096)]
C2_K = 2048


def c2_gemm(pk: dict, reps: int = 50, check: bool = True) -> list[dict]:
    """The int4 weight-only GEMM microbench: y = x @ dequant(W)^T, W N(0, 0.02) [N, 2048]
    quantised to int4 g128 (bf16 scales, 8 nibbles per int32), x bf16 N(0, 1) [M, 2048] (one
    bf16 plane: the activations are bf16), y fp32, for M in {1, 16, 256, 4096} and N in
    {6144, 2048}. Each shape launches `reps` times back to back through b200_linear, each launch
    on a different copy of the weight (the copies together exceed twice the 126 MB L2, so every
    launch streams its weight from HBM); time per launch = CUDA-event time / reps.

    At M = 4096 the time is that of the runtime's path for batches of 4096 tokens or more (the
    packed weight dequantised once per call into a bf16 copy, then the bf16-weight GEMM), with the
    one-kernel packed path's time beside it.

    roofline: bytes = N K / 2 (codes) + N K / 64 (bf16 scale per 128) + 2 M K (x) + 4 M N (y);
    flops = 2 M N K; bound time = max(bytes / measured HBM copy bandwidth, flops / measured bf16
    GEMM peak); frac = bound time / measured time. Parity: y against an fp64 product of x and the
    oracle's dequantisation of the packed bytes (read back), as the largest error relative to
    max |y| (up to 256 rows checked)."""
    import numpy as np

    from oracle import quant as OQ
    from strands_decider_b200.weights import packed_to_numpy

    torch.cuda.set_device(0)
    st = torch.cuda.current_stream()
    out = []
    for n in sorted({n for _, n in C2_SHAPES}, reverse=True):
        g = torch.Generator(device="cuda").manual_seed(n)
        base = WT.quantize("int4", torch.randn(n, C2_K, device="cuda", generator=g) * 0.02)
        base.ensure_tiles()
        per_copy = base.tiles.numel() + base.tile_scales.numel()
        copies = [base] + [WT.PackedWeight("int4", n, C2_K, base.data, base.scales, None, base.tiles.clone(),
                                           base.tile_scales.clone())
                           for _ in range(max(1, int(2 * 126e6 * 1.2 // per_copy)))]
        qws = [c.qweight() for c in copies]
        w64 = torch.from_numpy(OQ.dequantize("int4", packed_to_numpy(base)).astype(np.float64)) if check else None
        for m, nn in C2_SHAPES:
            if nn != n:
                continue
            x = torch.randn(m, C2_K, device="cuda", generator=g).to(torch.bfloat16)
            y = torch.empty(m, n, device="cuda")
            o = _lib.LinearOut(_lib.EP_STORE, n, _lib.ptr(y), n, 0)

            def launch(i, stream):
                _lib.call("b200_linear", _lib.ptr(x), None, m, C2_K, C2_K, C.byref(qws[i % len(qws)]), C.byref(o),
                          stream.cuda_stream)

            for i in range(3):
                launch(i, st)
            torch.cuda.synchronize()
            # the reps launches replay as one CUDA graph, as the forward runs its GEMMs: the time
            # is the device's, not the host's launch rate
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                cs = torch.cuda.current_stream()
                for i in range(reps):
                    launch(3 + i, cs)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            graph.replay()
            e1.record(st)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            del graph
            us_dq = None
            if m >= 4096:
                # the runtime's path at this size: the packed weight dequantised once into a bf16
                # copy (b200_dequantize), then the bf16-weight GEMM (CTA pairs)
                wbf = torch.empty(n, C2_K, dtype=torch.bfloat16, device="cuda")
                qb = _lib.QWeight()
                qb.format, qb.n, qb.k, qb.data = _lib.FMT["bf16"], n, C2_K, _lib.ptr(wbf)

                def launch_dq(i, stream):
                    _lib.call("b200_dequantize", C.byref(qws[i % len(qws)]), _lib.ptr(wbf), stream.cuda_stream)
                    _lib.call("b200_linear", _lib.ptr(x), None, m, C2_K, C2_K, C.byref(qb), C.byref(o),
                              stream.cuda_stream)

                for i in range(3):
                    launch_dq(i, st)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    cs = torch.cuda.current_stream()
                    for i in range(reps):
                        launch_dq(3 + i, cs)
                graph.replay()
                torch.cuda.synchronize()
                e0.record(st)
                graph.replay()
                e1.record(st)
                torch.cuda.synchronize()
                us_dq = e0.elapsed_time(e1) / reps * 1e3
                del graph
            nbytes = n * C2_K // 2 + n * C2_K // 64 + 2 * m * C2_K + 4 * m * n
            flops = 2.0 * m * n * C2_K
            t_hbm = nbytes / (pk["hbm_gbs"] * 1e9) * 1e6
            t_mma = flops / (pk["bf16_tflops"] * 1e12) * 1e6
            path = ("dequantised once + bf16 GEMM" if us_dq is not None else
                    "weights streamed through registers (<= 16 rows)" if m <= 16 else "packed tiles unpacked in the GEMM")
            us_best = us if us_dq is None else us_dq
            rec = {"m": m, "n": n, "k": C2_K, "us": round(us_best, 3), "path": path,
                   "gbs": round(nbytes / us_best / 1e3, 1), "tflops": round(flops / us_best / 1e6, 1),
                   "bound": "hbm" if t_hbm >= t_mma else "tensor", "roofline_us": round(max(t_hbm, t_mma), 3),
                   "frac": round(max(t_hbm, t_mma) / us_best, 3)}
            if us_dq is not None:
                rec["us_packed_path"] = round(us, 3)
            if check:
                if us_dq is not None:
                    launch_dq(0, st)
                else:
                    launch(0, st)
                rows = min(m, 256)
                ref = x[:rows].double().cpu() @ w64.T
                got = y[:rows].double().cpu()
                rec["max_rel_err"] = float((got - ref).abs().max() / ref.abs().max())
            out.append(rec)
        del copies, qws
        torch.cuda.empty_cache()
    assert _lib.read_fault() == 0
    return out


def c2_native_fp4(pk: dict, reps: int = 50) -> list[dict]:
    """The native NVFP4 (W4A4) GEMM at the microbench's shapes: W the same N(0, 0.02) latent
    quantised to NVFP4, x bf16 N(0, 1) quantised to NVFP4 activations (b200_quantize_act_nvfp4,
    timed apart), y fp32, b200_linear_nvfp4_native, 50 launches on rotating weight copies in one
    CUDA graph. The tensor bound is taken at 4 x the measured bf16 GEMM peak (the dense e2m1 :
    bf16 tensor-rate ratio, 9 : 2.25 PFLOP/s nominal)."""
    torch.cuda.set_device(0)
    st = torch.cuda.current_stream()
    fp4_peak = 4 * pk["bf16_tflops"]
    out = []

    def gtime(fn):
        for i in range(3):
            fn(i, st)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for i in range(reps):
                fn(3 + i, cs)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    for n in sorted({n for _, n in C2_SHAPES}, reverse=True):
        g = torch.Generator(device="cuda").manual_seed(n)
        base = WT.quantize("nvfp4", torch.randn(n, C2_K, device="cuda", generator=g) * 0.02)
        nb = C.c_size_t()
        _lib.check(_lib.load().b200_nvfp4_sf_atom_bytes(n, C2_K, C.byref(nb)))
        atoms = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        _lib.call("b200_nvfp4_sf_atoms", _lib.ptr(base.scales), n, C2_K, _lib.ptr(atoms), st.cuda_stream)
        per_copy = base.data.numel() + atoms.numel()
        ncop = max(1, int(2 * 126e6 * 1.2 // per_copy))
        copies = [(WT.PackedWeight("nvfp4", n, C2_K, base.data.clone(), base.scales, base.row_scale), atoms.clone())
                  for _ in range(ncop)]
        qws = [(c.qweight(), a) for c, a in copies]
        for m, nn in C2_SHAPES:
            if nn != n:
                continue
            x = torch.randn(m, C2_K, device="cuda", generator=g).to(torch.bfloat16).float()
            codes = torch.empty(m, C2_K // 2, dtype=torch.uint8, device="cuda")
            _lib.check(_lib.load().b200_nvfp4_sf_atom_bytes(m, C2_K, C.byref(nb)))
            xsf = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
            y = torch.empty(m, n, device="cuda")
            o = _lib.LinearOut(_lib.EP_STORE, n, _lib.ptr(y), n, 0, 0)

            def quant(i, stream):
                _lib.call("b200_quantize_act_nvfp4", _lib.ptr(x), m, C2_K, C2_K, _lib.ptr(codes), _lib.ptr(xsf),
                          stream.cuda_stream)

            def gemm(i, stream):
                qw, wa = qws[i % len(qws)]
                _lib.call("b200_linear_nvfp4_native", _lib.ptr(codes), _lib.ptr(xsf), m, C2_K, C.byref(qw),
                          _lib.ptr(wa), C.byref(o), stream.cuda_stream)

            quant(0, st)
            us_q, us = gtime(quant), gtime(gemm)
            nbytes = n * C2_K // 2 + n * C2_K // 16 + m * C2_K // 2 + m * C2_K // 16 + 4 * m * n
            flops = 2.0 * m * n * C2_K
            t_hbm = nbytes / (pk["hbm_gbs"] * 1e9) * 1e6
            t_mma = flops / (fp4_peak * 1e12) * 1e6
            out.append({"m": m, "n": n, "us": round(us, 3), "us_act_quant": round(us_q, 3),
                        "tflops": round(flops / us / 1e6, 1), "bound": "hbm" if t_hbm >= t_mma else "tensor",
                        "roofline_us": round(max(t_hbm, t_mma), 3), "frac": round(max(t_hbm, t_mma) / us, 3)})
        del copies, qws
        torch.cuda.empty_cache()
    assert _lib.read_fault() == 0
    return out


def c2_main(args) -> None:
    pk = peaks()
    shapes = c2_gemm(pk, reps=max(args.steps, 20))
    worst = min(r["frac"] for r in shapes)
    line = {"metric": "int4 g128 weight-only GEMM time per launch (K=2048)", "value": round(worst, 3),
            "unit": "min roofline fraction over shapes", "n_gpus": 1, "higher_is_better": True,
            "dtype": "bf16 x int4", "data": "synthetic",
            "config": {"workload": "int4-gemm-microbench", "k": C2_K, "m": [1, 16, 256, 4096], "n": [6144, 2048],
                       "l2": "weight copies rotated per launch (together > 2 x L2)",
                       "peaks": f"{pk['src']}: HBM {pk['hbm_gbs']} GB/s, bf16 {pk['bf16_tflops']} TFLOP/s"},
            "shapes": shapes,
            "nvfp4_native": {"what": "W4A4 on the block-scaled tensor cores (kind::mxf4nvf4); activations "
                                     "quantised to NVFP4 first (us_act_quant); not the runtime's path (4-bit "
                                     "activations move the decider's probabilities by up to 0.5)",
                             "peak_tflops": 4 * pk["bf16_tflops"], "shapes": c2_native_fp4(pk, reps=max(args.steps, 20))}}
    print(json.dumps(line), flush=True)


WORKLOADS = {
    "nvfp4": (config.HYBRID_2B, config.HYBRID_2B_WORKLOAD, 128, True),
    "prefix": (config.HYBRID_2B, config.PREFIX_CACHE_WORKLOAD, 32, True),
    "ternary-batch": (config.HYBRID_2B.with_format("ternary"),
                      dataclasses.replace(config.LATENCY_WORKLOAD, name="hybrid-2b-ternary-4096x96", n_requests=4096),
                      1024, False),
}


def _kmax(wl: config.Workload) -> int:
    return wl.option_range[1] if wl.option_range else max(wl.options)


def other_workload(name: str, steps: int = 3, warmup: int = 3, cpu_sample: int = 3) -> dict:
    """One more workload's line, measured in a child process of this run (its own model, CUDA
    graphs, timed region, clocks, CPU baseline and parity), summarised for the default line so
    that every configuration's number comes out of the same command."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE")}
    cmd = [sys.executable, os.path.abspath(__file__), "--workload", name, "--steps", str(steps), "--warmup",
           str(warmup), "--cpu-sample", str(cpu_sample), "--no-extras"]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env, cwd=ROOT)
    except subprocess.TimeoutExpired:
        return {"workload": name, "error": "timed out after 900 s"}
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"workload": name, "error": f"exit {r.returncode}: {r.stderr.strip()[-300:]}"}
    d = json.loads(lines[-1])
    cb = d.get("cpu_baseline") or {}
    return {"workload": d["config"]["workload"], "value": d["value"], "unit": d["unit"], "steps": d["steps"],
            "warmup": d["warmup"], "ms_per_step": d["ms_per_step"], "e2e": d["e2e"]["value"],
            "decisions_per_step": d["config"]["decisions_per_step"], "tokens_per_step": d["config"]["tokens_per_step"],
            "path": d["config"]["path"], "gpu_launches": d["gpu_launches"], "clocks": d["clocks"],
            "parity": d.get("parity"), "cpu_baseline": {k: cb.get(k) for k in ("value", "cores", "kind", "sample")}}


def latency(args, emit: bool = True, cpu: bool = True) -> dict:
    """p50 / p99 single-request latency: one 96-token request (93-token state + 3-token
    question, one 3-way choice) as one full-prompt forward of the ternary 2B-shape decider,
    CUDA-graphed, each replay timed alone with CUDA events (inputs resident; e2e adds the
    96 ids' upload and the answer's download to every replay). Returns the JSON line (printed
    when emit); cpu=False leaves out the CPU baseline."""
    from strands_decider_b200 import _lib
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.synth import request_batch
    from strands_decider_b200.weights import DeviceWeights

    spec, wl = config.HYBRID_2B.with_format("ternary"), config.LATENCY_WORKLOAD
    torch.cuda.set_device(0)
    weights = DeviceWeights.synthetic(spec, seed=0, device="cuda", latent_device="cuda")
    model = DecisionModel(weights, max_tokens=128, pool_slots=1, pool_kv_tokens=128, lo_plane=args.lo_plane)
    reqs = request_batch(wl, spec.vocab, 0, 1)
    reqs[0]["id"] = 0
    b = Batch(reqs, "cuda", pinned=True, kmax=3, prefix=False)
    g = StepGraph(model, b)
    runs = max(args.steps, 1000)
    for _ in range(max(args.warmup, 20)):
        g.replay()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()    # a profiler started with capture off records this one replay
    g.replay()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
    clocks = ClockSampler(0)
    clocks.start()
    for e0, e1 in ev:
        e0.record(st)
        g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    ms = sorted(e0.elapsed_time(e1) for e0, e1 in ev)
    out_host = torch.empty(b.n_decisions, 3, pin_memory=True)
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
    for e0, e1 in ev2:
        e0.record(st)
        b.upload()
        dec = g.replay()
        out_host.copy_(dec.probs, non_blocking=True)
        e1.record(st)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms2 = sorted(e0.elapsed_time(e1) for e0, e1 in ev2)
    assert _lib.read_fault() == 0

    def pct(v, q):
        return v[min(len(v) - 1, int(q * len(v)))]

    cb = cpu_baseline(spec, wl, 1, full_prompt=True) if (cpu and args.cpu_sample > 0) else None
    if cb:
        cb.pop("_probs")
    # Latency roofline: the forward must stream every linear's ternary weights (2 bits each) from
    # HBM once; its algorithmic FLOPs (2 x params x tokens) at the bf16 peak are the other bound.
    pk = peaks()
    p50 = pct(ms, 0.5)
    wbytes = spec.linear_params() * 0.25
    flops = 2.0 * spec.linear_params() * b.tokens
    roof = {"bound": "hbm", "achieved": round(wbytes / (p50 * 1e-3) / 1e9, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(wbytes / (p50 * 1e-3) / 1e9 / pk["hbm_gbs"], 4), "traffic": None,
            "kernel": "whole forward: every linear's packed weights streamed once",
            "hbm_bound_ms": round(wbytes / (pk["hbm_gbs"] * 1e9) * 1e3, 4),
            "mma_bound_ms": round(flops / (pk["bf16_tflops"] * 1e12) * 1e3, 4),
            "peak_src": pk["src"] + " copy bandwidth"}
    line = {"metric": METRIC, "value": round(pct(ms, 0.5), 4), "unit": "ms", "n_gpus": 1, "steps": runs,
            "warmup": max(args.warmup, 20), "ms_per_step": round(statistics.mean(ms), 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": wl.name, "model": spec.name, "weights": "ternary", "tokens": b.tokens, "lo_plane": args.lo_plane,
                       "path": "full prompt, one CUDA graph per request",
                       "l2": "weights (0.34 GB ternary + 1 GB embedding) exceed L2; no flush between replays"},
            "latency_ms": {"p50": round(pct(ms, 0.5), 4), "p99": round(pct(ms, 0.99), 4),
                           "min": round(ms[0], 4), "runs": runs},
            "e2e": {"value": round(pct(ms2, 0.5), 4), "unit": "ms", "p99": round(pct(ms2, 0.99), 4),
                    "h2d_bytes_per_step": b.h2d_bytes, "d2h_bytes_per_step": out_host.numel() * 4},
            "gpu_launches": runs * launches_per_forward(spec, True, b.tokens), "roofline": roof, "clocks": clk,
            "cpu_baseline": cb}
    if cb:
        cb["ms_per_request"] = round(1e3 / cb["value"], 1)
    if emit:
        print(json.dumps(line), flush=True)
    del g, model, weights
    torch.cuda.empty_cache()
    return line


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="nvfp4", choices=sorted(WORKLOADS) + ["latency", "gemm"])
    ap.add_argument("--requests-per-step", type=int, default=0, help="0 = the workload's default")
    ap.add_argument("--cpu-sample", type=int, default=3, help="requests in the CPU baseline sample (0 = skip)")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying CUDA graphs")
    ap.add_argument("--extras", action=argparse.BooleanOptionalAction, default=True,
                    help="one GPU, default workload: add the int4 GEMM microbench summary and the "
                         "single-request latency to the line")
    ap.add_argument("--lo-plane", default="e4m3", choices=["bf16", "e4m3"],
                    help="low activation plane of the large-batch GEMMs (DecisionModel lo_plane)")
    ap.add_argument("--case", choices=["gemm", "gdn", "attention", "small"],
                    help="time (and profile) one kernel alone (small: the head, norm, embedding and (de)quantisers)")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--fmt", default="nvfp4", choices=list(config.WEIGHT_FORMATS))
    ap.add_argument("--ep", default="swiglu", choices=["swiglu", "store", "resid"])
    ap.add_argument("--n", type=int, default=2 * 6144)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--planes", default="split", choices=["split", "lo8", "one"],
                    help="gemm case: activation planes (two bf16, bf16 + e4m3, or one bf16 plane)")
    ap.add_argument("--seqs", type=int, default=32)
    ap.add_argument("--len", type=int, default=512)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--scan", default="auto", choices=sorted(GDN_ENTRY))
    ap.add_argument("--prefix", default="", choices=["", "read", "append"],
                    help="gdn case: sequences start from (read) or continue and save (append) pool slots")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.workload == "gemm":
        c2_main(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "latency":
        if args.impl == "reference":
            if rank == 0:
                spec, wl = config.HYBRID_2B.with_format("ternary"), config.LATENCY_WORKLOAD
                cb = cpu_baseline(spec, wl, 1, full_prompt=True)
                cb.pop("_probs")
                ms = 1e3 / cb["value"]
                print(json.dumps({"metric": METRIC, "value": round(ms, 2), "unit": "ms", "impl": "reference",
                                  "higher_is_better": False, "config": {"workload": wl.name, "model": spec.name},
                                  "cpu_baseline": cb, "e2e": {"value": round(ms, 2), "unit": "ms",
                                                              "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
            return
        if rank == 0:
            latency(args)
        return
    spec, wl, r_default, prefix = WORKLOADS[args.workload]
    R = args.requests_per_step or r_default
    kmax = _kmax(wl)

    if args.impl == "reference":
        if rank != 0:
            return
        n_q = None if wl.n_questions <= 3 else 4
        cb = cpu_baseline(spec, wl, max(args.cpu_sample, 1), n_questions=n_q, full_prompt=not prefix)
        cb.pop("_probs")
        line = {"metric": METRIC, "value": round(cb["value"], 4), "unit": UNIT, "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": {"workload": wl.name, "model": spec.name},
                "cpu_baseline": cb, "e2e": {"value": round(cb["value"], 4), "unit": UNIT,
                                            "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch.distributed as dist

    from strands_decider_b200 import _lib, dispatch
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.synth import request_batch
    from strands_decider_b200.weights import DeviceWeights

    torch.cuda.set_device(local)
    extras = {}
    if world == 1 and args.extras and args.workload == "nvfp4":
        # the int4 GEMM microbench first, on a GPU that has not just run the power-capped main
        # workload (its small launches follow the SM clock), with the clocks it ran at
        csamp = ClockSampler(local)
        csamp.start()
        extras["c2_gemm"] = [{k: r[k] for k in ("m", "n", "us", "bound", "roofline_us", "frac", "path")}
                             for r in c2_gemm(peaks(), reps=30, check=False)]
        extras["c2_gemm_clocks"] = csamp.stop()
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    # every rank holds the whole workload's request list and plans the same LPT shards;
    # rank r forwards shards[r] in batches of R requests (weak scaling: each rank's share
    # is the full single-GPU workload, so N GPUs answer N times the questions)
    n_total = wl.n_requests * world
    need = (args.steps + args.warmup) * R
    reqs_all = request_batch(wl, spec.vocab, 0, min(n_total, need * world))
    for i, r in enumerate(reqs_all):
        r["id"] = i
    shards = dispatch.plan_shards([dispatch.request_cost(r) for r in reqs_all], world)
    mine = [reqs_all[i] for i in shards[rank]]
    n_batches = max(1, min(len(mine) // R, args.steps + args.warmup))
    batches = [Batch(mine[j * R:(j + 1) * R], "cuda", pinned=True, kmax=kmax, prefix=prefix)
               for j in range(n_batches)]
    max_tok = max(max(b.n_state_tokens, b.n_suffix_tokens) for b in batches)
    slots = R if prefix else 1
    kv = max(b.n_state_tokens for b in batches) if prefix else 1
    parity = world == 1 and args.cpu_sample > 0
    weights = DeviceWeights.synthetic(spec, seed=0, device="cuda", latent_device="cuda", keep_logical=parity)
    model = DecisionModel(weights, max_tokens=max_tok, pool_slots=slots, pool_kv_tokens=max(kv, 1),
                          lo_plane=args.lo_plane, graphs=False)
    stream = torch.cuda.current_stream()
    use_graph = not args.no_graph
    graphs = [StepGraph(model, b) for b in batches] if use_graph else None

    cap = R * wl.n_questions

    def step(i, upload=False):
        j = i % len(batches)
        b = batches[j]
        if upload:
            b.upload()
        dec = graphs[j].replay() if use_graph else run_step(model, b, stream)
        rec = records(dec, b)
        # every batch of every rank holds R requests: one fixed-size all-gather, no host sync
        out = dispatch.gather_answers(rec, cap, total=world * cap) if world > 1 else rec.rows
        return b, out

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0

    # timed: inputs resident in HBM
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.cudart().cudaProfilerStart()    # a profiler started with capture off records this region only
    e0.record(stream)
    decisions = 0
    tokens = 0
    for i in range(args.steps):
        b, _ = step(args.warmup + i)
        decisions += b.n_decisions
        tokens += b.tokens
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    ms = e0.elapsed_time(e1)

    # e2e: host inputs uploaded and the gathered answers read back every step
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    d2h = 0
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    h2d = 0
    for i in range(args.steps):
        b, out = step(args.warmup + i, upload=True)
        host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        host.copy_(out, non_blocking=True)
        d2h += out.numel() * 4
        h2d += b.h2d_bytes
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    clk = clocks.stop()

    # the timed graphs' last answers for the first batch (its first requests are the CPU sample's)
    b0_probs = (graphs[0].out.probs if use_graph else run_step(model, batches[0], stream).probs).cpu()
    t = torch.tensor([ms, ms_e2e, float(decisions), float(tokens)], device="cuda")
    per_rank = None
    if world > 1:
        g = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(g, t)
        ms = max(float(x[0]) for x in g)
        ms_e2e = max(float(x[1]) for x in g)
        total = sum(float(x[2]) for x in g)
        total_tok = sum(float(x[3]) for x in g)
        # each rank's own device time and work per step: the LPT shards' balance
        per_rank = [{"rank": r, "ms_per_step": round(float(x[0]) / args.steps, 3),
                     "tokens_per_step": int(float(x[3]) / args.steps),
                     "decisions_per_step": int(float(x[2]) / args.steps)} for r, x in enumerate(g)]
    else:
        total, total_tok = float(decisions), float(tokens)
    value = total / (ms * 1e-3)
    e2e = total / (ms_e2e * 1e-3)
    pk = peaks()
    del graphs
    roof = gemm_roofline(model, batches[0].n_state_tokens or batches[0].n_suffix_tokens, pk) if rank == 0 else None
    assert _lib.read_fault() == 0
    if world == 1 and args.extras and args.workload == "nvfp4":
        # the single-request latency, measured in the same run
        lat = latency(args, emit=False, cpu=False)
        extras["latency"] = {"workload": lat["config"]["workload"], "p50_ms": lat["latency_ms"]["p50"],
                             "p99_ms": lat["latency_ms"]["p99"], "e2e_p50_ms": lat["e2e"]["value"],
                             "roofline": {k: lat["roofline"][k] for k in ("bound", "frac", "hbm_bound_ms",
                                                                           "mma_bound_ms")},
                             "clocks": lat["clocks"]}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cb, par = None, None
    if parity:
        from oracle import synth as osynth

        W = osynth.device_logical_weights(weights, seed=0)
        del model, weights
        torch.cuda.empty_cache()
        n_q = None if wl.n_questions <= 3 else 4
        cb = cpu_baseline(spec, wl, args.cpu_sample, n_questions=n_q, full_prompt=not prefix, W=W)
        del W
        sample = [r for r in reqs_all[: args.cpu_sample]]
        assert all(r["id"] == i for i, r in enumerate(sample)) and batches[0].prefix == prefix
        rows = [i * wl.n_questions + q for i in range(len(sample)) for q in range(n_q or wl.n_questions)]
        assert shards[0][: len(sample)] == list(range(len(sample)))   # batch 0 starts with the sample
        par = parity_check(b0_probs[rows], cb.pop("_probs"),
                           [r["n_opts"][q] for r in sample for q in range(n_q or wl.n_questions)])
    if world == 1 and args.extras and args.workload == "nvfp4":
        # the prefix-cache workload (512 x U[64, 2048] + 32 x 48) and the 4096 x 96 ternary batch,
        # each a few steps in a child process
        extras["prefix_cache"] = other_workload("prefix")
        extras["ternary_batch"] = other_workload("ternary-batch")
    b0 = batches[0]
    fl = 2.0 * spec.linear_params() * total_tok
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": wl.name, "model": spec.name, "weights": spec.weight_format,
                   "requests_per_step": R, "decisions_per_step": b0.n_decisions,
                   "tokens_per_step": b0.tokens, "question_tokens": wl.question_len,
                   "path": "prefix cache (state once, questions against its pool slot)" if prefix else "full prompts",
                   "cuda_graphs": use_graph, "lo_plane": args.lo_plane,
                   "l2": "inputs larger than L2 (0.8 GB weights + GBs of activations per step)",
                   "parallelism": f"dp{world} (requests LPT-sharded, answers all-gathered over NCCL)"},
        "linear_tflops": round(fl / (ms * 1e-3) / 1e12 / world, 1),
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        "gpu_launches": sum(((launches_per_forward(spec, False, b.n_state_tokens, True, args.lo_plane) if prefix else 0)
                             + launches_per_forward(spec, True, b.n_suffix_tokens, lo_plane=args.lo_plane))
                            for b in (batches[(args.warmup + i) % len(batches)] for i in range(args.steps))) * world,
        "roofline": roof, "clocks": clk, "cpu_baseline": cb, "parity": par, **extras,
    }
    if per_rank:
        line["per_rank"] = per_rank
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
