"""Decisions/s of the batched scoring prefill on B200 (the hybrid-2B NVFP4 workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (one GPU): the 2B-shape hybrid decider (hidden 2048, 24 layers at 3:1
GDN:attention, GDN 16 heads x 128, attention 8q/2kv x 256, FFN 6144, vocab 248320 tied)
with NVFP4 weights; 1024 requests of 512 uniform-random tokens, each with 3 questions
(3-way choice, yes/no noul, 3-level score) of 32 tokens. A step is one batch of
--requests-per-step requests through the prefix-cache path: every state is forwarded once
into a pool slot, then all question suffixes are forwarded against their slots and decided
by the fused head. Data are synthetic (seeded), weights random-init.

Under torchrun (N > 1) every rank takes its own requests (weak scaling, no collective in the
forward) and the per-step answer records are all-gathered over NCCL.
"""

from __future__ import annotations

import argparse
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

from strands_decider_b200 import config  # noqa: E402

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
        self.index = index
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


def cpu_baseline(spec: config.ModelSpec, n_requests: int = 1) -> dict:
    """The CPU oracle (a restatement of the reference's torso and readout) on a bounded
    sample of the same workload: n_requests requests through the prefix-cache path,
    fp32, all host threads. Weights are fp32 tensors of the same shapes (the per-token
    arithmetic does not depend on their values)."""
    from oracle import head as OH
    from oracle import synth as osynth
    from oracle import torso as OT
    from strands_decider_b200 import synth

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = osynth.torso_config(spec)
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
    reqs = synth.request_batch(config.HYBRID_2B_WORKLOAD, spec.vocab, 0, n_requests)
    decisions = 0
    t0 = time.perf_counter()
    with torch.inference_mode():
        for r in reqs:
            _, cache = OT.forward_sequence(cfg, W, torch.tensor(r["state"]), keep_cache=True)
            for qi, q in enumerate(r["questions"]):
                hid, _ = OT.forward_sequence(cfg, W, torch.tensor(q), cache=cache)
                n = r["n_opts"][qi]
                OH.decide(hid[-1:], W["embed"], torch.tensor([r["opt_ids"][qi]]), torch.tensor([n]),
                          torch.tensor([1.0]))
                decisions += 1
    dt = time.perf_counter() - t0
    return {"value": decisions / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n_requests} request(s) x (512-token state + 3 x 32-token questions), prefix-cache path, "
                      f"fp32 torch on {cores} threads, {dt:.1f} s"}


# ----------------------------------------------------------------------------- GPU arm


def launches_per_forward(spec: config.ModelSpec, decide: bool) -> int:
    n = 1 + (1 if decide else 0)
    for lt in spec.layer_types:
        n += 2 + 4 + (1 if lt == config.GDN else 2)
    return n


class Batch:
    """One step's inputs, resident on the device (or in pinned host memory for e2e)."""

    def __init__(self, reqs: list[dict], device, pinned: bool = False):
        flat_s, cu_s, flat_q, cu_q = [], [0], [], [0]
        slots, qslots, opt, nopt, kinds = [], [], [], [], []
        for i, r in enumerate(reqs):
            flat_s += r["state"]
            cu_s.append(len(flat_s))
            slots.append(i)
            for qi, q in enumerate(r["questions"]):
                flat_q += q
                cu_q.append(len(flat_q))
                qslots.append(i)
                opt.append(r["opt_ids"][qi] + [0] * (3 - len(r["opt_ids"][qi])))
                nopt.append(r["n_opts"][qi])
                kinds.append(r["kinds"][qi])
        self.n_state_tokens, self.n_suffix_tokens = len(flat_s), len(flat_q)
        self.max_state, self.max_q = max(map(len, (r["state"] for r in reqs))), max(
            len(q) for r in reqs for q in r["questions"])
        I = torch.int32
        host = {
            "s_ids": torch.tensor(flat_s, dtype=I), "s_cu": torch.tensor(cu_s, dtype=I),
            "s_slot": torch.tensor(slots, dtype=I), "slot_kv": torch.tensor(cu_s[:-1], dtype=I),
            "q_ids": torch.tensor(flat_q, dtype=I), "q_cu": torch.tensor(cu_q, dtype=I),
            "q_slot": torch.tensor(qslots, dtype=I), "last_tok": torch.tensor([c - 1 for c in cu_q[1:]], dtype=I),
            "opt_ids": torch.tensor(opt, dtype=I), "n_opts": torch.tensor(nopt, dtype=I),
            "kinds": torch.tensor(kinds, dtype=I), "temps": torch.ones(len(nopt), dtype=torch.float32)}
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in host.values())
        if pinned:
            self.host = {k: v.pin_memory() for k, v in host.items()}
            self.dev = {k: torch.empty_like(v, device=device) for k, v in host.items()}
        else:
            self.host = None
            self.dev = {k: v.to(device) for k, v in host.items()}
        self.n_decisions = len(nopt)


def run_step(model, b: Batch, stream) -> object:
    d = b.dev
    model.slot_kv[: d["slot_kv"].numel()].copy_(d["slot_kv"], non_blocking=True)
    model.forward(d["s_ids"], d["s_cu"], save_slot=d["s_slot"], max_len=b.max_state, stream=stream)
    dec = {"last_tok": d["last_tok"], "opt_ids": d["opt_ids"], "n_opts": d["n_opts"], "kinds": d["kinds"],
           "temps": d["temps"]}
    return model.forward(d["q_ids"], d["q_cu"], prefix_slot=d["q_slot"], decide=dec, max_len=b.max_q, stream=stream)


def gemm_roofline(model, tokens: int, pk: dict, reps: int = 20) -> dict:
    """Time the dominant kernel (the gate/up projection GEMM with its SwiGLU epilogue, the
    largest GEMM of every layer) alone with CUDA events at a state-prefill batch's M.

    achieved = algorithmic FLOPs (2 M N K) / time. The activations enter as two bf16 planes
    (hi + lo, fp32-level precision), so the tensor pipe executes 2x the algorithmic FLOPs;
    frac is against the measured bf16 peak and is therefore bounded by 0.5."""
    import ctypes as C

    from strands_decider_b200 import _lib

    s = model.spec
    pw = model.w.layers[0]["gate_up"]
    xp = torch.randn(2, tokens, s.hidden, device="cuda").to(torch.bfloat16)
    out = torch.empty(2, tokens, s.inter, dtype=torch.bfloat16, device="cuda")
    o = _lib.LinearOut(_lib.EP_SWIGLU, 2 * s.inter, _lib.ptr(out), s.inter, tokens * s.inter)
    qw = pw.qweight()
    st = torch.cuda.current_stream()

    def launch():
        _lib.call("b200_linear", _lib.ptr(xp[0]), _lib.ptr(xp[1]), tokens, s.hidden, s.hidden, C.byref(qw),
                  C.byref(o), st.cuda_stream)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * tokens * (2 * s.inter) * s.hidden
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        per_tok = json.load(open(tp)).get("gate_up_dram_bytes_per_token")
        if per_tok:
            traffic = per_tok * tokens
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": traffic,
            "kernel": f"gemm_tc_kernel<256,nvfp4,swiglu,split> M={tokens} N={2 * s.inter} K={s.hidden}",
            "ms_per_launch": round(ms, 4), "mma_flops_per_algorithmic_flop": 2,
            "peak_src": pk["src"] + " bf16 burst (tcgen05 kind::f16)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--requests-per-step", type=int, default=128)
    ap.add_argument("--cpu-sample", type=int, default=1, help="requests in the CPU baseline sample (0 = skip)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    spec = config.HYBRID_2B
    wl = config.HYBRID_2B_WORKLOAD

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(spec, max(args.cpu_sample, 1))
        line = {"metric": METRIC, "value": round(cb["value"], 4), "unit": UNIT, "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": {"workload": wl.name, "model": spec.name},
                "cpu_baseline": cb, "e2e": {"value": round(cb["value"], 4), "unit": UNIT,
                                            "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch.distributed as dist

    from strands_decider_b200 import _lib
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.synth import request_batch
    from strands_decider_b200.weights import DeviceWeights

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    R = args.requests_per_step
    weights = DeviceWeights.synthetic(spec, seed=0, device="cuda", latent_device="cuda")
    model = DecisionModel(weights, max_tokens=R * wl.state_len[1], pool_slots=R, pool_kv_tokens=R * wl.state_len[1])
    # this rank's share of the workload (uniform lengths: round robin), cycled per step
    mine = list(range(rank, wl.n_requests, world))
    n_batches = max(1, len(mine) // R)
    batches, hbatches = [], []
    for b in range(min(n_batches, args.steps + args.warmup)):
        ids = mine[b * R:(b + 1) * R]
        reqs = [request_batch(wl, spec.vocab, i, 1)[0] for i in ids]
        batches.append(Batch(reqs, "cuda"))
        hbatches.append(Batch(reqs, "cuda", pinned=True))
    stream = torch.cuda.current_stream()
    gather_buf = None

    def gather(dec, n):
        nonlocal gather_buf
        if world == 1:
            return
        rec = torch.cat([dec.probs, dec.argmax.float()[:, None], dec.confidence[:, None], dec.score[:, None]], 1)
        if gather_buf is None or gather_buf.shape[1:] != rec.shape:
            gather_buf = torch.empty(world, *rec.shape, device="cuda")
        dist.all_gather_into_tensor(gather_buf, rec.contiguous())

    # warm-up
    for i in range(args.warmup):
        dec = run_step(model, batches[i % len(batches)], stream)
        gather(dec, batches[i % len(batches)].n_decisions)
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0

    # timed: inputs resident in HBM
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    decisions = 0
    for i in range(args.steps):
        b = batches[(args.warmup + i) % len(batches)]
        dec = run_step(model, b, stream)
        gather(dec, b.n_decisions)
        decisions += b.n_decisions
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()

    # e2e: through the public path with pinned host inputs, H2D + D2H every step
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    out_host = None
    d2h = 0
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(args.steps):
        b = hbatches[(args.warmup + i) % len(hbatches)]
        for k, v in b.host.items():
            b.dev[k].copy_(v, non_blocking=True)
        dec = run_step(model, b, stream)
        gather(dec, b.n_decisions)
        res = torch.cat([dec.probs, dec.argmax.float()[:, None], dec.confidence[:, None], dec.score[:, None]], 1)
        if out_host is None:
            out_host = torch.empty(res.shape, dtype=res.dtype, pin_memory=True)
        out_host.copy_(res, non_blocking=True)
        d2h = res.numel() * 4
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)

    t = torch.tensor([ms, ms_e2e, float(decisions)], device="cuda")
    if world > 1:
        g = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(g, t)
        ms = max(float(x[0]) for x in g)
        ms_e2e = max(float(x[1]) for x in g)
        total = sum(float(x[2]) for x in g)
    else:
        total = float(decisions)
    value = total / (ms * 1e-3)
    e2e = total / (ms_e2e * 1e-3)
    pk = peaks()
    roof = gemm_roofline(model, R * wl.state_len[1], pk) if rank == 0 else None
    assert _lib.read_fault() == 0
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cb = None
    if world == 1 and args.cpu_sample > 0:
        del model, weights
        torch.cuda.empty_cache()
        cb = cpu_baseline(spec, args.cpu_sample)
    b0 = batches[0]
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": wl.name, "model": spec.name, "weights": spec.weight_format,
                   "requests_per_step": R, "decisions_per_step": b0.n_decisions,
                   "tokens_per_step": b0.n_state_tokens + b0.n_suffix_tokens, "question_tokens": wl.question_len,
                   "l2": "inputs larger than L2 (0.8 GB weights + GBs of activations per step)",
                   "parallelism": f"dp{world} (requests sharded, answers all-gathered)"},
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": b0.h2d_bytes, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (launches_per_forward(spec, False) + launches_per_forward(spec, True)),
        "roofline": roof, "clocks": clk, "cpu_baseline": cb,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
