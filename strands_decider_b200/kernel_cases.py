"""Standalone launches of the hot kernels at the 2B shape, for timing and profiling.

    python -m strands_decider_b200.kernel_cases gemm [--m 8192] [--fmt nvfp4] [--ep swiglu] [--planes split]
    python -m strands_decider_b200.kernel_cases gdn [--seqs 32] [--len 512] [--scan auto|chunked|recurrent] [--prefix read|append]
    python -m strands_decider_b200.kernel_cases attention [--seqs 1] [--len 96]

Each case builds seeded synthetic operands on cuda:0, runs a few warm-up launches, prints
the CUDA-event time per launch, then runs ONE more launch between cudaProfilerStart and
cudaProfilerStop, so a profiler started with capture off (`ncu --profile-from-start off`)
records exactly that launch.

Shapes: the gate/up projection (N = 2 x 6144, K = 2048) or another linear of the 2B
decider; the GDN token mixer (16 heads x 128) over `seqs` sequences of `len` tokens; the
gated attention layer (8 query / 2 kv heads x 256) over `seqs` sequences of `len` tokens.
"""

from __future__ import annotations

import argparse
import ctypes as C

import torch

from . import _lib, config
from . import weights as W


def _time(fn, reps: int) -> float:
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


def _profiled(fn) -> None:
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
        gate = W.quantize(fmt, torch.randn(n // 2, k, device="cuda", generator=g) * 0.02)
        up = W.quantize(fmt, torch.randn(n // 2, k, device="cuda", generator=g) * 0.02)
        pw = W.interleave_gate_up(gate, up)
    else:
        pw = W.concat_rows([W.quantize(fmt, torch.randn(n, k, device="cuda", generator=g) * 0.02)])
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
        _lib.call("b200_linear", _lib.ptr(keep[1][0]), _lib.ptr(keep[1][1]), m, k, k, C.byref(qw), C.byref(o),
                  _lib.stream_ptr())

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
    from .runtime import rope_tables

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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "gdn", "attention"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--fmt", default="nvfp4", choices=list(config.WEIGHT_FORMATS))
    ap.add_argument("--ep", default="swiglu", choices=["swiglu", "store", "resid"])
    ap.add_argument("--n", type=int, default=2 * 6144)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--planes", default="split", choices=["split", "lo8"])
    ap.add_argument("--seqs", type=int, default=32)
    ap.add_argument("--len", type=int, default=512)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--scan", default="auto", choices=sorted(GDN_ENTRY))
    ap.add_argument("--prefix", default="", choices=["", "read", "append"],
                    help="gdn: sequences start from (read) or continue and save (append) pool slots")
    args = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("kernel_cases needs a CUDA device")
    _lib.load()
    if args.case == "gemm":
        launch, flops = gemm_case(args.m, args.fmt, args.ep, args.n, args.k, args.planes)
        label = f"gemm {args.fmt} {args.ep} {args.planes} M={args.m} N={args.n} K={args.k}"
    elif args.case == "gdn":
        launch, flops = gdn_case(args.seqs, args.len, scan=args.scan, prefix=args.prefix)
        label = (f"gdn {args.seqs} x {args.len} tokens, 16 heads (prep + {args.scan} scan"
                 f"{', prefix ' + args.prefix if args.prefix else ''})")
    else:
        launch, flops = attention_case(args.seqs, args.len)
        label = f"attention {args.seqs} x {args.len} tokens (prep + flash kernels)"
    ms = _time(launch, args.reps)
    rate = f", {flops / ms / 1e9:.1f} TFLOP/s algorithmic" if flops else ""
    print(f"{label}: {ms * 1e3:.1f} us per call{rate}", flush=True)
    _profiled(launch)


if __name__ == "__main__":
    main()
