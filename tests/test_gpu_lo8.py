"""The e4m3 low activation plane (B200_LO_E4M3) on the B200.

* b200_dequantize_lo8 writes W * 2^12 in bf16 (exactly b200_dequantize's output rescaled) and
  e4m3(W * 2^6), both bit-compared with torch's round-to-nearest-even conversions.
* The plane bytes RMSNorm and the SwiGLU epilogue write decode to the fp32 activation within
  e4m3's rounding of the low term.
* b200_linear_lo8 equals an fp64 evaluation of the same bf16 / e4m3 operands (fp32
  accumulation order aside) for every epilogue, the 128- and 256-column tiles, the K split
  and an M tail, and stays within 1e-3 of the exact product x W^T.
* A whole forward on e4m3 low planes keeps the reduced decider's probabilities within 2e-3
  of the reference's golden output with the same argmax."""

from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q
from strands_decider_b200 import config
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

SHIFT, X_SHIFT, W_SHIFT = 12, 6, 6


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    from strands_decider_b200 import _lib

    _lib.load()
    assert (_lib.LO8_SHIFT, _lib.LO8_X_SHIFT, _lib.LO8_W_SHIFT) == (SHIFT, X_SHIFT, W_SHIFT)
    yield
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0, "a device-side bounded wait or index check fired"


def _weights(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    w[3] = 0.0
    w[7, 0] = 0.3
    return w


def _e4m3_bytes(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float8_e4m3fn).view(torch.uint8)


def _e4m3_values(u8: torch.Tensor) -> torch.Tensor:
    return u8.view(torch.float8_e4m3fn).double()


def _lo8_copies(fmt, n, k, seed):
    """(packed weight, w_hi bf16 [n, k], w_lo8 uint8 [n, k], plain bf16 dequant [n, k])."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    pw = W.concat_rows([W.quantize(fmt, _weights(n, k, seed).cuda())])
    qw = pw.qweight()
    plain = torch.empty(n, k, dtype=torch.bfloat16, device="cuda")
    hi = torch.empty_like(plain)
    lo8 = torch.empty(n, k, dtype=torch.uint8, device="cuda")
    _lib.call("b200_dequantize", C.byref(qw), _lib.ptr(plain), _lib.stream_ptr())
    _lib.call("b200_dequantize_lo8", C.byref(qw), _lib.ptr(hi), _lib.ptr(lo8), _lib.stream_ptr())
    torch.cuda.synchronize()
    return pw, hi, lo8, plain


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary", "bf16"])
def test_dequantize_lo8_copies_are_exact_rescalings(fmt):
    from strands_decider_b200 import weights as W

    pw, hi, lo8, plain = _lo8_copies(fmt, 256, 512, 1)
    want = Q.f32_to_bf16_bits(Q.dequantize(fmt, W.packed_to_numpy(pw)))
    assert np.array_equal(plain.view(torch.int16).cpu().numpy().view(np.uint16), want)
    assert torch.equal(hi.float(), plain.float() * 2.0 ** SHIFT)
    assert torch.equal(lo8, _e4m3_bytes(plain.float() * 2.0 ** W_SHIFT))


def _x_planes(x: torch.Tensor):
    """bf16 hi plane and e4m3 low plane of an fp32 activation, both [m, k] on the device."""
    hi = x.to(torch.bfloat16)
    return hi.cuda(), _e4m3_bytes((x - hi.float()) * 2.0 ** X_SHIFT).cuda()


def _run_lo8(xh, xl8, whi, wlo8, ep, n_valid, lo_format=0):
    from strands_decider_b200 import _lib

    m, k = xh.shape
    n = whi.shape[0]
    lo_off = 0
    if ep == _lib.EP_STORE:
        out = torch.full((m, n_valid), 7.0, device="cuda")
        ldo = n_valid
    elif ep == _lib.EP_RESID_ADD:
        out = torch.randn(m, n_valid, device="cuda")
        ldo = n_valid
    else:
        ldo = n_valid // 2
        out = torch.zeros(2 * m * ldo, dtype=torch.bfloat16, device="cuda")
        lo_off = m * ldo
    before = out.clone()
    o = _lib.LinearOut(ep, n_valid, _lib.ptr(out), ldo, lo_off, lo_format)
    _lib.call("b200_linear_lo8", _lib.ptr(xh), _lib.ptr(xl8), m, k, k, _lib.ptr(whi), _lib.ptr(wlo8), n, C.byref(o),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    return out, before


def _operand_product(xh, xl8, whi, wlo8):
    """fp64 value of what the tensor cores compute: (x_hi w_hi + x_lo8 w_lo8) / 2^12."""
    return (xh.double().cpu() @ whi.double().cpu().T + _e4m3_values(xl8.cpu()) @ _e4m3_values(wlo8.cpu()).T) / 2.0 ** SHIFT


@pytest.mark.parametrize("m", [1, 77, 300, 2048])
@pytest.mark.parametrize("ep", ["store", "resid"])
def test_linear_lo8_matches_its_operands_and_the_exact_product(m, ep):
    """m = 1 / 77 / 300: 128-column tiles with a K split (atomic partial sums); 2048: 256-column
    tiles, whole K per tile."""
    from strands_decider_b200 import _lib

    k, n = 1024, 2560 if m == 2048 else 512
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m))
    xh, xl8 = _x_planes(x)
    pw, whi, wlo8, plain = _lo8_copies("int4", n, k, 2)
    e = _lib.EP_STORE if ep == "store" else _lib.EP_RESID_ADD
    out, before = _run_lo8(xh, xl8, whi, wlo8, e, n)
    got = out.double().cpu() - (before.double().cpu() if ep == "resid" else 0)
    ref = _operand_product(xh, xl8, whi, wlo8)
    scale = ref.abs().max().item()
    assert (got - ref).abs().max().item() < 2e-5 * scale + 1e-6
    exact = x.double() @ plain.double().cpu().T
    assert (got - exact).abs().max().item() < 1e-3 * scale


def test_linear_lo8_m_tail_and_large_k():
    from strands_decider_b200 import _lib

    m, k, n = 333, 6144, 512
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(9))
    xh, xl8 = _x_planes(x)
    _, whi, wlo8, _ = _lo8_copies("nvfp4", n, k, 7)
    out, _ = _run_lo8(xh, xl8, whi, wlo8, _lib.EP_STORE, n)
    ref = _operand_product(xh, xl8, whi, wlo8)
    assert (out.double().cpu() - ref).abs().max().item() < 2e-5 * ref.abs().max().item()


@pytest.mark.parametrize("m", [150, 2048])
@pytest.mark.parametrize("lo_format", [0, 1])
def test_linear_lo8_swiglu_writes_either_plane_format(m, lo_format):
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, inter = 1024, 1280 if m == 2048 else 384
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(5))
    xh, xl8 = _x_planes(x)
    gate = W.quantize("nvfp4", _weights(inter, k, seed=5).cuda())
    up = W.quantize("nvfp4", _weights(inter, k, seed=6).cuda())
    pw = W.interleave_gate_up(gate, up)
    qw = pw.qweight()
    whi = torch.empty(pw.n, k, dtype=torch.bfloat16, device="cuda")
    wlo8 = torch.empty(pw.n, k, dtype=torch.uint8, device="cuda")
    _lib.call("b200_dequantize_lo8", C.byref(qw), _lib.ptr(whi), _lib.ptr(wlo8), _lib.stream_ptr())
    out, _ = _run_lo8(xh, xl8, whi, wlo8, _lib.EP_SWIGLU, 2 * inter, lo_format)
    y = _operand_product(xh, xl8, whi, wlo8)          # interleaved blocks of 64: gate | up
    yb = y.view(m, -1, 2, 64)
    ref = (torch.nn.functional.silu(yb[:, :, 0]) * yb[:, :, 1]).reshape(m, inter)
    hi = out[: m * inter].view(m, inter).double().cpu()
    if lo_format == _lib.LO_E4M3:
        lo = _e4m3_values(out[m * inter:].view(torch.uint8)[: m * inter].view(m, inter).cpu()) / 2.0 ** X_SHIFT
        tol = 3e-4   # plus e4m3 rounding of the low term: 2^-4 of at most 2^-9 relative
    else:
        lo = out[m * inter:].view(m, inter).double().cpu()
        tol = 1e-4   # fp32 accumulation of y, amplified through silu(gate) * up
    assert (hi + lo - ref).abs().max().item() / ref.abs().max().item() < tol


@pytest.mark.parametrize("rows", [5, 3000])
def test_rmsnorm_lo8_planes(rows):
    """Same hi plane as b200_rmsnorm; the e4m3 low plane decodes to the fp32 normed value
    within e4m3's rounding of the low term."""
    from strands_decider_b200 import _lib

    hidden = 2048
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, hidden, generator=g) * 3).cuda()
    w = (torch.randn(hidden, generator=g) * 0.1).cuda()
    plain = torch.zeros(2 * rows * hidden, dtype=torch.bfloat16, device="cuda")
    lo8 = torch.zeros_like(plain)
    off = rows * hidden
    _lib.call("b200_rmsnorm", _lib.ptr(x), rows, hidden, _lib.ptr(w), 1e-6, _lib.ptr(plain), off, _lib.stream_ptr())
    _lib.call("b200_rmsnorm_lo8", _lib.ptr(x), rows, hidden, _lib.ptr(w), 1e-6, _lib.ptr(lo8), off, _lib.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(plain[:off], lo8[:off])
    y = plain[:off].double() + plain[off:].double()           # two bf16 planes: fp32-level
    dec = lo8[:off].double() + _e4m3_values(lo8[off:].view(torch.uint8)[:off]) / 2.0 ** X_SHIFT
    # e4m3 keeps 4 significant bits of the low term (<= 2^-9 |y|); below its normal range
    # (|lo| * 2^6 < 2^-6) the absolute step is 2^-9 / 2^6
    assert torch.all((dec - y).abs() <= 2.0 ** -12 * y.abs() + 2.0 ** -16)


def test_lo8_rejects_unaligned_rows():
    from strands_decider_b200 import _lib

    xh = torch.zeros(4, 1032, dtype=torch.bfloat16, device="cuda")
    xl8 = torch.zeros(4, 1032, dtype=torch.uint8, device="cuda")
    whi = torch.zeros(256, 1024, dtype=torch.bfloat16, device="cuda")
    wlo8 = torch.zeros(256, 1024, dtype=torch.uint8, device="cuda")
    out = torch.zeros(4, 256, device="cuda")
    o = _lib.LinearOut(0, 256, _lib.ptr(out), 256, 0, 0)
    with pytest.raises(_lib.B200Error) as e:      # ldx = 1032 is not a multiple of 16
        _lib.call("b200_linear_lo8", _lib.ptr(xh), _lib.ptr(xl8), 4, 1024, 1032, _lib.ptr(whi), _lib.ptr(wlo8), 256,
                  C.byref(o), _lib.stream_ptr())
    assert e.value.status == 2


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_forward_on_e4m3_low_planes_matches_reference_golden(fmt):
    """The reduced decider's golden prompts with every GEMM forced onto e4m3 low planes."""
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.weights import DeviceWeights

    g = np.load(os.path.join(GOLDEN, "reduced_1024_int4.npz"))
    spec = config.REDUCED_1024.with_format(fmt)
    w = DeviceWeights.synthetic(spec, seed=0, latent_device="cpu")
    rows = g["ids"].tolist()
    outs = {}
    for lo in ("bf16", "e4m3"):
        m = DecisionModel(w, max_tokens=4096, pool_slots=4, pool_kv_tokens=4096, dequant_min_tokens=1, lo_plane=lo)
        outs[lo] = m.score_prompts(rows, [[11, 12, 13]] * 4, [3] * 4, ["choice"] * 4, [1.0] * 4).cpu()
        del m
    d = np.abs(outs["e4m3"].probs.numpy() - outs["bf16"].probs.numpy()).max()
    assert d < 1e-3, d
    if fmt == "int4":
        assert np.abs(outs["e4m3"].probs.numpy() - g["probs"]).max() < 2e-3
        assert np.array_equal(outs["e4m3"].argmax.numpy(), g["probs"].argmax(1))


# ----------------------------------------------------------------------------- CTA pairs
# Batches with at least one 256 x 256 tile per SM pair run the bf16-weight GEMMs (two bf16
# planes, one plane, or the e4m3 low plane above) on CTA pairs (tcgen05 .cta_group::2).


@pytest.mark.parametrize("planes", ["split", "one"])
@pytest.mark.parametrize("ep", ["store", "resid", "swiglu"])
def test_pair_gemm_bf16_weights_large_m_with_tail(planes, ep):
    """M = 2125: 9 row tiles of 256, the last one's second CTA entirely past M."""
    from strands_decider_b200 import _lib

    m, k, n = 2125, 1024, 2560
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(31))
    xp = _lib.split_planes(x).cuda()
    w = _weights(n, k, 32).to(torch.bfloat16).cuda()
    qw = _lib.QWeight()
    qw.format, qw.n, qw.k, qw.data = _lib.FMT["bf16"], n, k, _lib.ptr(w)
    lo_off = 0
    if ep == "store":
        out, ldo, e = torch.full((m, n), 7.0, device="cuda"), n, _lib.EP_STORE
    elif ep == "resid":
        out, ldo, e = torch.randn(m, n, device="cuda"), n, _lib.EP_RESID_ADD
    else:
        ldo, e = n // 2, _lib.EP_SWIGLU
        out = torch.zeros(2, m, ldo, dtype=torch.bfloat16, device="cuda")
        lo_off = m * ldo
    before = out.clone()
    o = _lib.LinearOut(e, n, _lib.ptr(out), ldo, lo_off, 0)
    _lib.call("b200_linear", _lib.ptr(xp[0]), _lib.ptr(xp[1]) if planes == "split" else None, m, k, k, C.byref(qw),
              C.byref(o), _lib.stream_ptr())
    torch.cuda.synchronize()
    xv = xp[0].double().cpu() + (xp[1].double().cpu() if planes == "split" else 0)
    y = xv @ w.double().cpu().T
    if ep == "swiglu":
        yb = y.view(m, -1, 2, 64)
        ref = (torch.nn.functional.silu(yb[:, :, 0]) * yb[:, :, 1]).reshape(m, n // 2)
        got = out[0].double().cpu() + out[1].double().cpu()
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4
        return
    got = out.double().cpu() - (before.double().cpu() if ep == "resid" else 0)
    assert (got - y).abs().max().item() < 2e-5 * y.abs().max().item() + 1e-6


def test_pair_gemm_lo8_tail():
    from strands_decider_b200 import _lib

    m, k, n = 2125, 2048, 2560
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(33))
    xh, xl8 = _x_planes(x)
    _, whi, wlo8, _ = _lo8_copies("nvfp4", n, k, 34)
    out, before = _run_lo8(xh, xl8, whi, wlo8, _lib.EP_RESID_ADD, n)
    ref = _operand_product(xh, xl8, whi, wlo8)
    got = out.double().cpu() - before.double().cpu()
    assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item()


def test_e4m3_low_planes_on_the_2b_decider_stay_inside_the_bar():
    """The 2B-shape NVFP4 decider, 3 prompts x 512 tokens with every GEMM on the dequantised
    path (CTA pairs): e4m3 low planes against two bf16 planes (the latter within 1e-5 of the
    fp32 oracle). The CPU emulation of this case measures 6.9e-4 against fp32."""
    from strands_decider_b200.runtime import DecisionModel
    from strands_decider_b200.weights import DeviceWeights

    spec = config.HYBRID_2B
    w = DeviceWeights.synthetic(spec, seed=0, device="cuda", latent_device="cuda")
    g = torch.Generator().manual_seed(0)
    rows = [torch.randint(0, spec.vocab, (512,), generator=g).tolist() for _ in range(3)]
    outs = {}
    for lo in ("bf16", "e4m3"):
        m = DecisionModel(w, max_tokens=2048, pool_slots=1, pool_kv_tokens=16, dequant_min_tokens=1, lo_plane=lo)
        outs[lo] = m.score_prompts(rows, [[11, 12, 13]] * 3, [3] * 3, ["choice"] * 3, [1.0] * 3).cpu().probs
        del m
    d = (outs["e4m3"] - outs["bf16"]).abs().max().item()
    assert d < 1.5e-3, d
    top2 = outs["bf16"].topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * d
    assert torch.equal(outs["e4m3"].argmax(1)[clear], outs["bf16"].argmax(1)[clear])
