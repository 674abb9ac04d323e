"""The native NVFP4 path (W4A4 on tcgen05.mma kind::mxf4nvf4) against its oracle.

* The activation quantiser (b200_quantize_act_nvfp4): codes and scale atoms bit-exact with
  oracle.quant.quantize_act_nvfp4 / nvfp4_sf_atoms, including the zero-scale padding rows.
* The weight scale re-layout (b200_nvfp4_sf_atoms): bit-exact.
* The GEMM (b200_linear_nvfp4_native): against the fp64 sum of the exact block products
  (oracle.quant.nvfp4_native_product), within 1e-5 of max |y| (the device accumulates in
  fp32), for the store, residual and SwiGLU epilogues and ragged M.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    from strands_decider_b200 import _lib

    _lib.load()
    yield
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _atom_bytes(rows, k):
    from strands_decider_b200 import _lib

    n = C.c_size_t()
    _lib.check(_lib.load().b200_nvfp4_sf_atom_bytes(rows, k, C.byref(n)))
    return n.value


def _quant_act(x: torch.Tensor):
    """Device quantisation of an fp32 [m, k] CPU tensor -> (codes, atoms) device tensors."""
    from strands_decider_b200 import _lib

    m, k = x.shape
    xd = x.cuda().contiguous()
    codes = torch.empty(m, k // 2, dtype=torch.uint8, device="cuda")
    atoms = torch.full((_atom_bytes(m, k),), 0xAB, dtype=torch.uint8, device="cuda")
    _lib.call("b200_quantize_act_nvfp4", _lib.ptr(xd), m, k, k, _lib.ptr(codes), _lib.ptr(atoms), _lib.stream_ptr())
    torch.cuda.synchronize()
    return codes, atoms


@pytest.mark.parametrize("m,k", [(200, 512), (128, 2048), (1, 256)])
def test_activation_quantiser_is_bit_exact(m, k):
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + k)) * 3.0
    x[0, :16] = 0.0                    # a zero block: zero scale, zero codes
    if m > 5:
        x[5, 16:32] *= 1e-4            # a tiny block: a subnormal e4m3 scale
    codes, atoms = _quant_act(x)
    want_c, want_s = Q.quantize_act_nvfp4(x.numpy())
    assert np.array_equal(codes.cpu().numpy(), want_c)
    assert np.array_equal(atoms.cpu().numpy(), Q.nvfp4_sf_atoms(want_s))


def _weight(n, k, seed):
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    w = torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02
    pw = W.quantize("nvfp4", w.cuda())
    atoms = torch.empty(_atom_bytes(n, k), dtype=torch.uint8, device="cuda")
    _lib.call("b200_nvfp4_sf_atoms", _lib.ptr(pw.scales), n, k, _lib.ptr(atoms), _lib.stream_ptr())
    return pw, atoms


def test_weight_scale_atoms_are_bit_exact():
    from strands_decider_b200 import weights as W

    pw, atoms = _weight(384, 1024, 3)
    torch.cuda.synchronize()
    parts = W.packed_to_numpy(pw)
    assert np.array_equal(atoms.cpu().numpy(), Q.nvfp4_sf_atoms(parts["scales"]))


def _reference(x, pw):
    from strands_decider_b200 import weights as W

    parts = W.packed_to_numpy(pw)
    c, s = Q.quantize_act_nvfp4(x.numpy())
    return torch.from_numpy(Q.nvfp4_native_product(c, s, parts["data"], parts["scales"], pw.row_scale.cpu().numpy()))


def _run(x, pw, w_atoms, ep, n_valid):
    from strands_decider_b200 import _lib

    m = x.shape[0]
    codes, atoms = _quant_act(x)
    if ep == _lib.EP_SWIGLU:
        out = torch.zeros(2, m, n_valid // 2, dtype=torch.bfloat16, device="cuda")
        o = _lib.LinearOut(ep, n_valid, _lib.ptr(out), n_valid // 2, m * (n_valid // 2), 0)
    else:
        out = torch.randn(m, n_valid, device="cuda") if ep == _lib.EP_RESID_ADD else torch.full((m, n_valid), 7.0,
                                                                                               device="cuda")
        o = _lib.LinearOut(ep, n_valid, _lib.ptr(out), n_valid, 0, 0)
    before = out.clone()
    qw = pw.qweight()
    _lib.call("b200_linear_nvfp4_native", _lib.ptr(codes), _lib.ptr(atoms), m, x.shape[1], C.byref(qw),
              _lib.ptr(w_atoms), C.byref(o), _lib.stream_ptr())
    torch.cuda.synchronize()
    return out, before


@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (200, 768, 2048), (1000, 1280, 1024)])
def test_native_gemm_store_and_residual(m, n, k):
    from strands_decider_b200 import _lib

    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m))
    pw, w_atoms = _weight(n, k, m + 1)
    ref = _reference(x, pw)
    out, _ = _run(x, pw, w_atoms, _lib.EP_STORE, n)
    assert (out.double().cpu() - ref).abs().max().item() < 1e-5 * ref.abs().max().item()
    out, before = _run(x, pw, w_atoms, _lib.EP_RESID_ADD, n)
    got = out.double().cpu() - before.double().cpu()
    assert (got - ref).abs().max().item() < 1e-5 * ref.abs().max().item() + 1e-6


def test_native_gemm_swiglu():
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    m, k, inter = 300, 1024, 384
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(9))
    gate = W.quantize("nvfp4", torch.randn(inter, k, generator=torch.Generator().manual_seed(10)).cuda() * 0.02)
    up = W.quantize("nvfp4", torch.randn(inter, k, generator=torch.Generator().manual_seed(11)).cuda() * 0.02)
    pw = W.interleave_gate_up(gate, up)
    w_atoms = torch.empty(_atom_bytes(pw.n, k), dtype=torch.uint8, device="cuda")
    _lib.call("b200_nvfp4_sf_atoms", _lib.ptr(pw.scales), pw.n, k, _lib.ptr(w_atoms), _lib.stream_ptr())
    ref = torch.nn.functional.silu(_reference(x, gate)) * _reference(x, up)
    out, _ = _run(x, pw, w_atoms, _lib.EP_SWIGLU, 2 * inter)
    got = out[0].double().cpu() + out[1].double().cpu()
    assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4


def test_native_gemm_rejects_other_formats_and_shapes():
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    pw = W.quantize("int4", torch.zeros(256, 512, device="cuda"))
    b = torch.zeros(64, dtype=torch.uint8, device="cuda")
    out = torch.zeros(4, 256, device="cuda")
    o = _lib.LinearOut(_lib.EP_STORE, 256, _lib.ptr(out), 256, 0, 0)
    qw = pw.qweight()
    rs = torch.ones(256, device="cuda")
    qw.row_scale = _lib.ptr(rs)        # everything present: the format is what is refused
    with pytest.raises(_lib.B200Error) as e:
        _lib.call("b200_linear_nvfp4_native", _lib.ptr(b), _lib.ptr(b), 4, 512, C.byref(qw), _lib.ptr(b), C.byref(o),
                  _lib.stream_ptr())
    assert e.value.status == 3
