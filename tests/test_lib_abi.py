"""The C ABI, without a GPU: the library builds for sm_100a, loads, exports every entry
point include/strands_b200.h declares, and validates arguments on the host (status codes,
never an abort)."""

from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "strands_b200.h")


@pytest.fixture(scope="module")
def lib():
    from strands_decider_b200 import _lib, build

    build.build()
    return _lib.load()


def header_functions() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int)\s+(b200_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_runtime_and_kernels():
    names = header_functions()
    for want in ("b200_linear", "b200_quantize", "b200_gdn_mixer", "b200_attention", "b200_decide",
                 "b200_model_forward", "b200_read_fault"):
        assert want in names


def test_every_declared_symbol_is_exported(lib):
    from strands_decider_b200 import _lib

    for name in header_functions():
        assert hasattr(lib, name), name
    assert set(header_functions()) == set(_lib.exported_symbols())


def test_version(lib):
    assert lib.b200_version() == 100


def test_null_arguments_return_status_not_abort(lib):
    from strands_decider_b200 import _lib

    o = _lib.LinearOut()
    w = _lib.QWeight()
    assert lib.b200_linear(None, None, 1, 128, 128, C.byref(w), C.byref(o), None) == 1
    assert b"null" in lib.b200_last_error()
    assert lib.b200_quantize(1, None, 1, 128, None, None, None, None) == 1
    assert lib.b200_decide(None, 64, None, 1e-6, None, None, None) == 1


def test_linear_shape_checks_on_host(lib):
    from strands_decider_b200 import _lib

    buf = (C.c_uint8 * 64)()
    p = C.cast(buf, C.c_void_p).value
    p16 = (p + 15) // 16 * 16
    w = _lib.QWeight(1, 256, 1000, p16, p16, None)   # k not a multiple of 128
    o = _lib.LinearOut(0, 256, p16, 256, 0)
    assert lib.b200_linear(p16, None, 4, 1000, 1000, C.byref(w), C.byref(o), None) == 2
    w = _lib.QWeight(1, 200, 1024, p16, p16, None)   # n not a multiple of 256
    assert lib.b200_linear(p16, None, 4, 1024, 1024, C.byref(w), C.byref(o), None) == 2
    w = _lib.QWeight(9, 256, 1024, p16, p16, None)   # unknown format
    assert lib.b200_linear(p16, None, 4, 1024, 1024, C.byref(w), C.byref(o), None) == 3
    w = _lib.QWeight(1, 256, 1024, p16, p16, None)
    o = _lib.LinearOut(0, 200, p16, 256, 0)             # n_valid not a multiple of 32
    assert lib.b200_linear(p16, None, 4, 1024, 1024, C.byref(w), C.byref(o), None) == 2
    o = _lib.LinearOut(0, 256, p16, 256, 0)
    assert lib.b200_linear(p16, p16 + 8, 4, 1024, 1024, C.byref(w), C.byref(o), None) == 2  # lo plane unaligned


@pytest.mark.parametrize("entry", ["b200_gdn_mixer", "b200_gdn_mixer_chunked", "b200_gdn_mixer_recurrent"])
def test_gdn_mixer_argument_checks_on_host(lib, entry):
    """Every GDN entry point refuses bad arguments with a status before touching the device."""
    from strands_decider_b200 import _lib

    buf = (C.c_uint8 * 256)()
    p16 = (C.cast(buf, C.c_void_p).value + 15) // 16 * 16
    f = getattr(lib, entry)
    params = _lib.GdnParams(2, 128, 128, 4, 1e-6, p16, p16, p16, p16)
    seqs = _lib.Seqs(1, 4, 4, p16, None, None)
    ld = 3 * 256 + 256 + 4
    assert f(None, C.byref(seqs), p16, ld, p16, 0, None, 0, p16, None) == 1            # null params
    bad = _lib.GdnParams(2, 64, 128, 4, 1e-6, p16, p16, p16, p16)
    assert f(C.byref(bad), C.byref(seqs), p16, ld, p16, 0, None, 0, p16, None) == 7     # dk 64 is not built
    many = _lib.Seqs(70000, 70000, 1, p16, None, None)
    assert f(C.byref(params), C.byref(many), p16, ld, p16, 0, None, 0, p16, None) == 2  # grid limit
    slotted = _lib.Seqs(1, 4, 4, p16, p16, None)
    assert f(C.byref(params), C.byref(slotted), p16, ld, p16, 0, None, 0, p16, None) == 1  # slots need a pool
    assert f(C.byref(params), C.byref(seqs), p16, ld, p16, 0, None, 0, None, None) == 1    # no scratch
    assert f(C.byref(params), C.byref(seqs), p16, ld - 4, p16, 0, None, 0, p16, None) == 2  # ld_mix too narrow


def test_model_context_host_side(lib):
    from strands_decider_b200 import _lib, config

    s = config.REDUCED_1024
    cfg = _lib.ModelConfig()
    cfg.vocab, cfg.hidden, cfg.inter, cfg.n_layers = s.vocab, s.hidden, s.inter, s.n_layers
    for i, t in enumerate(s.layer_types):
        cfg.layer_kind[i] = 0 if t == config.GDN else 1
    cfg.gdn_heads, cfg.gdn_dk, cfg.gdn_dv, cfg.conv_width = s.gdn_heads, 128, 128, 4
    cfg.attn_heads, cfg.attn_kv_heads, cfg.head_dim, cfg.rope_dim, cfg.max_pos = 8, 2, 128, 32, 4096
    cfg.eps, cfg.weight_format = 1e-6, 1
    h = C.c_void_p()
    assert lib.b200_model_create(C.byref(cfg), C.byref(h)) == 0
    nbytes = C.c_size_t()
    assert lib.b200_model_workspace_bytes(h, 1024, C.byref(nbytes)) == 0
    # residual fp32 + normed bf16 + the widest bf16 projection output, at least
    assert nbytes.value >= 1024 * (1024 * 6 + 6144 * 2)
    # a forward before any weight is registered is refused on the host
    ids = (C.c_int32 * 4)()
    seqs = _lib.Seqs(1, 4, 4, C.cast(ids, C.c_void_p), None, None)
    assert lib.b200_model_forward(h, C.cast(ids, C.c_void_p), C.byref(seqs), None, None,
                                  C.cast(ids, C.c_void_p), 16, None) == 1
    assert lib.b200_model_destroy(h) == 0
    cfg.gdn_dk = 64
    assert lib.b200_model_create(C.byref(cfg), C.byref(h)) == 7   # unsupported GDN head dim


def test_library_without_gpu_has_no_fallback():
    """The product path raises when the library is absent (no CPU fallback)."""
    from strands_decider_b200 import _lib

    saved = _lib._lib
    try:
        _lib._lib = None
        with pytest.raises(RuntimeError, match="missing"):
            _lib.load("/nonexistent/libstrands_b200.so")
    finally:
        _lib._lib = saved
