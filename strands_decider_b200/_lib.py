"""ctypes binding of libstrands_b200.so (the C ABI in include/strands_b200.h).

The library is the only compute path: there is no CPU or pure-torch fallback. Loading
fails loudly when the shared library is missing; every call raises B200Error on a
non-zero status. Tensors are passed as raw device pointers (torch owns the memory).
"""

from __future__ import annotations

import ctypes as C
import os
import threading

import torch

from . import build as _build

LIB_PATH = _build.LIB

B200_OK = 0
STATUS = {1: "ARG", 2: "SHAPE", 3: "FORMAT", 4: "CUDA", 5: "WORKSPACE", 6: "TIMEOUT", 7: "UNSUPPORTED"}

FMT = {"bf16": 0, "int4": 1, "nvfp4": 2, "ternary": 3}
EP_STORE, EP_RESID_ADD, EP_SWIGLU = 0, 1, 2
LO_BF16, LO_E4M3 = 0, 1
LO8_X_SHIFT, LO8_W_SHIFT = 6, 6
LO8_SHIFT = LO8_X_SHIFT + LO8_W_SHIFT
LAYER_GDN, LAYER_ATTN = 0, 1


class B200Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b200 status {status} ({STATUS.get(status, '?')}): {msg}")
        self.status = status


class QWeight(C.Structure):
    _fields_ = [("format", C.c_int32), ("n", C.c_int32), ("k", C.c_int32), ("data", C.c_void_p),
                ("scales", C.c_void_p), ("row_scale", C.c_void_p), ("tiles", C.c_void_p),
                ("tile_scales", C.c_void_p)]


class LinearOut(C.Structure):
    _fields_ = [("epilogue", C.c_int32), ("n_valid", C.c_int32), ("out", C.c_void_p), ("ldo", C.c_int32),
                ("lo_offset", C.c_int64), ("lo_format", C.c_int32)]


class Seqs(C.Structure):
    _fields_ = [("n_seqs", C.c_int32), ("n_tokens", C.c_int32), ("max_len", C.c_int32),
                ("cu_seqlens", C.c_void_p), ("prefix_slot", C.c_void_p), ("save_slot", C.c_void_p)]


class PrefixPool(C.Structure):
    _fields_ = [("n_slots", C.c_int32), ("kv_capacity", C.c_int32), ("slot_len", C.c_void_p),
                ("slot_kv", C.c_void_p), ("gdn_state", C.c_void_p), ("conv_hist", C.c_void_p),
                ("k_cache", C.c_void_p), ("v_cache", C.c_void_p)]


class GdnParams(C.Structure):
    _fields_ = [("heads", C.c_int32), ("dk", C.c_int32), ("dv", C.c_int32), ("conv_width", C.c_int32),
                ("eps", C.c_float), ("conv_w", C.c_void_p), ("a_log", C.c_void_p), ("dt_bias", C.c_void_p),
                ("norm_w", C.c_void_p)]


class AttnParams(C.Structure):
    _fields_ = [("heads", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32), ("rope_dim", C.c_int32),
                ("max_pos", C.c_int32), ("eps", C.c_float), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p)]


class DecideArgs(C.Structure):
    _fields_ = [("n_rows", C.c_int32), ("kmax", C.c_int32), ("last_tok", C.c_void_p), ("opt_ids", C.c_void_p),
                ("n_opts", C.c_void_p), ("kinds", C.c_void_p), ("temperature", C.c_void_p),
                ("ordinal_smoothing", C.c_float), ("probs", C.c_void_p), ("argmax", C.c_void_p),
                ("confidence", C.c_void_p), ("score", C.c_void_p), ("opt_tok", C.c_void_p)]


HEAD_OPTION_TOKEN, HEAD_SLOT, HEAD_POINTER = 0, 1, 2


class Readout(C.Structure):
    _fields_ = [("kind", C.c_int32), ("hidden", C.c_int32), ("out", C.c_int32), ("mlp_hidden", C.c_int32),
                ("ln_eps", C.c_float), ("ln_w", C.c_void_p), ("ln_b", C.c_void_p), ("w1", C.c_void_p),
                ("b1", C.c_void_p), ("w2", C.c_void_p), ("b2", C.c_void_p)]


class ModelConfig(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32), ("n_layers", C.c_int32),
                ("layer_kind", C.c_int32 * 64), ("gdn_heads", C.c_int32), ("gdn_dk", C.c_int32),
                ("gdn_dv", C.c_int32), ("conv_width", C.c_int32), ("attn_heads", C.c_int32),
                ("attn_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("rope_dim", C.c_int32),
                ("max_pos", C.c_int32), ("eps", C.c_float), ("weight_format", C.c_int32),
                ("dequant_min_tokens", C.c_int32), ("lo_format", C.c_int32)]


class LayerWeights(C.Structure):
    _fields_ = [("input_norm", C.c_void_p), ("post_norm", C.c_void_p), ("mix_in", QWeight), ("mix_out", QWeight),
                ("gate_up", QWeight), ("down", QWeight), ("gdn", GdnParams), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p)]


_P = C.c_void_p
_I = C.c_int32
_SIGS = {
    "b200_version": ([], C.c_int),
    "b200_last_error": ([], C.c_char_p),
    "b200_read_fault": ([C.POINTER(C.c_uint)], C.c_int),
    "b200_quantize": ([_I, _P, _I, _I, _P, _P, _P, _P], C.c_int),
    "b200_dequantize": ([C.POINTER(QWeight), _P, _P], C.c_int),
    "b200_dequantize_lo8": ([C.POINTER(QWeight), _P, _P, _P], C.c_int),
    "b200_tile_bytes": ([_I, _I, _I, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)], C.c_int),
    "b200_tile_weights": ([C.POINTER(QWeight), _P, _P, _P], C.c_int),
    "b200_linear": ([_P, _P, _I, _I, _I, C.POINTER(QWeight), C.POINTER(LinearOut), _P], C.c_int),
    "b200_linear_simt": ([_P, _P, _I, _I, _I, C.POINTER(QWeight), C.POINTER(LinearOut), _P], C.c_int),
    "b200_linear_lo8": ([_P, _P, _I, _I, _I, _P, _P, _I, C.POINTER(LinearOut), _P], C.c_int),
    "b200_embed": ([_P, _I, _P, _I, _P, _P], C.c_int),
    "b200_rmsnorm": ([_P, _I, _I, _P, C.c_float, _P, C.c_int64, _P], C.c_int),
    "b200_rmsnorm_lo8": ([_P, _I, _I, _P, C.c_float, _P, C.c_int64, _P], C.c_int),
    "b200_gdn_mixer": ([C.POINTER(GdnParams), C.POINTER(Seqs), _P, _I, _P, C.c_int64, C.POINTER(PrefixPool), _I,
                        _P, _P], C.c_int),
    "b200_gdn_mixer_recurrent": ([C.POINTER(GdnParams), C.POINTER(Seqs), _P, _I, _P, C.c_int64,
                                  C.POINTER(PrefixPool), _I, _P, _P], C.c_int),
    "b200_gdn_mixer_chunked": ([C.POINTER(GdnParams), C.POINTER(Seqs), _P, _I, _P, C.c_int64,
                                C.POINTER(PrefixPool), _I, _P, _P], C.c_int),
    "b200_gdn_scratch_floats": ([_I, _I], C.c_int),
    "b200_attention": ([C.POINTER(AttnParams), C.POINTER(Seqs), _P, _I, _P, _P, _P, _P, C.c_int64,
                        C.POINTER(PrefixPool), _I, _P], C.c_int),
    "b200_attention_noalloc": ([C.POINTER(AttnParams), C.POINTER(Seqs), _P, _I, _P, C.c_int64,
                                C.POINTER(PrefixPool), _I, _P], C.c_int),
    "b200_decide": ([_P, _I, _P, C.c_float, _P, C.POINTER(DecideArgs), _P], C.c_int),
    "b200_nvfp4_sf_atom_bytes": ([_I, _I, C.POINTER(C.c_size_t)], C.c_int),
    "b200_quantize_act_nvfp4": ([_P, _I, _I, _I, _P, _P, _P], C.c_int),
    "b200_nvfp4_sf_atoms": ([_P, _I, _I, _P, _P], C.c_int),
    "b200_linear_nvfp4_native": ([_P, _P, _I, _I, C.POINTER(QWeight), _P, C.POINTER(LinearOut), _P], C.c_int),
    "b200_decide_readout": ([_P, _I, _P, C.c_float, C.POINTER(Readout), C.POINTER(DecideArgs), _I, _P], C.c_int),
    "b200_model_create": ([C.POINTER(ModelConfig), C.POINTER(C.c_void_p)], C.c_int),
    "b200_model_destroy": ([_P], C.c_int),
    "b200_model_set_layer": ([_P, _I, C.POINTER(LayerWeights)], C.c_int),
    "b200_model_set_globals": ([_P, _P, _P, _P, _P], C.c_int),
    "b200_model_set_readout": ([_P, C.POINTER(Readout)], C.c_int),
    "b200_model_workspace_bytes": ([_P, _I, C.POINTER(C.c_size_t)], C.c_int),
    "b200_model_forward": ([_P, _P, C.POINTER(Seqs), C.POINTER(PrefixPool), C.POINTER(DecideArgs), _P,
                            C.c_size_t, _P], C.c_int),
}

_lib: C.CDLL | None = None
_lock = threading.Lock()


def load(path: str | None = None) -> C.CDLL:
    """Load (once) and type the shared library. Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"{p} is missing: build it with `python -m strands_decider_b200.build` "
                "(this backend has no fallback path)")
        lib = C.CDLL(p)
        for name, (args, res) in _SIGS.items():
            f = getattr(lib, name)
            f.argtypes = args
            f.restype = res
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    return sorted(_SIGS)


def check(status: int) -> None:
    if status != B200_OK:
        msg = load().b200_last_error()
        raise B200Error(status, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("b200 kernels take CUDA tensors only")
    return t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def split_planes(x: torch.Tensor) -> torch.Tensor:
    """fp32 [..., k] -> bf16 [2, ..., k]: hi = bf16_rn(x), lo = bf16_rn(x - hi) (the
    activation format of every GEMM input)."""
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return torch.stack([hi, lo]).contiguous()


def read_fault() -> int:
    v = C.c_uint(0)
    check(load().b200_read_fault(C.byref(v)))
    return int(v.value)
