"""b200_attention_noalloc, the attention entry point that allocates nothing.

Some callers cannot call cudaMalloc: a host runtime whose device memory belongs to its own
arena or caching allocator (a serving process that preallocated its pool, or a Go / Java
host that hands the library only its request buffers) must not allocate or free in the middle
of a request. This entry point keeps its q / k / v scratch in a static device array of the
library instead of taking a scratch buffer. Checked here, through the C ABI, against
b200_attention (which takes caller scratch) on the same inputs, for two calls in a row.
This file is collected last so that a failure here cannot hide another test's result.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

NQ, NKV, HD = 8, 2, 256


def _inputs(seed, lens, prefix):
    from strands_decider_b200 import config
    from strands_decider_b200.runtime import rope_tables

    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    cols = 2 * NQ * HD + 2 * NKV * HD
    cos, sin = rope_tables(config.HYBRID_2B, "cpu")
    kv_cap = max(sum(prefix), 1)
    d = dict(qkv=torch.randn(T, cols, generator=g), qn=0.1 * torch.randn(HD, generator=g),
             kn=0.1 * torch.randn(HD, generator=g), cos=cos, sin=sin,
             kpool=torch.randn(1, kv_cap, NKV, HD, generator=g).to(torch.bfloat16),
             vpool=torch.randn(1, kv_cap, NKV, HD, generator=g).to(torch.bfloat16),
             slot_kv=torch.tensor([sum(prefix[:i]) for i in range(len(prefix))], dtype=torch.int32),
             slot_len=torch.tensor(prefix, dtype=torch.int32))
    d = {k: v.cuda() for k, v in d.items()}
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    d["cu"] = torch.tensor(cu, dtype=torch.int32, device="cuda")
    d["pslot"] = torch.arange(len(lens), dtype=torch.int32, device="cuda")
    return d, T, cols, kv_cap


def _run(noalloc: bool, d, T, cols, kv_cap, lens):
    from strands_decider_b200 import _lib

    out = torch.zeros(2, T, NQ * HD, dtype=torch.bfloat16, device="cuda")
    p = _lib.AttnParams(NQ, NKV, HD, HD // 4, d["cos"].shape[0], 1e-6, _lib.ptr(d["qn"]), _lib.ptr(d["kn"]),
                        _lib.ptr(d["cos"]), _lib.ptr(d["sin"]))
    seqs = _lib.Seqs(len(lens), T, max(lens), _lib.ptr(d["cu"]), _lib.ptr(d["pslot"]), None)
    pool = _lib.PrefixPool(len(lens), kv_cap, _lib.ptr(d["slot_len"]), _lib.ptr(d["slot_kv"]), None, None,
                           _lib.ptr(d["kpool"]), _lib.ptr(d["vpool"]))
    if noalloc:
        _lib.call("b200_attention_noalloc", C.byref(p), C.byref(seqs), _lib.ptr(d["qkv"]), cols, _lib.ptr(out),
                  T * NQ * HD, C.byref(pool), 0, _lib.stream_ptr())
    else:
        qb = torch.empty(T, NQ, HD, dtype=torch.bfloat16, device="cuda")
        kb = torch.empty(T, NKV, HD, dtype=torch.bfloat16, device="cuda")
        vb = torch.empty_like(kb)
        _lib.call("b200_attention", C.byref(p), C.byref(seqs), _lib.ptr(d["qkv"]), cols, _lib.ptr(qb),
                  _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(out), T * NQ * HD, C.byref(pool), 0, _lib.stream_ptr())
    torch.cuda.synchronize()
    return out


def test_noalloc_attention_matches_scratch_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    from strands_decider_b200 import _lib

    _lib.load()
    for seed, lens, prefix in [(0, [1, 37, 64, 130], [5, 0, 70, 2]), (1, [200, 3], [0, 40])]:
        d, T, cols, kv_cap = _inputs(seed, lens, prefix)
        want = _run(False, d, T, cols, kv_cap, lens)
        got = _run(True, d, T, cols, kv_cap, lens)
        ref = want.float()
        err = (got.float() - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6)
        assert err <= 1e-6, (seed, err)
    assert _lib.read_fault() == 0


def test_noalloc_attention_refuses_batches_beyond_its_scratch():
    from strands_decider_b200 import _lib

    _lib.load()
    lens = [1400]                       # 1400 * (8 + 4) * 256 * 2 bytes > 8 MiB
    d, T, cols, kv_cap = _inputs(2, lens, [0])
    with pytest.raises(_lib.B200Error) as e:
        _run(True, d, T, cols, kv_cap, lens)
    assert e.value.status == 2 and "8 MiB" in str(e.value)
