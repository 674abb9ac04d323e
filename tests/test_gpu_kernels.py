"""Kernel-level parity on the B200: every comparison runs the CUDA path through the C ABI
against the CPU oracle (bit-exact for the integer/byte work, stated tolerances for fp)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu

FORMATS = ["int4", "nvfp4", "ternary", "bf16"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("the -m gpu tests need a CUDA device")
    from strands_decider_b200 import _lib

    _lib.load()
    yield
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0, "a device-side bounded wait or index check fired"


def _weights(n, k, seed=0, zero_row=3):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    w[zero_row] = 0.0
    w[5, :16] = 0.0        # an all-zero NVFP4 block / partial int4 group
    w[7, 0] = 0.3          # an outlier
    return w


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_quantize_bit_exact(fmt):
    from strands_decider_b200 import weights as W

    w = _weights(384, 1024)
    pw = W.quantize(fmt, w.cuda())
    got = W.packed_to_numpy(pw)
    want = Q.quantize(fmt, w.numpy())
    assert np.array_equal(got["data"].view(np.uint8), want["data"].view(np.uint8))
    assert np.array_equal(np.asarray(got["scales"]).view(np.uint8), np.asarray(want["scales"]).view(np.uint8))
    if fmt == "nvfp4":
        assert np.array_equal(pw.row_scale.cpu().numpy(), np.full(384, want["global_scale"][0], np.float32))


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequantize_bit_exact(fmt):
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    w = _weights(256, 512, seed=1)
    pw = W.quantize(fmt, w.cuda())
    out = torch.empty(256, 512, dtype=torch.int16, device="cuda")
    qw = pw.qweight()
    _lib.call("b200_dequantize", _ref(qw), _lib.ptr(out), _lib.stream_ptr())
    got = out.cpu().numpy().view(np.uint16)
    want = Q.f32_to_bf16_bits(Q.dequantize(fmt, W.packed_to_numpy(pw)))
    assert np.array_equal(got, want)


def _ref(s):
    import ctypes as C

    return C.byref(s)


def _planes(m, k, seed):
    """An fp32 activation [m, k] and its two bf16 planes [2, m, k] on the device."""
    from strands_decider_b200 import _lib

    x = torch.randn(m, k, generator=torch.Generator().manual_seed(seed))
    return x, _lib.split_planes(x).cuda()


def _linear(fn, xp, pw, ep, n_valid=None, split=True):
    """Run b200_linear / b200_linear_simt on planes xp [2, m, k]; returns (out, out_before)."""
    from strands_decider_b200 import _lib

    _, m, k = xp.shape
    n_valid = n_valid or pw.n
    lo_off = 0
    if ep == _lib.EP_STORE:
        out = torch.full((m, n_valid), 7.0, device="cuda")  # the store must overwrite it (split K zeroes it first)
        ldo = n_valid
    elif ep == _lib.EP_RESID_ADD:
        out = torch.randn(m, n_valid, device="cuda")
        ldo = n_valid
    else:
        out = torch.zeros(2, m, n_valid // 2, dtype=torch.bfloat16, device="cuda")
        ldo = n_valid // 2
        lo_off = m * ldo
    before = out.clone()
    o = _lib.LinearOut(ep, n_valid, _lib.ptr(out), ldo, lo_off)
    qw = pw.qweight()
    _lib.call(fn, _lib.ptr(xp[0]), _lib.ptr(xp[1]) if split else None, m, k, k, _ref(qw), _ref(o),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    return out, before


def _reference(xp, pw, split=True):
    from strands_decider_b200 import weights as W

    wd = torch.from_numpy(Q.dequantize(pw.fmt, W.packed_to_numpy(pw))).double()
    x = xp[0].double().cpu() + (xp[1].double().cpu() if split else 0)
    return x @ wd.T


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 77, 128, 300])
def test_linear_store_matches_reference(fmt, m):
    """fp32 store of x W^T with x carried as two bf16 planes (fp32-level precision)."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, n = 1024, 512
    _, xp = _planes(m, k, m)
    pw = W.concat_rows([W.quantize(fmt, _weights(n - 32, k, seed=2).cuda())])   # n_valid < n (padding)
    ref = _reference(xp, pw)[:, : n - 32]
    for fn in ("b200_linear", "b200_linear_simt"):
        out, _ = _linear(fn, xp, pw, _lib.EP_STORE, n_valid=n - 32)
        err = (out.double().cpu() - ref).abs().max().item() / ref.abs().max().item()
        assert err < 2e-5, (fn, err)


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
def test_linear_single_plane(fmt):
    """x_lo = NULL: one bf16 pass."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, n = 2048, 768
    _, xp = _planes(200, k, 9)
    pw = W.concat_rows([W.quantize(fmt, _weights(n, k, seed=3).cuda())])
    ref = _reference(xp, pw, split=False)
    out, _ = _linear("b200_linear", xp, pw, _lib.EP_STORE, split=False)
    assert (out.double().cpu() - ref).abs().max().item() / ref.abs().max().item() < 2e-5


@pytest.mark.parametrize("fmt", ["int4", "ternary", "nvfp4"])
def test_linear_residual_add(fmt):
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, n = 2048, 512
    _, xp = _planes(130, k, 4)
    pw = W.concat_rows([W.quantize(fmt, _weights(n, k, seed=4).cuda())])
    ref = _reference(xp, pw)
    for fn in ("b200_linear", "b200_linear_simt"):
        out, before = _linear(fn, xp, pw, _lib.EP_RESID_ADD)
        got = (out.double() - before.double()).cpu()
        assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item() + 1e-6, fn


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "bf16"])
def test_linear_swiglu(fmt):
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, inter = 1024, 384
    _, xp = _planes(150, k, 5)
    gate = W.quantize(fmt, _weights(inter, k, seed=5).cuda())
    up = W.quantize(fmt, _weights(inter, k, seed=6).cuda())
    pw = W.interleave_gate_up(gate, up)
    ref = torch.nn.functional.silu(_reference(xp, gate)) * _reference(xp, up)
    for fn in ("b200_linear", "b200_linear_simt"):
        out, _ = _linear(fn, xp, pw, _lib.EP_SWIGLU, n_valid=2 * inter)
        got = out[0].double().cpu() + out[1].double().cpu()      # hi + lo planes
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4, fn


@pytest.mark.parametrize("ep", ["store", "resid", "swiglu"])
def test_linear_many_tiles_without_k_split(ep):
    """M large enough that every SM gets whole output tiles: 256-column tiles, no K split
    (the small-M tests above run the split-K and 128-column paths)."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    m, k, n = 2048, 1024, 2560          # 16 x 10 = 160 tiles of 128 x 256
    _, xp = _planes(m, k, 21)
    if ep == "swiglu":
        gate = W.quantize("nvfp4", _weights(n // 2, k, seed=22).cuda())
        up = W.quantize("nvfp4", _weights(n // 2, k, seed=23).cuda())
        pw = W.interleave_gate_up(gate, up)
        ref = torch.nn.functional.silu(_reference(xp, gate)) * _reference(xp, up)
        out, _ = _linear("b200_linear", xp, pw, _lib.EP_SWIGLU, n_valid=n)
        got = out[0].double().cpu() + out[1].double().cpu()
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4
        return
    pw = W.concat_rows([W.quantize("int4", _weights(n, k, seed=24).cuda())])
    ref = _reference(xp, pw)
    out, before = _linear("b200_linear", xp, pw, _lib.EP_STORE if ep == "store" else _lib.EP_RESID_ADD)
    got = out.double().cpu() - (before.double().cpu() if ep == "resid" else 0)
    assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item() + 1e-6


def test_linear_large_k_and_m_tail():
    """K = 6144 (the down projection), M not a multiple of the 128-row tile."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, n = 6144, 512
    _, xp = _planes(333, k, 11)
    pw = W.concat_rows([W.quantize("nvfp4", _weights(n, k, seed=7).cuda())])
    ref = _reference(xp, pw)
    out, _ = _linear("b200_linear", xp, pw, _lib.EP_STORE)
    assert (out.double().cpu() - ref).abs().max().item() / ref.abs().max().item() < 2e-5


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 5, 9, 16, 17, 64, 96, 128])
@pytest.mark.parametrize("ep", ["store", "resid", "swiglu"])
def test_linear_small_m_matches_reference(fmt, m, ep):
    """Batches of at most 16 rows on packed weights run the register-streamed kernel (weights
    decoded in registers into mma.sync A fragments, one or two 8-token tiles, the 8 warps' K
    partials summed in shared memory); 17 to 128 rows run the swap-AB kernel (weights decoded
    into tensor memory as the MMA's 128-row A operand, both activation planes in one B operand
    of N = 2 x 16, 64 or 128 tokens; split K for the store and residual epilogues, whole K with
    the weight ring refilled for the SwiGLU; bf16 weights take the general kernel): fp64 product
    of the same operands, and the CUDA-core cross-check."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k = 2048
    _, xp = _planes(m, k, 40 + m)
    if ep == "swiglu":
        inter = 384
        gate = W.quantize(fmt, _weights(inter, k, seed=41).cuda())
        up = W.quantize(fmt, _weights(inter, k, seed=42).cuda())
        pw = W.interleave_gate_up(gate, up)
        ref = torch.nn.functional.silu(_reference(xp, gate)) * _reference(xp, up)
        for fn in ("b200_linear", "b200_linear_simt"):
            out, _ = _linear(fn, xp, pw, _lib.EP_SWIGLU, n_valid=2 * inter)
            got = out[0].double().cpu() + out[1].double().cpu()
            assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4, fn
        return
    pw = W.concat_rows([W.quantize(fmt, _weights(736, k, seed=43).cuda())])   # 768 rows, 736 valid
    ref = _reference(xp, pw)[:, :736]
    e = _lib.EP_STORE if ep == "store" else _lib.EP_RESID_ADD
    for fn in ("b200_linear", "b200_linear_simt"):
        out, before = _linear(fn, xp, pw, e, n_valid=736)
        got = out.double().cpu() - (before.double().cpu() if ep == "resid" else 0)
        assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item() + 1e-6, fn


@pytest.mark.parametrize("m", [3, 12])
def test_linear_small_m_swiglu_e4m3_low_plane(m):
    """The SwiGLU of a batch of at most 16 rows written with an e4m3 low plane: hi = bf16_rn(h),
    lo byte = e4m3_rn_satfinite((h - hi) 2^6); the planes recombine to the fp64 SwiGLU within the
    e4m3 plane's precision, and the hi plane equals the bf16-low-plane call's hi plane."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, inter = 2048, 768
    _, xp = _planes(m, k, 70 + m)
    gate = W.quantize("nvfp4", _weights(inter, k, seed=71).cuda())
    up = W.quantize("nvfp4", _weights(inter, k, seed=72).cuda())
    pw = W.interleave_gate_up(gate, up)
    ref = torch.nn.functional.silu(_reference(xp, gate)) * _reference(xp, up)
    buf = torch.zeros(3 * m * inter, dtype=torch.uint8, device="cuda")  # hi plane (bf16), then the e4m3 bytes
    hi = buf[: 2 * m * inter].view(torch.bfloat16).view(m, inter)
    lo8 = buf[2 * m * inter:].view(m, inter)
    o = _lib.LinearOut(_lib.EP_SWIGLU, 2 * inter, _lib.ptr(hi), inter, m * inter, 1)
    qw = pw.qweight()
    _lib.call("b200_linear", _lib.ptr(xp[0]), _lib.ptr(xp[1]), m, k, k, _ref(qw), _ref(o), _lib.stream_ptr())
    torch.cuda.synchronize()
    lo = torch.from_numpy(Q.e4m3_decode(lo8.cpu().numpy())).double() / 64.0
    got = hi.double().cpu() + lo
    # bf16 hi plane + e4m3 residual: about 12 significant bits per element
    assert (got - ref).abs().max().item() / ref.abs().max().item() < 3e-4
    out, _ = _linear("b200_linear", xp, pw, _lib.EP_SWIGLU, n_valid=2 * inter)
    assert torch.equal(out[0], hi)


@pytest.mark.parametrize("split", [True, False])
def test_linear_small_m_whole_k_with_weight_ring(split):
    """96 weight tiles of 128 rows leave no room to split K: each CTA streams all 32 k-blocks
    through its weight ring (the refill path), one or two activation planes."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    m, k, n = 9, 2048, 12288
    _, xp = _planes(m, k, 50)
    pw = W.concat_rows([W.quantize("nvfp4", _weights(n, k, seed=51).cuda())])
    ref = _reference(xp, pw, split=split)
    out, _ = _linear("b200_linear", xp, pw, _lib.EP_STORE, split=split)
    assert (out.double().cpu() - ref).abs().max().item() / ref.abs().max().item() < 2e-5


@pytest.mark.parametrize("m,split", [(8, False), (16, True), (32, True), (96, True)])
def test_linear_small_m_ragged_k_ranges(m, split):
    """A down-projection shape (K = 6144, 16 weight tiles): K splits 9 ways into ranges of 10 and
    11 k-blocks, so the two MMA issuers (alternate k-blocks) get ranges of unequal length and
    the activation slots wrap at different points, one or two planes."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    k, n = 6144, 2048
    _, xp = _planes(m, k, 60 + m)
    pw = W.concat_rows([W.quantize("ternary", _weights(n, k, seed=61).cuda())])
    ref = _reference(xp, pw, split=split)
    out, before = _linear("b200_linear", xp, pw, _lib.EP_RESID_ADD, split=split)
    got = out.double().cpu() - before.double().cpu()
    assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item() + 1e-6


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
@pytest.mark.parametrize("ep", ["store", "resid", "swiglu"])
@pytest.mark.parametrize("split", [True, False])
def test_linear_register_path_down_projection(fmt, ep, split):
    """The register-streamed kernel (at most 16 rows) at a down-projection depth: K = 6144 gives
    each of a CTA's 8 warps 12 k-blocks, so the 4-deep weight ring and 2-deep activation ring
    wrap; 13 rows (two token tiles, the second partly past the batch), n_valid below the weight's
    rows, one or two activation planes; fp64 product of the same operands."""
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    m, k = 13, 6144
    _, xp = _planes(m, k, 80)
    if ep == "swiglu":
        inter = 256
        gate = W.quantize(fmt, _weights(inter, k, seed=81).cuda())
        up = W.quantize(fmt, _weights(inter, k, seed=82).cuda())
        pw = W.interleave_gate_up(gate, up)
        ref = torch.nn.functional.silu(_reference(xp, gate, split)) * _reference(xp, up, split)
        out, _ = _linear("b200_linear", xp, pw, _lib.EP_SWIGLU, n_valid=2 * inter, split=split)
        got = out[0].double().cpu() + out[1].double().cpu()
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-4
        return
    pw = W.concat_rows([W.quantize(fmt, _weights(480, k, seed=83).cuda())])   # 512 rows, 480 valid
    ref = _reference(xp, pw, split)[:, :480]
    e = _lib.EP_STORE if ep == "store" else _lib.EP_RESID_ADD
    out, before = _linear("b200_linear", xp, pw, e, n_valid=480, split=split)
    got = out.double().cpu() - (before.double().cpu() if ep == "resid" else 0)
    assert (got - ref).abs().max().item() < 2e-5 * ref.abs().max().item() + 1e-6


def test_linear_rejects_bad_shapes():
    from strands_decider_b200 import _lib
    from strands_decider_b200 import weights as W

    pw = W.concat_rows([W.quantize("int4", _weights(256, 1024).cuda())])
    x = torch.zeros(4, 1000, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, 256, device="cuda")
    o = _lib.LinearOut(0, 256, _lib.ptr(out), 256, 0)
    qw = pw.qweight()
    with pytest.raises(_lib.B200Error) as e:
        _lib.call("b200_linear", _lib.ptr(x), None, 4, 1000, 1000, _ref(qw), _ref(o), _lib.stream_ptr())
    assert e.value.status == 2


# ----------------------------------------------------------------------------- GDN mixer


@pytest.mark.parametrize("batch", ["few", "many", "large"])
def test_gdn_mixer_matches_oracle_chunk_rule(batch):
    """conv + gating + chunked delta rule + gated norm, ragged sequences, against the
    oracle's restatement of TF:462-530 on the same bf16 inputs. A few sequences run on
    clusters of CTAs that split each head's value columns; many run one CTA per head."""
    import torch.nn.functional as F

    from oracle import torso as T
    from strands_decider_b200 import _lib

    H, dk = (16 if batch == "large" else 2), 128
    conv_dim, vdim = 3 * H * dk, H * dk
    g = torch.Generator().manual_seed(0)
    if batch == "few":
        lens = [1, 31, 32, 33, 100]
    elif batch == "many":   # 40 sequences x 2 heads: more CTAs than half the SMs
        lens = [int(x) for x in torch.randint(1, 80, (40,), generator=g)]
    else:   # 4200 tokens x 16 heads: the prep kernel's large-batch form
        lens = [1, 2, 3, 700, 1500, 1994]   # (4200 x 16 >= 64K token-heads: 8 tokens per warp)
    Ttot = sum(lens)
    mix = torch.randn(Ttot, conv_dim + vdim + 2 * H, generator=g)
    ab = mix[:, conv_dim + vdim:]
    conv_w = torch.rand(conv_dim, 4, generator=g) - 0.5
    a_log = torch.log(torch.rand(H, generator=g) * 0.99 + 0.01)
    dt_bias = torch.ones(H)
    norm_w = 1 + 0.1 * torch.randn(dk, generator=g)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    out = torch.zeros(2, Ttot, vdim, dtype=torch.bfloat16, device="cuda")
    keep = [conv_w.cuda(), a_log.cuda(), dt_bias.cuda(), norm_w.cuda()]
    p = _lib.GdnParams(H, 128, 128, 4, 1e-6, *[_lib.ptr(t) for t in keep])
    cu_d = torch.tensor(cu, dtype=torch.int32, device="cuda")
    seqs = _lib.Seqs(len(lens), Ttot, max(lens), _lib.ptr(cu_d), None, None)
    mix_d = mix.cuda()
    scratch = torch.empty(_lib.load().b200_gdn_scratch_floats(H, Ttot), device="cuda")
    _lib.call("b200_gdn_mixer", _ref(p), _ref(seqs), _lib.ptr(mix_d), mix.shape[1], _lib.ptr(out),
              Ttot * vdim, None, 0, _lib.ptr(scratch), _lib.stream_ptr())
    torch.cuda.synchronize()
    got = out[0].float().cpu() + out[1].float().cpu()
    for i, n in enumerate(lens):
        rows = slice(cu[i], cu[i + 1])
        x = mix[rows].float()
        conv = torch.zeros(n, conv_dim)
        xin = torch.cat([torch.zeros(3, conv_dim), x[:, :conv_dim]], 0)
        for j in range(4):
            conv = conv + xin[j:j + n] * conv_w[:, j]
        conv = F.silu(conv)
        q, k, v = conv[:, :H * dk].view(n, H, dk), conv[:, H * dk:2 * H * dk].view(n, H, dk), conv[:, 2 * H * dk:].view(n, H, dk)
        beta = ab[rows, :H].sigmoid()
        gg = -a_log.exp() * F.softplus(ab[rows, H:] + dt_bias)
        o, _ = T.chunk_gated_delta_rule(q, k, v, gg, beta)
        z = x[:, conv_dim:conv_dim + vdim].reshape(-1, dk)
        want = T.gated_rms_norm(o.reshape(-1, dk), z, norm_w, 1e-6).reshape(n, vdim)
        err = (got[rows] - want).abs().max().item() / (want.abs().max().item() + 1e-6)
        assert err < 2e-4, (n, err)


@pytest.mark.parametrize("lens", [[1] * 37, [0, 1, 1, 2, 5, 40]], ids=["single-token", "ragged"])
def test_gdn_recurrent_appends_match_oracle(lens):
    """The token-by-token kernel (what b200_gdn_mixer runs for single-token appends) continues
    every sequence from its pool slot's state and conv history and saves the continued ones
    back into the same slot. Outputs, saved states and saved conv histories against the
    oracle's recurrent rule (TF:314-353) with the gated norm; the chunked kernel on the same
    batch agrees with it, and the automatic choice for one token per sequence is the
    recurrent kernel itself (bit-identical)."""
    import torch.nn.functional as F

    from oracle import torso as T
    from strands_decider_b200 import _lib

    H, dk = 2, 128
    conv_dim, vdim = 3 * H * dk, H * dk
    n = len(lens)
    g = torch.Generator().manual_seed(3)
    Ttot = sum(lens)
    mix = torch.randn(Ttot, conv_dim + vdim + 2 * H, generator=g)
    ab = mix[:, conv_dim + vdim:]
    conv_w = torch.rand(conv_dim, 4, generator=g) - 0.5
    a_log = torch.log(torch.rand(H, generator=g) * 0.99 + 0.01)
    dt_bias = torch.ones(H)
    norm_w = 1 + 0.1 * torch.randn(dk, generator=g)
    state0 = 0.05 * torch.randn(1, n, H, dk, dk, generator=g)
    hist0 = torch.randn(1, n, 3, conv_dim, generator=g)
    cu = [0]
    for m in lens:
        cu.append(cu[-1] + m)
    keep = [conv_w.cuda(), a_log.cuda(), dt_bias.cuda(), norm_w.cuda()]
    p = _lib.GdnParams(H, 128, 128, 4, 1e-6, *[_lib.ptr(t) for t in keep])
    cu_d = torch.tensor(cu, dtype=torch.int32, device="cuda")
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    seqs = _lib.Seqs(n, Ttot, max(lens), _lib.ptr(cu_d), _lib.ptr(slots), _lib.ptr(slots))
    mix_d = mix.cuda()
    slot_len = torch.zeros(n, dtype=torch.int32, device="cuda")
    slot_kv = torch.zeros(n, dtype=torch.int32, device="cuda")

    def run(entry):
        st, hist = state0.cuda(), hist0.cuda()
        pool = _lib.PrefixPool(n, 0, _lib.ptr(slot_len), _lib.ptr(slot_kv), _lib.ptr(st), _lib.ptr(hist), None, None)
        out = torch.zeros(2, Ttot, vdim, dtype=torch.bfloat16, device="cuda")
        scratch = torch.empty(_lib.load().b200_gdn_scratch_floats(H, Ttot), device="cuda")
        _lib.call(entry, _ref(p), _ref(seqs), _lib.ptr(mix_d), mix.shape[1], _lib.ptr(out), Ttot * vdim,
                  _ref(pool), 0, _lib.ptr(scratch), _lib.stream_ptr())
        torch.cuda.synchronize()
        return out.float().cpu(), st.cpu(), hist.cpu()

    out_r, st_r, hist_r = run("b200_gdn_mixer_recurrent")
    got = out_r[0] + out_r[1]
    for i, m in enumerate(lens):
        rows = slice(cu[i], cu[i + 1])
        x = mix[rows].float()
        xin = torch.cat([hist0[0, i], x[:, :conv_dim]], 0)
        conv = torch.zeros(m, conv_dim)
        for j in range(4):
            conv = conv + xin[j:j + m] * conv_w[:, j]
        conv = F.silu(conv)
        q, k, v = conv[:, :H * dk].view(m, H, dk), conv[:, H * dk:2 * H * dk].view(m, H, dk), conv[:, 2 * H * dk:].view(m, H, dk)
        beta = ab[rows, :H].sigmoid()
        gg = -a_log.exp() * F.softplus(ab[rows, H:] + dt_bias)
        o, s_want = T.recurrent_gated_delta_rule(q, k, v, gg, beta, initial_state=state0[0, i])
        err_s = (st_r[0, i] - s_want).abs().max().item() / s_want.abs().max().item()
        assert err_s < 1e-4, (i, m, err_s)
        assert torch.equal(hist_r[0, i], xin[-3:]), (i, m)   # the last 3 raw inputs, bit-exact
        if m:
            z = x[:, conv_dim:conv_dim + vdim].reshape(-1, dk)
            want = T.gated_rms_norm(o.reshape(-1, dk), z, norm_w, 1e-6).reshape(m, vdim)
            err = (got[rows] - want).abs().max().item() / (want.abs().max().item() + 1e-6)
            assert err < 2e-4, (i, m, err)

    out_c, st_c, hist_c = run("b200_gdn_mixer_chunked")
    assert ((out_c[0] + out_c[1]) - got).abs().max().item() < 4e-4 * got.abs().max().item()
    assert (st_c - st_r).abs().max().item() < 5e-4 * st_r.abs().max().item()
    assert torch.equal(hist_c, hist_r)
    if Ttot <= n:
        out_a, st_a, _ = run("b200_gdn_mixer")
        assert torch.equal(out_a, out_r) and torch.equal(st_a, st_r)


@pytest.mark.parametrize("fmt", ["int4", "nvfp4", "ternary"])
def test_tile_weights_layout(fmt):
    """The GEMM's streaming copy holds exactly the canonical bytes, chunked per
    (256-row tile, 64-column stage)."""
    from strands_decider_b200 import weights as W

    n, k = 512, 1024
    pw = W.concat_rows([W.quantize(fmt, _weights(n, k, seed=8).cuda())])
    pw.ensure_tiles()
    torch.cuda.synchronize()
    data = pw.data.cpu().numpy().view(np.uint8).reshape(n, -1)
    rb = data.shape[1] // (k // 64)
    want = data.reshape(n // 256, 256, k // 64, rb).transpose(0, 2, 1, 3).reshape(-1)
    assert np.array_equal(pw.tiles.cpu().numpy(), want)
    if fmt in ("int4", "nvfp4"):
        sc = pw.scales.cpu().numpy().view(np.uint8).reshape(n, -1)
        if fmt == "int4":   # one bf16 scale per 128 columns, repeated for both 64-column stages
            sc = np.repeat(sc.reshape(n, k // 128, 2), 2, axis=1).reshape(n, -1)
        srb = sc.shape[1] // (k // 64)
        want_s = sc.reshape(n // 256, 256, k // 64, srb).transpose(0, 2, 1, 3).reshape(-1)
        assert np.array_equal(pw.tile_scales.cpu().numpy()[: want_s.size], want_s)


@pytest.mark.parametrize("with_prefix", [False, True])
@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("heads", [(8, 2), (4, 4), (8, 1), (6, 2)])
def test_attention_matches_reference(with_prefix, hd, heads):
    """q/k RMSNorm(1+w), partial RoPE, causal GQA softmax over (prefix-pool keys +) own
    keys, times sigmoid(gate) (TF:647-690), ragged lengths around the 64/32 tile sizes.
    Query groups of 4, 1 and 8 heads per kv head run the tcgen05 kernel (128-row tiles of
    32, 128 and 16 positions); 3 runs the mma.sync kernel.

    Three bounds, from tight to loose: (1) the prep kernel's q / k / v (bf16 after norm and
    RoPE, the kernel's storage format) within one bf16 rounding of the fp64 values; (2) the
    attention output within 5e-3 (relative to its max) of fp64 attention over those same bf16
    q / k / v, the remaining error being the bf16 probabilities of the P V product and fp32
    accumulation; (3) end to end against fp64 from the fp32 inputs within 2e-2, which also
    carries the bf16 rounding of q and k into the scores (whole-model parity is checked in
    probabilities elsewhere)."""
    from oracle import torso as OT
    from strands_decider_b200 import _lib, config
    from strands_decider_b200.runtime import rope_tables

    nq, nkv = heads
    spec = {256: config.HYBRID_2B, 128: config.REDUCED_1024, 64: config.TINY}[hd]
    g = torch.Generator().manual_seed(hd)
    lens = [1, 37, 64, 65, 130]
    P = [0, 0, 0, 0, 0] if not with_prefix else [5, 0, 70, 33, 2]
    T = sum(lens)
    cols = 2 * nq * hd + 2 * nkv * hd
    qkv = torch.randn(T, cols, generator=g)
    qn, kn = 0.1 * torch.randn(hd, generator=g), 0.1 * torch.randn(hd, generator=g)
    cos, sin = rope_tables(spec, "cpu")
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    # prefix pool: per-sequence slot i holding P[i] keys (post norm+rope) at offset sum(P[:i])
    kv_cap = max(sum(P), 1)
    kpool = torch.randn(1, kv_cap, nkv, hd, generator=g).to(torch.bfloat16)
    vpool = torch.randn(1, kv_cap, nkv, hd, generator=g).to(torch.bfloat16)
    slot_kv = torch.tensor([sum(P[:i]) for i in range(len(P))], dtype=torch.int32)
    slot_len = torch.tensor(P, dtype=torch.int32)
    dev = {k: v.cuda() for k, v in dict(qkv=qkv, qn=qn, kn=kn, cos=cos, sin=sin, kpool=kpool, vpool=vpool,
                                        slot_kv=slot_kv, slot_len=slot_len).items()}
    cu_d = torch.tensor(cu, dtype=torch.int32, device="cuda")
    pslot = torch.arange(len(lens), dtype=torch.int32, device="cuda") if with_prefix else None
    qb = torch.empty(T, nq, hd, dtype=torch.bfloat16, device="cuda")
    kb = torch.empty(T, nkv, hd, dtype=torch.bfloat16, device="cuda")
    vb = torch.empty_like(kb)
    out = torch.zeros(2, T, nq * hd, dtype=torch.bfloat16, device="cuda")
    p = _lib.AttnParams(nq, nkv, hd, hd // 4, cos.shape[0], 1e-6, _lib.ptr(dev["qn"]), _lib.ptr(dev["kn"]),
                        _lib.ptr(dev["cos"]), _lib.ptr(dev["sin"]))
    seqs = _lib.Seqs(len(lens), T, max(lens), _lib.ptr(cu_d), _lib.ptr(pslot), None)
    pool = _lib.PrefixPool(len(lens), kv_cap, _lib.ptr(dev["slot_len"]), _lib.ptr(dev["slot_kv"]), None, None,
                           _lib.ptr(dev["kpool"]), _lib.ptr(dev["vpool"]))
    _lib.call("b200_attention", _ref(p), _ref(seqs), _lib.ptr(dev["qkv"]), cols, _lib.ptr(qb), _lib.ptr(kb),
              _lib.ptr(vb), _lib.ptr(out), T * nq * hd, _ref(pool) if with_prefix else None, 0, _lib.stream_ptr())
    torch.cuda.synchronize()
    got = (out[0].double() + out[1].double()).cpu()
    cfg = OT.TorsoConfig(vocab=1, hidden=1, inter=1, layer_types=(), gdn_heads=1, attn_heads=nq,
                         attn_kv_heads=nkv, head_dim=hd)
    for i, n in enumerate(lens):
        x = qkv[cu[i]:cu[i + 1]].double()
        qg = x[:, : 2 * nq * hd].view(n, nq, 2 * hd)
        q, gate = qg[..., :hd], qg[..., hd:].reshape(n, -1)
        k = x[:, 2 * nq * hd: 2 * nq * hd + nkv * hd].view(n, nkv, hd)
        v = x[:, 2 * nq * hd + nkv * hd:].view(n, nkv, hd)
        q = OT.rms_norm_1p(q, qn, 1e-6).double()
        k = OT.rms_norm_1p(k, kn, 1e-6).double()
        pos = torch.arange(P[i], P[i] + n)
        q = OT.apply_rope(q, cos[pos].repeat(1, 2).double(), sin[pos].repeat(1, 2).double())
        k = OT.apply_rope(k, cos[pos].repeat(1, 2).double(), sin[pos].repeat(1, 2).double())
        kp = kpool[0, slot_kv[i]:slot_kv[i] + P[i]].double()
        vp = vpool[0, slot_kv[i]:slot_kv[i] + P[i]].double()
        ka, va = torch.cat([kp, k]), torch.cat([vp, v])
        kr, vr = ka.repeat_interleave(nq // nkv, 1), va.repeat_interleave(nq // nkv, 1)
        s = torch.einsum("thd,shd->hts", q, kr) * hd ** -0.5
        s = s.masked_fill((torch.arange(P[i] + n)[None, :] > pos[:, None])[None], float("-inf"))
        o = torch.einsum("hts,shd->thd", s.softmax(-1), vr).reshape(n, -1) * torch.sigmoid(gate)
        err = (got[cu[i]:cu[i + 1]] - o).abs().max().item() / o.abs().max().item()
        assert err < 2e-2, (n, P[i], err)
        # (1) the stored q / k / v are the fp64 values rounded to bf16 (one rounding, 2^-8 relative)
        qd, kd, vd = (t[cu[i]:cu[i + 1]].double().cpu() for t in (qb, kb, vb))
        for stored, exact in ((qd, q), (kd, k), (vd, v)):
            assert ((stored - exact).abs() <= exact.abs() * 2.0 ** -8 + 1e-6).all()
        # (2) attention over exactly the stored bf16 q / k / v and pool keys
        ka, va = torch.cat([kp, kd]), torch.cat([vp, vd])
        kr, vr = ka.repeat_interleave(nq // nkv, 1), va.repeat_interleave(nq // nkv, 1)
        s = torch.einsum("thd,shd->hts", qd, kr) * hd ** -0.5
        s = s.masked_fill((torch.arange(P[i] + n)[None, :] > pos[:, None])[None], float("-inf"))
        o = torch.einsum("hts,shd->thd", s.softmax(-1), vr).reshape(n, -1) * torch.sigmoid(gate)
        err = (got[cu[i]:cu[i + 1]] - o).abs().max().item() / o.abs().max().item()
        assert err < 5e-3, (n, P[i], err)


@pytest.mark.parametrize("rows,hidden", [(5, 2048), (96, 1024), (3000, 2048), (40, 256)])
def test_rmsnorm_planes_match_reference(rows, hidden):
    """Qwen3_5RMSNorm (TF:711-728): x * rsqrt(mean x^2 + eps) * (1 + w), as hi/lo bf16 planes;
    both the block-per-row (few rows) and warp-per-row kernels."""
    from strands_decider_b200 import _lib

    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, hidden, generator=g) * 3
    w = 0.1 * torch.randn(hidden, generator=g)
    out = torch.zeros(2, rows, hidden, dtype=torch.bfloat16, device="cuda")
    xd, wd = x.cuda(), w.cuda()
    _lib.call("b200_rmsnorm", _lib.ptr(xd), rows, hidden, _lib.ptr(wd), 1e-6, _lib.ptr(out), rows * hidden,
              _lib.stream_ptr())
    torch.cuda.synchronize()
    xx = x.double()
    ref = xx * torch.rsqrt(xx.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + w.double())
    got = out[0].double().cpu() + out[1].double().cpu()
    assert (got - ref).abs().max().item() < 1e-5 * ref.abs().max().item()
