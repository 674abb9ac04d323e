"""Bit-exact numpy restatement of the packed weight formats and their dequantisation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference (strands-decider) has no quantisation code at all: its torso runs the
bf16/fp32 `nn.Linear`s of transformers' Qwen3.5 module (TF:398-420, TF:632-644,
TF:699-703). The formats below are therefore defined here, from the published
descriptions, and this file is the single source of truth that the CUDA quantisers
and the in-kernel unpackers are tested against, bit for bit.

Formats (weights W[N, K], row n = output feature, K contiguous):

int4 group-128, symmetric
    scale[n, g] = bf16_rn(amax(|W[n, 128g:128g+128]|) / 7)          (fp32 divide)
    code[n, k]  = clamp(rint_half_even(W[n, k] / float(scale)), -8, 7)  (fp32 divide),
                  0 where the scale is 0
    packed      int32 [N, K/8]; element k sits in bits 4*(k%8) .. 4*(k%8)+3 of word k/8,
                  as a 4-bit two's-complement value
    dequant     bf16_rn(float(code) * float(scale))

NVFP4 (e2m1 values, e4m3 scale per 16 elements, fp32 per-tensor scale)
    gs          = amax(|W|) / 2688  (= 6 * 448), or 1 if W is all zero     (fp32 divide)
    sb[n, b]    = e4m3_rn_sat(amax(|W[n, 16b:16b+16]|) / fp32(gs * 6))
    scale[n, b] = bf16_rn(fp32(e4m3_value(sb) * gs))      (the block's effective scale)
    code[n, k]  = e2m1_rn_sat(W[n, k] / scale[n, b]), 0 where scale is 0  (fp32 divide)
    packed      uint8 [N, K/2]; element k in the low nibble of byte k/2 when k is even,
                  the high nibble when odd. Nibble = sign(bit 3) | magnitude code(bits 0-2);
                  a value that rounds to zero is stored as +0.
    scales      uint8 [N, K/16] (e4m3 bit patterns), per-tensor scale fp32 (stored per row
                  on the device, constant within one logical tensor)
    dequant     bf16_rn(e2m1_value(code) * scale[n, b])  (the product is exact in fp32)

Ternary (BitNet b1.58 absmean, Ma et al. 2024), per-output-row scale
    scale[n]    = bf16_rn(fp32(mean(|W[n, :]|)))   (mean accumulated in float64)
    t[n, k]     = clamp(rint_half_even(W[n, k] / float(scale[n])), -1, 1), 0 where scale is 0
    packed      uint8 [N, K/4]; element k in bits 2*(k%4) .. 2*(k%4)+1 of byte k/4;
                  00 = 0, 01 = +1, 11 = -1
    dequant     bf16_rn(t * float(scale[n]))  (exact)

bf16_rn is IEEE round-to-nearest-even of an fp32 value to bfloat16.
"""

from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------- bf16


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest, ties to even. In uint32: no
    finite or infinite input overflows (the largest is 0xFF807FFF), and NaNs are replaced."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    r = ((u + bias) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = r.copy()
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 value, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ----------------------------------------------------------------------------- e4m3 / e2m1

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 (fn variant: bias 7, max 448, no inf) bit patterns, RNE, saturating."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = (x < 0).astype(np.uint8) << 7
    a = np.abs(x)
    out = np.zeros(a.shape, dtype=np.uint8)
    sub = a < 2.0 ** -6
    # subnormals: m * 2^-9, m in 0..7; m == 8 rounds up into the first normal (code 0x08)
    m = np.rint(a[sub] / 2.0 ** -9).astype(np.int64)
    out[sub] = m.astype(np.uint8)  # m == 8 -> 0x08 is exactly the min normal encoding
    nrm = ~sub
    an = a[nrm]
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(an)).astype(np.int64)
    # guard log2 rounding at exact powers of two
    e = np.where(an < 2.0 ** e, e - 1, e)
    e = np.where(an >= 2.0 ** (e + 1), e + 1, e)
    mant = np.rint((an / 2.0 ** e - 1.0) * 8.0).astype(np.int64)
    carry = mant == 8
    e = np.where(carry, e + 1, e)
    mant = np.where(carry, 0, mant)
    sat = (e > 8) | ((e == 8) & (mant > 6))
    code = ((e + 7) << 3) | mant
    code = np.where(sat, 0x7E, code)
    out[nrm] = code.astype(np.uint8)
    return out | sign


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e - 7))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return (s * val).astype(np.float32)


def e2m1_encode(v: np.ndarray) -> np.ndarray:
    """fp32 -> e2m1 nibble (sign bit 3, magnitude code bits 0-2), RNE, saturating at 6."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v)
    code = np.zeros(a.shape, dtype=np.uint8)
    code = np.where(a > 0.25, 1, code)
    code = np.where(a >= 0.75, 2, code)
    code = np.where(a > 1.25, 3, code)
    code = np.where(a >= 1.75, 4, code)
    code = np.where(a > 2.5, 5, code)
    code = np.where(a >= 3.5, 6, code)
    code = np.where(a > 5.0, 7, code)
    code = code.astype(np.uint8)
    sign = ((v < 0) & (code != 0)).astype(np.uint8) << 3
    return code | sign


def e2m1_decode(n: np.ndarray) -> np.ndarray:
    n = np.asarray(n, dtype=np.uint8)
    mag = E2M1_VALUES[n & 7]
    return np.where(n & 8, -mag, mag).astype(np.float32)


# ----------------------------------------------------------------------------- int4 g128

INT4_GROUP = 128


def quantize_int4g128(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """W fp32 [N, K] -> (packed int32 [N, K/8], scales bf16 bits uint16 [N, K/128])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % INT4_GROUP == 0
    g = w.reshape(n, k // INT4_GROUP, INT4_GROUP)
    amax = np.abs(g).max(axis=2)
    scale_bits = f32_to_bf16_bits((amax / np.float32(7.0)).astype(np.float32))
    scale = bf16_bits_to_f32(scale_bits)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint((g / scale[:, :, None]).astype(np.float32))
    q = np.where(scale[:, :, None] == 0, 0, q)
    q = np.clip(q, -8, 7).astype(np.int64).reshape(n, k)
    nib = (q & 0xF).astype(np.uint32).reshape(n, k // 8, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    packed = np.bitwise_or.reduce(nib << shifts, axis=2).astype(np.uint32).view(np.int32)
    return packed, scale_bits


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed).view(np.uint32)
    n, kw = p.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    nib = ((p[:, :, None] >> shifts) & 0xF).astype(np.int64)
    q = np.where(nib >= 8, nib - 16, nib)
    return q.reshape(n, kw * 8)


def dequantize_int4g128(packed: np.ndarray, scale_bits: np.ndarray) -> np.ndarray:
    """-> fp32 [N, K] holding the bf16 dequantised values."""
    q = unpack_int4(packed).astype(np.float32)
    n, k = q.shape
    s = bf16_bits_to_f32(scale_bits)
    prod = (q.reshape(n, k // INT4_GROUP, INT4_GROUP) * s[:, :, None]).astype(np.float32)
    return bf16_round(prod.reshape(n, k))


# ----------------------------------------------------------------------------- NVFP4

NVFP4_BLOCK = 16


def nvfp4_global_scale(w: np.ndarray) -> np.float32:
    amax = np.float32(np.abs(np.asarray(w, dtype=np.float32)).max()) if w.size else np.float32(0)
    if amax == 0:
        return np.float32(1.0)
    return np.float32(amax / np.float32(2688.0))


def quantize_nvfp4(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.float32]:
    """W fp32 [N, K] -> (packed uint8 [N, K/2], scales e4m3 uint8 [N, K/16], global scale)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % NVFP4_BLOCK == 0
    gs = nvfp4_global_scale(w)
    b = w.reshape(n, k // NVFP4_BLOCK, NVFP4_BLOCK)
    amax_b = np.abs(b).max(axis=2)
    denom = np.float32(gs * np.float32(6.0))
    sb = e4m3_encode((amax_b / denom).astype(np.float32))
    scale = nvfp4_block_scale(sb, gs)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (b / scale[:, :, None]).astype(np.float32)
    v = np.where(scale[:, :, None] == 0, np.float32(0), v)
    codes = e2m1_encode(v).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, sb, gs


def unpack_nvfp4(packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    n, kb = p.shape
    out = np.empty((n, kb * 2), dtype=np.uint8)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = p >> 4
    return out


def nvfp4_block_scale(sb: np.ndarray, gs) -> np.ndarray:
    """Effective block scale bf16_rn(fp32(e4m3(sb) * gs)) as fp32."""
    return bf16_round((e4m3_decode(sb) * np.float32(gs)).astype(np.float32))


def dequantize_nvfp4_elementwise(packed: np.ndarray, sb: np.ndarray, gs: float) -> np.ndarray:
    """bf16_rn(e2m1_value(code) * scale[n, b]) element by element (the definition)."""
    codes = unpack_nvfp4(packed)
    n, k = codes.shape
    vals = e2m1_decode(codes).reshape(n, k // NVFP4_BLOCK, NVFP4_BLOCK)
    scale = nvfp4_block_scale(sb, gs)
    prod = (vals * scale[:, :, None]).astype(np.float32)
    return bf16_round(prod.reshape(n, k))


def dequantize_nvfp4(packed: np.ndarray, sb: np.ndarray, gs: float) -> np.ndarray:
    """The same values as dequantize_nvfp4_elementwise, table-driven: for one tensor (one gs)
    a value depends only on the (scale byte, code nibble) pair, so the definition is applied
    once to all 256 x 16 pairs and every element is a table lookup. Bit-identical by
    construction; fast enough for billions of weights."""
    codes16 = np.arange(16, dtype=np.uint8)
    pairs = np.repeat(codes16[None, :], 256, axis=0)                       # [256 scale bytes, 16 codes]
    packed_tab = (pairs[:, 0::2] | (pairs[:, 1::2] << 4)).astype(np.uint8)  # [256, 8]: 16 codes per row
    sb_tab = np.arange(256, dtype=np.uint8)[:, None]                        # one block of 16 per row
    lut = dequantize_nvfp4_elementwise(packed_tab, sb_tab, gs).reshape(256 * 16)
    codes = unpack_nvfp4(packed)
    n, k = codes.shape
    sbe = np.repeat(np.ascontiguousarray(sb, dtype=np.uint8).astype(np.uint16), NVFP4_BLOCK, axis=1)
    return lut[sbe * 16 + codes]


# ----------------------------------------------------------------------------- NVFP4 activations (W4A4)
# The block-scaled tensor-core path quantises the activations too. Per row and 16-block of
# an activation x [M, K]: scale byte sb = e4m3_rn_sat(amax / 6) (fp32 divide; no tensor scale),
# code = e2m1_rn_sat(x / e4m3_value(sb)) (fp32 divide), 0 where the scale is 0; packed as the
# weights are. The MMA then forms, in fp32, sum_b sa[t, b] * sw[n, b] * sum e2m1(a) * e2m1(w)
# over each 16-block b, and the epilogue multiplies by the weight's tensor scale: every product
# is exact, so an fp64 sum is the reference (the device differs by fp32 accumulation only).


def quantize_act_nvfp4(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x fp32 [M, K] -> (packed uint8 [M, K/2], scale bytes uint8 [M, K/16])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    assert k % NVFP4_BLOCK == 0
    b = x.reshape(m, k // NVFP4_BLOCK, NVFP4_BLOCK)
    sb = e4m3_encode((np.abs(b).max(axis=2) / np.float32(6.0)).astype(np.float32))
    s = e4m3_decode(sb)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (b / s[:, :, None]).astype(np.float32)
    v = np.where(s[:, :, None] == 0, np.float32(0), v)
    codes = e2m1_encode(v).reshape(m, k)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8), sb


def nvfp4_sf_atoms(scales: np.ndarray) -> np.ndarray:
    """Scale bytes [rows, K/16] -> the 512-byte atoms the block-scaled MMA reads, rows padded
    with zero scales to a multiple of 128: byte 16 (r % 32) + 4 ((r % 128) / 32) + (b % 4) of
    atom [r / 128][b / 4] is the scale of row r, 16-block b."""
    scales = np.asarray(scales, dtype=np.uint8)
    rows, nb = scales.shape
    rp = (rows + 127) // 128 * 128
    pad = np.zeros((rp, nb), np.uint8)
    pad[:rows] = scales
    # [tile, m1, m0, atom, j] -> [tile, atom, m0, m1, j]
    a = pad.reshape(rp // 128, 4, 32, nb // 4, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(a).reshape(-1)


def nvfp4_values(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """e2m1 code x its block's e4m3 scale, exactly, as float64 [rows, K]."""
    codes = unpack_nvfp4(packed)
    rows, k = codes.shape
    v = e2m1_decode(codes).astype(np.float64).reshape(rows, k // NVFP4_BLOCK, NVFP4_BLOCK)
    return (v * e4m3_decode(scales).astype(np.float64)[:, :, None]).reshape(rows, k)


def nvfp4_native_product(act_packed, act_scales, w_packed, w_scales, w_gs) -> np.ndarray:
    """What the block-scaled GEMM computes, in float64: x_q @ w_q^T times the weight's tensor
    scale (w_gs: a scalar or one value per weight row)."""
    y = nvfp4_values(act_packed, act_scales) @ nvfp4_values(w_packed, w_scales).T
    return y * np.asarray(w_gs, dtype=np.float64).reshape(1, -1)


# ----------------------------------------------------------------------------- ternary


def ternary_row_scale(w: np.ndarray) -> np.ndarray:
    """Per-row absmean scale as bf16 bits (mean accumulated in float64)."""
    w = np.asarray(w, dtype=np.float32)
    m = np.abs(w).astype(np.float64).mean(axis=1).astype(np.float32)
    return f32_to_bf16_bits(m)


def pack_ternary(t: np.ndarray) -> np.ndarray:
    t = np.asarray(t, dtype=np.int64)
    n, k = t.shape
    assert k % 4 == 0
    code = (t & 3).astype(np.uint8).reshape(n, k // 4, 4)  # 0->00, 1->01, -1->11
    shifts = (np.arange(4, dtype=np.uint8) * 2)[None, None, :]
    return np.bitwise_or.reduce(code << shifts, axis=2).astype(np.uint8)


def _ternary_byte_table() -> np.ndarray:
    """[256, 4] int8: the four codes of a byte (low bits first), 01 -> +1, 11 -> -1, else 0."""
    c = (np.arange(256, dtype=np.int64)[:, None] >> (2 * np.arange(4))[None, :]) & 3
    return np.where(c == 3, -1, np.where(c == 1, 1, 0)).astype(np.int8)


_TERNARY_BYTES = _ternary_byte_table()


def unpack_ternary(packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    n, kb = p.shape
    return _TERNARY_BYTES[p].reshape(n, kb * 4)


def quantize_ternary(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """W fp32 [N, K] -> (packed uint8 [N, K/4], scales bf16 bits [N])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    sbits = ternary_row_scale(w)
    s = bf16_bits_to_f32(sbits)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.rint((w / s[:, None]).astype(np.float32))
    t = np.where(s[:, None] == 0, 0, t)
    t = np.clip(t, -1, 1).astype(np.int64)
    return pack_ternary(t), sbits


def dequantize_ternary(packed: np.ndarray, sbits: np.ndarray) -> np.ndarray:
    """t * s with t in {-1, 0, +1} and s a bf16 value: already a bf16 value (its bf16 rounding
    is the identity)."""
    t = unpack_ternary(packed).astype(np.float32)
    s = bf16_bits_to_f32(sbits)
    return (t * s[:, None]).astype(np.float32)


# ----------------------------------------------------------------------------- dispatch

FORMATS = ("bf16", "int4", "nvfp4", "ternary")


def dequantize(fmt: str, parts: dict) -> np.ndarray:
    """Dequantise a packed weight given as the dict the product's packers produce."""
    if fmt == "bf16":
        return bf16_bits_to_f32(parts["data"])
    if fmt == "int4":
        return dequantize_int4g128(parts["data"], parts["scales"])
    if fmt == "nvfp4":
        return dequantize_nvfp4(parts["data"], parts["scales"], float(np.asarray(parts["global_scale"]).reshape(-1)[0]))
    if fmt == "ternary":
        return dequantize_ternary(parts["data"], parts["scales"])
    raise ValueError(fmt)


def quantize(fmt: str, w: np.ndarray) -> dict:
    if fmt == "bf16":
        return {"data": f32_to_bf16_bits(w)}
    if fmt == "int4":
        d, s = quantize_int4g128(w)
        return {"data": d, "scales": s}
    if fmt == "nvfp4":
        d, s, g = quantize_nvfp4(w)
        return {"data": d, "scales": s, "global_scale": np.array([g], dtype=np.float32)}
    if fmt == "ternary":
        d, s = quantize_ternary(w)
        return {"data": d, "scales": s}
    raise ValueError(fmt)
