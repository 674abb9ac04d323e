// Device-side weight formats: encoders (quantisers) and the unpackers the GEMM runs in
// shared memory. Bit-exact definitions: oracle/quant.py (module docstring).
#pragma once

#include "common.cuh"

namespace sdb {

// ----------------------------------------------------------------------------- e4m3 / e2m1

// fp32 -> e4m3 (fn: bias 7, max 448, no inf), round to nearest even, saturating.
// Every step below is exact in fp32, so the result equals the float64 restatement.
__device__ __forceinline__ uint8_t e4m3_encode(float x) {
  uint8_t sign = x < 0.0f ? 0x80 : 0;
  float a = fabsf(x);
  if (a < 0.015625f) {  // 2^-6: subnormal range, m * 2^-9
    int m = __float2int_rn(a * 512.0f);
    return sign | uint8_t(m);  // m == 8 is exactly the min-normal code 0x08
  }
  int e = int((__float_as_uint(a) >> 23) & 0xFF) - 127;
  float f = (__fmul_rn(a, __uint_as_float(uint32_t(127 - e) << 23)) - 1.0f) * 8.0f;
  int mant = __float2int_rn(f);
  if (mant == 8) {
    e += 1;
    mant = 0;
  }
  if (e > 8 || (e == 8 && mant > 6)) return sign | 0x7E;
  return sign | uint8_t(((e + 7) << 3) | mant);
}

__device__ __forceinline__ float e4m3_decode(uint8_t b) {
  int e = (b >> 3) & 0xF, m = b & 7;
  float v = e == 0 ? float(m) * 0.001953125f : (1.0f + float(m) * 0.125f) * __uint_as_float(uint32_t(e - 7 + 127) << 23);
  return (b & 0x80) ? -v : v;
}

__device__ __forceinline__ uint8_t e2m1_encode(float v) {
  float a = fabsf(v);
  uint8_t c = 0;
  c = a > 0.25f ? 1 : c;
  c = a >= 0.75f ? 2 : c;
  c = a > 1.25f ? 3 : c;
  c = a >= 1.75f ? 4 : c;
  c = a > 2.5f ? 5 : c;
  c = a >= 3.5f ? 6 : c;
  c = a > 5.0f ? 7 : c;
  return (v < 0.0f && c != 0) ? uint8_t(c | 8) : c;
}

__device__ __forceinline__ float e2m1_decode(uint32_t n) {
  // magnitude code c = (e << 1) | m: c = 1 is 0.5, c >= 2 is 2^(e-1) * (1 + m/2)
  const uint32_t c = n & 7;
  uint32_t bits = c >= 2 ? ((((c >> 1) + 126u) << 23) | ((c & 1u) << 22)) : (c ? 0x3F000000u : 0u);
  bits |= (n & 8u) << 28;
  return __uint_as_float(bits);
}

__device__ __forceinline__ float bf16_round(float x) { return bf16_to_f32(f32_to_bf16_rn(x)); }

// Effective NVFP4 block scale: bf16_rn(fp32(e4m3(sb) * gs)).
__device__ __forceinline__ float nvfp4_block_scale(uint8_t sb, float gs) {
  return bf16_round(__fmul_rn(e4m3_decode(sb), gs));
}

// ----------------------------------------------------------------------------- unpackers
// Each produces 8 consecutive bf16 weights (one 16-byte chunk of a 128-byte K row) with
// packed bf16x2 arithmetic. Every product below is a single round-to-nearest-even of an
// exact product, so the results equal the fp32 definitions bit for bit.

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// int4: one word = 8 two's-complement nibbles; s2 = the bf16 group scale in both halves.
// n ^ 8 placed in the mantissa of bf16 128.0 gives 128 + (n ^ 8); minus 136 is q exactly;
// times s is bf16_rn(q * s).
__device__ __forceinline__ uint4 unpack8_int4(uint32_t word, uint32_t s2) {
  const uint32_t x = word ^ 0x88888888u;
  const uint32_t ev = x & 0x0F0F0F0Fu;          // elements 0, 2, 4, 6
  const uint32_t od = (x >> 4) & 0x0F0F0F0Fu;   // elements 1, 3, 5, 7
  const uint32_t t01 = prmt(ev, od, 0x5140);    // elements 0, 1, 2, 3
  const uint32_t t23 = prmt(ev, od, 0x7362);    // elements 4, 5, 6, 7
  const uint32_t K = 0x43434343u, C136 = 0x43084308u;
  uint4 o;
  o.x = bf16x2_mul(bf16x2_sub(prmt(t01, K, 0x4140), C136), s2);
  o.y = bf16x2_mul(bf16x2_sub(prmt(t01, K, 0x4342), C136), s2);
  o.z = bf16x2_mul(bf16x2_sub(prmt(t23, K, 0x4140), C136), s2);
  o.w = bf16x2_mul(bf16x2_sub(prmt(t23, K, 0x4342), C136), s2);
  return o;
}

// NVFP4: one word = 8 e2m1 codes (low nibble first); s2 = the bf16 block scale in both halves.
// The magnitude (3 bits) indexes byte tables of the bf16 encodings of 0, .5, 1, 1.5, 2, 3, 4, 6;
// the sign bit is moved to bit 15 / 31; times s is bf16_rn(e2m1 * s).
__device__ __forceinline__ uint4 unpack8_nvfp4(uint32_t word, uint32_t s2) {
  const uint32_t m = word & 0x77777777u;
  const uint32_t HI_A = 0x3F3F3F00u, HI_B = 0x40404040u, LO_A = 0xC0800000u, LO_B = 0xC0804000u;
  const uint32_t hi03 = prmt(HI_A, HI_B, m), lo03 = prmt(LO_A, LO_B, m);
  const uint32_t hi47 = prmt(HI_A, HI_B, m >> 16), lo47 = prmt(LO_A, LO_B, m >> 16);
  const uint32_t sg = word & 0x88888888u;
  const uint32_t A = sg << 4, B = sg;           // bit 7 of byte j: sign of element 2j (A), 2j+1 (B)
  uint4 o;
  o.x = bf16x2_mul(prmt(lo03, hi03, 0x5140) ^ (prmt(A, B, 0x4000) & 0x80008000u), s2);
  o.y = bf16x2_mul(prmt(lo03, hi03, 0x7362) ^ (prmt(A, B, 0x5111) & 0x80008000u), s2);
  o.z = bf16x2_mul(prmt(lo47, hi47, 0x5140) ^ (prmt(A, B, 0x6222) & 0x80008000u), s2);
  o.w = bf16x2_mul(prmt(lo47, hi47, 0x7362) ^ (prmt(A, B, 0x7333) & 0x80008000u), s2);
  return o;
}

// ternary: 16 bits = 8 two-bit codes (00 = 0, 01 = +1, 11 = -1); `lut` maps a pair's 4 bits
// to the bf16x2 of its two t values; times s (both halves) is exact.
__device__ __forceinline__ uint4 unpack8_ternary(uint32_t bits16, uint32_t s2, const uint32_t* lut) {
  uint4 o;
  o.x = bf16x2_mul(lut[bits16 & 0xF], s2);
  o.y = bf16x2_mul(lut[(bits16 >> 4) & 0xF], s2);
  o.z = bf16x2_mul(lut[(bits16 >> 8) & 0xF], s2);
  o.w = bf16x2_mul(lut[(bits16 >> 12) & 0xF], s2);
  return o;
}

// bf16x2 of the two t values {0, +1, -1} coded by 4 bits (low code first).
__host__ __device__ constexpr uint32_t ternary_pair_bits(uint32_t x) {
  return ((x & 3) == 1 ? 0x3F80u : (x & 3) == 3 ? 0xBF80u : 0u) |
         ((((x >> 2) & 3) == 1 ? 0x3F80u : ((x >> 2) & 3) == 3 ? 0xBF80u : 0u) << 16);
}

// Unpack 32 consecutive weights k0 .. k0+31 (k0 a multiple of 32) of row n into four
// 16-byte chunks. `raw` holds the row's packed bytes for those 32 weights (16 bytes for
// int4 / NVFP4, 8 for ternary), `sc` the raw scale bits the caller loaded:
//   int4: bf16 scale of group k0/128 (low 16 bits)
//   NVFP4: e4m3 scales of blocks k0/16 and k0/16+1 (bytes 0 and 1), gs the row scale
//   ternary: bf16 row scale (low 16 bits)
template <int FMT>
__device__ __forceinline__ void unpack32(const uint4& raw, uint32_t sc, float gs, uint4 (&out)[4],
                                         const uint32_t* lut = nullptr) {
  if constexpr (FMT == B200_W_INT4G128) {
    const uint32_t s2 = (sc & 0xFFFFu) * 0x10001u;
    out[0] = unpack8_int4(raw.x, s2);
    out[1] = unpack8_int4(raw.y, s2);
    out[2] = unpack8_int4(raw.z, s2);
    out[3] = unpack8_int4(raw.w, s2);
  } else if constexpr (FMT == B200_W_NVFP4) {
    const uint32_t s0 = uint32_t(f32_to_bf16_rn(__fmul_rn(e4m3_decode(uint8_t(sc & 0xFF)), gs))) * 0x10001u;
    const uint32_t s1 = uint32_t(f32_to_bf16_rn(__fmul_rn(e4m3_decode(uint8_t((sc >> 8) & 0xFF)), gs))) * 0x10001u;
    out[0] = unpack8_nvfp4(raw.x, s0);
    out[1] = unpack8_nvfp4(raw.y, s0);
    out[2] = unpack8_nvfp4(raw.z, s1);
    out[3] = unpack8_nvfp4(raw.w, s1);
  } else if constexpr (FMT == B200_W_TERNARY) {
    const uint32_t s2 = (sc & 0xFFFFu) * 0x10001u;
    out[0] = unpack8_ternary(raw.x & 0xFFFF, s2, lut);
    out[1] = unpack8_ternary(raw.x >> 16, s2, lut);
    out[2] = unpack8_ternary(raw.y & 0xFFFF, s2, lut);
    out[3] = unpack8_ternary(raw.y >> 16, s2, lut);
  } else {  // bf16: 64 bytes of raw data do not fit `raw`; handled by the caller
    out[0] = out[1] = out[2] = out[3] = make_uint4(0, 0, 0, 0);
  }
}

// Streaming-copy geometry: bytes of one row's 64 columns, and of their scales.
__host__ __device__ constexpr int tile_row_bytes(int fmt) {
  return fmt == B200_W_INT4G128 ? 32 : fmt == B200_W_NVFP4 ? 32 : fmt == B200_W_TERNARY ? 16 : 128;
}
__host__ __device__ constexpr int tile_scale_row_bytes(int fmt) {
  return fmt == B200_W_INT4G128 ? 2 : fmt == B200_W_NVFP4 ? 4 : 0;
}

// Bytes of packed data per 32 weights, and per-row pitch helpers.
__host__ __device__ constexpr int packed_bytes_per32(int fmt) {
  return fmt == B200_W_INT4G128 ? 16 : fmt == B200_W_NVFP4 ? 16 : fmt == B200_W_TERNARY ? 8 : 64;
}

// Load the packed bytes + scale bits for weights [k0, k0+32) of row n.
template <int FMT>
__device__ __forceinline__ void load32(const b200_qweight& w, int n, int k0, uint4& raw, uint32_t& sc, float& gs) {
  const int K = w.k;
  if constexpr (FMT == B200_W_INT4G128) {
    const uint8_t* row = reinterpret_cast<const uint8_t*>(w.data) + size_t(n) * (K / 2);
    raw = __ldg(reinterpret_cast<const uint4*>(row + k0 / 2));
    sc = __ldg(reinterpret_cast<const uint16_t*>(w.scales) + size_t(n) * (K / 128) + k0 / 128);
    gs = 1.0f;
  } else if constexpr (FMT == B200_W_NVFP4) {
    const uint8_t* row = reinterpret_cast<const uint8_t*>(w.data) + size_t(n) * (K / 2);
    raw = __ldg(reinterpret_cast<const uint4*>(row + k0 / 2));
    const uint8_t* srow = reinterpret_cast<const uint8_t*>(w.scales) + size_t(n) * (K / 16) + k0 / 16;
    sc = uint32_t(__ldg(srow)) | (uint32_t(__ldg(srow + 1)) << 8);
    gs = __ldg(w.row_scale + n);
  } else if constexpr (FMT == B200_W_TERNARY) {
    const uint8_t* row = reinterpret_cast<const uint8_t*>(w.data) + size_t(n) * (K / 4);
    uint2 v = __ldg(reinterpret_cast<const uint2*>(row + k0 / 4));
    raw = make_uint4(v.x, v.y, 0, 0);
    sc = __ldg(reinterpret_cast<const uint16_t*>(w.scales) + n);
    gs = 1.0f;
  } else {
    raw = make_uint4(0, 0, 0, 0);
    sc = 0;
    gs = 1.0f;
  }
}

}  // namespace sdb
