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
// Each produces 8 consecutive bf16 weights (one 16-byte chunk of a 128-byte K row).

// int4: one 32-bit word = 8 nibbles; w = bf16_rn(q * s), s a bf16 value.
__device__ __forceinline__ uint4 unpack8_int4(uint32_t word, float s) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int q0 = int(word << (28 - 8 * j)) >> 28;          // nibble 2j, sign-extended
    int q1 = int(word << (24 - 8 * j)) >> 28;          // nibble 2j+1
    o[j] = pack_bf16x2(__fmul_rn(float(q0), s), __fmul_rn(float(q1), s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// NVFP4: 4 bytes = 8 e2m1 values (low nibble first); s the effective block scale.
__device__ __forceinline__ uint4 unpack8_nvfp4(uint32_t word, float s) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t byte = (word >> (8 * j)) & 0xFF;
    o[j] = pack_bf16x2(__fmul_rn(e2m1_decode(byte & 0xF), s), __fmul_rn(e2m1_decode(byte >> 4), s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ternary: 16 bits = 8 two-bit codes (00 = 0, 01 = +1, 11 = -1); s the row scale.
__device__ __forceinline__ uint4 unpack8_ternary(uint32_t bits16, float s) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t c0 = (bits16 >> (4 * j)) & 3, c1 = (bits16 >> (4 * j + 2)) & 3;
    float t0 = c0 == 1 ? 1.0f : (c0 == 3 ? -1.0f : 0.0f);
    float t1 = c1 == 1 ? 1.0f : (c1 == 3 ? -1.0f : 0.0f);
    o[j] = pack_bf16x2(t0 * s, t1 * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Unpack 32 consecutive weights k0 .. k0+31 (k0 a multiple of 32) of row n into four
// 16-byte chunks. `raw` holds the row's packed bytes for those 32 weights (16 bytes for
// int4 / NVFP4, 8 for ternary), `sc` the raw scale bits the caller loaded:
//   int4: bf16 scale of group k0/128 (low 16 bits)
//   NVFP4: e4m3 scales of blocks k0/16 and k0/16+1 (bytes 0 and 1), gs the row scale
//   ternary: bf16 row scale (low 16 bits)
template <int FMT>
__device__ __forceinline__ void unpack32(const uint4& raw, uint32_t sc, float gs, uint4 (&out)[4]) {
  if constexpr (FMT == B200_W_INT4G128) {
    float s = bf16_to_f32(uint16_t(sc & 0xFFFF));
    out[0] = unpack8_int4(raw.x, s);
    out[1] = unpack8_int4(raw.y, s);
    out[2] = unpack8_int4(raw.z, s);
    out[3] = unpack8_int4(raw.w, s);
  } else if constexpr (FMT == B200_W_NVFP4) {
    float s0 = nvfp4_block_scale(uint8_t(sc & 0xFF), gs);
    float s1 = nvfp4_block_scale(uint8_t((sc >> 8) & 0xFF), gs);
    out[0] = unpack8_nvfp4(raw.x, s0);
    out[1] = unpack8_nvfp4(raw.y, s0);
    out[2] = unpack8_nvfp4(raw.z, s1);
    out[3] = unpack8_nvfp4(raw.w, s1);
  } else if constexpr (FMT == B200_W_TERNARY) {
    float s = bf16_to_f32(uint16_t(sc & 0xFFFF));
    out[0] = unpack8_ternary(raw.x & 0xFFFF, s);
    out[1] = unpack8_ternary(raw.x >> 16, s);
    out[2] = unpack8_ternary(raw.y & 0xFFFF, s);
    out[3] = unpack8_ternary(raw.y >> 16, s);
  } else {  // bf16: 64 bytes of raw data do not fit `raw`; handled by the caller
    out[0] = out[1] = out[2] = out[3] = make_uint4(0, 0, 0, 0);
  }
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
