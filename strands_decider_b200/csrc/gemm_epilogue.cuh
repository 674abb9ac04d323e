// Shared by the GEMM kernels (gemm.cu, gemm_fp4.cu): the launch arguments and the fused
// epilogues that turn 32 consecutive fp32 accumulators of one output row into the layer's
// output (fp32 store, residual add, split-K partial, or SwiGLU into the next GEMM's planes).
#pragma once

#include "common.cuh"

namespace sdb {

struct GemmArgs {
  b200_qweight w;
  b200_linear_out o;
  int m, k;
  int ksplit;  // > 1: each output tile is summed from ksplit K-ranges by fp32 atomic adds
  int ngroup;  // CTA pairs: N tiles per group (units walk all row tiles of one group, then the next)
  int tile_m;  // small-M kernel: token rows per activation plane (m rounded up to 16)
  int xslots;  // small-M kernel: activation k-blocks held in shared memory at once
  int accs;    // small-M kernel: TMEM accumulators (= MMA-issuing threads), 1 or 2
};

// --------------------------------------------------------------------------- epilogue
// One thread holds 32 consecutive fp32 accumulators of its row.
template <int EP>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int row, int gcol, const uint32_t (&v)[32]) {
  const b200_linear_out& o = a.o;
  if (row >= a.m || gcol >= o.n_valid) return;
  const int nv = min(32, o.n_valid - gcol);
  float* dst = reinterpret_cast<float*>(o.out) + size_t(row) * o.ldo + gcol;
  if constexpr (EP == B200_EP_STORE) {
    if (nv == 32) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<float4*>(dst)[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                        __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) dst[j] = __uint_as_float(v[j]);
    }
  } else if constexpr (EP == B200_EP_RESID_ADD) {
    if (nv == 32) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 r = reinterpret_cast<float4*>(dst)[j];
        r.x += __uint_as_float(v[4 * j]);
        r.y += __uint_as_float(v[4 * j + 1]);
        r.z += __uint_as_float(v[4 * j + 2]);
        r.w += __uint_as_float(v[4 * j + 3]);
        reinterpret_cast<float4*>(dst)[j] = r;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) dst[j] += __uint_as_float(v[j]);
    }
  }
}

// Split-K partial: out[row, gcol..] += v (fp32 atomic adds; the store epilogue's output was
// zeroed before the launch, the residual epilogue adds into the residual itself).
__device__ __forceinline__ void epilogue_chunk_atomic(const GemmArgs& a, int row, int gcol, const uint32_t (&v)[32]) {
  const b200_linear_out& o = a.o;
  if (row >= a.m || gcol >= o.n_valid) return;
  const int nv = min(32, o.n_valid - gcol);
  float* dst = reinterpret_cast<float*>(o.out) + size_t(row) * o.ldo + gcol;
  if (nv == 32) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + 4 * j), "r"(v[4 * j]), "r"(v[4 * j + 1]),
                   "r"(v[4 * j + 2]), "r"(v[4 * j + 3])
                   : "memory");
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) atomicAdd(dst + j, __uint_as_float(v[j]));
  }
}

// PL_LO8 accumulates y * 2^B200_LO8_SHIFT: scale 32 accumulators back (exact).
__device__ __forceinline__ void lo8_unscale(uint32_t (&v)[32]) {
  constexpr float s = 1.0f / float(1 << B200_LO8_SHIFT);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * s);
}

// hi = bf16_rn(x), lo = bf16_rn(x - hi): the two planes of an fp32 activation.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  lo = lo_pair(a, b, hi);
}

// SwiGLU: gate chunk g and up chunk u (same 32 intermediate features) -> 32 outputs as
// hi/lo bf16 planes.
__device__ __forceinline__ void epilogue_swiglu(const GemmArgs& a, int row, int ocol, const uint32_t (&g)[32],
                                                const uint32_t (&u)[32]) {
  const b200_linear_out& o = a.o;
  if (row >= a.m || 2 * ocol >= o.n_valid) return;
  uint16_t* dst = reinterpret_cast<uint16_t*>(o.out) + size_t(row) * o.ldo + ocol;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = silu_approx(__uint_as_float(g[8 * j + e])) * __uint_as_float(u[8 * j + e]);
    uint4 hi, lo;
    split_bf16x2(h[0], h[1], hi.x, lo.x);
    split_bf16x2(h[2], h[3], hi.y, lo.y);
    split_bf16x2(h[4], h[5], hi.z, lo.z);
    split_bf16x2(h[6], h[7], hi.w, lo.w);
    reinterpret_cast<uint4*>(dst)[j] = hi;
    if (!o.lo_offset) continue;
    if (o.lo_format == B200_LO_E4M3) {
      const uint16_t* hb = reinterpret_cast<const uint16_t*>(&hi);
      float l[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) l[e] = lo8_value(h[e], hb[e]);
      // the e4m3 plane: one byte per element at the hi plane's element index
      uint8_t* lo8 = reinterpret_cast<uint8_t*>(reinterpret_cast<uint16_t*>(o.out) + o.lo_offset) +
                     size_t(row) * o.ldo + ocol;
      reinterpret_cast<uint2*>(lo8)[j] = make_uint2(e4m3x4(l[0], l[1], l[2], l[3]), e4m3x4(l[4], l[5], l[6], l[7]));
    } else {
      reinterpret_cast<uint4*>(dst + o.lo_offset)[j] = lo;
    }
  }
}

}  // namespace sdb
