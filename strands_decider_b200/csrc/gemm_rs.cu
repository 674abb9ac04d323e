// Quantised linears for batches of at most 16 token rows: the weights stream through
// registers.
//
// At this size a linear is a matrix-vector product. Its cost is reading the packed weight
// once (int4 N = 6144, K = 2048: 6.3 MB, about 1 us of HBM time), and the 16 tokens need
// little arithmetic. The kernel below has no barrier, shared-memory ring or tensor memory on
// its path to the first MMA: every warp loads its own packed weight bytes into registers
// straight from the b200_tile_weights layout, decodes them in registers (the same unpackers,
// so the bf16 weights are bit-exact with b200_dequantize) and feeds them to mma.sync
// m16n8k16 as the A operand, with the tokens as the N = 8 operand. The weights depend on no
// earlier kernel, so each warp issues its first weight loads before the programmatic-launch
// wait, and they overlap the tail of the kernel before it.
//
// Work split: CTA c owns RT 16-row weight tiles (16 output features each) over the whole K;
// its 8 warps take the 64-column k-blocks w, w + 8, w + 16, ... and sum their partials
// through shared memory, so no output is written twice and nothing is zeroed first.
// For the SwiGLU the CTA's two tiles are a gate tile and its up tile (the same 16 features
// of a 64-row gate / 64-row up block), so the CTA applies silu(g) * u itself.
//
// Fragment mapping. Lane (g, t) = (lane / 4, lane % 4) of a warp holds, per 64-column k-block,
// 16 weights of row g and 16 of row g + 8 of its tile: physical columns 16 t .. 16 t + 15 of
// the block (8 bytes of packed int4 / NVFP4, 4 bytes of ternary). Decoded, these are 8 bf16
// pairs per row, P[0..7] and Q[0..7] (pair p = columns 16 t + 2 p, + 1). The k-block's four
// MMAs j = 0..3 use A = {P[2j], Q[2j], P[2j+1], Q[2j+1]}: the MMA's k-slots 2t, 2t+1 are
// columns 16 t + 4 j + {0, 1} and its k-slots 2t + 8, 2t + 9 are columns 16 t + 4 j + {2, 3}.
// The B fragment of token g must follow the same column order, and it does with no shuffle:
// lane (g, t) loads columns 16 t .. 16 t + 15 of its token (32 bytes) and MMA j takes the
// pairs 2j and 2j + 1 of them. A sum over k is the same sum in any column order, so
// y[token][row] = sum_k x[token][k] W[row][k] comes out of the C fragment unchanged.
#include <algorithm>

#include "dequant.cuh"
#include "gemm_epilogue.cuh"

namespace sdb {

constexpr int RS_THREADS = 256;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_MAX_M = 16;
constexpr int RS_BK = 64;     // columns of one k-block (one b200_tile_weights stage)
constexpr int RS_WDEPTH = 4;  // weight k-blocks in flight per warp
constexpr int RS_XDEPTH = 2;  // activation k-blocks in flight per warp

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Streaming loads of packed weights (read once per call: no L1 allocation).
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// One lane's share of one k-block of one row: the packed words of its 16 columns and the raw
// scale bits (int4: the bf16 group scale; NVFP4: the e4m3 scale of its 16-column block;
// ternary: unused, the row scale is loaded once).
struct RsRow {
  uint32_t w0, w1, sc;
};

template <int FMT>
__device__ __forceinline__ RsRow rs_load_row(const b200_qweight& w, int nkb, int kb, int row, int t) {
  const int tn = row >> 8, r = row & 255;
  const size_t chunk = (size_t(tn) * nkb + kb) * 256 + r;
  const uint8_t* tiles = reinterpret_cast<const uint8_t*>(w.tiles);
  const uint8_t* tsc = reinterpret_cast<const uint8_t*>(w.tile_scales);
  RsRow o{0u, 0u, 0u};
  if constexpr (FMT == B200_W_TERNARY) {
    o.w0 = ld_stream_u32(tiles + chunk * 16 + 4 * t);
  } else {
    const uint2 v = ld_stream_u2(tiles + chunk * 32 + 8 * t);
    o.w0 = v.x;
    o.w1 = v.y;
    if constexpr (FMT == B200_W_INT4G128) o.sc = __ldg(reinterpret_cast<const uint16_t*>(tsc) + chunk);
    else o.sc = __ldg(tsc + chunk * 4 + t);
  }
  return o;
}

// The row's 16 columns as 8 bf16 pairs, bit-exact with b200_dequantize. `rs2` is the ternary
// row scale in both halves, `gs` the NVFP4 row scale.
template <int FMT>
__device__ __forceinline__ void rs_decode_row(const RsRow& r, uint32_t rs2, float gs, const uint32_t* lut,
                                              uint32_t (&p)[8]) {
  uint4 a, b;
  if constexpr (FMT == B200_W_INT4G128) {
    const uint32_t s2 = (r.sc & 0xFFFFu) * 0x10001u;
    a = unpack8_int4(r.w0, s2);
    b = unpack8_int4(r.w1, s2);
  } else if constexpr (FMT == B200_W_NVFP4) {
    const uint32_t s2 = uint32_t(f32_to_bf16_rn(__fmul_rn(e4m3_decode(uint8_t(r.sc)), gs))) * 0x10001u;
    a = unpack8_nvfp4(r.w0, s2);
    b = unpack8_nvfp4(r.w1, s2);
  } else {
    a = unpack8_ternary(r.w0 & 0xFFFFu, rs2, lut);
    b = unpack8_ternary(r.w0 >> 16, rs2, lut);
  }
  p[0] = a.x, p[1] = a.y, p[2] = a.z, p[3] = a.w;
  p[4] = b.x, p[5] = b.y, p[6] = b.z, p[7] = b.w;
}

// Columns 16 t .. 16 t + 15 of k-block kb of token `tok` (zeros past the batch): 8 bf16 pairs.
__device__ __forceinline__ void rs_load_x(const uint16_t* x, int ldx, int m, int tok, int kb, int t,
                                          uint32_t (&v)[8]) {
  uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
  if (tok < m) {
    const uint4* p = reinterpret_cast<const uint4*>(x + size_t(tok) * ldx + kb * RS_BK + 16 * t);
    a = p[0];
    b = p[1];
  }
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
  v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// grid: one CTA per group of RT 16-row weight tiles (row0 below); 8 warps over the k-blocks.
// NT8 token tiles of 8 (m <= 8 NT8); SPLIT adds the x_lo plane (a second MMA per A fragment
// into the same accumulator).
template <int FMT, int EP, bool SPLIT, int RT, int NT8>
__global__ void __launch_bounds__(RS_THREADS, 2) gemm_rs_kernel(const uint16_t* __restrict__ x,
                                                             const uint16_t* __restrict__ xl, int ldx,
                                                             const GemmArgs a) {
  static_assert(EP != B200_EP_SWIGLU || RT == 2, "a SwiGLU CTA holds a gate tile and its up tile");
  constexpr int PLANES = SPLIT ? 2 : 1;
  __shared__ float4 red[RS_WARPS][RT][NT8][32];  // each warp's C fragments, summed over the warps
  __shared__ uint32_t lut[16];                   // ternary code pairs -> bf16x2
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nkb = a.k / RS_BK;
  // the first row of tile rt: consecutive tiles, or for the SwiGLU the gate rows 16 j.. of a
  // 128-row (64 gate, 64 up) block and the matching up rows
  int row0[RT];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
    if constexpr (EP == B200_EP_SWIGLU) row0[rt] = (blockIdx.x >> 2) * 128 + rt * 64 + (blockIdx.x & 3) * 16;
    else row0[rt] = (blockIdx.x * RT + rt) * 16;
  }
  if constexpr (FMT == B200_W_TERNARY) {
    if (threadIdx.x < 16) lut[threadIdx.x] = ternary_pair_bits(threadIdx.x);
  }
  // per-row constants: the ternary row scale (bf16 pair), the NVFP4 row scale
  uint32_t rs2[RT][2] = {};
  float gs[RT][2] = {};
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row0[rt] + g + 8 * h;
      if constexpr (FMT == B200_W_TERNARY)
        rs2[rt][h] = uint32_t(__ldg(reinterpret_cast<const uint16_t*>(a.w.scales) + row)) * 0x10001u;
      if constexpr (FMT == B200_W_NVFP4) gs[rt][h] = __ldg(a.w.row_scale + row);
    }
  }

  // this warp's k-blocks: warp, warp + 8, ... (s-th one: warp + 8 s)
  const int ns = warp < nkb ? (nkb - warp + RS_WARPS - 1) / RS_WARPS : 0;
  RsRow wr[RS_WDEPTH][RT][2];
  uint32_t xr[RS_XDEPTH][NT8][PLANES][8];
  float acc[RT][NT8][4] = {};

  auto load_w = [&](RsRow (&dst)[RT][2], int s) {
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h) dst[rt][h] = rs_load_row<FMT>(a.w, nkb, warp + RS_WARPS * s, row0[rt] + g + 8 * h, t);
  };
  auto load_x = [&](uint32_t (&dst)[NT8][PLANES][8], int s) {
#pragma unroll
    for (int i = 0; i < NT8; ++i) {
      rs_load_x(x, ldx, a.m, 8 * i + g, warp + RS_WARPS * s, t, dst[i][0]);
      if constexpr (SPLIT) rs_load_x(xl, ldx, a.m, 8 * i + g, warp + RS_WARPS * s, t, dst[i][PLANES - 1]);
    }
  };

  // the weights first (they depend on no earlier kernel), then wait for the activations
#pragma unroll
  for (int d = 0; d < RS_WDEPTH; ++d)
    if (d < ns) load_w(wr[d], d);
  pdl_wait();
  pdl_trigger();
  __syncthreads();  // the ternary table
#pragma unroll
  for (int d = 0; d < RS_XDEPTH; ++d)
    if (d < ns) load_x(xr[d], d);

  for (int s0 = 0; s0 < ns; s0 += RS_WDEPTH) {
#pragma unroll
    for (int d = 0; d < RS_WDEPTH; ++d) {
      const int s = s0 + d;
      if (s < ns) {
        uint32_t (&xs)[NT8][PLANES][8] = xr[d % RS_XDEPTH];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
          uint32_t p[8], q[8];
          rs_decode_row<FMT>(wr[d][rt][0], rs2[rt][0], gs[rt][0], lut, p);
          rs_decode_row<FMT>(wr[d][rt][1], rs2[rt][1], gs[rt][1], lut, q);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t af[4] = {p[2 * j], q[2 * j], p[2 * j + 1], q[2 * j + 1]};
#pragma unroll
            for (int i = 0; i < NT8; ++i) {
#pragma unroll
              for (int pl = 0; pl < PLANES; ++pl) mma_bf16_16816(acc[rt][i], af, xs[i][pl][2 * j], xs[i][pl][2 * j + 1]);
            }
          }
        }
        if (s + RS_WDEPTH < ns) load_w(wr[d], s + RS_WDEPTH);
        if (s + RS_XDEPTH < ns) load_x(xs, s + RS_XDEPTH);
      }
    }
  }

  // ---- the warps' partial sums -> shared memory -> one thread per (tile, token tile, lane)
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int i = 0; i < NT8; ++i)
      red[warp][rt][i][lane] = make_float4(acc[rt][i][0], acc[rt][i][1], acc[rt][i][2], acc[rt][i][3]);
  __syncthreads();
  const b200_linear_out& o = a.o;
  constexpr int SETS = (EP == B200_EP_SWIGLU ? 1 : RT) * NT8;  // (tile, token tile) pairs summed
  if (threadIdx.x >= SETS * 32) return;
  const int set = threadIdx.x >> 5, rt = set / NT8, i = set % NT8;
  // C fragment of lane (g, t): c0 (row g, token 2t), c1 (row g, 2t + 1), c2 (row g + 8, 2t), c3
  auto sum_set = [&](int r) {
    float4 s = red[0][r][i][lane];
#pragma unroll
    for (int w = 1; w < RS_WARPS; ++w) {
      const float4 v = red[w][r][i][lane];
      s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
    }
    return s;
  };
  const int tok0 = 8 * i + 2 * t;
  if constexpr (EP == B200_EP_SWIGLU) {
    const float4 gsum = sum_set(0), usum = sum_set(1);
    const float gv[4] = {gsum.x, gsum.y, gsum.z, gsum.w}, uv[4] = {usum.x, usum.y, usum.z, usum.w};
    const int f0 = (blockIdx.x >> 2) * 64 + (blockIdx.x & 3) * 16 + g;  // output feature of row g
    uint16_t* dst = reinterpret_cast<uint16_t*>(o.out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = tok0 + (e & 1), f = f0 + 8 * (e >> 1);
      if (tok >= a.m || 2 * f >= o.n_valid) continue;
      const float h = silu_approx(gv[e]) * uv[e];
      const uint16_t hb = f32_to_bf16_rn(h);
      const size_t idx = size_t(tok) * o.ldo + f;
      dst[idx] = hb;
      if (!o.lo_offset) continue;
      if (o.lo_format == B200_LO_E4M3)
        reinterpret_cast<uint8_t*>(dst + o.lo_offset)[idx] = uint8_t(f32x2_to_e4m3x2(lo8_value(h, hb), 0.0f));
      else
        dst[o.lo_offset + idx] = f32_to_bf16_rn(h - bf16_to_f32(hb));
    }
  } else {
    const float4 ssum = sum_set(rt);
    const float yv[4] = {ssum.x, ssum.y, ssum.z, ssum.w};
    float* out = reinterpret_cast<float*>(o.out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = tok0 + (e & 1), row = row0[rt] + g + 8 * (e >> 1);
      if (tok >= a.m || row >= o.n_valid) continue;
      float* p = out + size_t(tok) * o.ldo + row;
      if constexpr (EP == B200_EP_RESID_ADD) *p += yv[e];
      else *p = yv[e];
    }
  }
}

template <int FMT, int EP, bool SPLIT, int RT, int NT8>
static int launch_rs(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  // n_valid rows of 16 RT (the SwiGLU: n_valid / 128 blocks of 4 CTAs, the same count)
  const int grid = (a.o.n_valid + 16 * RT - 1) / (16 * RT);
  SDB_CUDA(launch_pdl(gemm_rs_kernel<FMT, EP, SPLIT, RT, NT8>, dim3(grid), dim3(RS_THREADS), 0, st, x, xl, ldx, a));
  return B200_OK;
}

// Two tiles per CTA when the batch has a second token tile and there are rows enough to keep
// every SM busy (each CTA then reads the activations once for 32 weight rows); one otherwise.
template <int FMT, int EP, bool SPLIT, int NT8>
static int dispatch_rs_rt(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  if constexpr (EP == B200_EP_SWIGLU) {
    return launch_rs<FMT, EP, SPLIT, 2, NT8>(x, xl, ldx, a, st);
  } else {
    if (NT8 == 2 && a.o.n_valid >= 32 * sm_count()) return launch_rs<FMT, EP, SPLIT, 2, NT8>(x, xl, ldx, a, st);
    return launch_rs<FMT, EP, SPLIT, 1, NT8>(x, xl, ldx, a, st);
  }
}

template <int FMT, bool SPLIT>
static int dispatch_rs_ep(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  const bool two = a.m > 8;
  switch (a.o.epilogue) {
    case B200_EP_STORE:
      return two ? dispatch_rs_rt<FMT, B200_EP_STORE, SPLIT, 2>(x, xl, ldx, a, st)
                 : dispatch_rs_rt<FMT, B200_EP_STORE, SPLIT, 1>(x, xl, ldx, a, st);
    case B200_EP_RESID_ADD:
      return two ? dispatch_rs_rt<FMT, B200_EP_RESID_ADD, SPLIT, 2>(x, xl, ldx, a, st)
                 : dispatch_rs_rt<FMT, B200_EP_RESID_ADD, SPLIT, 1>(x, xl, ldx, a, st);
    default:
      return two ? dispatch_rs_rt<FMT, B200_EP_SWIGLU, SPLIT, 2>(x, xl, ldx, a, st)
                 : dispatch_rs_rt<FMT, B200_EP_SWIGLU, SPLIT, 1>(x, xl, ldx, a, st);
  }
}

template <bool SPLIT>
static int dispatch_rs_fmt(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  switch (a.w.format) {
    case B200_W_INT4G128: return dispatch_rs_ep<B200_W_INT4G128, SPLIT>(x, xl, ldx, a, st);
    case B200_W_NVFP4: return dispatch_rs_ep<B200_W_NVFP4, SPLIT>(x, xl, ldx, a, st);
    default: return dispatch_rs_ep<B200_W_TERNARY, SPLIT>(x, xl, ldx, a, st);
  }
}

// Batches b200_linear sends here: at most 16 rows on packed weights.
bool linear_rs(int32_t m, int32_t format) { return m <= RS_MAX_M && format != B200_W_BF16; }

// The caller (b200_linear) has checked the shapes and the streaming copy. The activation rows
// are read 16 bytes at a time: ldx % 8 == 0 and 16-byte aligned planes (b200_linear's rules).
int sdb_linear_rs(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  if (a.m < 1 || a.m > RS_MAX_M) return sdb_fail(B200_ERR_SHAPE, "b200_linear: small-batch path takes 1..16 rows");
  return xl ? dispatch_rs_fmt<true>(x, xl, ldx, a, st) : dispatch_rs_fmt<false>(x, xl, ldx, a, st);
}

}  // namespace sdb
