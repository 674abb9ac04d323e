// Weight quantisers and the standalone dequantiser (bit-exact to oracle/quant.py).
#include "dequant.cuh"

namespace sdb {

// int4 group-128: one thread per (row, group).
__global__ void quant_int4_kernel(const float* __restrict__ w, int n, int k, uint32_t* __restrict__ data,
                                  uint16_t* __restrict__ scales) {
  const int groups = k / 128;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * groups) return;
  const int row = idx / groups, g = idx % groups;
  const float* src = w + size_t(row) * k + g * 128;
  float amax = 0.0f;
  for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(src[i]));
  const uint16_t sb = f32_to_bf16_rn(__fdiv_rn(amax, 7.0f));
  const float s = bf16_to_f32(sb);
  scales[size_t(row) * groups + g] = sb;
  uint32_t* dst = data + size_t(row) * (k / 8) + g * 16;
  for (int wd = 0; wd < 16; ++wd) {
    uint32_t word = 0;
    for (int j = 0; j < 8; ++j) {
      int q = 0;
      if (s != 0.0f) {
        q = __float2int_rn(__fdiv_rn(src[wd * 8 + j], s));
        q = max(-8, min(7, q));
      }
      word |= (uint32_t(q) & 0xFu) << (4 * j);
    }
    dst[wd] = word;
  }
}

// |x| max of a tensor into *out (non-negative floats order like their bit patterns).
__global__ void absmax_kernel(const float* __restrict__ w, size_t count, unsigned int* __restrict__ out) {
  float m = 0.0f;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < count; i += size_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(w[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// row_scale[0] holds the tensor's |max| as bits; one block turns it into gs and writes gs
// to every row (a single block, so the read of row 0 happens before any write).
__global__ void nvfp4_gs_kernel(float* __restrict__ row_scale, int n) {
  __shared__ float gs_sh;
  if (threadIdx.x == 0) {
    const float amax = __uint_as_float(reinterpret_cast<const unsigned int*>(row_scale)[0]);
    gs_sh = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 2688.0f);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) row_scale[i] = gs_sh;
}

// NVFP4: one thread per (row, 16-block).
__global__ void quant_nvfp4_kernel(const float* __restrict__ w, int n, int k, const float* __restrict__ row_scale,
                                   uint8_t* __restrict__ data, uint8_t* __restrict__ scales) {
  const int blocks = k / 16;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * blocks) return;
  const int row = idx / blocks, b = idx % blocks;
  const float gs = row_scale[row];
  const float* src = w + size_t(row) * k + b * 16;
  float amax_b = 0.0f;
  for (int i = 0; i < 16; ++i) amax_b = fmaxf(amax_b, fabsf(src[i]));
  const uint8_t sb = e4m3_encode(__fdiv_rn(amax_b, __fmul_rn(gs, 6.0f)));
  scales[size_t(row) * blocks + b] = sb;
  const float s = nvfp4_block_scale(sb, gs);
  uint8_t* dst = data + size_t(row) * (k / 2) + b * 8;
  for (int j = 0; j < 8; ++j) {
    uint8_t lo = 0, hi = 0;
    if (s != 0.0f) {
      lo = e2m1_encode(__fdiv_rn(src[2 * j], s));
      hi = e2m1_encode(__fdiv_rn(src[2 * j + 1], s));
    }
    dst[j] = uint8_t(lo | (hi << 4));
  }
}

// ternary: one block per row; absmean accumulated in float64.
__global__ void quant_ternary_kernel(const float* __restrict__ w, int n, int k, uint8_t* __restrict__ data,
                                     uint16_t* __restrict__ scales) {
  const int row = blockIdx.x;
  const float* src = w + size_t(row) * k;
  double acc = 0.0;
  for (int i = threadIdx.x; i < k; i += blockDim.x) acc += double(fabsf(src[i]));
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) t += red[i];
    red[0] = t;
  }
  __syncthreads();
  const uint16_t sb = f32_to_bf16_rn(float(red[0] / double(k)));
  const float s = bf16_to_f32(sb);
  if (threadIdx.x == 0) scales[row] = sb;
  for (int byte = threadIdx.x; byte < k / 4; byte += blockDim.x) {
    uint8_t v = 0;
    for (int j = 0; j < 4; ++j) {
      int t = 0;
      if (s != 0.0f) t = max(-1, min(1, __float2int_rn(__fdiv_rn(src[byte * 4 + j], s))));
      v |= uint8_t((t & 3) << (2 * j));
    }
    data[size_t(row) * (k / 4) + byte] = v;
  }
}

// Standalone dequantiser: one thread per 32 weights, through the GEMM's own unpackers. With
// out8, the two copies of b200_linear_lo8 instead: out = W * 2^B200_LO8_SHIFT (bf16, exact)
// and out8 = e4m3(W * 2^B200_LO8_W_SHIFT).
template <int FMT>
__global__ void dequant_kernel(b200_qweight w, uint16_t* __restrict__ out, uint8_t* __restrict__ out8) {
  __shared__ uint32_t lut[16];
  // the packed weights are constant, but `out` may still be read by the GEMM before this kernel
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  if (threadIdx.x < 16) lut[threadIdx.x] = ternary_pair_bits(threadIdx.x);
  __syncthreads();
  const int per_row = w.k / 32;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= w.n * per_row) return;
  const int row = idx / per_row, k0 = (idx % per_row) * 32;
  uint4 dst[4];
  if constexpr (FMT == B200_W_BF16) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w.data) + size_t(row) * w.k + k0);
    for (int c = 0; c < 4; ++c) dst[c] = src[c];
  } else {
    uint4 raw;
    uint32_t sc;
    float gs;
    load32<FMT>(w, row, k0, raw, sc, gs);
    unpack32<FMT>(raw, sc, gs, dst, lut);
  }
  if (out8) {
    uint16_t* h = reinterpret_cast<uint16_t*>(dst);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = bf16_to_f32(h[4 * i + e]);
      constexpr float ws = float(1 << B200_LO8_W_SHIFT), hs = float(1 << B200_LO8_SHIFT);
      q[i] = e4m3x4(f[0] * ws, f[1] * ws, f[2] * ws, f[3] * ws);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[4 * i + e] = f32_to_bf16_rn(f[e] * hs);  // a power of two: exact
    }
    uint4* o8 = reinterpret_cast<uint4*>(out8 + size_t(row) * w.k + k0);
    o8[0] = make_uint4(q[0], q[1], q[2], q[3]);
    o8[1] = make_uint4(q[4], q[5], q[6], q[7]);
  }
  uint4* o = reinterpret_cast<uint4*>(out + size_t(row) * w.k + k0);
  for (int c = 0; c < 4; ++c) o[c] = dst[c];
}

// Streaming copy for the GEMM: one thread per (row, 64-column stage) copies the row's
// packed bytes of that stage (and its scales) into the stage's contiguous chunk.
__global__ void tile_kernel(b200_qweight w, uint8_t* __restrict__ tiles, uint8_t* __restrict__ tile_scales) {
  const int stages = w.k / 64;
  const long idx = blockIdx.x * long(blockDim.x) + threadIdx.x;
  if (idx >= long(w.n) * stages) return;
  const int row = int(idx / stages), st = int(idx % stages);
  const int tile = row / 256, r = row % 256;
  const size_t chunk = size_t(tile) * stages + st;
  const int rb = tile_row_bytes(w.format);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(w.data) + size_t(row) * (size_t(w.k) * rb / 64) + size_t(st) * rb;
  uint8_t* dst = tiles + (chunk * 256 + r) * rb;
  for (int b = 0; b < rb; b += 4) *reinterpret_cast<uint32_t*>(dst + b) = *reinterpret_cast<const uint32_t*>(src + b);
  if (w.format == B200_W_INT4G128) {
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(w.scales) + size_t(row) * (w.k / 128) + st / 2;
    reinterpret_cast<uint16_t*>(tile_scales)[chunk * 256 + r] = *sc;
  } else if (w.format == B200_W_NVFP4) {
    const uint8_t* sc = reinterpret_cast<const uint8_t*>(w.scales) + size_t(row) * (w.k / 16) + st * 4;
    uint8_t* d = tile_scales + (chunk * 256 + r) * 4;
    for (int b = 0; b < 4; ++b) d[b] = sc[b];
  }
}

}  // namespace sdb

using namespace sdb;

extern "C" int b200_tile_bytes(int32_t format, int32_t n, int32_t k, size_t* tile_bytes, size_t* tile_scale_bytes) {
  if (!tile_bytes || !tile_scale_bytes) return sdb_fail(B200_ERR_ARG, "b200_tile_bytes: null pointer");
  if (n <= 0 || k <= 0 || n % 256 != 0 || k % 128 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_tile_bytes: bad shape");
  if (format < 0 || format > 3) return sdb_fail(B200_ERR_FORMAT, "b200_tile_bytes: unknown format");
  if (format == B200_W_BF16) {
    *tile_bytes = *tile_scale_bytes = 0;
    return B200_OK;
  }
  *tile_bytes = size_t(n) * (k / 64) * tile_row_bytes(format);
  *tile_scale_bytes = size_t(n) * (k / 64) * tile_scale_row_bytes(format);
  return B200_OK;
}

extern "C" int b200_tile_weights(const b200_qweight* w, void* tiles, void* tile_scales, b200_stream stream) {
  if (!w || !w->data) return sdb_fail(B200_ERR_ARG, "b200_tile_weights: null pointer");
  if (w->n % 256 != 0 || w->k % 128 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_tile_weights: bad shape");
  if (w->format == B200_W_BF16) return B200_OK;
  if (!tiles || (tile_scale_row_bytes(w->format) && !tile_scales))
    return sdb_fail(B200_ERR_ARG, "b200_tile_weights: null output");
  const long total = long(w->n) * (w->k / 64);
  tile_kernel<<<int((total + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      *w, reinterpret_cast<uint8_t*>(tiles), reinterpret_cast<uint8_t*>(tile_scales));
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

extern "C" int b200_quantize(int32_t format, const float* w, int32_t n, int32_t k, void* data, void* scales,
                             float* row_scale, b200_stream stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!w || !data || n <= 0 || k <= 0) return sdb_fail(B200_ERR_ARG, "b200_quantize: null pointer or empty shape");
  if (k % 128 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_quantize: k must be a multiple of 128");
  switch (format) {
    case B200_W_INT4G128: {
      if (!scales) return sdb_fail(B200_ERR_ARG, "b200_quantize: int4 needs scales");
      const int total = n * (k / 128);
      quant_int4_kernel<<<(total + 127) / 128, 128, 0, st>>>(w, n, k, reinterpret_cast<uint32_t*>(data),
                                                             reinterpret_cast<uint16_t*>(scales));
      break;
    }
    case B200_W_NVFP4: {
      if (!scales || !row_scale) return sdb_fail(B200_ERR_ARG, "b200_quantize: nvfp4 needs scales and row_scale");
      unsigned int* amax = reinterpret_cast<unsigned int*>(row_scale);
      SDB_CUDA(cudaMemsetAsync(amax, 0, sizeof(unsigned int), st));
      absmax_kernel<<<592, 256, 0, st>>>(w, size_t(n) * k, amax);
      nvfp4_gs_kernel<<<1, 1024, 0, st>>>(row_scale, n);
      const int total = n * (k / 16);
      quant_nvfp4_kernel<<<(total + 127) / 128, 128, 0, st>>>(w, n, k, row_scale, reinterpret_cast<uint8_t*>(data),
                                                              reinterpret_cast<uint8_t*>(scales));
      break;
    }
    case B200_W_TERNARY: {
      if (!scales) return sdb_fail(B200_ERR_ARG, "b200_quantize: ternary needs scales");
      quant_ternary_kernel<<<n, 256, 0, st>>>(w, n, k, reinterpret_cast<uint8_t*>(data),
                                              reinterpret_cast<uint16_t*>(scales));
      break;
    }
    default:
      return sdb_fail(B200_ERR_FORMAT, "b200_quantize: unknown or non-quantised format");
  }
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

static int dequantize(const b200_qweight* w, uint16_t* out, uint8_t* out8, cudaStream_t st) {
  if (!w || !out || !w->data) return sdb_fail(B200_ERR_ARG, "b200_dequantize: null pointer");
  if (w->n <= 0 || w->k <= 0 || w->k % 128 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_dequantize: bad shape");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(out8)) & 15)
    return sdb_fail(B200_ERR_SHAPE, "b200_dequantize: outputs must be 16-byte aligned");
  const int total = w->n * (w->k / 32);
  const dim3 grid((total + 255) / 256), block(256);
  switch (w->format) {
    case B200_W_BF16: SDB_CUDA(launch_pdl(dequant_kernel<B200_W_BF16>, grid, block, 0, st, *w, out, out8)); break;
    case B200_W_INT4G128:
      SDB_CUDA(launch_pdl(dequant_kernel<B200_W_INT4G128>, grid, block, 0, st, *w, out, out8));
      break;
    case B200_W_NVFP4:
      if (!w->row_scale) return sdb_fail(B200_ERR_ARG, "b200_dequantize: nvfp4 needs row_scale");
      SDB_CUDA(launch_pdl(dequant_kernel<B200_W_NVFP4>, grid, block, 0, st, *w, out, out8));
      break;
    case B200_W_TERNARY:
      SDB_CUDA(launch_pdl(dequant_kernel<B200_W_TERNARY>, grid, block, 0, st, *w, out, out8));
      break;
    default: return sdb_fail(B200_ERR_FORMAT, "b200_dequantize: unknown format");
  }
  return B200_OK;
}

extern "C" int b200_dequantize(const b200_qweight* w, uint16_t* out, b200_stream stream) {
  return dequantize(w, out, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b200_dequantize_lo8(const b200_qweight* w, uint16_t* w_hi, uint8_t* w_lo8, b200_stream stream) {
  if (!w_lo8) return sdb_fail(B200_ERR_ARG, "b200_dequantize_lo8: null e4m3 output");
  return dequantize(w, w_hi, w_lo8, reinterpret_cast<cudaStream_t>(stream));
}
