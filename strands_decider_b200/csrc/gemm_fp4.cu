// Native NVFP4 GEMM (W4A4) on the block-scaled tensor cores: tcgen05.mma kind::mxf4nvf4 with
// e2m1 operands and an unsigned-e4m3 scale per 16 elements of K on both sides.
//
// y[t, n] = gs_w[n] * sum_b (sa[t, b] * sw[n, b] * sum_{i in b} a[t, i] * w[n, i])
// where a / w are e2m1 values, sa / sw their block scales (block b = 16 consecutive k) and gs_w
// the weight's per-tensor fp32 scale (row_scale). The activations carry no tensor scale: their
// block scale is e4m3_rn(amax / 6) of the 16 values, so block maxima from about 2^-9 * 6 up to
// 448 * 6 are representable (b200_quantize_act_nvfp4). The weights are the packed NVFP4 format
// the rest of the library uses (element k in the low nibble of byte k/2 when k is even), read
// by the MMA as they are; only their scales are re-laid out (b200_nvfp4_sf_atoms).
//
// Scale factors reach the MMA through tensor memory. Their layout (the one the block-scaled
// MMA reads after tcgen05.cp.32x128b.warpx4) is built per 128 rows and 64 k as a 512-byte atom:
// byte 16 * (r % 32) + 4 * (r / 32) + j holds the scale of row r, 16-block j (j = 0..3), so
// one 16-byte line carries rows r, r + 32, r + 64, r + 96. A matrix's atoms are stored
// [row tile of 128][k / 64][512 bytes].
//
// Kernel: persistent CTAs over 128 x 128 output tiles (N fastest), 256 k per stage (128 bytes
// of e2m1 per row, 128-byte swizzle), 4 stages, double-buffered accumulators.
//   warp 0      TMA loads of the activation and weight tiles, bulk copies of their scale atoms
//   warp 1      per stage: 8 tcgen05.cp (4 SFA + 4 SFB atoms into the stage's TMEM columns),
//               then 4 block-scaled MMAs (M = 128, N = 128, K = 64)
//   warps 2..5  epilogue: accumulators times gs_w, then the fused store / residual / SwiGLU
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "dequant.cuh"
#include "gemm_epilogue.cuh"

namespace sdb {

constexpr int F4_BM = 128, F4_BN = 128, F4_BK = 256;  // BK in elements (128 bytes of e2m1)
constexpr int F4_STAGES = 4;
constexpr int F4_THREADS = 192;
constexpr int F4_SF_ATOM = 512;                          // bytes: 128 rows x 4 scales
constexpr int F4_TILE_BYTES = F4_BM * F4_BK / 2;         // 16 KB of e2m1 per operand tile and stage
constexpr int F4_SF_STAGE = 4 * F4_SF_ATOM;              // 4 atoms (256 k) per operand and stage
constexpr int F4_STAGE = 2 * F4_TILE_BYTES + 2 * F4_SF_STAGE;
constexpr int F4_SMEM = F4_STAGES * F4_STAGE + 1024 + (2 * F4_STAGES + 4) * 8 + 16;
// TMEM: two accumulators of 128 columns, then per stage 32 columns of scale factors
// (4 SFA atoms x 4 columns, 4 SFB atoms x 4 columns)
constexpr uint32_t F4_TMEM_COLS = 512;
constexpr uint32_t F4_SF_COL0 = 2 * F4_BN;

__host__ __device__ constexpr int sf_atom_offset(int r, int b, int k_blocks16) {
  // row r, 16-block b of a matrix with k_blocks16 = K / 16 blocks per row
  return ((r / 128) * (k_blocks16 / 4) + b / 4) * F4_SF_ATOM + 16 * (r % 32) + 4 * ((r % 128) / 32) + (b % 4);
}

// Instruction descriptor, kind::mxf4nvf4 block16: e2m1 A and B (format 1), unsigned-e4m3
// scales (format 0), both K-major, M x N, scale-factor ids 0, K = 64.
__host__ __device__ constexpr uint32_t umma_idesc_fp4(int M, int N) {
  return (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void umma_fp4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// Shared-memory descriptor of one scale atom as tcgen05.cp reads it: 32 lines of 16 bytes
// (no swizzle), 8-line groups 128 bytes apart.
__device__ __forceinline__ uint64_t sf_atom_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(128 >> 4) << 16) | (uint64_t(128 >> 4) << 32) |
         (uint64_t(1) << 46);
}

// One atom (32 lines x 128 bits) into 4 TMEM columns, copied to all four lane quarters.
__device__ __forceinline__ void tmem_cp_sf_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// ----------------------------------------------------------------------------- quantisers
// Activations: one thread per (row, 16-block). scale byte = e4m3_rn_sat(amax / 6), scale =
// its value, code = e2m1_rn_sat(x / scale) (0 where the scale is 0). Rows m .. round_up(m, 128)
// of the scale atoms are written as zeros (the GEMM reads them for its last row tile).
__global__ void act_nvfp4_kernel(const float* __restrict__ x, int m, int k, int ldx, uint8_t* __restrict__ codes,
                                 uint8_t* __restrict__ sf) {
  pdl_wait();
  pdl_trigger();
  const int nb = k / 16;
  const int rows = (m + 127) / 128 * 128;
  const long idx = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= long(rows) * nb) return;
  const int r = int(idx / nb), b = int(idx % nb);
  uint8_t sb = 0;
  if (r < m) {
    const float4* src = reinterpret_cast<const float4*>(x + size_t(r) * ldx + b * 16);
    float v[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 q = src[i];
      v[4 * i] = q.x;
      v[4 * i + 1] = q.y;
      v[4 * i + 2] = q.z;
      v[4 * i + 3] = q.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    sb = e4m3_encode(__fdiv_rn(amax, 6.0f));
    const float s = e4m3_decode(sb);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t c = s > 0.0f ? e2m1_encode(__fdiv_rn(v[i], s)) : 0u;
      if (i < 8) lo |= c << (4 * i);
      else hi |= c << (4 * (i - 8));
    }
    *reinterpret_cast<uint2*>(codes + size_t(r) * (k / 2) + b * 8) = make_uint2(lo, hi);
  }
  sf[sf_atom_offset(r, b, nb)] = sb;
}

// Row-major block scales [rows][k / 16] -> atoms.
__global__ void sf_atoms_kernel(const uint8_t* __restrict__ scales, int rows, int k, uint8_t* __restrict__ sf) {
  const int nb = k / 16;
  const long idx = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= long(rows) * nb) return;
  const int r = int(idx / nb), b = int(idx % nb);
  sf[sf_atom_offset(r, b, nb)] = scales[idx];
}

// ----------------------------------------------------------------------------- GEMM
struct Fp4Args {
  GemmArgs g;                 // weight (NVFP4: n, k, row_scale), output, m, k
  const uint8_t* sfa;         // activation scale atoms
  const uint8_t* sfb;         // weight scale atoms
};

template <int EP>
__global__ void __launch_bounds__(F4_THREADS, 1)
    gemm_fp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const Fp4Args fa) {
  const GemmArgs& args = fa.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                 // STAGES x 16 KB
  uint8_t* sB = sA + F4_STAGES * F4_TILE_BYTES;       // STAGES x 16 KB
  uint8_t* sSFA = sB + F4_STAGES * F4_TILE_BYTES;     // STAGES x 2 KB
  uint8_t* sSFB = sSFA + F4_STAGES * F4_SF_STAGE;     // STAGES x 2 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + F4_STAGES * F4_SF_STAGE);
  uint64_t* full = bars;                              // [STAGES]
  uint64_t* empty = bars + F4_STAGES;                 // [STAGES]
  uint64_t* acc_full = bars + 2 * F4_STAGES;          // [2]
  uint64_t* acc_empty = acc_full + 2;                 // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = args.k / F4_BK;
  const int n_tiles_n = args.w.n / F4_BN, m_tiles = (args.m + F4_BM - 1) / F4_BM;
  const int n_units = n_tiles_n * m_tiles;
  const int kb16 = args.k / 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < F4_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, F4_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const int nt = u % n_tiles_n, mt = u / n_tiles_n;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % F4_STAGES;
          const uint32_t ph = (it / F4_STAGES) & 1;
          mbar_wait(&empty[s], ph ^ 1, FAULT_GEMM_WAIT_EMPTY);
          mbar_arrive_expect_tx(&full[s], 2 * F4_TILE_BYTES + 2 * F4_SF_STAGE);
          // x coordinates in bytes: kt * 128 (a multiple of 16)
          tma_load_2d(sA + s * F4_TILE_BYTES, &tmA, &full[s], kt * (F4_BK / 2), mt * F4_BM);
          tma_load_2d(sB + s * F4_TILE_BYTES, &tmB, &full[s], kt * (F4_BK / 2), nt * F4_BN);
          // the 4 atoms of 64 k each: contiguous per (row tile, k)
          bulk_load(sSFA + s * F4_SF_STAGE, fa.sfa + (size_t(mt) * (kb16 / 4) + kt * 4) * F4_SF_ATOM, F4_SF_STAGE,
                    &full[s]);
          bulk_load(sSFB + s * F4_SF_STAGE, fa.sfb + (size_t(nt) * (kb16 / 4) + kt * 4) * F4_SF_ATOM, F4_SF_STAGE,
                    &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_fp4(F4_BM, F4_BN);
      uint32_t it = 0, local = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++local) {
        const uint32_t ab = local & 1, aph = (local >> 1) & 1;
        mbar_wait(&acc_empty[ab], aph ^ 1, FAULT_GEMM_WAIT_ACCUM);
        tc_fence_after();
        const uint32_t acc = tmem_base + ab * F4_BN;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % F4_STAGES;
          const uint32_t ph = (it / F4_STAGES) & 1;
          mbar_wait(&full[s], ph, FAULT_GEMM_WAIT_FULL_A);
          tc_fence_after();
          const uint32_t sf_col = tmem_base + F4_SF_COL0 + uint32_t(s) * 32;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tmem_cp_sf_atom(sf_col + j * 4, sf_atom_desc(smem_addr(sSFA + s * F4_SF_STAGE + j * F4_SF_ATOM)));
            tmem_cp_sf_atom(sf_col + 16 + j * 4, sf_atom_desc(smem_addr(sSFB + s * F4_SF_STAGE + j * F4_SF_ATOM)));
          }
          const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * F4_TILE_BYTES));
          const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * F4_TILE_BYTES));
#pragma unroll
          for (int j = 0; j < 4; ++j)  // 64 e2m1 = 32 bytes of K per MMA = +2 in 16-byte units
            umma_fp4(acc, ad + 2 * j, bd + 2 * j, idesc, sf_col + j * 4, sf_col + 16 + j * 4,
                     (kt != 0 || j != 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[ab]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warp (2..5) owns TMEM lanes 32*(warp%4)..+31
    const int q = warp & 3;
    uint32_t local = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++local) {
      const int nt = u % n_tiles_n, mt = u / n_tiles_n;
      const int m0 = mt * F4_BM, n0 = nt * F4_BN;
      const uint32_t ab = local & 1, aph = (local >> 1) & 1;
      mbar_wait(&acc_full[ab], aph, FAULT_GEMM_WAIT_ACCUM);
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tl = tmem_base + ab * F4_BN + (uint32_t(q * 32) << 16);
      if constexpr (EP == B200_EP_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // 128-column block: gate cols 0..63, up cols 64..127
          uint32_t g[32], v[32];
          tmem_ld_32x32b_x32(tl + c * 32, g);
          tmem_ld_32x32b_x32(tl + 64 + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            g[j] = __float_as_uint(__uint_as_float(g[j]) * __ldg(args.w.row_scale + n0 + c * 32 + j));
            v[j] = __float_as_uint(__uint_as_float(v[j]) * __ldg(args.w.row_scale + n0 + 64 + c * 32 + j));
          }
          epilogue_swiglu(args, row, n0 / 2 + c * 32, g, v);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < F4_BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tl + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__uint_as_float(v[j]) * __ldg(args.w.row_scale + n0 + c * 32 + j));
          epilogue_chunk<EP>(args, row, n0 + c * 32, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, F4_TMEM_COLS);
  }
}

}  // namespace sdb

using namespace sdb;

static PFN_cuTensorMapEncodeTiled_v12000 g_encode_fp4 = nullptr;
static std::once_flag g_encode_fp4_once;

// An [rows, cols] uint8 matrix (row pitch `pitch` bytes) as 128-byte x box_rows tiles with
// 128-byte swizzle.
static int make_byte_map(CUtensorMap* map, const void* base, int rows, int cols, size_t pitch, int box_rows) {
  std::call_once(g_encode_fp4_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_fp4 = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode_fp4) return sdb_fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(pitch)};
  cuuint32_t box[2] = {128, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode_fp4(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: tensor map rejected");
}

extern "C" int b200_nvfp4_sf_atom_bytes(int32_t rows, int32_t k, size_t* bytes) {
  if (!bytes || rows <= 0 || k <= 0 || k % 64 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_nvfp4_sf_atom_bytes: bad shape");
  *bytes = size_t((rows + 127) / 128) * (k / 64) * F4_SF_ATOM;
  return B200_OK;
}

extern "C" int b200_quantize_act_nvfp4(const float* x, int32_t m, int32_t k, int32_t ldx, uint8_t* codes,
                                       uint8_t* sf_atoms, b200_stream stream) {
  if (!x || !codes || !sf_atoms) return sdb_fail(B200_ERR_ARG, "b200_quantize_act_nvfp4: null pointer");
  if (m <= 0 || k <= 0 || k % 64 != 0 || ldx < k || ldx % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(codes) & 7))
    return sdb_fail(B200_ERR_SHAPE,
                    "b200_quantize_act_nvfp4: k % 64 == 0, ldx % 4 == 0, x 16-byte and codes 8-byte aligned");
  const long threads = long((m + 127) / 128 * 128) * (k / 16);
  SDB_CUDA(launch_pdl(act_nvfp4_kernel, dim3(unsigned((threads + 255) / 256)), dim3(256), 0,
                      reinterpret_cast<cudaStream_t>(stream), x, m, k, ldx, codes, sf_atoms));
  return B200_OK;
}

extern "C" int b200_nvfp4_sf_atoms(const uint8_t* scales, int32_t rows, int32_t k, uint8_t* sf_atoms,
                                   b200_stream stream) {
  if (!scales || !sf_atoms) return sdb_fail(B200_ERR_ARG, "b200_nvfp4_sf_atoms: null pointer");
  if (rows <= 0 || rows % 128 != 0 || k <= 0 || k % 64 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_nvfp4_sf_atoms: rows % 128 == 0 and k % 64 == 0");
  const long threads = long(rows) * (k / 16);
  sf_atoms_kernel<<<unsigned((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      scales, rows, k, sf_atoms);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

template <int EP>
static int launch_fp4(const CUtensorMap& ma, const CUtensorMap& mb, const Fp4Args& fa, cudaStream_t st) {
  static_assert(F4_SMEM <= 227 * 1024, "FP4 GEMM shared memory exceeds the 227 KB per-CTA limit");
  static DeviceOnce attr;
  const int r = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(gemm_fp4_kernel<EP>, cudaFuncAttributeMaxDynamicSharedMemorySize, F4_SMEM));
    return B200_OK;
  });
  if (r != B200_OK) return r;
  const int units = (fa.g.w.n / F4_BN) * ((fa.g.m + F4_BM - 1) / F4_BM);
  SDB_CUDA(launch_pdl(gemm_fp4_kernel<EP>, dim3(std::min(units, sm_count())), dim3(F4_THREADS), F4_SMEM, st, ma, mb,
                      fa));
  return B200_OK;
}

extern "C" int b200_linear_nvfp4_native(const uint8_t* x_codes, const uint8_t* x_sf, int32_t m, int32_t k,
                                        const b200_qweight* w, const uint8_t* w_sf, const b200_linear_out* out,
                                        b200_stream stream) {
  if (!x_codes || !x_sf || !w || !w_sf || !out || !w->data || !w->row_scale || !out->out)
    return sdb_fail(B200_ERR_ARG, "b200_linear_nvfp4_native: null pointer");
  if (w->format != B200_W_NVFP4) return sdb_fail(B200_ERR_FORMAT, "b200_linear_nvfp4_native: NVFP4 weights only");
  if (m <= 0 || k <= 0 || w->k != k || k % F4_BK != 0 || w->n % F4_BN != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: k % 256 == 0 and n % 128 == 0");
  if (out->n_valid <= 0 || out->n_valid > w->n || out->n_valid % 32 != 0 || out->ldo % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(out->out) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: n_valid % 32, ldo % 8, 16-byte aligned output");
  if (out->epilogue == B200_EP_SWIGLU && (out->n_valid % 128 != 0 || out->lo_offset % 8 != 0))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: SwiGLU needs n_valid % 128 == 0");
  if (out->epilogue != B200_EP_SWIGLU && out->ldo < out->n_valid)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: ldo < n_valid");
  if ((reinterpret_cast<uintptr_t>(x_codes) | reinterpret_cast<uintptr_t>(w->data) |
       reinterpret_cast<uintptr_t>(x_sf) | reinterpret_cast<uintptr_t>(w_sf)) & 15)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_nvfp4_native: operands must be 16-byte aligned");
  CUtensorMap ma, mb;
  if (int rc = make_byte_map(&ma, x_codes, m, k / 2, size_t(k) / 2, F4_BM)) return rc;
  if (int rc = make_byte_map(&mb, w->data, w->n, k / 2, size_t(k) / 2, F4_BN)) return rc;
  Fp4Args fa{GemmArgs{*w, *out, m, k, 1, 1}, x_sf, w_sf};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (out->epilogue) {
    case B200_EP_STORE: return launch_fp4<B200_EP_STORE>(ma, mb, fa, st);
    case B200_EP_RESID_ADD: return launch_fp4<B200_EP_RESID_ADD>(ma, mb, fa, st);
    case B200_EP_SWIGLU: return launch_fp4<B200_EP_SWIGLU>(ma, mb, fa, st);
    default: return sdb_fail(B200_ERR_ARG, "b200_linear_nvfp4_native: unknown epilogue");
  }
}
