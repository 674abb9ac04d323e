// Weight-only quantised linear layers on the 5th-generation tensor cores (tcgen05).
//
// y[m, n] = sum_k x[m, k] * W[n, k] with x bf16 and W packed (int4 g128, NVFP4, ternary or
// bf16). One CTA computes a 128 x BN tile (BN = 256 by default) with the accumulator in
// tensor memory:
//   warp 0      one lane issues TMA loads of the x tile (128 rows x 64 k, 128-byte swizzle)
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128, N=BN, K=16) x 4 per stage
//   warps 2..5  unpack the packed weights of the stage to bf16 directly into the same
//               128-byte-swizzled K-major layout the MMA reads, then run the epilogue
//               (TMEM -> registers -> fused op -> global)
// A 4-stage ring of shared-memory stages is guarded by mbarriers: full_a (TMA bytes),
// full_b (128 unpacking threads), empty (tcgen05.commit). Every wait is bounded.
#include <cudaTypedefs.h>

#include <mutex>

#include "dequant.cuh"

namespace sdb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_STAGES = 4;
constexpr int GEMM_THREADS = 192;

struct GemmArgs {
  b200_qweight w;
  b200_linear_out o;
  int m, k;
};

template <int BN>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return GEMM_STAGES * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) + 1024 + (3 * GEMM_STAGES + 1) * 8 + 16;
}

// --------------------------------------------------------------------------- epilogue
template <int EP>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int row, int gcol, const uint32_t (&v)[32]) {
  const b200_linear_out& o = a.o;
  if (row >= a.m || gcol >= o.n_valid) return;
  const int nv = min(32, o.n_valid - gcol);
  if constexpr (EP == B200_EP_STORE) {
    if (gcol >= o.split_n) {
      float* dst = o.out_f32 + size_t(row) * o.ldo_f32 + (gcol - o.split_n);
      if (nv == 32) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          reinterpret_cast<float4*>(dst)[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                          __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
      } else {
        for (int j = 0; j < nv; ++j) dst[j] = __uint_as_float(v[j]);
      }
    } else {
      uint16_t* dst = reinterpret_cast<uint16_t*>(o.out) + size_t(row) * o.ldo + gcol;
      if (nv == 32) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 p;
          p.x = pack_bf16x2(__uint_as_float(v[8 * j + 0]), __uint_as_float(v[8 * j + 1]));
          p.y = pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
          p.z = pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
          p.w = pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
          reinterpret_cast<uint4*>(dst)[j] = p;
        }
      } else {
        for (int j = 0; j < nv; ++j) dst[j] = f32_to_bf16_rn(__uint_as_float(v[j]));
      }
    }
  } else if constexpr (EP == B200_EP_RESID_ADD) {
    float* dst = reinterpret_cast<float*>(o.out) + size_t(row) * o.ldo + gcol;
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
      for (int j = 0; j < nv; ++j) dst[j] += __uint_as_float(v[j]);
    }
  }
}

// SwiGLU: gate chunk g and up chunk u (same 32 intermediate features) -> 32 bf16 outputs.
__device__ __forceinline__ void epilogue_swiglu(const GemmArgs& a, int row, int ocol, const uint32_t (&g)[32],
                                                const uint32_t (&u)[32]) {
  const b200_linear_out& o = a.o;
  if (row >= a.m || 2 * ocol >= o.n_valid) return;
  uint16_t* dst = reinterpret_cast<uint16_t*>(o.out) + size_t(row) * o.ldo + ocol;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = silu(__uint_as_float(g[8 * j + e])) * __uint_as_float(u[8 * j + e]);
    uint4 p;
    p.x = pack_bf16x2(h[0], h[1]);
    p.y = pack_bf16x2(h[2], h[3]);
    p.z = pack_bf16x2(h[4], h[5]);
    p.w = pack_bf16x2(h[6], h[7]);
    reinterpret_cast<uint4*>(dst)[j] = p;
  }
}

// --------------------------------------------------------------------------- B unpack
// Raw packed data for one (row, half) unit: 32 weights.
template <int FMT>
struct Raw32 {
  uint4 d0, d1, d2, d3;  // bf16 needs 64 bytes; the packed formats use d0 only
  uint32_t sc;
  float gs;
};

template <int FMT>
__device__ __forceinline__ void load_unit(const b200_qweight& w, int n, int k0, Raw32<FMT>& r) {
  if constexpr (FMT == B200_W_BF16) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w.data) + size_t(n) * w.k + k0);
    r.d0 = __ldg(src);
    r.d1 = __ldg(src + 1);
    r.d2 = __ldg(src + 2);
    r.d3 = __ldg(src + 3);
    r.sc = 0;
    r.gs = 1.0f;
  } else {
    load32<FMT>(w, n, k0, r.d0, r.sc, r.gs);
  }
}

template <int FMT>
__device__ __forceinline__ void store_unit(uint8_t* sB, int r, int half, const Raw32<FMT>& raw) {
  uint4 out[4];
  if constexpr (FMT == B200_W_BF16) {
    out[0] = raw.d0;
    out[1] = raw.d1;
    out[2] = raw.d2;
    out[3] = raw.d3;
  } else {
    unpack32<FMT>(raw.d0, raw.sc, raw.gs, out);
  }
  uint8_t* rowp = sB + r * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int chunk = half * 4 + c;
    *reinterpret_cast<uint4*>(rowp + ((chunk ^ (r & 7)) << 4)) = out[c];
  }
}

// --------------------------------------------------------------------------- kernel
template <int BN, int FMT, int EP>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  constexpr int B_BYTES = BN * GEMM_BK * 2;
  uint8_t* sA = smem;
  uint8_t* sB = smem + GEMM_STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + GEMM_STAGES * B_BYTES);
  uint64_t* full_a = bars;
  uint64_t* full_b = bars + GEMM_STAGES;
  uint64_t* empty = bars + 2 * GEMM_STAGES;
  uint64_t* accum = bars + 3 * GEMM_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * GEMM_STAGES + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * GEMM_BM;
  const int nk = args.k / GEMM_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMM_STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_b[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % GEMM_STAGES;
        const uint32_t ph = (kt / GEMM_STAGES) & 1;
        mbar_wait(&empty[s], ph ^ 1, FAULT_GEMM_WAIT_EMPTY);
        mbar_arrive_expect_tx(&full_a[s], A_BYTES);
        tma_load_2d(sA + s * A_BYTES, &tmA, &full_a[s], kt * GEMM_BK, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(GEMM_BM, BN);
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % GEMM_STAGES;
        const uint32_t ph = (kt / GEMM_STAGES) & 1;
        mbar_wait(&full_a[s], ph, FAULT_GEMM_WAIT_FULL_A);
        mbar_wait(&full_b[s], ph, FAULT_GEMM_WAIT_FULL_B);
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * A_BYTES));
        const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * B_BYTES));
#pragma unroll
        for (int j = 0; j < GEMM_BK / 16; ++j)  // +32 bytes of K per MMA = +2 in 16-byte units
          umma_bf16(tmem_base, ad + 2 * j, bd + 2 * j, idesc, (kt | j) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
    __syncwarp();
  } else {
    // ---------------- weight unpack producers (128 threads)
    const int t = threadIdx.x - 64;
    constexpr int UNITS = BN * 2 / 128;
    Raw32<FMT> cur[UNITS], nxt[UNITS];
#pragma unroll
    for (int i = 0; i < UNITS; ++i) {
      const int u = t + 128 * i;
      load_unit<FMT>(args.w, n0 + (u >> 1), (u & 1) * 32, cur[i]);
    }
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % GEMM_STAGES;
      const uint32_t ph = (kt / GEMM_STAGES) & 1;
      if (kt + 1 < nk) {
#pragma unroll
        for (int i = 0; i < UNITS; ++i) {
          const int u = t + 128 * i;
          load_unit<FMT>(args.w, n0 + (u >> 1), (kt + 1) * GEMM_BK + (u & 1) * 32, nxt[i]);
        }
      }
      mbar_wait(&empty[s], ph ^ 1, FAULT_GEMM_WAIT_EMPTY);
      uint8_t* stage = sB + s * B_BYTES;
#pragma unroll
      for (int i = 0; i < UNITS; ++i) {
        const int u = t + 128 * i;
        store_unit<FMT>(stage, u >> 1, u & 1, cur[i]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full_b[s]);
#pragma unroll
      for (int i = 0; i < UNITS; ++i) cur[i] = nxt[i];
    }

    // ---------------- epilogue: this warp owns TMEM lanes 32*(warp%4) .. +31
    mbar_wait(accum, 0, FAULT_GEMM_WAIT_ACCUM);
    tc_fence_after();
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const uint32_t tl = tmem_base + (uint32_t(q * 32) << 16);
    if constexpr (EP == B200_EP_SWIGLU) {
#pragma unroll 1
      for (int b = 0; b < BN / 128; ++b) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tl + b * 128 + c * 32, g);
          tmem_ld_32x32b_x32(tl + b * 128 + 64 + c * 32, u);
          tmem_ld_wait();
          epilogue_swiglu(args, row, (n0 + b * 128) / 2 + c * 32, g, u);
        }
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tl + c * 32, v);
        tmem_ld_wait();
        epilogue_chunk<EP>(args, row, n0 + c * 32, v);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

// --------------------------------------------------------------------------- SIMT cross-check
template <int FMT>
__device__ __forceinline__ void load_row32_f32(const b200_qweight& w, int n, int k0, float (&out)[32]) {
  Raw32<FMT> r;
  load_unit<FMT>(w, n, k0, r);
  uint4 u[4];
  if constexpr (FMT == B200_W_BF16) {
    u[0] = r.d0;
    u[1] = r.d1;
    u[2] = r.d2;
    u[3] = r.d3;
  } else {
    unpack32<FMT>(r.d0, r.sc, r.gs, u);
  }
  const uint16_t* h = reinterpret_cast<const uint16_t*>(u);
#pragma unroll
  for (int j = 0; j < 32; ++j) out[j] = bf16_to_f32(h[j]);
}

template <int FMT>
__device__ float simt_dot(const GemmArgs& a, const uint16_t* x, int ldx, int m, int n) {
  float acc = 0.0f;
  for (int k0 = 0; k0 < a.k; k0 += 32) {
    float wv[32];
    load_row32_f32<FMT>(a.w, n, k0, wv);
#pragma unroll
    for (int j = 0; j < 32; ++j) acc = fmaf(bf16_to_f32(x[size_t(m) * ldx + k0 + j]), wv[j], acc);
  }
  return acc;
}

template <int FMT, int EP>
__global__ void gemm_simt_kernel(const uint16_t* __restrict__ x, int ldx, const GemmArgs a) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  const b200_linear_out& o = a.o;
  if (m >= a.m) return;
  if constexpr (EP == B200_EP_SWIGLU) {
    if (2 * n >= o.n_valid) return;
    const int blk = n / 64, i = n % 64;
    const float g = simt_dot<FMT>(a, x, ldx, m, blk * 128 + i);
    const float u = simt_dot<FMT>(a, x, ldx, m, blk * 128 + 64 + i);
    reinterpret_cast<uint16_t*>(o.out)[size_t(m) * o.ldo + n] = f32_to_bf16_rn(silu(g) * u);
  } else {
    if (n >= o.n_valid) return;
    const float y = simt_dot<FMT>(a, x, ldx, m, n);
    if constexpr (EP == B200_EP_STORE) {
      if (n >= o.split_n)
        o.out_f32[size_t(m) * o.ldo_f32 + (n - o.split_n)] = y;
      else
        reinterpret_cast<uint16_t*>(o.out)[size_t(m) * o.ldo + n] = f32_to_bf16_rn(y);
    } else {
      reinterpret_cast<float*>(o.out)[size_t(m) * o.ldo + n] += y;
    }
  }
}

// --------------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static int get_encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? B200_OK : sdb_fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
}

static int make_act_map(CUtensorMap* map, const uint16_t* x, int m, int k, int ldx) {
  if (int rc = get_encode_fn()) return rc;
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
  cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
  cuuint32_t box[2] = {GEMM_BK, GEMM_BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return sdb_fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activation tile");
  return B200_OK;
}

static int check_linear(const uint16_t* x, int m, int k, int ldx, const b200_qweight* w, const b200_linear_out* o) {
  if (!x || !w || !o || !w->data || !o->out) return sdb_fail(B200_ERR_ARG, "b200_linear: null pointer");
  if (m <= 0 || k <= 0) return sdb_fail(B200_ERR_SHAPE, "b200_linear: empty shape");
  if (w->k != k) return sdb_fail(B200_ERR_SHAPE, "b200_linear: x and W disagree on k");
  if (k % 128 != 0 || w->n % 256 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_linear: k % 128 and n % 256 must be 0");
  if (ldx < k || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: x must be 16-byte aligned with ldx a multiple of 8");
  if (o->n_valid <= 0 || o->n_valid > w->n) return sdb_fail(B200_ERR_SHAPE, "b200_linear: bad n_valid");
  if (o->ldo % 8 != 0 || (reinterpret_cast<uintptr_t>(o->out) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: out must be 16-byte aligned with ldo a multiple of 8");
  if (o->epilogue == B200_EP_STORE && o->split_n < o->n_valid) {
    if (!o->out_f32 || o->split_n % 32 != 0 || o->ldo_f32 % 4 != 0 || (reinterpret_cast<uintptr_t>(o->out_f32) & 15))
      return sdb_fail(B200_ERR_SHAPE, "b200_linear: split store needs aligned out_f32, split_n % 32 == 0");
  }
  if (o->epilogue == B200_EP_SWIGLU && o->n_valid % 128 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: SwiGLU needs n_valid % 128 == 0");
  if (o->epilogue == B200_EP_RESID_ADD && o->n_valid % 32 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: residual add needs n_valid % 32 == 0");
  if (o->epilogue < 0 || o->epilogue > 2) return sdb_fail(B200_ERR_ARG, "b200_linear: unknown epilogue");
  if (w->format < 0 || w->format > 3) return sdb_fail(B200_ERR_FORMAT, "b200_linear: unknown weight format");
  if (w->format != B200_W_BF16 && !w->scales) return sdb_fail(B200_ERR_ARG, "b200_linear: missing scales");
  if (w->format == B200_W_NVFP4 && !w->row_scale) return sdb_fail(B200_ERR_ARG, "b200_linear: missing row_scale");
  return B200_OK;
}

template <int BN, int FMT, int EP>
static int launch_tc(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  constexpr int smem = gemm_smem_bytes<BN>();
  static bool attr_set = false;  // per instantiation; set before first launch on this device
  if (!attr_set) {
    SDB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, FMT, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  dim3 grid(a.w.n / BN, (a.m + GEMM_BM - 1) / GEMM_BM);
  gemm_tc_kernel<BN, FMT, EP><<<grid, GEMM_THREADS, smem, st>>>(map, a);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

template <int FMT>
static int dispatch_ep(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  switch (a.o.epilogue) {
    case B200_EP_STORE: return launch_tc<256, FMT, B200_EP_STORE>(map, a, st);
    case B200_EP_RESID_ADD: return launch_tc<256, FMT, B200_EP_RESID_ADD>(map, a, st);
    default: return launch_tc<256, FMT, B200_EP_SWIGLU>(map, a, st);
  }
}

template <int FMT>
static int dispatch_simt(const uint16_t* x, int ldx, const GemmArgs& a, cudaStream_t st) {
  const int ncols = a.o.epilogue == B200_EP_SWIGLU ? a.o.n_valid / 2 : a.o.n_valid;
  dim3 grid((ncols + 127) / 128, a.m);
  switch (a.o.epilogue) {
    case B200_EP_STORE: gemm_simt_kernel<FMT, B200_EP_STORE><<<grid, 128, 0, st>>>(x, ldx, a); break;
    case B200_EP_RESID_ADD: gemm_simt_kernel<FMT, B200_EP_RESID_ADD><<<grid, 128, 0, st>>>(x, ldx, a); break;
    default: gemm_simt_kernel<FMT, B200_EP_SWIGLU><<<grid, 128, 0, st>>>(x, ldx, a); break;
  }
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace sdb

using namespace sdb;

extern "C" int b200_linear(const uint16_t* x, int32_t m, int32_t k, int32_t ldx, const b200_qweight* w,
                           const b200_linear_out* out, b200_stream stream) {
  if (int rc = check_linear(x, m, k, ldx, w, out)) return rc;
  CUtensorMap map;
  if (int rc = make_act_map(&map, x, m, k, ldx)) return rc;
  GemmArgs a{*w, *out, m, k};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (w->format) {
    case B200_W_BF16: return dispatch_ep<B200_W_BF16>(map, a, st);
    case B200_W_INT4G128: return dispatch_ep<B200_W_INT4G128>(map, a, st);
    case B200_W_NVFP4: return dispatch_ep<B200_W_NVFP4>(map, a, st);
    default: return dispatch_ep<B200_W_TERNARY>(map, a, st);
  }
}

extern "C" int b200_linear_simt(const uint16_t* x, int32_t m, int32_t k, int32_t ldx, const b200_qweight* w,
                                const b200_linear_out* out, b200_stream stream) {
  if (int rc = check_linear(x, m, k, ldx, w, out)) return rc;
  GemmArgs a{*w, *out, m, k};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (w->format) {
    case B200_W_BF16: return dispatch_simt<B200_W_BF16>(x, ldx, a, st);
    case B200_W_INT4G128: return dispatch_simt<B200_W_INT4G128>(x, ldx, a, st);
    case B200_W_NVFP4: return dispatch_simt<B200_W_NVFP4>(x, ldx, a, st);
    default: return dispatch_simt<B200_W_TERNARY>(x, ldx, a, st);
  }
}
