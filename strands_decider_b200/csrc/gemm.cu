// Weight-only quantised linear layers on the 5th-generation tensor cores (tcgen05).
//
// y[m, n] = sum_k x[m, k] * W[n, k] with W packed (int4 g128, NVFP4, ternary or bf16) and x
// held as two bf16 planes x_hi + x_lo (fp32-level precision). A persistent CTA per SM walks
// 128 x BN output tiles (BN = 256, N fastest so concurrent CTAs share activation tiles),
// with two accumulators in tensor memory (2 x 256 columns) so the epilogue of one tile
// overlaps the main loop of the next:
//   warp 0      one lane streams each stage: TMA loads of the x tiles (128 rows x 64 k
//               per plane, 128-byte swizzle) and bulk copies of the stage's packed weight
//               chunk and scales (the b200_tile_weights layout); bf16 weights come as a
//               swizzled TMA tile straight into the B stage
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128, N=BN, K=16): per 16 k,
//               one MMA for x_hi and one for x_lo against the same weight tile
//   warps 2..5  epilogue: TMEM -> registers -> fused op -> global, one TMEM lane quarter each
//   warps 6..13 unpack the stage's packed weights from shared memory to bf16, directly into
//               the 128-byte-swizzled K-major layout the MMA reads
// A 3-stage ring of shared-memory stages is guarded by mbarriers: full_a (activation TMA
// bytes), full_w (packed weight bytes), full_b (256 unpacking threads), empty
// (tcgen05.commit); the two accumulators by acc_full (tcgen05.commit) and acc_empty (the 4
// epilogue warps). Every wait is bounded.
//
// The e4m3-low-plane form (PL_LO8, bf16 weight copies only): the low activation plane is
// e4m3(lo * 2^6) and meets an e4m3 copy of W * 2^6, while the hi plane meets W * 2^12 in bf16,
// so both products share one accumulator at scale 2^12 (undone in the epilogue). Per 64 k:
// four bf16 MMAs (K = 16) and two e4m3 MMAs (K = 32, 64-byte swizzled tiles) instead of
// eight bf16 MMAs.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "dequant.cuh"
#include "gemm_epilogue.cuh"

namespace sdb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
// warp 0 streams stages, warp 1 issues MMAs, warps 2..5 run the epilogue (one per TMEM lane
// quarter), warps 6..13 unpack weights
constexpr int GEMM_THREADS = 448;
constexpr int GEMM_UNPACK_THREADS = 256;
constexpr int GEMM_EPI_WARP0 = 2;
constexpr int GEMM_UNPACK_WARP0 = 6;

// Shared-memory stages: 3 of 72 KB for 256-column tiles, 4 of 52 KB for 128-column tiles
// (the narrow tiles serve small M, where the depth hides the weights' HBM latency).
constexpr int gemm_stages(int bn) { return bn == 128 ? 4 : 3; }
// Packed weight tiles are prefetched into L2 this many k-blocks ahead of the copy into a stage.
constexpr int GEMM_L2_AHEAD = 6;

// activation planes: hi only, hi + bf16 lo, hi + e4m3 lo (the last with bf16 weights only)
constexpr int PL_ONE = 0, PL_SPLIT = 1, PL_LO8 = 2;

constexpr int GEMM_TILE_ROWS = 256;  // rows of one b200_tile_weights tile (a 128-column tile reads half of one)

// Work unit u -> output tile (m0, n0) and its K range [kb0, kb1) in GEMM_BK blocks. N is
// fastest so the CTAs running at one time share activation tiles; then the K split.
struct GemmUnit {
  int m0, n0, kb0, kb1;
};
template <int BN>
__device__ __forceinline__ GemmUnit gemm_unit(const GemmArgs& a, int u, int nk) {
  const int n_tiles_n = a.w.n / BN;
  const int nt = u % n_tiles_n, rest = u / n_tiles_n;
  const int ks = rest % a.ksplit, mt = rest / a.ksplit;
  return {mt * GEMM_BM, nt * BN, ks * nk / a.ksplit, (ks + 1) * nk / a.ksplit};
}

template <int BN, int FMT, int PL>
struct GemmSmem {
  static_assert(PL != PL_LO8 || FMT == B200_W_BF16, "the e4m3 low plane pairs with bf16 weight copies");
  static constexpr bool PACKED = FMT != B200_W_BF16;
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;          // the hi activation plane
  static constexpr int A_LO_BYTES = PL == PL_SPLIT ? A_BYTES : PL == PL_LO8 ? GEMM_BM * GEMM_BK : 0;
  static constexpr int A_STAGE = A_BYTES + A_LO_BYTES;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;               // unpacked bf16 weight tile
  static constexpr int B8_BYTES = PL == PL_LO8 ? BN * GEMM_BK : 0;  // e4m3 weight tile
  static constexpr int W_BYTES = PACKED ? BN * tile_row_bytes(FMT) : 0;
  static constexpr int S_BYTES = BN * tile_scale_row_bytes(FMT);
  static constexpr int STAGE = A_STAGE + B_BYTES + B8_BYTES + W_BYTES + S_BYTES;
  static constexpr int STAGES = gemm_stages(BN);
  static constexpr int BARS = 4 * STAGES + 4;
  static constexpr int TOTAL = STAGES * STAGE + 1024 + BARS * 8 + 16 + 64;
};

// --------------------------------------------------------------------------- B unpack
// Raw packed data for one (row, half) unit: 32 weights.
template <int FMT>
struct Raw32 {
  uint4 d0;
  uint32_t sc;
  float gs;
};
template <>
struct Raw32<B200_W_BF16> {
  uint4 d0, d1, d2, d3;  // 64 bytes of bf16
};

template <int FMT>
__device__ __forceinline__ void load_unit(const b200_qweight& w, int n, int k0, Raw32<FMT>& r) {
  if constexpr (FMT == B200_W_BF16) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w.data) + size_t(n) * w.k + k0);
    r.d0 = __ldg(src);
    r.d1 = __ldg(src + 1);
    r.d2 = __ldg(src + 2);
    r.d3 = __ldg(src + 3);
  } else {
    load32<FMT>(w, n, k0, r.d0, r.sc, r.gs);
  }
}

template <int FMT>
__device__ __forceinline__ void unit_values(const Raw32<FMT>& raw, uint4 (&out)[4], const uint32_t* lut) {
  if constexpr (FMT == B200_W_BF16) {
    out[0] = raw.d0;
    out[1] = raw.d1;
    out[2] = raw.d2;
    out[3] = raw.d3;
  } else {
    unpack32<FMT>(raw.d0, raw.sc, raw.gs, out, lut);
  }
}

// Unpack unit (row r, half h) of a stage from its shared-memory chunk into the swizzled
// B tile. `rowc` is the per-row constant (ternary scale bits / NVFP4 row scale).
template <int FMT>
__device__ __forceinline__ void unpack_unit_regs(const uint8_t* sW, const uint8_t* sS, int r, int h, uint32_t row_sc,
                                                 float row_gs, const uint32_t* lut, uint4 (&out)[4]) {
  constexpr int RB = tile_row_bytes(FMT);
  uint4 raw;
  if constexpr (FMT == B200_W_TERNARY) {
    const uint2 v = *reinterpret_cast<const uint2*>(sW + r * RB + h * 8);
    raw = make_uint4(v.x, v.y, 0, 0);
  } else {
    raw = *reinterpret_cast<const uint4*>(sW + r * RB + h * 16);
  }
  uint32_t sc;
  if constexpr (FMT == B200_W_INT4G128) sc = *reinterpret_cast<const uint16_t*>(sS + r * 2);
  else if constexpr (FMT == B200_W_NVFP4) sc = *reinterpret_cast<const uint16_t*>(sS + r * 4 + h * 2);
  else sc = row_sc;
  unpack32<FMT>(raw, sc, row_gs, out, lut);
}

template <int FMT>
__device__ __forceinline__ void unpack_unit_smem(uint8_t* sB, const uint8_t* sW, const uint8_t* sS, int r, int h,
                                                 uint32_t row_sc, float row_gs, const uint32_t* lut) {
  uint4 out[4];
  unpack_unit_regs<FMT>(sW, sS, r, h, row_sc, row_gs, lut, out);
  uint8_t* rowp = sB + r * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int chunk = h * 4 + c;
    *reinterpret_cast<uint4*>(rowp + ((chunk ^ (r & 7)) << 4)) = out[c];
  }
}

// --------------------------------------------------------------------------- kernel
template <int BN, int FMT, int EP, int PL>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB8,
                   const GemmArgs args) {
  using SM = GemmSmem<BN, FMT, PL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                   // STAGES x A_STAGE
  uint8_t* sB = sA + SM::STAGES * SM::A_STAGE;         // STAGES x B_BYTES
  uint8_t* sB8 = sB + SM::STAGES * SM::B_BYTES;        // STAGES x B8_BYTES (PL_LO8)
  uint8_t* sW = sB8 + SM::STAGES * SM::B8_BYTES;       // STAGES x W_BYTES
  uint8_t* sS = sW + SM::STAGES * SM::W_BYTES;         // STAGES x S_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sS + SM::STAGES * SM::S_BYTES);
  uint64_t* full_a = bars;
  uint64_t* full_w = bars + SM::STAGES;
  uint64_t* full_b = bars + 2 * SM::STAGES;
  uint64_t* empty = bars + 3 * SM::STAGES;
  uint64_t* acc_full = bars + 4 * SM::STAGES;       // [2]
  uint64_t* acc_empty = bars + 4 * SM::STAGES + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + SM::BARS);
  uint32_t* lut = tmem_slot + 4;  // 16 words: ternary pair table

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = args.k / GEMM_BK;
  const int n_units = (args.w.n / BN) * ((args.m + GEMM_BM - 1) / GEMM_BM) * args.ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SM::STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_w[s], 1);
      mbar_init(&full_b[s], GEMM_UNPACK_THREADS / 32);  // one arrival per unpack warp
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_fence_init();
  }
  if (threadIdx.x < 16) lut[threadIdx.x] = ternary_pair_bits(threadIdx.x);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above touched only this CTA's shared memory and tensor memory: with PDL it
  // overlapped the previous kernel's tail; from here on inputs and outputs are shared
  pdl_wait();
  // With one unit per CTA (small M) the next kernel may be scheduled now, so its launch
  // overlaps this one. A persistent multi-unit grid lets it start only at exit: its CTAs
  // would otherwise sit on the SMs for the whole GEMM and slow it.
  if (n_units <= int(gridDim.x)) pdl_trigger();

  if (warp == 0) {
    // ---------------- producer: activations (TMA) and packed weights (bulk copies)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      if constexpr (PL != PL_ONE) tma_prefetch_desc(&tmA_lo);
      if constexpr (!SM::PACKED) tma_prefetch_desc(&tmB);
      if constexpr (PL == PL_LO8) tma_prefetch_desc(&tmB8);
      constexpr int RB = SM::PACKED ? tile_row_bytes(FMT) : 0, SB = tile_scale_row_bytes(FMT);
      const uint64_t keep = l2_evict_last_policy();  // weight tiles: re-read for every row tile
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const GemmUnit w = gemm_unit<BN>(args, u, nk);
        const int m0 = w.m0, n0 = w.n0;
        // this tile's rows inside the 256-row streaming tiles: tile n0 / 256, row offset n0 % 256
        const size_t lt = size_t(n0 / GEMM_TILE_ROWS) * nk, sub = n0 % GEMM_TILE_ROWS;
        const uint8_t* wtiles = reinterpret_cast<const uint8_t*>(args.w.tiles) + sub * RB;
        const uint8_t* stiles = reinterpret_cast<const uint8_t*>(args.w.tile_scales) + sub * SB;
        if constexpr (SM::PACKED) {
          for (int kt = w.kb0; kt < min(w.kb1, w.kb0 + GEMM_L2_AHEAD); ++kt)
            bulk_prefetch_l2(wtiles + (lt + kt) * GEMM_TILE_ROWS * RB, SM::W_BYTES);
        }
        for (int kt = w.kb0; kt < w.kb1; ++kt, ++it) {
          const int s = it % SM::STAGES;
          const uint32_t ph = (it / SM::STAGES) & 1;
          if constexpr (SM::PACKED) {
            if (kt + GEMM_L2_AHEAD < w.kb1)
              bulk_prefetch_l2(wtiles + (lt + kt + GEMM_L2_AHEAD) * GEMM_TILE_ROWS * RB, SM::W_BYTES);
          }
          mbar_wait(&empty[s], ph ^ 1, FAULT_GEMM_WAIT_EMPTY);
          if constexpr (SM::PACKED) {
            mbar_arrive_expect_tx(&full_w[s], SM::W_BYTES + SM::S_BYTES);
            bulk_load(sW + s * SM::W_BYTES, wtiles + (lt + kt) * GEMM_TILE_ROWS * RB, SM::W_BYTES, &full_w[s]);
            if constexpr (SM::S_BYTES > 0)
              bulk_load(sS + s * SM::S_BYTES, stiles + (lt + kt) * GEMM_TILE_ROWS * SB, SM::S_BYTES, &full_w[s]);
          }
          mbar_arrive_expect_tx(&full_a[s], SM::A_STAGE + (SM::PACKED ? 0 : SM::B_BYTES) + SM::B8_BYTES);
          tma_load_2d(sA + s * SM::A_STAGE, &tmA, &full_a[s], kt * GEMM_BK, m0);
          // (an e4m3 tile's x coordinate is in bytes = elements: kt * 64, a multiple of 16)
          if constexpr (PL != PL_ONE)
            tma_load_2d(sA + s * SM::A_STAGE + SM::A_BYTES, &tmA_lo, &full_a[s], kt * GEMM_BK, m0);
          if constexpr (!SM::PACKED) tma_load_2d_hint(sB + s * SM::B_BYTES, &tmB, &full_a[s], kt * GEMM_BK, n0, keep);
          if constexpr (PL == PL_LO8)
            tma_load_2d_hint(sB8 + s * SM::B8_BYTES, &tmB8, &full_a[s], kt * GEMM_BK, n0, keep);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(GEMM_BM, BN);
      constexpr uint32_t idesc8 = umma_idesc_e4m3(GEMM_BM, BN);
      uint32_t it = 0, local = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++local) {
        const GemmUnit w = gemm_unit<BN>(args, u, nk);
        const uint32_t ab = local & 1, aph = (local >> 1) & 1;
        mbar_wait(&acc_empty[ab], aph ^ 1, FAULT_GEMM_WAIT_ACCUM);
        tc_fence_after();
        const uint32_t acc = tmem_base + ab * BN;
        for (int kt = w.kb0; kt < w.kb1; ++kt, ++it) {
          const int s = it % SM::STAGES;
          const uint32_t ph = (it / SM::STAGES) & 1;
          mbar_wait(&full_a[s], ph, FAULT_GEMM_WAIT_FULL_A);
          if constexpr (SM::PACKED) mbar_wait(&full_b[s], ph, FAULT_GEMM_WAIT_FULL_B);
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * SM::A_STAGE));
          const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * SM::B_BYTES));
#pragma unroll
          for (int j = 0; j < GEMM_BK / 16; ++j) {  // +32 bytes of K per MMA = +2 in 16-byte units
            umma_bf16(acc, ad + 2 * j, bd + 2 * j, idesc, (kt != w.kb0 || j != 0) ? 1u : 0u);
            if constexpr (PL == PL_SPLIT) umma_bf16(acc, ad + (SM::A_BYTES >> 4) + 2 * j, bd + 2 * j, idesc, 1u);
          }
          if constexpr (PL == PL_LO8) {  // 64-byte e4m3 rows: K = 32 per MMA, +32 bytes = +2
            const uint64_t ald = umma_desc_sw64(smem_addr(sA + s * SM::A_STAGE + SM::A_BYTES));
            const uint64_t bld = umma_desc_sw64(smem_addr(sB8 + s * SM::B8_BYTES));
#pragma unroll
            for (int j = 0; j < GEMM_BK / 32; ++j) umma_e4m3(acc, ald + 2 * j, bld + 2 * j, idesc8, 1u);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[ab]);
      }
    }
    __syncwarp();
  } else if (warp < GEMM_UNPACK_WARP0) {
    // ---------------- epilogue: warp (2..5) owns TMEM lanes 32*(warp%4)..+31, all columns
    const int q = warp & 3;
    uint32_t local = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++local) {
      const GemmUnit w = gemm_unit<BN>(args, u, nk);
      const int m0 = w.m0, n0 = w.n0;
      const uint32_t ab = local & 1, aph = (local >> 1) & 1;
      mbar_wait(&acc_full[ab], aph, FAULT_GEMM_WAIT_ACCUM);
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tl = tmem_base + ab * BN + (uint32_t(q * 32) << 16);
      if constexpr (EP == B200_EP_SWIGLU) {
#pragma unroll 1
        for (int b = 0; b < BN / 128; ++b) {  // 128-column block: gate cols 0..63, up cols 64..127
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t g[32], u[32];
            tmem_ld_32x32b_x32(tl + b * 128 + c * 32, g);
            tmem_ld_32x32b_x32(tl + b * 128 + 64 + c * 32, u);
            tmem_ld_wait();
            if constexpr (PL == PL_LO8) {
              lo8_unscale(g);
              lo8_unscale(u);
            }
            epilogue_swiglu(args, row, (n0 + b * 128) / 2 + c * 32, g, u);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tl + c * 32, v);
          tmem_ld_wait();
          if constexpr (PL == PL_LO8) lo8_unscale(v);
          if (args.ksplit > 1) epilogue_chunk_atomic(args, row, n0 + c * 32, v);
          else epilogue_chunk<EP>(args, row, n0 + c * 32, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  } else {
    // ---------------- weight unpack (256 threads): shared chunk -> swizzled bf16 tile
    if constexpr (SM::PACKED) {
      const int t = threadIdx.x - GEMM_UNPACK_WARP0 * 32;
      constexpr int UNITS = BN * 2 / GEMM_UNPACK_THREADS;
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const GemmUnit w = gemm_unit<BN>(args, u, nk);
        const int n0 = w.n0;
        uint32_t row_sc[UNITS];
        float row_gs[UNITS];
#pragma unroll
        for (int i = 0; i < UNITS; ++i) {
          const int r = (t + GEMM_UNPACK_THREADS * i) >> 1;
          row_sc[i] =
              FMT == B200_W_TERNARY ? uint32_t(__ldg(reinterpret_cast<const uint16_t*>(args.w.scales) + n0 + r)) : 0u;
          row_gs[i] = FMT == B200_W_NVFP4 ? __ldg(args.w.row_scale + n0 + r) : 1.0f;
        }
        for (int kt = w.kb0; kt < w.kb1; ++kt, ++it) {
          const int s = it % SM::STAGES;
          const uint32_t ph = (it / SM::STAGES) & 1;
          mbar_wait(&full_w[s], ph, FAULT_GEMM_WAIT_FULL_W);
          uint8_t* stage = sB + s * SM::B_BYTES;
#pragma unroll
          for (int i = 0; i < UNITS; ++i) {
            const int u = t + GEMM_UNPACK_THREADS * i;
            unpack_unit_smem<FMT>(stage, sW + s * SM::W_BYTES, sS + s * SM::S_BYTES, u >> 1, u & 1, row_sc[i],
                                  row_gs[i], lut);
          }
          // each thread makes its own stores visible to the tensor cores; then one arrival
          // per warp (256 arrivals on one barrier would serialise for hundreds of cycles)
          fence_proxy_async_smem();
          __syncwarp();
          if ((threadIdx.x & 31) == 0) mbar_arrive(&full_b[s]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// --------------------------------------------------------------------------- CTA pairs
// Large M with bf16 weight copies (the dequantised path, hi + bf16 or e4m3 lo planes): a
// cluster of two CTAs computes 256 x 256 tiles with tcgen05.mma.cta_group::2 (M = 256). Each
// CTA stages its own 128 activation rows and its half (128 rows) of the weight tile; the
// leader CTA's MMAs read both CTAs' shared memory at the same offsets, and each CTA's tensor
// memory holds its 128 accumulator rows x 256 columns (x 2 buffers). Per FLOP every SM then
// streams and reads half the weight bytes of a one-CTA 128 x 256 tile, which is what bounds
// the one-CTA kernel here (shared-memory operand traffic, not the tensor pipe's rate).
//   warp 0 (both CTAs)   one lane streams the stage: TMA loads signalled on the leader's
//                        full barrier (the leader also posts the pair's expected bytes)
//   warp 1 (leader)      one lane issues the pair MMAs; commits release both CTAs' stage
//                        (empty) and accumulator (acc_full) barriers
//   warps 2..5 (both)    epilogue of the CTA's 128 rows; one arrival per warp on the
//                        leader's acc_empty (8 per tile)
constexpr int GEMM2_THREADS = 192;
constexpr int GEMM2_STAGES = 4;

template <int PL>
struct Gemm2Smem {
  static constexpr int A_BYTES = 128 * GEMM_BK * 2;
  static constexpr int A_LO_BYTES = PL == PL_SPLIT ? A_BYTES : PL == PL_LO8 ? 128 * GEMM_BK : 0;
  static constexpr int A_STAGE = A_BYTES + A_LO_BYTES;
  static constexpr int B_BYTES = 128 * GEMM_BK * 2;                 // this CTA's half of the bf16 weight tile
  static constexpr int B8_BYTES = PL == PL_LO8 ? 128 * GEMM_BK : 0;  // and of the e4m3 copy
  static constexpr int STAGE = A_STAGE + B_BYTES + B8_BYTES;
  static constexpr int STAGES = GEMM2_STAGES;
  static constexpr int BARS = 2 * STAGES + 4;
  static constexpr int TOTAL = STAGES * STAGE + 1024 + BARS * 8 + 16;
};

template <int EP, int PL>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM2_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA_lo,
                     const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB8,
                     const GemmArgs args) {
  using SM = Gemm2Smem<PL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                              // STAGES x A_STAGE
  uint8_t* sB = sA + SM::STAGES * SM::A_STAGE;    // STAGES x B_BYTES
  uint8_t* sB8 = sB + SM::STAGES * SM::B_BYTES;   // STAGES x B8_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB8 + SM::STAGES * SM::B8_BYTES);
  uint64_t* full = bars;                           // [STAGES], the leader's are used
  uint64_t* empty = bars + SM::STAGES;             // [STAGES], both CTAs'
  uint64_t* acc_full = bars + 2 * SM::STAGES;      // [2], both CTAs'
  uint64_t* acc_empty = bars + 2 * SM::STAGES + 2; // [2], the leader's are used
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + SM::BARS);

  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = args.k / GEMM_BK;
  const int n_tiles_n = args.w.n / 256, m_tiles = (args.m + 255) / 256;
  const int n_units = n_tiles_n * m_tiles;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  // unit -> (row tile, column tile): groups of ngroup column tiles, row tiles within a group,
  // so the weight rows a group re-reads stay in L2 while the activations stream past
  const int G = args.ngroup;
  auto tile_of = [&](int u, int& mt, int& nt) {
    const int g = u / (G * m_tiles), r = u - g * G * m_tiles;
    const int gs = min(G, n_tiles_n - g * G);
    mt = r / gs;
    nt = g * G + r % gs;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SM::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  if (n_units <= n_pairs) pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      if constexpr (PL != PL_ONE) tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB);
      if constexpr (PL == PL_LO8) tma_prefetch_desc(&tmB8);
      const uint32_t full0 = mapa_shared(smem_addr(full), 0);
      const uint64_t keep = l2_evict_last_policy();  // weight tiles: re-read for every row tile
      uint32_t it = 0;
      for (int u = pair; u < n_units; u += n_pairs) {
        int mt, nt;
        tile_of(u, mt, nt);
        const int m0 = mt * 256 + int(rank) * 128, n0 = nt * 256 + int(rank) * 128;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % SM::STAGES;
          const uint32_t ph = (it / SM::STAGES) & 1;
          mbar_wait(&empty[s], ph ^ 1, FAULT_GEMM_WAIT_EMPTY);
          const uint32_t fb = full0 + 8u * s;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * SM::STAGE);
          tma_load_2d_pair(sA + s * SM::A_STAGE, &tmA, fb, kt * GEMM_BK, m0);
          if constexpr (PL != PL_ONE) tma_load_2d_pair(sA + s * SM::A_STAGE + SM::A_BYTES, &tmA_lo, fb, kt * GEMM_BK, m0);
          tma_load_2d_pair_hint(sB + s * SM::B_BYTES, &tmB, fb, kt * GEMM_BK, n0, keep);
          if constexpr (PL == PL_LO8)
            tma_load_2d_pair_hint(sB8 + s * SM::B8_BYTES, &tmB8, fb, kt * GEMM_BK, n0, keep);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(256, 256);
      constexpr uint32_t idesc8 = umma_idesc_e4m3(256, 256);
      const uint32_t empty1 = mapa_shared(smem_addr(empty), 1), acc_full1 = mapa_shared(smem_addr(acc_full), 1);
      uint32_t it = 0, local = 0;
      for (int u = pair; u < n_units; u += n_pairs, ++local) {
        const uint32_t ab = local & 1, aph = (local >> 1) & 1;
        mbar_wait(&acc_empty[ab], aph ^ 1, FAULT_GEMM_WAIT_ACCUM);
        tc_fence_after();
        const uint32_t acc = tmem_base + ab * 256;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % SM::STAGES;
          const uint32_t ph = (it / SM::STAGES) & 1;
          mbar_wait(&full[s], ph, FAULT_GEMM_WAIT_FULL_A);
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * SM::A_STAGE));
          const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * SM::B_BYTES));
#pragma unroll
          for (int j = 0; j < GEMM_BK / 16; ++j) {
            umma_pair_bf16(acc, ad + 2 * j, bd + 2 * j, idesc, (kt != 0 || j != 0) ? 1u : 0u);
            if constexpr (PL == PL_SPLIT) umma_pair_bf16(acc, ad + (SM::A_BYTES >> 4) + 2 * j, bd + 2 * j, idesc, 1u);
          }
          if constexpr (PL == PL_LO8) {
            const uint64_t ald = umma_desc_sw64(smem_addr(sA + s * SM::A_STAGE + SM::A_BYTES));
            const uint64_t bld = umma_desc_sw64(smem_addr(sB8 + s * SM::B8_BYTES));
#pragma unroll
            for (int j = 0; j < GEMM_BK / 32; ++j) umma_pair_e4m3(acc, ald + 2 * j, bld + 2 * j, idesc8, 1u);
          }
          umma_pair_commit(smem_addr(&empty[s]));  // both CTAs may refill stage s
          umma_pair_commit(empty1 + 8u * s);
        }
        umma_pair_commit(smem_addr(&acc_full[ab]));
        umma_pair_commit(acc_full1 + 8u * ab);
      }
    }
    __syncwarp();
  } else {
    // epilogue: warp (2..5) owns TMEM lanes 32*(warp%4)..+31 of this CTA's 128 rows
    const int q = warp & 3;
    const uint32_t acc_empty0 = mapa_shared(smem_addr(acc_empty), 0);
    uint32_t local = 0;
    for (int u = pair; u < n_units; u += n_pairs, ++local) {
      int mt, nt;
      tile_of(u, mt, nt);
      const int m0 = mt * 256 + int(rank) * 128, n0 = nt * 256;
      const uint32_t ab = local & 1, aph = (local >> 1) & 1;
      mbar_wait(&acc_full[ab], aph, FAULT_GEMM_WAIT_ACCUM);
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tl = tmem_base + ab * 256 + (uint32_t(q * 32) << 16);
      if constexpr (EP == B200_EP_SWIGLU) {
#pragma unroll 1
        for (int b = 0; b < 2; ++b) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t g[32], v[32];
            tmem_ld_32x32b_x32(tl + b * 128 + c * 32, g);
            tmem_ld_32x32b_x32(tl + b * 128 + 64 + c * 32, v);
            tmem_ld_wait();
            if constexpr (PL == PL_LO8) {
              lo8_unscale(g);
              lo8_unscale(v);
            }
            epilogue_swiglu(args, row, (n0 + b * 128) / 2 + c * 32, g, v);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tl + c * 32, v);
          tmem_ld_wait();
          if constexpr (PL == PL_LO8) lo8_unscale(v);
          epilogue_chunk<EP>(args, row, n0 + c * 32, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * ab);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the other may still read or signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// --------------------------------------------------------------------------- SIMT cross-check
template <int FMT>
__device__ __forceinline__ void load_row32_f32(const b200_qweight& w, int n, int k0, float (&out)[32]) {
  uint32_t lut[16];  // per-thread copy: this cross-check kernel has threads that exit early
#pragma unroll
  for (int i = 0; i < 16; ++i) lut[i] = ternary_pair_bits(i);
  Raw32<FMT> r;
  load_unit<FMT>(w, n, k0, r);
  uint4 u[4];
  unit_values<FMT>(r, u, lut);
  const uint16_t* h = reinterpret_cast<const uint16_t*>(u);
#pragma unroll
  for (int j = 0; j < 32; ++j) out[j] = bf16_to_f32(h[j]);
}

template <int FMT>
__device__ float simt_dot(const GemmArgs& a, const uint16_t* x, const uint16_t* xl, int ldx, int m, int n) {
  float acc = 0.0f;
  for (int k0 = 0; k0 < a.k; k0 += 32) {
    float wv[32];
    load_row32_f32<FMT>(a.w, n, k0, wv);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const size_t i = size_t(m) * ldx + k0 + j;
      const float xv = bf16_to_f32(x[i]) + (xl ? bf16_to_f32(xl[i]) : 0.0f);
      acc = fmaf(xv, wv[j], acc);
    }
  }
  return acc;
}

template <int FMT, int EP>
__global__ void gemm_simt_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ xl, int ldx,
                                 const GemmArgs a) {
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  const b200_linear_out& o = a.o;
  if (m >= a.m) return;
  if constexpr (EP == B200_EP_SWIGLU) {
    if (2 * n >= o.n_valid) return;
    const int blk = n / 64, i = n % 64;
    const float g = simt_dot<FMT>(a, x, xl, ldx, m, blk * 128 + i);
    const float u = simt_dot<FMT>(a, x, xl, ldx, m, blk * 128 + 64 + i);
    const float h = silu(g) * u;
    uint16_t* dst = reinterpret_cast<uint16_t*>(o.out) + size_t(m) * o.ldo + n;
    const uint16_t hb = f32_to_bf16_rn(h);
    dst[0] = hb;
    if (o.lo_offset) dst[o.lo_offset] = f32_to_bf16_rn(h - bf16_to_f32(hb));
  } else {
    if (n >= o.n_valid) return;
    const float y = simt_dot<FMT>(a, x, xl, ldx, m, n);
    if constexpr (EP == B200_EP_STORE) {
      reinterpret_cast<float*>(o.out)[size_t(m) * o.ldo + n] = y;
    } else {
      reinterpret_cast<float*>(o.out)[size_t(m) * o.ldo + n] += y;
    }
  }
}

// Zero rows [m][0, n) of an fp32 [m, ld] output before a split-K store accumulates into it
// (a kernel rather than a memset so that it joins the programmatic-dependent-launch chain).
// n % 4 == 0 and ld % 4 == 0 (b200_linear's n_valid % 32 and ldo % 8 rules).
__global__ void zero_rows_kernel(float* __restrict__ out, int ld, int n) {
  pdl_wait();
  pdl_trigger();
  float4* row = reinterpret_cast<float4*>(out + size_t(blockIdx.x) * ld);
  for (int i = threadIdx.x; i < n / 4; i += blockDim.x) row[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// Vector fp32 atomic add (sm_90+): one split-K partial of four consecutive outputs.
__device__ __forceinline__ void red_add_v4(float* p, const float4& v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Rows of the swap-AB epilogue's staging tile sT[token][weight row] (floats; 128 + 4 so that
// the column-wise writes and the row-wise 16-byte reads are both conflict-free).
constexpr int SWAP_LD = 132;

// The swap-AB epilogue for tokens t0 .. t0 + TC - 1 of a 128-row weight tile at n0. Epilogue
// warp q (TMEM lane quarter q) holds in v[t] the sum of weight row 32 q + lane for token
// t0 + t. The chunk is turned around in shared memory so that each warp then writes whole
// token rows (tokens t0 + q, t0 + q + 4, ...): the tile's 128 output columns as one float4 per
// lane (fp32 store, residual add, or red.global.add.v4 of a split-K partial), or, for the
// SwiGLU (tile rows 0..63 = gate features n0/2 .. n0/2 + 63, rows 64..127 the matching up
// features), its 64 features as one bf16 pair per lane and plane. The 4 epilogue warps meet
// at named barrier 1 before the reads and after them (the next chunk reuses sT).
template <int EP, int TC>
__device__ __forceinline__ void swap_ab_epilogue(const GemmArgs& args, int n0, int q, int lane, int t0,
                                                 const float (&v)[TC], float* sT) {
  const b200_linear_out& o = args.o;
  constexpr int NTOK = TC / 4;  // tokens per warp
#pragma unroll
  for (int t = 0; t < TC; ++t) sT[t * SWAP_LD + 32 * q + lane] = v[t];
  asm volatile("bar.sync 1, 128;" ::: "memory");
  // every shared-memory (and residual) read of the warp's tokens comes before its first store,
  // so the reads overlap instead of each waiting behind the previous token's store
  if constexpr (EP == B200_EP_SWIGLU) {
    const int ocol = n0 / 2 + 2 * lane;  // features ocol, ocol + 1
    float2 g[NTOK], u[NTOK];
#pragma unroll
    for (int tt = 0; tt < NTOK; ++tt) {
      const float* st = sT + (q + 4 * tt) * SWAP_LD;
      g[tt] = *reinterpret_cast<const float2*>(st + 2 * lane);
      u[tt] = *reinterpret_cast<const float2*>(st + 64 + 2 * lane);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // sT may be rewritten by the next chunk now
    if (2 * ocol + 2 <= o.n_valid) {
      uint16_t* dst = reinterpret_cast<uint16_t*>(o.out);
#pragma unroll
      for (int tt = 0; tt < NTOK; ++tt) {
        const int t = q + 4 * tt;
        if (t0 + t >= args.m) break;
        const size_t row = size_t(t0 + t) * o.ldo;
        const float h0 = silu_approx(g[tt].x) * u[tt].x, h1 = silu_approx(g[tt].y) * u[tt].y;
        const uint32_t hb = pack_bf16x2(h0, h1);
        *reinterpret_cast<uint32_t*>(dst + row + ocol) = hb;
        if (o.lo_offset) {
          if (o.lo_format == B200_LO_E4M3)
            *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(dst + o.lo_offset) + row + ocol) =
                f32x2_to_e4m3x2(lo8_value(h0, uint16_t(hb & 0xFFFFu)), lo8_value(h1, uint16_t(hb >> 16)));
          else
            *reinterpret_cast<uint32_t*>(dst + o.lo_offset + row + ocol) = lo_pair(h0, h1, hb);
        }
      }
    }
  } else {
    const int col = n0 + 4 * lane;
    float4 val[NTOK], res[NTOK];
#pragma unroll
    for (int tt = 0; tt < NTOK; ++tt) {
      const int t = q + 4 * tt;
      val[tt] = *reinterpret_cast<const float4*>(sT + t * SWAP_LD + 4 * lane);
      res[tt] = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (EP == B200_EP_RESID_ADD) {
        if (args.ksplit == 1 && col < o.n_valid && t0 + t < args.m)
          res[tt] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(o.out) +
                                                      size_t(t0 + t) * o.ldo + col);
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // sT may be rewritten by the next chunk now
    if (col < o.n_valid) {
#pragma unroll
      for (int tt = 0; tt < NTOK; ++tt) {
        const int t = q + 4 * tt;
        if (t0 + t >= args.m) break;
        float* p = reinterpret_cast<float*>(o.out) + size_t(t0 + t) * o.ldo + col;
        if (args.ksplit > 1) {
          red_add_v4(p, val[tt]);
        } else if constexpr (EP == B200_EP_RESID_ADD) {
          *reinterpret_cast<float4*>(p) =
              make_float4(res[tt].x + val[tt].x, res[tt].y + val[tt].y, res[tt].z + val[tt].z, res[tt].w + val[tt].w);
        } else {
          *reinterpret_cast<float4*>(p) = val[tt];
        }
      }
    }
  }
}

constexpr int SK_ROWS = 128;  // weight rows per swap-AB tile (the MMA's M)

// --------------------------------------------------------------------------- small M, weights in TMEM
// Batches of at most 128 rows on packed weights (the forward of a single request of about
// 100 tokens, small request batches, state appends, the int4 microbench at M = 1 and 16).
// Swap-AB: the 128-row weight tile is the MMA's A operand (M = 128) and the tokens its B
// operand (N = NT or 2 NT), so no MMA work goes to padding token rows. The decoded weight
// tile never goes through shared memory: the unpack warps write it into tensor memory with
// tcgen05.st and each tcgen05.mma reads A (128 weight rows x 16 k) from there, so the
// shared-memory port carries only the activations. One CTA = one weight tile over one K
// range (K split across CTAs for the store and residual epilogues).
// The two activation planes form one B operand (hi tokens in rows 0..NT-1, lo tokens in rows
// NT..2NT-1 of the slot), so one MMA per 16 k covers both and the epilogue adds the column
// halves of the accumulator.
//   warp 0      activation producer: both planes of each k-block (TMA, tile_m rows x 64 k per
//               plane; rows past m read as zeros) into as many slots as shared memory holds
//   warp 1      TMEM and the MMAs: per 16 k one tcgen05.mma, M = 128, N = NT or 2 NT,
//               A = the weight stage in TMEM, B = the activation slot
//   warps 2..5  first the weights: one lane runs the packed weight ring (1-D bulk copies into
//               TS_WSLOTS slots, each refilled once decoded), the others pull later k-blocks
//               into L2; then the epilogue: TMEM lane quarter -> registers -> swap_ab_epilogue
//   warps 6..13 unpack: warp w decodes the 32-k half (w - 6) / 4 of rows 32 (w % 4) ..
//               32 (w % 4) + 31 (its TMEM lane quarter) of each k-block into 16 columns of a
//               32-column TMEM stage (two bf16 per column, lower k in the low half); same
//               decode as every other GEMM here, bit-exact with b200_dequantize
constexpr int TS_STAGES = 4;
constexpr int TS_WSLOTS = 8;
constexpr int TS_MAX_XSLOTS = 16;
constexpr int TS_MAX_M = 128;
constexpr int TS_UNPACK_WARPS = 8;
constexpr int TS_THREADS = 32 * (GEMM_UNPACK_WARP0 + TS_UNPACK_WARPS);  // 448
constexpr int TS_SMEM_LIMIT = 227 * 1024;

constexpr int pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

// Shared memory: activation slots (args.xslots x X_STAGE, 1024-aligned), then the packed weight
// slots, their scales, the epilogue's staging tile, the barriers, the TMEM address and the
// ternary table. NT is the token capacity (16 or 128); the tile actually loaded and multiplied
// is args.tile_m rows (m rounded up to 16), so the MMA's N, the slot size and the slot count
// follow the batch at run time.
template <int FMT, int PL, int NT>
struct TsSmem {
  static_assert(FMT != B200_W_BF16 && PL != PL_LO8, "packed weights and one or two bf16 activation planes");
  static_assert(NT == 16 || NT == 128, "token capacities of 16 or 128");
  static constexpr int PLANES = PL == PL_SPLIT ? 2 : 1;
  static constexpr int W_BYTES = SK_ROWS * tile_row_bytes(FMT);
  static constexpr int S_BYTES = SK_ROWS * tile_scale_row_bytes(FMT);
  static constexpr int TC = NT < 32 ? NT : 32;                // epilogue tokens per chunk
  static constexpr int SWAP_BYTES = TC * SWAP_LD * 4;         // the epilogue's staging tile
  // TMEM: args.accs accumulators of acc_stride(tile_m) columns from column 0, then the weight
  // stages (stage s at columns a_col0 + 32 s); capacity 16 allocates 256 columns, 128 all 512
  static constexpr int TM_COLS = NT < 32 ? 256 : 512;
  static constexpr int acc_stride(int tile_m) { return (PLANES * tile_m + 31) / 32 * 32; }
  static constexpr int max_accs(int tile_m) { return 2 * acc_stride(tile_m) + 32 * TS_STAGES <= TM_COLS ? 2 : 1; }
  static constexpr int BARS = 2 * TS_WSLOTS + 2 * TS_MAX_XSLOTS + 2 * TS_STAGES + 1;
  static constexpr int FIXED = TS_WSLOTS * (W_BYTES + S_BYTES) + SWAP_BYTES + BARS * 8 + 16 + 64;
  static constexpr int x_stage(int tile_m) { return PLANES * tile_m * GEMM_BK * 2; }
  static_assert(acc_stride(NT) + 32 * TS_STAGES <= TM_COLS, "TMEM columns");
};

template <int FMT, int EP, int PL, int NT>
__global__ void __launch_bounds__(TS_THREADS, 1)
    gemm_ts_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmX_lo,
                   const GemmArgs args) {
  using SM = TsSmem<FMT, PL, NT>;
  extern __shared__ uint8_t smem_raw[];
  const int tile_m = args.tile_m, xslots = args.xslots, accs = args.accs;
  const int acc_stride = SM::acc_stride(tile_m), a_col0 = accs * acc_stride;
  const int x_plane = tile_m * GEMM_BK * 2, x_stage = SM::x_stage(tile_m);
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;                                // xslots x x_stage
  uint8_t* sW = sX + xslots * x_stage;               // TS_WSLOTS x W_BYTES
  uint8_t* sS = sW + TS_WSLOTS * SM::W_BYTES;        // TS_WSLOTS x S_BYTES
  float* sT = reinterpret_cast<float*>(sS + TS_WSLOTS * SM::S_BYTES);  // [TC][SWAP_LD]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sT) + SM::SWAP_BYTES);
  uint64_t* full_w = bars;                           // [WSLOTS] weight slot landed
  uint64_t* empty_w = bars + TS_WSLOTS;              // [WSLOTS] weight slot decoded
  uint64_t* full_x = bars + 2 * TS_WSLOTS;           // [xslots] activation slot landed
  uint64_t* empty_x = full_x + TS_MAX_XSLOTS;        // [xslots] the slot's MMAs are done
  uint64_t* full_a = empty_x + TS_MAX_XSLOTS;        // [STAGES] TMEM weight stage written
  uint64_t* empty_a = full_a + TS_STAGES;            // [STAGES] the stage's MMAs are done
  uint64_t* acc_full = empty_a + TS_STAGES;          // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  uint32_t* lut = tmem_slot + 4;                     // 16 words: ternary pair table
  constexpr uint32_t TM_COLS = SM::TM_COLS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = args.k / GEMM_BK;
  const int n_tiles = args.w.n / SK_ROWS;
  const int n0 = (int(blockIdx.x) % n_tiles) * SK_ROWS, ks = int(blockIdx.x) / n_tiles;
  const int kb0 = ks * nk / args.ksplit, kb1 = (ks + 1) * nk / args.ksplit;
  const int nkb = kb1 - kb0;

  // this tile's packed rows inside the 256-row streaming tiles: tile n0 / 256, row offset n0 % 256
  constexpr int RB = tile_row_bytes(FMT), SB = tile_scale_row_bytes(FMT);
  const size_t lt = size_t(n0 / GEMM_TILE_ROWS) * nk, sub = n0 % GEMM_TILE_ROWS;
  const uint8_t* wtiles = reinterpret_cast<const uint8_t*>(args.w.tiles) + sub * RB;
  const uint8_t* stiles = reinterpret_cast<const uint8_t*>(args.w.tile_scales) + sub * SB;
  auto issue_w = [&](int i) {  // k-block kb0 + i into slot i % WSLOTS
    const int slot = i % TS_WSLOTS;
    const size_t kt = lt + kb0 + i;
    mbar_arrive_expect_tx(&full_w[slot], SM::W_BYTES + SM::S_BYTES);
    bulk_load(sW + slot * SM::W_BYTES, wtiles + kt * GEMM_TILE_ROWS * RB, SM::W_BYTES, &full_w[slot]);
    if constexpr (SM::S_BYTES > 0)
      bulk_load(sS + slot * SM::S_BYTES, stiles + kt * GEMM_TILE_ROWS * SB, SM::S_BYTES, &full_w[slot]);
  };

  if (warp == 0) {  // barriers: one lane each
    for (int b = lane; b < SM::BARS; b += 32) {
      uint32_t count = 1;
      if (b < 2 * TS_WSLOTS) count = b < TS_WSLOTS ? 1 : TS_UNPACK_WARPS;       // full_w, empty_w
      else if (b >= 2 * TS_WSLOTS + 2 * TS_MAX_XSLOTS && b < 2 * TS_WSLOTS + 2 * TS_MAX_XSLOTS + TS_STAGES)
        count = TS_UNPACK_WARPS;                                                  // full_a
      else if (b == SM::BARS - 1) count = accs;                                   // acc_full
      mbar_init(&bars[b], count);
    }
    mbar_fence_init();
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      if constexpr (PL == PL_SPLIT) tma_prefetch_desc(&tmX_lo);
    }
  }
  if (threadIdx.x < 16) lut[threadIdx.x] = ternary_pair_bits(threadIdx.x);
  if (warp == 1) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();  // one unit per CTA: the next kernel may be scheduled now (it waits for this one's results)

  // One MMA-issuing thread: k-blocks first, first + accs, ... into accumulator `first`. Issuing a
  // tcgen05.mma costs its thread a fixed time whatever N is, so at small N two threads
  // (accumulators) issue twice as fast; the epilogue adds them. With two, the activation slots
  // are even in number, so each slot (and each of the 4 weight stages) serves one issuer. The
  // activation slot and its phase are counters: this thread's loop is the critical path, and a
  // division by the run-time slot count costs it tens of dependent instructions.
  auto mma_loop = [&](int first) {
    const uint32_t idesc = umma_idesc_bf16(SK_ROWS, SM::PLANES * tile_m);
    const uint32_t acc = tmem_base + uint32_t(first * acc_stride);
    for (int i = first, xs = first, xph = 0; i < nkb; i += accs) {  // k-block i: slot i % xslots, phase (i / xslots) & 1
      const int s = i % TS_STAGES;
      mbar_wait(&full_x[xs], uint32_t(xph), FAULT_GEMM_WAIT_FULL_A);
      mbar_wait(&full_a[s], (i / TS_STAGES) & 1, FAULT_GEMM_WAIT_FULL_B);
      tc_fence_after();
      const uint64_t bd = umma_desc_sw128(smem_addr(sX + xs * x_stage));
      const uint32_t ta = tmem_base + uint32_t(a_col0 + 32 * s);
#pragma unroll
      for (int j = 0; j < GEMM_BK / 16; ++j)  // 16 k = 8 TMEM columns of A, 32 bytes of B
        umma_bf16_ts(acc, ta + uint32_t(8 * j), bd + 2 * j, idesc, (i >= accs || j != 0) ? 1u : 0u);
      umma_commit(&empty_a[s]);
      umma_commit(&empty_x[xs]);
      xs += accs;
      if (xs >= xslots) xs -= xslots, xph ^= 1;
    }
    umma_commit(&acc_full[0]);
  };

  if (warp == 0) {
    // ---------------- activation producer (the weight ring has its own thread, warp 2)
    if (lane == 0) {
      pdl_wait();  // the activations come from the kernel before this one
      for (int i = 0, xs = 0, xph = 0; i < nkb; ++i) {  // slot i % xslots, phase (i / xslots) & 1
        mbar_wait(&empty_x[xs], uint32_t(xph ^ 1), FAULT_GEMM_WAIT_EMPTY);
        mbar_arrive_expect_tx(&full_x[xs], uint32_t(x_stage));
        tma_load_2d(sX + xs * x_stage, &tmX, &full_x[xs], (kb0 + i) * GEMM_BK, 0);
        if constexpr (PL == PL_SPLIT)
          tma_load_2d(sX + xs * x_stage + x_plane, &tmX_lo, &full_x[xs], (kb0 + i) * GEMM_BK, 0);
        if (++xs == xslots) xs = 0, xph ^= 1;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: D[weight row][token] += W_stage (TMEM) . X_slot^T (k-blocks
    // of parity 0 when a second issuer in warp 3 takes parity 1)
    if (lane == 0) mma_loop(0);
    __syncwarp();
  } else if (warp < GEMM_UNPACK_WARP0) {
    // ---------------- epilogue: quarter q holds weight rows n0 + 32q .. n0 + 32q + 31
    const int q = warp & 3;
    // Until the accumulator is ready, the epilogue warps feed the weights (which do not depend
    // on the kernel before this one): lane 0 of warp 2 runs the weight ring (its first
    // TS_WSLOTS k-blocks, then a refill as each slot is decoded); warps 3..5 pull the K range's
    // later k-blocks into L2, one per thread, so that the refills come from L2.
    if (warp == GEMM_EPI_WARP0 + 1 && accs == 2) {  // ---------------- the second MMA issuer
      if (lane == 0) mma_loop(1);
      __syncwarp();
    }
    if (warp == GEMM_EPI_WARP0) {
      if (lane == 0) {
        for (int i = 0; i < min(nkb, TS_WSLOTS); ++i) issue_w(i);
        for (int i = TS_WSLOTS; i < nkb; ++i) {
          mbar_wait(&empty_w[i % TS_WSLOTS], ((i / TS_WSLOTS) - 1) & 1, FAULT_GEMM_WAIT_EMPTY);
          issue_w(i);
        }
      }
      __syncwarp();
    } else {
      const int i = TS_WSLOTS + (warp - GEMM_EPI_WARP0 - 1) * 32 + lane;
      if (i < nkb) {
        const size_t kt = lt + kb0 + i;
        bulk_prefetch_l2(wtiles + kt * GEMM_TILE_ROWS * RB, SM::W_BYTES);
        if constexpr (SM::S_BYTES > 0) bulk_prefetch_l2(stiles + kt * GEMM_TILE_ROWS * SB, SM::S_BYTES);
      }
    }
    pdl_wait();  // the output (or residual) may be read or written by the kernel before this one
    mbar_wait_idle(&acc_full[0], 0, FAULT_GEMM_WAIT_ACCUM);
    tc_fence_after();
    const uint32_t tl = tmem_base + (uint32_t(q * 32) << 16);
    constexpr int TC = SM::TC;
#pragma unroll 1
    for (int t0 = 0; t0 < tile_m && t0 < args.m; t0 += TC) {
      float v[TC];
#pragma unroll
      for (int t = 0; t < TC; ++t) v[t] = 0.0f;
      for (int a = 0; a < accs; ++a) {
        const uint32_t ta = tl + uint32_t(a * acc_stride);
        uint32_t r[32];
        tmem_ld_32x32b_x32(ta + uint32_t(t0), r);  // capacity 16: hi in columns 0..15, lo in 16..31
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < TC; ++t) v[t] += __uint_as_float(r[t]);
        if constexpr (PL == PL_SPLIT) {
          if constexpr (NT < 32) {
#pragma unroll
            for (int t = 0; t < TC; ++t) v[t] += __uint_as_float(r[NT + t]);
          } else {
            tmem_ld_32x32b_x32(ta + uint32_t(tile_m + t0), r);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < TC; ++t) v[t] += __uint_as_float(r[t]);
          }
        }
      }
      swap_ab_epilogue<EP, TC>(args, n0, q, lane, t0, v, sT);
    }
  } else {
    // ---------------- weight unpack into the TMEM stage
    const int u = warp - GEMM_UNPACK_WARP0, q = warp & 3, h = u >> 2;
    const int r = 32 * q + lane;  // weight row = TMEM lane
    const uint32_t row_sc =
        FMT == B200_W_TERNARY ? uint32_t(__ldg(reinterpret_cast<const uint16_t*>(args.w.scales) + n0 + r)) : 0u;
    const float row_gs = FMT == B200_W_NVFP4 ? __ldg(args.w.row_scale + n0 + r) : 1.0f;
    const uint32_t ta = tmem_base + (uint32_t(32 * q) << 16) + uint32_t(a_col0 + 16 * h);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % TS_STAGES, ws = i % TS_WSLOTS;
      mbar_wait(&full_w[ws], (i / TS_WSLOTS) & 1, FAULT_GEMM_WAIT_FULL_W);
      mbar_wait(&empty_a[s], ((i / TS_STAGES) & 1) ^ 1, FAULT_GEMM_WAIT_EMPTY);
      tc_fence_after();
      uint4 vals[4];
      unpack_unit_regs<FMT>(sW + ws * SM::W_BYTES, sS + ws * SM::S_BYTES, r, h, row_sc, row_gs, lut, vals);
      tmem_st_32x32b_x16(ta + uint32_t(32 * s), vals);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // one arrival per warp
        mbar_arrive(&full_a[s]);
        mbar_arrive(&empty_w[ws]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TM_COLS);
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

// [m, k] row-major tiles of GEMM_BK columns x box_rows rows: bf16 with 128-byte swizzle (128-byte
// rows), or e4m3 bytes with 64-byte swizzle (64-byte rows). ld is in elements.
static int make_tile_map(CUtensorMap* map, const void* x, bool e4m3, int m, int k, int ld, int box_rows) {
  if (int rc = get_encode_fn()) return rc;
  const int eb = e4m3 ? 1 : 2;
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * eb};
  cuuint32_t box[2] = {GEMM_BK, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, e4m3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        e4m3 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return sdb_fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed for a GEMM tile");
  return B200_OK;
}
int encode_bf16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box) {
  if (int rc = get_encode_fn()) return rc;
  if (rank < 1 || rank > 5) return sdb_fail(B200_ERR_ARG, "encode_bf16_sw128: rank");
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) st[i - 1] = strides[i - 1];
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void*>(base), d, st, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return sdb_fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return B200_OK;
}

static int make_act_map(CUtensorMap* map, const uint16_t* x, int m, int k, int ldx, int box_rows = GEMM_BM) {
  return make_tile_map(map, x, false, m, k, ldx, box_rows);
}

static int check_linear(const uint16_t* x, const uint16_t* xl, int m, int k, int ldx, const b200_qweight* w,
                        const b200_linear_out* o) {
  if (!x || !w || !o || !w->data || !o->out) return sdb_fail(B200_ERR_ARG, "b200_linear: null pointer");
  if (m <= 0 || k <= 0) return sdb_fail(B200_ERR_SHAPE, "b200_linear: empty shape");
  if (w->k != k) return sdb_fail(B200_ERR_SHAPE, "b200_linear: x and W disagree on k");
  if (k % 128 != 0 || w->n % 256 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_linear: k % 128 and n % 256 must be 0");
  if (ldx < k || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(xl) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: x planes must be 16-byte aligned with ldx a multiple of 8");
  if (o->n_valid <= 0 || o->n_valid > w->n || o->n_valid % 32 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: n_valid must be in (0, n] and a multiple of 32");
  if (o->ldo % 8 != 0 || (reinterpret_cast<uintptr_t>(o->out) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: out must be 16-byte aligned with ldo a multiple of 8");
  if (o->epilogue == B200_EP_SWIGLU && (o->n_valid % 128 != 0 || o->lo_offset % 8 != 0))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: SwiGLU needs n_valid % 128 == 0 and lo_offset % 8 == 0");
  if (o->epilogue != B200_EP_SWIGLU && o->ldo < o->n_valid)
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: ldo < n_valid");
  if (o->epilogue < 0 || o->epilogue > 2) return sdb_fail(B200_ERR_ARG, "b200_linear: unknown epilogue");
  if (o->lo_format != B200_LO_BF16 && o->lo_format != B200_LO_E4M3)
    return sdb_fail(B200_ERR_ARG, "b200_linear: unknown lo_format");
  if (w->format < 0 || w->format > 3) return sdb_fail(B200_ERR_FORMAT, "b200_linear: unknown weight format");
  if (w->format != B200_W_BF16 && !w->scales) return sdb_fail(B200_ERR_ARG, "b200_linear: missing scales");
  if (w->format == B200_W_NVFP4 && !w->row_scale) return sdb_fail(B200_ERR_ARG, "b200_linear: missing row_scale");
  return B200_OK;
}

static int check_tiles(const b200_qweight* w) {
  if (w->format == B200_W_BF16) return B200_OK;
  if (!w->tiles || (tile_scale_row_bytes(w->format) && !w->tile_scales))
    return sdb_fail(B200_ERR_ARG, "b200_linear: packed weights need their streaming copy (b200_tile_weights)");
  if ((reinterpret_cast<uintptr_t>(w->tiles) & 15) || (reinterpret_cast<uintptr_t>(w->tile_scales) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear: weight tiles must be 16-byte aligned");
  return B200_OK;
}

template <int BN, int FMT, int EP, int PL>
static int launch_tc(const CUtensorMap& map, const CUtensorMap& map_lo, const CUtensorMap& map_b,
                     const CUtensorMap& map_b8, const GemmArgs& a, cudaStream_t st) {
  constexpr int smem = GemmSmem<BN, FMT, PL>::TOTAL;
  static_assert(smem <= 227 * 1024, "GEMM shared memory exceeds the 227 KB per-CTA limit");
  static DeviceOnce attr;  // per instantiation and device
  const int r = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, FMT, EP, PL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem));
    return B200_OK;
  });
  if (r != B200_OK) return r;
  const int n_sm = sm_count();
  GemmArgs args = a;
  const int tiles = (a.w.n / BN) * ((a.m + GEMM_BM - 1) / GEMM_BM);
  const int nk = a.k / GEMM_BK;
  // Small M (few output tiles): split K so every SM has work; each unit keeps >= 2 k-blocks.
  // (The SwiGLU needs whole sums, so it is never split.)
  args.ksplit = 1;
  if (EP != B200_EP_SWIGLU && 2 * tiles <= n_sm) args.ksplit = std::max(1, std::min({n_sm / tiles, nk / 2, 16}));
  if (args.ksplit > 1 && EP == B200_EP_STORE)
    SDB_CUDA(launch_pdl(zero_rows_kernel, dim3(a.m), dim3(256), 0, st, reinterpret_cast<float*>(a.o.out), a.o.ldo,
                        a.o.n_valid));
  const int units = tiles * args.ksplit;
  // programmatic dependent launch: the CTA set-up (barriers, TMEM, descriptor prefetch)
  // overlaps the tail of the kernel before it in the stream (the kernel waits before its
  // first shared access)
  SDB_CUDA(launch_pdl(gemm_tc_kernel<BN, FMT, EP, PL>, dim3(std::min(units, n_sm)), dim3(GEMM_THREADS), smem, st,
                      map, map_lo, map_b, map_b8, args));
  return B200_OK;
}

// 128-column tiles when 256-column tiles would leave most SMs idle (small M): twice the
// tiles, a deeper stage ring, and (for the split-K epilogues) half the K split.
static int tile_bn(const GemmArgs& a) {
  const int tiles256 = (a.w.n / 256) * ((a.m + GEMM_BM - 1) / GEMM_BM);
  return 2 * tiles256 <= sm_count() ? 128 : 256;
}

template <int FMT, int PL>
static int dispatch_ep(const CUtensorMap& map, const CUtensorMap& map_lo, const CUtensorMap& map_b,
                       const CUtensorMap& map_b8, const GemmArgs& a, cudaStream_t st) {
  const bool narrow = tile_bn(a) == 128;
  switch (a.o.epilogue) {
    case B200_EP_STORE:
      return narrow ? launch_tc<128, FMT, B200_EP_STORE, PL>(map, map_lo, map_b, map_b8, a, st)
                    : launch_tc<256, FMT, B200_EP_STORE, PL>(map, map_lo, map_b, map_b8, a, st);
    case B200_EP_RESID_ADD:
      return narrow ? launch_tc<128, FMT, B200_EP_RESID_ADD, PL>(map, map_lo, map_b, map_b8, a, st)
                    : launch_tc<256, FMT, B200_EP_RESID_ADD, PL>(map, map_lo, map_b, map_b8, a, st);
    default:
      return narrow ? launch_tc<128, FMT, B200_EP_SWIGLU, PL>(map, map_lo, map_b, map_b8, a, st)
                    : launch_tc<256, FMT, B200_EP_SWIGLU, PL>(map, map_lo, map_b, map_b8, a, st);
  }
}

// The CTA-pair kernel: bf16 weight copies, 256 x 256 tiles, at least one tile per pair.
template <int EP, int PL>
static int launch_pair(const CUtensorMap& map, const CUtensorMap& map_lo, const CUtensorMap& map_b,
                       const CUtensorMap& map_b8, const GemmArgs& a, cudaStream_t st) {
  constexpr int smem = Gemm2Smem<PL>::TOTAL;
  static_assert(smem <= 227 * 1024, "GEMM shared memory exceeds the 227 KB per-CTA limit");
  static DeviceOnce attr;                       // per instantiation and device
  static int max_pairs_dev[kMaxDevices] = {};   // written under attr's lock, once per device
  const int r = once_per_device(attr, [](int dev) -> int {
    SDB_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<EP, PL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count() & ~1);
    cfg.blockDim = dim3(GEMM2_THREADS);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EP, PL>, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = sm_count() / 2;
    }
    max_pairs_dev[dev] = n;
    return B200_OK;
  });
  if (r != B200_OK) return r;
  int dev = 0;
  SDB_CUDA(cudaGetDevice(&dev));
  const int max_pairs = max_pairs_dev[dev];
  GemmArgs args = a;
  args.ksplit = 1;
  // Weight bytes of all column tiles beyond what L2 keeps alongside the activation stream
  // (about 48 MB here: the 126 MB L2 holds a line in each die's half when both dies read it)
  // -> groups of column tiles of at most about 40 MB each.
  const int n_tiles_n = a.w.n / 256;
  const double tile_bytes = 256.0 * a.k * (PL == PL_LO8 ? 3 : 2);
  const int groups = n_tiles_n * tile_bytes <= 48e6 ? 1 : int(std::ceil(n_tiles_n * tile_bytes / 40e6));
  args.ngroup = (n_tiles_n + groups - 1) / groups;
  const int units = n_tiles_n * ((a.m + 255) / 256);
  SDB_CUDA(launch_pdl(gemm_pair_kernel<EP, PL>, dim3(2 * std::min(units, max_pairs)), dim3(GEMM2_THREADS), smem, st,
                      map, map_lo, map_b, map_b8, args));
  return B200_OK;
}

template <int PL>
static int dispatch_pair(const CUtensorMap& map, const CUtensorMap& map_lo, const CUtensorMap& map_b,
                         const CUtensorMap& map_b8, const GemmArgs& a, cudaStream_t st) {
  switch (a.o.epilogue) {
    case B200_EP_STORE: return launch_pair<B200_EP_STORE, PL>(map, map_lo, map_b, map_b8, a, st);
    case B200_EP_RESID_ADD: return launch_pair<B200_EP_RESID_ADD, PL>(map, map_lo, map_b, map_b8, a, st);
    default: return launch_pair<B200_EP_SWIGLU, PL>(map, map_lo, map_b, map_b8, a, st);
  }
}

// Pairs pay off once every pair has a whole 256 x 256 tile.
static bool pair_path(const GemmArgs& a) {
  return (a.w.n / 256) * ((a.m + 255) / 256) >= sm_count() / 2;
}

template <int PL>
static int dispatch_fmt(const CUtensorMap& map, const CUtensorMap& map_lo, const CUtensorMap& map_b, const GemmArgs& a,
                        cudaStream_t st) {
  switch (a.w.format) {
    case B200_W_BF16: return dispatch_ep<B200_W_BF16, PL>(map, map_lo, map_b, map, a, st);
    case B200_W_INT4G128: return dispatch_ep<B200_W_INT4G128, PL>(map, map_lo, map_b, map, a, st);
    case B200_W_NVFP4: return dispatch_ep<B200_W_NVFP4, PL>(map, map_lo, map_b, map, a, st);
    default: return dispatch_ep<B200_W_TERNARY, PL>(map, map_lo, map_b, map, a, st);
  }
}

template <int FMT>
static int dispatch_simt(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st) {
  const int ncols = a.o.epilogue == B200_EP_SWIGLU ? a.o.n_valid / 2 : a.o.n_valid;
  dim3 grid((ncols + 127) / 128, a.m);
  switch (a.o.epilogue) {
    case B200_EP_STORE:
      SDB_CUDA(launch_pdl(gemm_simt_kernel<FMT, B200_EP_STORE>, grid, dim3(128), 0, st, x, xl, ldx, a));
      break;
    case B200_EP_RESID_ADD:
      SDB_CUDA(launch_pdl(gemm_simt_kernel<FMT, B200_EP_RESID_ADD>, grid, dim3(128), 0, st, x, xl, ldx, a));
      break;
    default: SDB_CUDA(launch_pdl(gemm_simt_kernel<FMT, B200_EP_SWIGLU>, grid, dim3(128), 0, st, x, xl, ldx, a)); break;
  }
  return B200_OK;
}

// The TMEM-weight kernel: K split so that about one unit per SM exists (the SwiGLU needs
// whole sums and is never split); a split store first zeroes its output. The activation tile is
// m rounded up to 16 rows; as many activation slots as the shared memory holds (at most 16).
template <int FMT, int EP, int PL, int NT>
static int launch_ts(const CUtensorMap& mx, const CUtensorMap& mx_lo, const GemmArgs& a, cudaStream_t st) {
  using SM = TsSmem<FMT, PL, NT>;
  static DeviceOnce attr;
  const int r = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(gemm_ts_kernel<FMT, EP, PL, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  TS_SMEM_LIMIT));
    return B200_OK;
  });
  if (r != B200_OK) return r;
  GemmArgs args = a;
  const int tiles = a.w.n / SK_ROWS, nk = a.k / GEMM_BK;
  args.ksplit = EP == B200_EP_SWIGLU ? 1 : std::max(1, std::min(sm_count() / tiles, nk / 2));
  args.tile_m = (a.m + 15) / 16 * 16;
  const int x_stage = SM::x_stage(args.tile_m);
  args.xslots = std::min(TS_MAX_XSLOTS, (TS_SMEM_LIMIT - 1024 - SM::FIXED) / x_stage);
  args.accs = SM::max_accs(args.tile_m);
  if (args.accs == 2) args.xslots &= ~1;  // each slot serves one of the two MMA issuers
  if (args.tile_m > NT || args.xslots < 2) return sdb_fail(B200_ERR_SHAPE, "b200_linear: small-M tile does not fit");
  const int smem = 1024 + args.xslots * x_stage + SM::FIXED;
  if (args.ksplit > 1 && EP == B200_EP_STORE)
    SDB_CUDA(launch_pdl(zero_rows_kernel, dim3(a.m), dim3(256), 0, st, reinterpret_cast<float*>(a.o.out), a.o.ldo,
                        a.o.n_valid));
  SDB_CUDA(launch_pdl(gemm_ts_kernel<FMT, EP, PL, NT>, dim3(tiles * args.ksplit), dim3(TS_THREADS), smem, st, mx,
                      mx_lo, args));
  return B200_OK;
}

template <int FMT, int PL, int NT>
static int dispatch_ts_ep(const CUtensorMap& mx, const CUtensorMap& mx_lo, const GemmArgs& a, cudaStream_t st) {
  switch (a.o.epilogue) {
    case B200_EP_STORE: return launch_ts<FMT, B200_EP_STORE, PL, NT>(mx, mx_lo, a, st);
    case B200_EP_RESID_ADD: return launch_ts<FMT, B200_EP_RESID_ADD, PL, NT>(mx, mx_lo, a, st);
    default: return launch_ts<FMT, B200_EP_SWIGLU, PL, NT>(mx, mx_lo, a, st);
  }
}

template <int PL, int NT>
static int dispatch_ts(const CUtensorMap& mx, const CUtensorMap& mx_lo, const GemmArgs& a, cudaStream_t st) {
  switch (a.w.format) {
    case B200_W_INT4G128: return dispatch_ts_ep<B200_W_INT4G128, PL, NT>(mx, mx_lo, a, st);
    case B200_W_NVFP4: return dispatch_ts_ep<B200_W_NVFP4, PL, NT>(mx, mx_lo, a, st);
    default: return dispatch_ts_ep<B200_W_TERNARY, PL, NT>(mx, mx_lo, a, st);
  }
}

template <int PL>
static int dispatch_ts_nt(const CUtensorMap& mx, const CUtensorMap& mx_lo, const GemmArgs& a, cudaStream_t st) {
  return a.m <= 16 ? dispatch_ts<PL, 16>(mx, mx_lo, a, st) : dispatch_ts<PL, 128>(mx, mx_lo, a, st);
}

// b200_linear takes the small-M kernel (whose store epilogue splits K and clears its output
// with a separate launch) for these batches.
bool linear_small_m(int32_t m, int32_t format) { return m <= TS_MAX_M && format != B200_W_BF16; }

// At most 16 rows on packed weights: the register-streamed kernel (gemm_rs.cu).
bool linear_rs(int32_t m, int32_t format);
int sdb_linear_rs(const uint16_t* x, const uint16_t* xl, int ldx, const GemmArgs& a, cudaStream_t st);

}  // namespace sdb

using namespace sdb;

extern "C" int b200_linear(const uint16_t* x_hi, const uint16_t* x_lo, int32_t m, int32_t k, int32_t ldx,
                           const b200_qweight* w, const b200_linear_out* out, b200_stream stream) {
  if (int rc = check_linear(x_hi, x_lo, m, k, ldx, w, out)) return rc;
  if (int rc = check_tiles(w)) return rc;
  CUtensorMap map, map_lo, map_b;
  if (int rc = make_act_map(&map, x_hi, m, k, ldx)) return rc;
  if (x_lo) {
    if (int rc = make_act_map(&map_lo, x_lo, m, k, ldx)) return rc;
  } else {
    map_lo = map;
  }
  GemmArgs a{*w, *out, m, k, 1};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (linear_rs(m, w->format)) return sdb_linear_rs(x_hi, x_lo, ldx, a, st);  // <= 16 rows, packed
  if (linear_small_m(m, w->format)) {  // small M, packed weights: decoded into TMEM (swap-AB)
    const int nt = (m + 15) / 16 * 16;
    CUtensorMap mx, mx_lo;
    if (int rc = make_act_map(&mx, x_hi, m, k, ldx, nt)) return rc;
    if (x_lo) {
      if (int rc = make_act_map(&mx_lo, x_lo, m, k, ldx, nt)) return rc;
    } else {
      mx_lo = mx;
    }
    return x_lo ? dispatch_ts_nt<PL_SPLIT>(mx, mx_lo, a, st) : dispatch_ts_nt<PL_ONE>(mx, mx_lo, a, st);
  }
  if (w->format == B200_W_BF16) {  // the weight tile streams through TMA as [n, k] bf16, one box per N tile
    if (reinterpret_cast<uintptr_t>(w->data) & 15) return sdb_fail(B200_ERR_SHAPE, "b200_linear: bf16 W unaligned");
    if (pair_path(a)) {  // each CTA of a pair loads 128 of the tile's 256 weight rows
      if (int rc = make_act_map(&map_b, reinterpret_cast<const uint16_t*>(w->data), w->n, k, k, 128)) return rc;
      return x_lo ? dispatch_pair<PL_SPLIT>(map, map_lo, map_b, map_b, a, st)
                  : dispatch_pair<PL_ONE>(map, map_lo, map_b, map_b, a, st);
    }
    const int bn = tile_bn(a);
    if (int rc = make_act_map(&map_b, reinterpret_cast<const uint16_t*>(w->data), w->n, k, k, bn)) return rc;
  } else {
    map_b = map;
  }
  return x_lo ? dispatch_fmt<PL_SPLIT>(map, map_lo, map_b, a, st) : dispatch_fmt<PL_ONE>(map, map_lo, map_b, a, st);
}

extern "C" int b200_linear_lo8(const uint16_t* x_hi, const uint8_t* x_lo8, int32_t m, int32_t k, int32_t ldx,
                               const uint16_t* w_hi, const uint8_t* w_lo8, int32_t n, const b200_linear_out* out,
                               b200_stream stream) {
  if (!x_lo8 || !w_lo8) return sdb_fail(B200_ERR_ARG, "b200_linear_lo8: null low plane or e4m3 weight");
  const b200_qweight w{B200_W_BF16, n, k, w_hi, nullptr, nullptr, nullptr, nullptr};
  if (int rc = check_linear(x_hi, reinterpret_cast<const uint16_t*>(x_lo8), m, k, ldx, &w, out)) return rc;
  if (ldx % 16 != 0 || (reinterpret_cast<uintptr_t>(w_hi) & 15) || (reinterpret_cast<uintptr_t>(w_lo8) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_linear_lo8: ldx % 16 and 16-byte aligned weight copies required");
  GemmArgs a{w, *out, m, k, 1};
  const bool pair = pair_path(a);
  const int bn = pair ? 128 : tile_bn(a);  // weight rows per TMA box (a pair CTA loads half a tile)
  CUtensorMap map, map_lo, map_b, map_b8;
  if (int rc = make_tile_map(&map, x_hi, false, m, k, ldx, GEMM_BM)) return rc;
  if (int rc = make_tile_map(&map_lo, x_lo8, true, m, k, ldx, GEMM_BM)) return rc;
  if (int rc = make_tile_map(&map_b, w_hi, false, n, k, k, bn)) return rc;
  if (int rc = make_tile_map(&map_b8, w_lo8, true, n, k, k, bn)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pair) return dispatch_pair<PL_LO8>(map, map_lo, map_b, map_b8, a, st);
  return dispatch_ep<B200_W_BF16, PL_LO8>(map, map_lo, map_b, map_b8, a, st);
}

extern "C" int b200_linear_simt(const uint16_t* x_hi, const uint16_t* x_lo, int32_t m, int32_t k, int32_t ldx,
                                const b200_qweight* w, const b200_linear_out* out, b200_stream stream) {
  if (int rc = check_linear(x_hi, x_lo, m, k, ldx, w, out)) return rc;
  GemmArgs a{*w, *out, m, k, 1};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (w->format) {
    case B200_W_BF16: return dispatch_simt<B200_W_BF16>(x_hi, x_lo, ldx, a, st);
    case B200_W_INT4G128: return dispatch_simt<B200_W_INT4G128>(x_hi, x_lo, ldx, a, st);
    case B200_W_NVFP4: return dispatch_simt<B200_W_NVFP4>(x_hi, x_lo, ldx, a, st);
    default: return dispatch_simt<B200_W_TERNARY>(x_hi, x_lo, ldx, a, st);
  }
}
