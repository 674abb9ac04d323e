// Gated-DeltaNet token mixer (after the in-projection GEMM) on tensor cores.
//
// Two kernels, restating TF:234-311 with TF:462-530 fused around it.
// gdn_prep_kernel, one warp per (head, TPW consecutive tokens), fully parallel:
//   causal depthwise conv (width 4) + SiLU over the head's q, k, v channels (the 3 previous
//   raw inputs come from the sequence itself or the prefix slot's history), l2norm(q) *
//   dk^-1/2, l2norm(k), beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias).
// gdn_mixer_kernel, one CTA (8 warps) per (sequence, head), chunks of GC = 32 tokens in order:
//   1. G = cumsum(g) within the chunk
//   2. q, k and [beta v | beta k e^G] as hi/lo planes in shared memory
//   3. A = strictly-lower(beta_i k_i.k_j e^{G_i-G_j}), P = lower(q_i.k_j e^{G_i-G_j})
//   4. T = (I + A)^{-1} by block forward substitution (fp32)
//   5. [U | W] = T [beta v | beta k e^G]
//   6. Vn = U - W S
//   7. O = e^G (q S) + P Vn;  S = e^{G_last} S + k^T (Vn e^{G_last - G})
//   8. gated RMSNorm: out = norm_w * O * rsqrt(mean O^2 + eps) * silu(z), as hi/lo planes
// Every matrix product runs on mma.sync m16n8k16 with fp32 accumulation and operands split
// into bf16 planes x = x_hi + x_lo; a product is hi*hi + hi*lo + lo*hi (about 16
// significant bits per operand). The fp32 state S [dk, dv] lives in the warps' accumulator
// registers (warp w holds rows 16w..16w+15) and is republished to shared memory as hi/lo
// planes for the next chunk's products.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace sdb {

constexpr int GC = 32;          // chunk length
static_assert(GC == 32, "the decay scan of a chunk is one warp scan");
constexpr int GD = 128;         // key / value head dim
constexpr int GQKV = 3 * GD;
constexpr int GPREP = GQKV + 4;   // per (token, head): q | k | v | beta, g, pad
constexpr int GDN_THREADS = 256;
constexpr int GDN_DV_SPLIT = 32;   // value columns per CTA when a head is split over a cluster

struct GdnArgs {
  b200_gdn_params p;
  const int32_t* cu;
  const int32_t* prefix_slot;
  const int32_t* save_slot;
  int n_seqs;
  int n_tokens;
  const float* mix;      // [T, ld_mix]: q | k | v | z | b | a
  int ld_mix;
  float* prep;           // [heads][T][GPREP]: q (128) | k (128) | v (128) | beta | g  (fp32); a chunk of
                         // one head is one contiguous run of GC records (GPREP * 4 = 1552 bytes each)
  uint16_t* out;         // hi plane [T, value_dim]; lo plane at out + lo_offset
  long long lo_offset;
  int lo8;               // lo plane as e4m3 bytes (B200_LO_E4M3) instead of bf16
  int32_t* slot_len;
  float* state_pool;     // this layer's [n_slots][heads][dk][dv]
  float* conv_pool;      // this layer's [n_slots][conv_width-1][conv_dim]
  int n_slots;
};

// bf16 planes, row-major, 16-byte chunks XOR-swizzled by row so ldmatrix is conflict-free
// Shared memory of one CTA that owns DV of the head's 128 value columns (DV = 128: the whole
// head; DV = 32: a quarter, four CTAs of a cluster per head).
template <int DV>
struct GdnSmem {
  static constexpr int RW = (DV + GD + 63) / 64 * 64;  // R row width: [beta v (DV) | beta k e^G (128) | pad]
  static constexpr int UP = DV + 4;                     // fp32 row stride of U / O (spreads stores over banks)
  float stage[GC * GPREP];                      // the chunk's prep records, filled by a bulk copy one chunk ahead
  uint64_t bar;                                 // completes when a stage copy has landed
  uint64_t pad_;
  uint16_t Sh[GD * DV], Sl[GD * DV];           // state slab, rows dk, cols: this CTA's dv columns
  uint16_t Qh[GC * GD], Ql[GC * GD];           // q (l2normed, scaled)
  uint16_t Kh[GC * GD], Kl[GC * GD];           // k (l2normed)
  union {
    struct {
      uint16_t Rh[GC * RW], Rl[GC * RW];
    } r;
    struct {
      float U[GC][UP];                          // fp32 U, then (same thread per element) the output O
      uint16_t Wh[GC * GD], Wl[GC * GD];
    } uw;
  } ru;
  uint16_t Vh[GC * DV], Vl[GC * DV];           // Vn
  uint16_t Th[GC * DV], Tl[GC * DV];           // Vn * e^{G_last - G} (named T for "tail-decayed")
  uint16_t Ph[GC * GC], Pl[GC * GC];           // P
  uint16_t Ih[GC * GC], Il[GC * GC];           // (I + A)^{-1}
  float A[GC][GC + 1];                          // A, then the inverse in fp32
  float G[GC], beta[GC], eG[GC], eL[GC];
  float part[2][GC];                            // per-row partial sums of O^2 (DV < 128; by chunk parity)
};

// ----------------------------------------------------------------------------- helpers
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// byte offset of element (r, col) in a swizzled plane whose rows hold RL bf16
template <int RL>
__device__ __forceinline__ uint32_t soff(int r, int col) {
  constexpr int CH = RL / 8;
  const int c = col >> 3;
  const int sw = CH >= 8 ? (r & 7) : ((r >> 1) & (CH - 1));
  return uint32_t(r * RL * 2 + ((c ^ sw) << 4) + (col & 7) * 2);
}

// four consecutive values (8-byte aligned offset): one 8-byte store per plane
__device__ __forceinline__ void split_store4(uint16_t* hi, uint16_t* lo, uint32_t off, float4 v) {
  const uint32_t h01 = pack_bf16x2(v.x, v.y), h23 = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(hi) + off) = make_uint2(h01, h23);
  *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(lo) + off) = make_uint2(lo_pair(v.x, v.y, h01), lo_pair(v.z, v.w, h23));
}

__device__ __forceinline__ void split_store(uint16_t* hi, uint16_t* lo, uint32_t off, float a, float b) {
  const uint32_t h = pack_bf16x2(a, b);
  *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(hi) + off) = h;
  *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(lo) + off) = lo_pair(a, b, h);
}

// A fragment (16 x 16) of a plane stored [m][k] with RL elements per row, rows m0.., cols k0..
template <int RL>
__device__ __forceinline__ void frag_a(uint32_t (&f)[4], const uint16_t* plane, int m0, int k0, int lane) {
  ldsm4(f, smem_addr(plane) + soff<RL>(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
}
// A fragment of the transpose of a plane stored [k][m]: A[m][k] = plane[k][m]
template <int RL>
__device__ __forceinline__ void frag_at(uint32_t (&f)[4], const uint16_t* plane, int m0, int k0, int lane) {
  ldsm4t(f, smem_addr(plane) + soff<RL>(k0 + (lane & 7) + ((lane >> 4) << 3), m0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of two n-tiles (n0..n0+15) x k16 from a plane stored [n][k] (B[k][n] = plane[n][k])
template <int RL>
__device__ __forceinline__ void frag_b(uint32_t (&f)[4], const uint16_t* plane, int n0, int k0, int lane) {
  ldsm4(f, smem_addr(plane) + soff<RL>(n0 + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of two n-tiles from a plane stored [k][n] (B[k][n] = plane[k][n])
template <int RL>
__device__ __forceinline__ void frag_bt(uint32_t (&f)[4], const uint16_t* plane, int n0, int k0, int lane) {
  ldsm4t(f, smem_addr(plane) + soff<RL>(k0 + (lane & 15), n0 + ((lane >> 4) << 3)));
}

// split product of one k16 step into two n-tiles: d0 (n0..n0+7), d1 (n0+8..)
__device__ __forceinline__ void mma3(float (&d0)[4], float (&d1)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                     const uint32_t (&bh)[4], const uint32_t (&bl)[4]) {
  mma16816(d0, ah, bh[0], bh[1]);
  mma16816(d0, ah, bl[0], bl[1]);
  mma16816(d0, al, bh[0], bh[1]);
  mma16816(d1, ah, bh[2], bh[3]);
  mma16816(d1, ah, bl[2], bl[3]);
  mma16816(d1, al, bh[2], bh[3]);
}

// ----------------------------------------------------------------------------- prep kernel
__device__ __forceinline__ int gdn_find_seq(const int32_t* cu, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// tokens per warp: 8 for large batches (each input row is loaded once, the conv window
// slides in registers), 1 for small ones (latency: every warp loads its 4 rows at once)
constexpr int PREP_TPW_LARGE = 8;

// grid (3 heads, ceil(T / (8 TPW))), 8 warps: warp w of block (3 h + part, b) handles head h,
// part (0 q, 1 k, 2 v) and tokens 8 TPW b + TPW w .. +TPW-1; lane l owns channels 4l..4l+3 of
// that part. Blocks run (head, part) fastest, so the blocks resident at one time read whole
// rows of the in-projection output (DRAM pages opened once) rather than one head's 512-byte
// strip down all T rows. The warp keeps the last 3 input rows in registers and loads each
// input row once, four tokens ahead for large batches (two for TPW = 1; token t's row is mix
// row t whatever its sequence, so the prefetch needs no sequence lookup). One part per warp
// keeps the registers low enough for 4 blocks per SM, whose loads in flight cover HBM latency.
template <int TPW>
__global__ void __launch_bounds__(256, 4) gdn_prep_kernel(const GdnArgs a) {
  __shared__ float4 wsm[4][32];  // conv taps (oldest first) of channel 4 lane + c of this part
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.x / 3, part = blockIdx.x % 3, H = a.p.heads, T = a.n_tokens;
  const int key_dim = H * GD, conv_dim = 3 * key_dim, value_dim = key_dim;
  const int ch0 = part * key_dim + h * GD;  // this part's first channel of the head
  if (threadIdx.x < GD) {
    const int ch = threadIdx.x;
    wsm[ch & 3][ch >> 2] = *reinterpret_cast<const float4*>(a.p.conv_w + size_t(ch0 + ch) * 4);
  }
  __syncthreads();
  // the conv taps above are weights; everything below comes from the kernels before this one
  pdl_wait();
  pdl_trigger();
  const int t_begin = (blockIdx.y * 8 + warp) * TPW;
  if (t_begin >= T) return;
  const int t_end = min(T, t_begin + TPW);
  int seq = gdn_find_seq(a.cu, a.n_seqs, t_begin);
  int tok0 = a.cu[seq], tend = a.cu[seq + 1];
  bool fresh = true;
  const float* xrow = a.mix + ch0 + lane * 4;  // + t * ld: token t's 4 channels of this lane
  float4 win[3];  // rows p-3, p-2, p-1
  // v warps, lanes 0 / 1: the gating inputs b / a of the head, loaded ahead like the rows
  const bool gate_lane = part == 2 && lane < 2;
  const float* grow = a.mix + conv_dim + value_dim + (lane == 0 ? h : H + h);
  const float a_coef = gate_lane ? -__expf(a.p.a_log[h]) : 0.0f, dt_bias = gate_lane ? a.p.dt_bias[h] : 0.0f;
  // rows t .. t + PD - 1 (and their gating inputs) in flight: xq[i] is row t + i
  constexpr int PD = TPW >= 8 ? 4 : 2;
  float4 xq[PD];
  float gq[PD];
#pragma unroll
  for (int i = 0; i < PD; ++i) {
    xq[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    gq[i] = 0.0f;
    if (t_begin + i < t_end) {
      xq[i] = *reinterpret_cast<const float4*>(xrow + size_t(t_begin + i) * a.ld_mix);
      if (gate_lane) gq[i] = grow[size_t(t_begin + i) * a.ld_mix];
    }
  }
  for (int t = t_begin; t < t_end; ++t) {
    const float4 x = xq[0];
    const float g = gq[0];
#pragma unroll
    for (int i = 0; i + 1 < PD; ++i) {
      xq[i] = xq[i + 1];
      gq[i] = gq[i + 1];
    }
    if (t + PD < t_end) {  // in flight meanwhile
      xq[PD - 1] = *reinterpret_cast<const float4*>(xrow + size_t(t + PD) * a.ld_mix);
      if (gate_lane) gq[PD - 1] = grow[size_t(t + PD) * a.ld_mix];
    }
    while (t >= tend) {  // next (possibly empty) sequence; ends because t < T = cu[n_seqs]
      ++seq;
      tok0 = tend;
      tend = a.cu[seq + 1];
      fresh = true;
    }
    const int p = t - tok0;
    if (fresh) {
      // rows p-3..p-1: the sequence's own for positions >= 0, else the prefix slot's conv
      // history, else zeros
      const int pslot = a.prefix_slot ? a.prefix_slot[seq] : -1;
      const bool pvalid = pslot >= 0 && pslot < a.n_slots;
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const int q = p - 3 + r;
        if (q >= 0) win[r] = *reinterpret_cast<const float4*>(xrow + size_t(tok0 + q) * a.ld_mix);
        else if (pvalid)
          win[r] = *reinterpret_cast<const float4*>(a.conv_pool + (size_t(pslot) * 3 + (3 + q)) * conv_dim + ch0 +
                                                    lane * 4);
        else win[r] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      fresh = false;
    }
    const float xi[4][4] = {{win[0].x, win[1].x, win[2].x, x.x},
                            {win[0].y, win[1].y, win[2].y, x.y},
                            {win[0].z, win[1].z, win[2].z, x.z},
                            {win[0].w, win[1].w, win[2].w, x.w}};
    float o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 w = wsm[c][lane];
      float acc = 0.0f;
      acc = fmaf(w.x, xi[c][0], acc);
      acc = fmaf(w.y, xi[c][1], acc);
      acc = fmaf(w.z, xi[c][2], acc);
      acc = fmaf(w.w, xi[c][3], acc);
      o[c] = silu_approx(acc);
    }
    win[0] = win[1];
    win[1] = win[2];
    win[2] = x;
    float r = 1.0f;
    if (part < 2) {  // q, k: l2norm over the head's 128 channels; q also takes 1 / sqrt(dk)
      const float ss = warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      r = rsqrtf(ss + 1e-6f) * (part == 0 ? rsqrtf(float(GD)) : 1.0f);
    }
    float* dst = a.prep + (size_t(h) * T + t) * GPREP;
    reinterpret_cast<float4*>(dst + part * GD)[lane] = make_float4(o[0] * r, o[1] * r, o[2] * r, o[3] * r);
    if (gate_lane)  // beta = sigmoid(b) (lane 0), g = -exp(A_log) softplus(a + dt_bias) (lane 1)
      dst[GQKV + lane] = lane == 0 ? __fdividef(1.0f, 1.0f + __expf(-g)) : a_coef * softplus(g + dt_bias);
  }
}

// ----------------------------------------------------------------------------- kernel

// Bulk-copy the prep records of chunk c (rows tok0 + c .., head h: one contiguous run of
// GPREP * 4 = 1552-byte records, 16-byte aligned) into the stage; completes on bar.
__device__ __forceinline__ void gdn_stage_chunk(float* stage, uint64_t* bar, const GdnArgs& a, int h, int tok0, int len,
                                                int c) {
  const uint32_t bytes = uint32_t(min(GC, len - c)) * GPREP * 4;
  mbar_arrive_expect_tx(bar, bytes);
  bulk_load(stage, a.prep + (size_t(h) * a.n_tokens + tok0 + c) * GPREP, bytes, bar);
}

// The saved conv history of head h (called by all GDN_THREADS threads of one CTA): the
// sequence's last 3 raw inputs of the head's q / k / v channels; positions before the
// sequence come from the prefix slot's history. Everything is read before anything is
// written, so a sequence may save into its own prefix slot (append).
__device__ __forceinline__ void gdn_save_conv(const GdnArgs& a, int h, int tok0, int len, int pslot, bool pvalid,
                                              int sslot) {
  const int key_dim = a.p.heads * GD, conv_dim = 3 * key_dim;
  constexpr int PER_T = (3 * 3 * GD + GDN_THREADS - 1) / GDN_THREADS;
  float hv[PER_T];
#pragma unroll
  for (int i = 0; i < PER_T; ++i) {
    const int idx = threadIdx.x + i * GDN_THREADS;
    hv[i] = 0.0f;
    if (idx < 3 * 3 * GD) {
      const int r = idx / (3 * GD), part = (idx / GD) % 3, c = idx % GD;
      const int q = len - 3 + r, ch = part * key_dim + h * GD + c;
      if (q >= 0) hv[i] = a.mix[size_t(tok0 + q) * a.ld_mix + ch];
      else if (pvalid) hv[i] = a.conv_pool[(size_t(pslot) * 3 + (3 + q)) * conv_dim + ch];
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < PER_T; ++i) {
    const int idx = threadIdx.x + i * GDN_THREADS;
    if (idx < 3 * 3 * GD) {
      const int r = idx / (3 * GD), part = (idx / GD) % 3, c = idx % GD;
      a.conv_pool[(size_t(sslot) * 3 + r) * conv_dim + part * key_dim + h * GD + c] = hv[i];
    }
  }
}

// grid (heads * NS, n_seqs), NS = 128 / DV CTAs per (sequence, head) forming one cluster; the
// CTA with cluster rank `slice` owns value columns col0 = slice * DV .. col0 + DV - 1 of the
// state, U, Vn and O. The dv columns of the delta rule are independent except for the gated
// RMSNorm's sum of squares, which the cluster exchanges through distributed shared memory.
// Steps 1-5 (decay, A, P, T, W) are computed by every CTA of the cluster.
template <int DV>
__global__ void __launch_bounds__(GDN_THREADS, 1) gdn_mixer_kernel(const GdnArgs a) {
  constexpr int NS = GD / DV;
  constexpr int NT = DV / 8;              // n8 tiles of the state slab per warp
  using SMT = GdnSmem<DV>;
  constexpr int RW = SMT::RW;
  extern __shared__ __align__(128) uint8_t gdn_smem_raw[];
  SMT& sm = *reinterpret_cast<SMT*>(gdn_smem_raw);
  float (*const O)[SMT::UP] = sm.ru.uw.U;
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int h = blockIdx.x / NS, slice = blockIdx.x % NS, col0 = slice * DV, seq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int H = a.p.heads;
  const int key_dim = H * GD, value_dim = H * GD, conv_dim = 2 * key_dim + value_dim;
  const int tok0 = a.cu[seq], len = a.cu[seq + 1] - tok0;
  const int pslot = a.prefix_slot ? a.prefix_slot[seq] : -1;
  const int sslot = a.save_slot ? a.save_slot[seq] : -1;
  const bool pvalid = pslot >= 0 && pslot < a.n_slots;
  const bool svalid = sslot >= 0 && sslot < a.n_slots;
  if ((pslot >= a.n_slots || sslot >= a.n_slots) && tid == 0) raise_fault(FAULT_BAD_INDEX);

  // ---- initial state (fp32 slab in registers)
  float S[NT][4];  // rows 16*warp + g8 (+8), cols col0 + 8*nt + 2*t4 (+1)
  {
    const float* src = pvalid ? a.state_pool + (size_t(pslot) * H + h) * GD * GD : nullptr;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {  // columns c, c + 1 as one 8-byte load
        const int r = 16 * warp + g8 + 8 * hr, c = 8 * nt + 2 * t4;
        const float2 v = src ? *reinterpret_cast<const float2*>(src + r * GD + col0 + c) : make_float2(0.f, 0.f);
        S[nt][2 * hr] = v.x;
        S[nt][2 * hr + 1] = v.y;
      }
    }
  }
  if (tid == 0) {
    mbar_init(&sm.bar, 1);
    mbar_fence_init();
    if (len > 0) gdn_stage_chunk(sm.stage, &sm.bar, a, h, tok0, len, 0);
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr)
      split_store(sm.Sh, sm.Sl, soff<DV>(16 * warp + g8 + 8 * hr, 8 * nt + 2 * t4), S[nt][2 * hr], S[nt][2 * hr + 1]);
  }
  __syncthreads();

  uint32_t phase = 0;
  for (int c0 = 0; c0 < len; c0 += GC) {
    const int L = min(GC, len - c0);
    const bool need_state = svalid || c0 + GC < len;  // the state after this chunk is used
    const bool landed = mbar_wait(&sm.bar, phase, FAULT_GDN_WAIT_STAGE);
    phase ^= 1u;
    if constexpr (NS == 1) {
      if (__syncthreads_or(!landed)) break;  // a copy that never landed: give up (fault recorded)
    } else {
      // a cluster keeps going (every CTA must reach every cluster barrier); the data of a
      // copy that never landed is garbage, and the fault word already reports it
      __syncthreads();
    }
    if (lane < GC / 8 && warp + 8 * lane < L)  // the z gate rows this warp reads in step 8
      bulk_prefetch_l2(a.mix + size_t(tok0 + c0 + warp + 8 * lane) * a.ld_mix + conv_dim + h * GD + col0, DV * 4);
    // ---- 1. cumulative decay within the chunk: every warp scans the chunk's g itself (lane l
    //         holds G_l), so the planes of step 2 need no barrier after it; warp 0 publishes
    //         G, beta, e^G and e^{G_{L-1} - G} for the later steps
    float bl = 0.0f, Gl = 0.0f;
    {
      if (lane < L) {
        bl = sm.stage[lane * GPREP + GQKV];
        Gl = sm.stage[lane * GPREP + GQKV + 1];
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive warp scan
        const float n = __shfl_up_sync(0xffffffffu, Gl, o);
        if (lane >= o) Gl += n;
      }
      if (warp == 0) {
        const float GL = __shfl_sync(0xffffffffu, Gl, L - 1);
        sm.G[lane] = Gl;
        sm.beta[lane] = bl;
        sm.eG[lane] = __expf(Gl);
        sm.eL[lane] = lane < L ? __expf(GL - Gl) : 0.0f;
      }
    }
    // ---- 2. q, k, [beta v | beta k e^G] as hi/lo planes (rows past L are zero)
#pragma unroll
    for (int j = warp; j < GC; j += GDN_THREADS / 32) {
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f), k = q, v = q;
      if (j < L) {
        const float* pr = sm.stage + j * GPREP;
        q = reinterpret_cast<const float4*>(pr)[lane];
        k = reinterpret_cast<const float4*>(pr + GD)[lane];
        if (lane < DV / 4) v = reinterpret_cast<const float4*>(pr + 2 * GD + col0)[lane];
      }
      const float bj = __shfl_sync(0xffffffffu, bl, j), bke = bj * __expf(__shfl_sync(0xffffffffu, Gl, j));
      const int c = lane * 4;
      split_store4(sm.Qh, sm.Ql, soff<GD>(j, c), q);
      split_store4(sm.Kh, sm.Kl, soff<GD>(j, c), k);
      if (lane < DV / 4)
        split_store4(sm.ru.r.Rh, sm.ru.r.Rl, soff<RW>(j, c), make_float4(bj * v.x, bj * v.y, bj * v.z, bj * v.w));
      split_store4(sm.ru.r.Rh, sm.ru.r.Rl, soff<RW>(j, DV + c),
                   make_float4(bke * k.x, bke * k.y, bke * k.z, bke * k.w));
    }
    __syncthreads();
    if (tid == 0 && c0 + GC < len) {  // every read of the stage is done: fetch the next chunk
      fence_proxy_async_smem();
      gdn_stage_chunk(sm.stage, &sm.bar, a, h, tok0, len, c0 + GC);
    }
    // ---- 3. A = beta k k^T, P = q k^T (x decay, masked): warp -> rows 16*(w>>2), cols 8*(w&3);
    //         each of the three split passes accumulates apart (three short dependency chains)
    {
      const int m0 = 16 * (warp >> 2), n0 = 8 * (warp & 3);
      float kk[4] = {0, 0, 0, 0}, qk[4] = {0, 0, 0, 0};
      float kk1[4] = {0, 0, 0, 0}, qk1[4] = {0, 0, 0, 0}, kk2[4] = {0, 0, 0, 0}, qk2[4] = {0, 0, 0, 0};
      // B fragment of the n-tile n0 (8 keys) x k16 from both planes in one ldmatrix.x4: lanes 0-15
      // address the hi plane, 16-31 the lo plane -> {hi b0, hi b1, lo b0, lo b1}
      const uint16_t* bplane = lane < 16 ? sm.Kh : sm.Kl;
#pragma unroll 2
      for (int k0 = 0; k0 < GD; k0 += 16) {
        uint32_t kh[4], kl[4], qh[4], ql[4], b[4];
        frag_a<GD>(kh, sm.Kh, m0, k0, lane);
        frag_a<GD>(kl, sm.Kl, m0, k0, lane);
        frag_a<GD>(qh, sm.Qh, m0, k0, lane);
        frag_a<GD>(ql, sm.Ql, m0, k0, lane);
        ldsm4(b, smem_addr(bplane) + soff<GD>(n0 + (lane & 7), k0 + (((lane >> 3) & 1) << 3)));
        mma16816(kk, kh, b[0], b[1]);
        mma16816(qk, qh, b[0], b[1]);
        mma16816(kk1, kh, b[2], b[3]);
        mma16816(qk1, qh, b[2], b[3]);
        mma16816(kk2, kl, b[0], b[1]);
        mma16816(qk2, ql, b[0], b[1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        kk[e] += kk1[e] + kk2[e];
        qk[e] += qk1[e] + qk2[e];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + g8 + 8 * (e >> 1), j = n0 + 2 * t4 + (e & 1);
        const bool ok = i < L && j < L;
        const float dec = ok && j <= i ? __expf(sm.G[i] - sm.G[j]) : 0.0f;
        sm.A[i][j] = (ok && j < i) ? sm.beta[i] * kk[e] * dec : 0.0f;
        qk[e] = (ok && j <= i) ? qk[e] * dec : 0.0f;
      }
      split_store(sm.Ph, sm.Pl, soff<GC>(m0 + g8, n0 + 2 * t4), qk[0], qk[1]);
      split_store(sm.Ph, sm.Pl, soff<GC>(m0 + g8 + 8, n0 + 2 * t4), qk[2], qk[3]);
    }
    __syncthreads();
    // ---- 4. (I + A)^{-1}: diagonal 16x16 blocks by forward substitution, then the
    //         off-diagonal block T10 = -T11 A10 T00; result in sm.A (fp32) and the I planes
    if (warp < 2 && lane < 16) {
      const int b = 16 * warp, c = lane;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float r = i == c ? 1.0f : 0.0f;
#pragma unroll
        for (int j = 0; j < i; ++j) r = fmaf(-sm.A[b + i][b + j], x[j], r);
        x[i] = r;
      }
      __syncwarp(0x0000FFFFu);
#pragma unroll
      for (int i = 0; i < 16; ++i) sm.A[b + i][b + c] = x[i];  // diagonal block now holds T_bb
    }
    __syncthreads();
    {
      // M = A10 T00 (16x16), then T10 = -T11 M; thread -> (row i, col c) with 256 threads
      const int i = tid >> 4, c = tid & 15;
      float mval = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) mval = fmaf(sm.A[16 + i][j], sm.A[j][c], mval);
      // Vh (>= 2 KB) is first written in step 6; its last reads (the previous chunk's step 7a)
      // are several barriers back
      float* scratch = reinterpret_cast<float*>(sm.Vh);
      scratch[i * 16 + c] = mval;
      __syncthreads();
      float t = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) t = fmaf(sm.A[16 + i][16 + j], scratch[j * 16 + c], t);
      sm.A[16 + i][c] = -t;  // A10 was last read above, before the barrier
    }
    __syncthreads();
    for (int i = tid; i < GC * GC / 2; i += GDN_THREADS) {
      const int r = i / (GC / 2), c = 2 * (i % (GC / 2));
      const float v0 = c <= r ? sm.A[r][c] : 0.0f, v1 = c + 1 <= r ? sm.A[r][c + 1] : 0.0f;
      split_store(sm.Ih, sm.Il, soff<GC>(r, c), v0, v1);
    }
    __syncthreads();
    // ---- 5. [U | W] = T R : job j = (rows 16*(j&1), cols 16*(j>>1) .. +16) of the DV + 128
    //         columns; warp w takes jobs w, w + 8, ... (all with rows 16*(w&1))
    {
      constexpr int NB = (DV + GD) / 16, PER = (2 * NB + 7) / 8;
      const int m0 = 16 * (warp & 1);
      float acc[PER][2][4];
#pragma unroll
      for (int i = 0; i < PER; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][0][e] = acc[i][1][e] = 0.0f;
#pragma unroll
      for (int k0 = 0; k0 < GC; k0 += 16) {
        uint32_t ah[4], al[4];
        frag_a<GC>(ah, sm.Ih, m0, k0, lane);
        frag_a<GC>(al, sm.Il, m0, k0, lane);
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int nb = (warp >> 1) + 4 * i;
          if (nb < NB) {
            uint32_t bh[4], bl[4];
            frag_bt<RW>(bh, sm.ru.r.Rh, 16 * nb, k0, lane);
            frag_bt<RW>(bl, sm.ru.r.Rl, 16 * nb, k0, lane);
            mma3(acc[i][0], acc[i][1], ah, al, bh, bl);
          }
        }
      }
      __syncthreads();  // R is fully read before U / W overwrite it
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int nb = (warp >> 1) + 4 * i;
        if (nb < NB) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              const int r = m0 + g8 + 8 * hr, c = 16 * nb + 8 * half + 2 * t4;
              if (c < DV) {
                *reinterpret_cast<float2*>(&sm.ru.uw.U[r][c]) =
                    make_float2(acc[i][half][2 * hr], acc[i][half][2 * hr + 1]);
              } else {
                split_store(sm.ru.uw.Wh, sm.ru.uw.Wl, soff<GD>(r, c - DV), acc[i][half][2 * hr],
                            acc[i][half][2 * hr + 1]);
              }
            }
          }
        }
      }
    }
    __syncthreads();
    // ---- 6. Vn = U - W S  and  O = e^G (q S): job j = (rows 16*(j&1), cols 16*(j>>1) .. +16)
    //         of the DV columns; warp w takes jobs w, w + 8
    constexpr int NB6 = DV / 16, PER6 = (2 * NB6 + 7) / 8;
    {
      const int m0 = 16 * (warp & 1);
      float ws[PER6][2][4], qs[PER6][2][4];
#pragma unroll
      for (int i = 0; i < PER6; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) ws[i][0][e] = ws[i][1][e] = qs[i][0][e] = qs[i][1][e] = 0.0f;
      if (warp < 2 * NB6) {
#pragma unroll 2
        for (int k0 = 0; k0 < GD; k0 += 16) {
          uint32_t wh[4], wl[4], qh[4], ql[4];
          frag_a<GD>(wh, sm.ru.uw.Wh, m0, k0, lane);
          frag_a<GD>(wl, sm.ru.uw.Wl, m0, k0, lane);
          frag_a<GD>(qh, sm.Qh, m0, k0, lane);
          frag_a<GD>(ql, sm.Ql, m0, k0, lane);
#pragma unroll
          for (int i = 0; i < PER6; ++i) {
            const int nb = (warp >> 1) + 4 * i;
            if (nb < NB6) {
              uint32_t bh[4], bl[4];
              frag_bt<DV>(bh, sm.Sh, 16 * nb, k0, lane);
              frag_bt<DV>(bl, sm.Sl, 16 * nb, k0, lane);
              mma3(ws[i][0], ws[i][1], wh, wl, bh, bl);
              mma3(qs[i][0], qs[i][1], qh, ql, bh, bl);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < PER6; ++i) {
        const int nb = (warp >> 1) + 4 * i;
        if (warp < 2 * NB6 && nb < NB6) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              const int r = m0 + g8 + 8 * hr, c = 16 * nb + 8 * half + 2 * t4;
              const bool ok = r < L;
              const float2 u2 = *reinterpret_cast<const float2*>(&sm.ru.uw.U[r][c]);  // c even
              const float v0 = ok ? u2.x - ws[i][half][2 * hr] : 0.0f;
              const float v1 = ok ? u2.y - ws[i][half][2 * hr + 1] : 0.0f;
              split_store(sm.Vh, sm.Vl, soff<DV>(r, c), v0, v1);
              if (need_state) split_store(sm.Th, sm.Tl, soff<DV>(r, c), v0 * sm.eL[r], v1 * sm.eL[r]);
              // overwrites U[r][c], U[r][c + 1], read just above by this thread (c even: 8-byte store)
              *reinterpret_cast<float2*>(&O[r][c]) =
                  make_float2(qs[i][half][2 * hr] * sm.eG[r], qs[i][half][2 * hr + 1] * sm.eG[r]);
            }
          }
        }
      }
    }
    __syncthreads();
    // ---- 7a. O += P Vn  (same jobs as step 6)
    if (warp < 2 * NB6) {
      const int m0 = 16 * (warp & 1);
      float pv[PER6][2][4];
#pragma unroll
      for (int i = 0; i < PER6; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) pv[i][0][e] = pv[i][1][e] = 0.0f;
#pragma unroll
      for (int k0 = 0; k0 < GC; k0 += 16) {
        uint32_t ph[4], pl[4];
        frag_a<GC>(ph, sm.Ph, m0, k0, lane);
        frag_a<GC>(pl, sm.Pl, m0, k0, lane);
#pragma unroll
        for (int i = 0; i < PER6; ++i) {
          const int nb = (warp >> 1) + 4 * i;
          if (nb < NB6) {
            uint32_t bh[4], bl[4];
            frag_bt<DV>(bh, sm.Vh, 16 * nb, k0, lane);
            frag_bt<DV>(bl, sm.Vl, 16 * nb, k0, lane);
            mma3(pv[i][0], pv[i][1], ph, pl, bh, bl);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < PER6; ++i) {
        const int nb = (warp >> 1) + 4 * i;
        if (nb < NB6) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              const int r = m0 + g8 + 8 * hr, c = 16 * nb + 8 * half + 2 * t4;
              float2* o2 = reinterpret_cast<float2*>(&O[r][c]);
              const float2 prev = *o2;
              *o2 = make_float2(prev.x + pv[i][half][2 * hr], prev.y + pv[i][half][2 * hr + 1]);
            }
          }
        }
      }
    }
    // ---- 7b. S = e^{G_last} S + k^T (Vn e^{G_last - G}): warp w owns S rows 16w..16w+15;
    //          skipped after the last chunk of a sequence that saves no state (a question)
    if (need_state) {
      const float el = __expf(sm.G[L - 1]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] *= el;
      }
#pragma unroll
      for (int k0 = 0; k0 < GC; k0 += 16) {
        uint32_t ah[4], al[4];
        frag_at<GD>(ah, sm.Kh, 16 * warp, k0, lane);
        frag_at<GD>(al, sm.Kl, 16 * warp, k0, lane);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t bh[4], bl[4];
          frag_bt<DV>(bh, sm.Th, 16 * np, k0, lane);
          frag_bt<DV>(bl, sm.Tl, 16 * np, k0, lane);
          mma3(S[2 * np], S[2 * np + 1], ah, al, bh, bl);
        }
      }
    }
    // the z gates of all the warp's step-8 rows (and the norm weights), loaded here so that their
    // latency passes under the barrier and the state-plane stores
    constexpr int CPL = DV / 32;
    float nw[CPL], zv[GC / 8][CPL];
#pragma unroll
    for (int e = 0; e < CPL; ++e) nw[e] = a.p.norm_w[col0 + lane * CPL + e];
#pragma unroll
    for (int i = 0; i < GC / 8; ++i) {
      const int j = warp + 8 * i;
      const float* z = a.mix + size_t(tok0 + c0 + (j < L ? j : 0)) * a.ld_mix + conv_dim + h * GD + col0 + lane * CPL;
      if constexpr (CPL == 4) {
        const float4 z4 = j < L ? *reinterpret_cast<const float4*>(z) : make_float4(0.f, 0.f, 0.f, 0.f);
        zv[i][0] = z4.x;
        zv[i][1] = z4.y;
        zv[i][2] = z4.z;
        zv[i][3] = z4.w;
      } else {
#pragma unroll
        for (int e = 0; e < CPL; ++e) zv[i][e] = j < L ? z[e] : 0.0f;
      }
    }
    __syncthreads();  // all reads of the old S planes (step 6) and of O's partials are done
    if (need_state) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr)
          split_store(sm.Sh, sm.Sl, soff<DV>(16 * warp + g8 + 8 * hr, 8 * nt + 2 * t4), S[nt][2 * hr],
                      S[nt][2 * hr + 1]);
      }
    }
    // ---- 8. gated RMSNorm of the O rows -> hi/lo planes; warp w owns rows w, w + 8, ...;
    //         lane l owns this CTA's columns CPL*l .. CPL*l + CPL - 1
    {
      const int cpar = (c0 / GC) & 1;
      float ov[GC / 8][CPL], ss[GC / 8];
#pragma unroll
      for (int i = 0; i < GC / 8; ++i) {
        const int j = warp + 8 * i;
        float q = 0.0f;
        if constexpr (CPL == 4) {  // one 16-byte load (rows of O are 16-byte aligned: UP % 4 == 0)
          const float4 o4 = *reinterpret_cast<const float4*>(&O[j][lane * 4]);
          ov[i][0] = o4.x;
          ov[i][1] = o4.y;
          ov[i][2] = o4.z;
          ov[i][3] = o4.w;
        } else {
#pragma unroll
          for (int e = 0; e < CPL; ++e) ov[i][e] = O[j][lane * CPL + e];
        }
#pragma unroll
        for (int e = 0; e < CPL; ++e) q += ov[i][e] * ov[i][e];
        ss[i] = warp_sum(q);
        if constexpr (NS > 1) {
          if (lane == 0) sm.part[cpar][j] = ss[i];
        }
      }
      if constexpr (NS > 1) {
        // the cluster's partial sums: each CTA reads every CTA's part[cpar] after this barrier;
        // part[cpar] is written again two chunks later, after the next chunk's barrier
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
#pragma unroll
        for (int i = 0; i < GC / 8; ++i) {
          const int j = warp + 8 * i;
          float tot = 0.0f;
#pragma unroll
          for (int r = 0; r < NS; ++r) tot += cluster.map_shared_rank(&sm.part[cpar][0], r)[j];
          ss[i] = tot;
        }
      }
#pragma unroll
      for (int i = 0; i < GC / 8; ++i) {
        const int j = warp + 8 * i;
        if (j < L) {  // uniform across the warp
          const float r = rsqrtf(ss[i] / float(GD) + a.p.eps);
          float y[CPL];
          uint16_t hb[CPL];
#pragma unroll
          for (int e = 0; e < CPL; ++e) {
            y[e] = nw[e] * (ov[i][e] * r) * silu_approx(zv[i][e]);
            hb[e] = f32_to_bf16_rn(y[e]);
          }
          const size_t e0 = size_t(tok0 + c0 + j) * value_dim + h * GD + col0 + lane * CPL;
          if constexpr (CPL == 4) {
            store_planes4(a.out, a.lo_offset, a.lo8, e0, y[0], y[1], y[2], y[3]);
          } else {
#pragma unroll
            for (int e = 0; e < CPL; ++e) {
              a.out[e0 + e] = hb[e];
              if (!a.lo_offset) continue;
              if (a.lo8)
                reinterpret_cast<uint8_t*>(a.out + a.lo_offset)[e0 + e] =
                    uint8_t(f32x2_to_e4m3x2(lo8_value(y[e], hb[e]), 0.0f));
              else
                a.out[e0 + e + a.lo_offset] = f32_to_bf16_rn(y[e] - bf16_to_f32(hb[e]));
            }
          }
        }
      }
    }
    // no barrier here: the next chunk's first shared-memory writes (step 1) come after the
    // barrier at the top of its iteration
  }

  if (svalid) {
    float* dst = a.state_pool + (size_t(sslot) * H + h) * GD * GD;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = 16 * warp + g8 + 8 * (e >> 1), c = 8 * nt + 2 * t4 + (e & 1);
        dst[r * GD + col0 + c] = S[nt][e];
      }
    }
    if (slice == 0) gdn_save_conv(a, h, tok0, len, pslot, pvalid, sslot);
  }
  if constexpr (NS > 1) {
    // no CTA leaves while another may still read its part[] (the last chunk's exchange)
    cg::this_cluster().sync();
  }
}

// ----------------------------------------------------------------------------- recurrent kernel

// Token-by-token form of the same rule (TF:314-353), for batches whose sequences are one
// token long (appends of a single token to a cached state) or a few: per token
//   S <- e^g S;  delta = beta (v - S^T k);  S <- S + k delta^T;  o = S^T q,
// computed as a = S^T k and b = S^T q over the state before the update, so that
//   delta = beta (v - e^g a)  and  o = e^g b + delta (k . q)
// come out of one pass over S. grid (heads, n_seqs), 8 warps: warp w owns the state rows (key
// dims) 16w..16w+15 and lane l the value columns 4l..4l+3, so one row of a warp is one
// coalesced 512-byte float4 access and the fp32 state stays in registers for the whole
// sequence. The prep records arrive in shared memory by bulk copies of GSTEP_TB tokens, one
// block ahead (double-buffered, bounded waits), so no token waits on DRAM. The column sums are
// reduced across the 8 warps through shared memory (one barrier per token; the partials are
// double-buffered by token parity, so the next token's writes never meet this token's reads).
// Every warp then holds o for all 128 columns; warp (t mod 8) applies the gated RMSNorm to
// token t, with its z gate row loaded when the token's block starts.
constexpr int GSTEP_TB = GDN_THREADS / 32;  // tokens per staged block: one per warp

__global__ void __launch_bounds__(GDN_THREADS, 2) gdn_step_kernel(const GdnArgs a) {
  __shared__ __align__(128) float stage[2][GSTEP_TB * GPREP];
  __shared__ float4 part[2][GDN_THREADS / 32][2][32];  // [parity][warp][S^T k | S^T q][lane]
  __shared__ float part_kq[2][GDN_THREADS / 32];
  __shared__ __align__(8) uint64_t bar[2];
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int h = blockIdx.x, seq = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.p.heads;
  const int key_dim = H * GD, value_dim = H * GD, conv_dim = 2 * key_dim + value_dim;
  const int tok0 = a.cu[seq], len = a.cu[seq + 1] - tok0;
  const int pslot = a.prefix_slot ? a.prefix_slot[seq] : -1;
  const int sslot = a.save_slot ? a.save_slot[seq] : -1;
  const bool pvalid = pslot >= 0 && pslot < a.n_slots;
  const bool svalid = sslot >= 0 && sslot < a.n_slots;
  if ((pslot >= a.n_slots || sslot >= a.n_slots) && threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
  const float* recs = a.prep + (size_t(h) * a.n_tokens + tok0) * GPREP;  // this head's records, token-major
  auto stage_block = [&](int b) {  // records of tokens b * TB .. (one thread)
    const uint32_t bytes = uint32_t(min(GSTEP_TB, len - b * GSTEP_TB)) * GPREP * 4;
    mbar_arrive_expect_tx(&bar[b & 1], bytes);
    bulk_load(stage[b & 1], recs + size_t(b) * GSTEP_TB * GPREP, bytes, &bar[b & 1]);
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
    if (len > 0) stage_block(0);
  }

  float4 S[16];  // S[i] = state row 16 * warp + i, columns 4 * lane .. 4 * lane + 3
  {
    const float* src = pvalid ? a.state_pool + (size_t(pslot) * H + h) * GD * GD : nullptr;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      S[i] = src ? reinterpret_cast<const float4*>(src + (16 * warp + i) * GD)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float4 nw = reinterpret_cast<const float4*>(a.p.norm_w)[lane];
  __syncthreads();  // barriers initialised

  for (int b = 0; b * GSTEP_TB < len; ++b) {
    const int nb = min(GSTEP_TB, len - b * GSTEP_TB);
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);  // the z gate of token b * TB + warp (normed by this warp)
    if (warp < nb)
      z = *reinterpret_cast<const float4*>(a.mix + size_t(tok0 + b * GSTEP_TB + warp) * a.ld_mix + conv_dim + h * GD +
                                           4 * lane);
    if (threadIdx.x == 0 && (b + 1) * GSTEP_TB < len) {
      // the other buffer was last read by block b - 1, before the barriers all threads passed since
      fence_proxy_async_smem();
      stage_block(b + 1);
    }
    const bool landed = mbar_wait(&bar[b & 1], (b >> 1) & 1, FAULT_GDN_WAIT_STAGE);
    if (__syncthreads_or(!landed)) break;  // a copy that never landed: give up (fault recorded)
    for (int tt = 0; tt < nb; ++tt) {
      const int t = b * GSTEP_TB + tt;
      const float* rec = stage[b & 1] + tt * GPREP;  // q | k | v | beta, g
      float qr[16], kr[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // the warp's 16 rows of q and k (a broadcast read)
        const float4 q4 = reinterpret_cast<const float4*>(rec + 16 * warp)[i];
        const float4 k4 = reinterpret_cast<const float4*>(rec + GD + 16 * warp)[i];
        qr[4 * i] = q4.x, qr[4 * i + 1] = q4.y, qr[4 * i + 2] = q4.z, qr[4 * i + 3] = q4.w;
        kr[4 * i] = k4.x, kr[4 * i + 1] = k4.y, kr[4 * i + 2] = k4.z, kr[4 * i + 3] = k4.w;
      }
      const float4 v = reinterpret_cast<const float4*>(rec + 2 * GD)[lane];
      const float beta = rec[GQKV], eg = expf(rec[GQKV + 1]);
      float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
      float kq = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        pk.x = fmaf(S[i].x, kr[i], pk.x), pk.y = fmaf(S[i].y, kr[i], pk.y);
        pk.z = fmaf(S[i].z, kr[i], pk.z), pk.w = fmaf(S[i].w, kr[i], pk.w);
        pq.x = fmaf(S[i].x, qr[i], pq.x), pq.y = fmaf(S[i].y, qr[i], pq.y);
        pq.z = fmaf(S[i].z, qr[i], pq.z), pq.w = fmaf(S[i].w, qr[i], pq.w);
        kq = fmaf(kr[i], qr[i], kq);
      }
      const int par = t & 1;
      part[par][warp][0][lane] = pk;
      part[par][warp][1][lane] = pq;
      if (lane == 0) part_kq[par][warp] = kq;
      __syncthreads();
      float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sq = sk;
      float kqs = 0.0f;
#pragma unroll
      for (int w = 0; w < GDN_THREADS / 32; ++w) {  // the same order in every warp: identical sums
        const float4 x = part[par][w][0][lane], y = part[par][w][1][lane];
        sk.x += x.x, sk.y += x.y, sk.z += x.z, sk.w += x.w;
        sq.x += y.x, sq.y += y.y, sq.z += y.z, sq.w += y.w;
        kqs += part_kq[par][w];
      }
      const float4 d = make_float4(beta * (v.x - eg * sk.x), beta * (v.y - eg * sk.y), beta * (v.z - eg * sk.z),
                                   beta * (v.w - eg * sk.w));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        S[i].x = fmaf(kr[i], d.x, eg * S[i].x), S[i].y = fmaf(kr[i], d.y, eg * S[i].y);
        S[i].z = fmaf(kr[i], d.z, eg * S[i].z), S[i].w = fmaf(kr[i], d.w, eg * S[i].w);
      }
      if (warp == tt) {  // gated RMSNorm (TF:175-190) of token t
        const float o[4] = {fmaf(eg, sq.x, d.x * kqs), fmaf(eg, sq.y, d.y * kqs), fmaf(eg, sq.z, d.z * kqs),
                            fmaf(eg, sq.w, d.w * kqs)};
        const float r =
            rsqrtf(warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]) / float(GD) + a.p.eps);
        store_planes4(a.out, a.lo_offset, a.lo8, size_t(tok0 + t) * value_dim + h * GD + 4 * lane,
                      nw.x * (o[0] * r) * silu_approx(z.x), nw.y * (o[1] * r) * silu_approx(z.y),
                      nw.z * (o[2] * r) * silu_approx(z.z), nw.w * (o[3] * r) * silu_approx(z.w));
      }
    }
  }

  if (svalid) {
    float* dst = a.state_pool + (size_t(sslot) * H + h) * GD * GD;
#pragma unroll
    for (int i = 0; i < 16; ++i) reinterpret_cast<float4*>(dst + (16 * warp + i) * GD)[lane] = S[i];
    gdn_save_conv(a, h, tok0, len, pslot, pvalid, sslot);
  }
}

}  // namespace sdb

using namespace sdb;

int sdb_gdn_prep_floats(int heads, int n_tokens) { return n_tokens * heads * GPREP; }

// mode: GDN_AUTO picks the recurrent kernel when no sequence of the batch can be longer than
// one token on average (n_tokens <= n_seqs: single-token appends), the chunk kernel otherwise;
// GDN_CHUNK / GDN_RECURRENT force one.
enum { GDN_AUTO = 0, GDN_CHUNK = 1, GDN_RECURRENT = 2 };

static int sdb_gdn_mixer_mode(const b200_gdn_params* p, const b200_seqs* s, const float* mix, int32_t ld_mix,
                              uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t layer,
                              float* prep, int lo8, int mode, cudaStream_t st) {
  if (!p || !s || !mix || !out) return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: null pointer");
  if (p->dk != GD || p->dv != GD || p->conv_width != 4)
    return sdb_fail(B200_ERR_UNSUPPORTED, "b200_gdn_mixer: only dk = dv = 128 and conv width 4 are built");
  if (!p->conv_w || !p->a_log || !p->dt_bias || !p->norm_w) return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: null param");
  if (s->n_seqs <= 0 || !s->cu_seqlens) return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: empty batch");
  if (s->n_seqs > 65535) return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: at most 65535 sequences per call");
  const bool uses_pool = s->prefix_slot || s->save_slot;
  if (uses_pool && (!pool || !pool->gdn_state || !pool->conv_hist || !pool->slot_len))
    return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: prefix/save slots need a pool");
  if (lo_offset % 4 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: lo_offset must be a multiple of 4");
  GdnArgs a;
  a.p = *p;
  a.cu = s->cu_seqlens;
  a.prefix_slot = s->prefix_slot;
  a.save_slot = s->save_slot;
  a.n_seqs = s->n_seqs;
  a.prep = prep;
  if (!prep) return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: null scratch");
  a.mix = mix;
  a.ld_mix = ld_mix;
  a.out = out;
  a.lo_offset = lo_offset;
  a.lo8 = lo8;
  const int conv_dim = 3 * p->heads * GD;
  if (ld_mix % 4 != 0 || (reinterpret_cast<uintptr_t>(mix) & 15) || (reinterpret_cast<uintptr_t>(out) & 7))
    return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: mix must be 16-byte aligned with ld_mix % 4 == 0, out 8-byte aligned");
  if (ld_mix < conv_dim + p->heads * GD + 2 * p->heads)
    return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: ld_mix is narrower than [q|k|v|z|b|a]");
  a.n_slots = uses_pool ? pool->n_slots : 0;
  a.slot_len = uses_pool ? pool->slot_len : nullptr;
  a.state_pool = uses_pool ? pool->gdn_state + size_t(layer) * pool->n_slots * p->heads * GD * GD : nullptr;
  a.conv_pool = uses_pool ? pool->conv_hist + size_t(layer) * pool->n_slots * 3 * conv_dim : nullptr;
  static DeviceOnce attr;
  const int attr_status = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(gdn_mixer_kernel<GD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(sizeof(GdnSmem<GD>))));
    SDB_CUDA(cudaFuncSetAttribute(gdn_mixer_kernel<GDN_DV_SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(sizeof(GdnSmem<GDN_DV_SPLIT>))));
    return B200_OK;
  });
  if (attr_status != B200_OK) return attr_status;
  a.n_tokens = s->n_tokens;
  const bool recurrent = mode == GDN_RECURRENT || (mode == GDN_AUTO && s->n_tokens <= s->n_seqs);
  if (recurrent && ((reinterpret_cast<uintptr_t>(p->norm_w) & 15) || (reinterpret_cast<uintptr_t>(prep) & 15) ||
                    (a.state_pool && (reinterpret_cast<uintptr_t>(a.state_pool) & 15))))
    return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: norm_w, scratch and the pool's gdn_state must be 16-byte aligned");
  if (s->n_tokens > 65535 * 8 * PREP_TPW_LARGE) return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: too many tokens");
  if (long(s->n_tokens) * p->heads >= 64L * 1024) {  // enough warps at 8 tokens each to fill the GPU
    constexpr int TPW = PREP_TPW_LARGE;
    SDB_CUDA(launch_pdl(gdn_prep_kernel<TPW>, dim3(3 * p->heads, (s->n_tokens + 8 * TPW - 1) / (8 * TPW)), dim3(256), 0,
                        st, a));
  } else {
    SDB_CUDA(launch_pdl(gdn_prep_kernel<1>, dim3(3 * p->heads, (s->n_tokens + 7) / 8), dim3(256), 0, st, a));
  }
  if (recurrent) {
    SDB_CUDA(launch_pdl(gdn_step_kernel, dim3(p->heads, s->n_seqs), dim3(GDN_THREADS), 0, st, a));
    return B200_OK;
  }
  if (long(s->n_seqs) * p->heads * 2 > 148) {  // enough (sequence, head) CTAs: one per head
    SDB_CUDA(launch_pdl(gdn_mixer_kernel<GD>, dim3(p->heads, s->n_seqs), dim3(GDN_THREADS), sizeof(GdnSmem<GD>), st,
                        a));
    return B200_OK;
  }
  // few sequences (latency): a cluster of 128 / GDN_DV_SPLIT CTAs per head, each owning a
  // slice of the value columns
  constexpr int NS = GD / GDN_DV_SPLIT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->heads * NS, s->n_seqs);
  cfg.blockDim = dim3(GDN_THREADS);
  cfg.dynamicSmemBytes = sizeof(GdnSmem<GDN_DV_SPLIT>);
  cfg.stream = st;
  cudaLaunchAttribute attr_cl[2];
  attr_cl[0].id = cudaLaunchAttributeClusterDimension;
  attr_cl[0].val.clusterDim.x = NS;
  attr_cl[0].val.clusterDim.y = 1;
  attr_cl[0].val.clusterDim.z = 1;
  attr_cl[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_cl[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_cl;
  cfg.numAttrs = 2;
  SDB_CUDA(cudaLaunchKernelEx(&cfg, gdn_mixer_kernel<GDN_DV_SPLIT>, a));
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

int sdb_gdn_mixer(const b200_gdn_params* p, const b200_seqs* s, const float* mix, int32_t ld_mix, uint16_t* out,
                  int64_t lo_offset, const b200_prefix_pool* pool, int32_t layer, float* prep, int lo8,
                  cudaStream_t st) {
  return sdb_gdn_mixer_mode(p, s, mix, ld_mix, out, lo_offset, pool, layer, prep, lo8, GDN_AUTO, st);
}

extern "C" int b200_gdn_mixer(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix, int32_t ld_mix,
                              uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t gdn_layer,
                              float* scratch, b200_stream stream) {
  return sdb_gdn_mixer_mode(p, seqs, mix, ld_mix, out, lo_offset, pool, gdn_layer, scratch, 0, GDN_AUTO,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b200_gdn_mixer_recurrent(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix,
                                        int32_t ld_mix, uint16_t* out, int64_t lo_offset,
                                        const b200_prefix_pool* pool, int32_t gdn_layer, float* scratch,
                                        b200_stream stream) {
  return sdb_gdn_mixer_mode(p, seqs, mix, ld_mix, out, lo_offset, pool, gdn_layer, scratch, 0, GDN_RECURRENT,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b200_gdn_mixer_chunked(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix,
                                      int32_t ld_mix, uint16_t* out, int64_t lo_offset,
                                      const b200_prefix_pool* pool, int32_t gdn_layer, float* scratch,
                                      b200_stream stream) {
  return sdb_gdn_mixer_mode(p, seqs, mix, ld_mix, out, lo_offset, pool, gdn_layer, scratch, 0, GDN_CHUNK,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b200_gdn_scratch_floats(int32_t heads, int32_t n_tokens) { return sdb_gdn_prep_floats(heads, n_tokens); }
