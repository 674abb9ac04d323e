// Gated GQA attention for the full-attention layers (TF:647-690).
//
// attn_prep_kernel: one block per token. Warps 0..heads-1 normalise (RMSNorm (1+w),
//   TF:644-645, 663-664) and rotate (partial RoPE on the first rope_dim dims, TF:544-579)
//   one query head each; the next kv_heads warps do the same for the keys, and the last
//   kv_heads warps copy the values. Keys and values go to the batch scratch, and, for a
//   sequence that saves its cache, to the prefix pool as well.
// attn_tc_kernel: flash attention on tcgen05 (S and O in tensor memory, P written back to
//   tensor memory as the A operand of P V) over the prefix slot's keys (positions 0..P-1) then
//   the sequence's own keys (P..P+j), causal, times sigmoid(gate); 128-row tiles of the query
//   heads that share a kv head. attn_flash_kernel (mma.sync) serves query groups of other
//   sizes.
#include <mutex>

#include "common.cuh"

namespace sdb {

struct AttnArgs {
  b200_attn_params p;
  const int32_t* cu;
  const int32_t* prefix_slot;
  const int32_t* save_slot;
  int n_seqs;
  const float* qkv;
  int ld_qkv;
  uint16_t* q_buf;
  uint16_t* k_buf;
  uint16_t* v_buf;
  uint16_t* out;
  long long lo_offset;
  int lo8;  // lo plane as e4m3 bytes (B200_LO_E4M3) instead of bf16
  const int32_t* slot_len;
  const int32_t* slot_kv;
  uint16_t* k_pool;   // this layer's [kv_capacity][kv_heads][head_dim]
  uint16_t* v_pool;
  int n_slots;
  int kv_capacity;
};

__device__ __forceinline__ int find_seq(const int32_t* cu, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int HD>
__global__ void attn_prep_kernel(const AttnArgs a) {
  constexpr int PER = HD / 32;
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.p.heads, nkv = a.p.kv_heads;
  if (warp >= nq + 2 * nkv) return;
  const int seq = find_seq(a.cu, a.n_seqs, t);
  const int j = t - a.cu[seq];
  const int ps = a.prefix_slot ? a.prefix_slot[seq] : -1;
  const int ss = a.save_slot ? a.save_slot[seq] : -1;
  const int P = (ps >= 0 && ps < a.n_slots) ? a.slot_len[ps] : 0;
  int pos = P + j;
  if (pos >= a.p.max_pos) {
    if (lane == 0) raise_fault(FAULT_BAD_INDEX);
    pos = a.p.max_pos - 1;
  }
  const float* row = a.qkv + size_t(t) * a.ld_qkv;
  const float* src;
  const float* nw = nullptr;
  uint16_t* dst;
  uint16_t* pool_dst = nullptr;
  // a saving sequence stores its keys / values after the slot's existing ones when it saves
  // into its own prefix slot (append), at the slot's start when it has no prefix; saving into
  // a different slot than its prefix would need the prefix copied and is refused
  bool save = ss >= 0 && ss < a.n_slots && a.k_pool;
  const bool pvalid = ps >= 0 && ps < a.n_slots;
  const int kv0 = save ? a.slot_kv[ss] + (pvalid ? P : 0) : 0;
  if (save && ((pvalid && ps != ss) || a.slot_kv[ss] < 0 || kv0 + j >= a.kv_capacity)) {
    if (lane == 0) raise_fault(FAULT_BAD_INDEX);
    save = false;
  }
  if (warp < nq) {  // query head: columns [h*2*HD, h*2*HD + HD) (TF:658-661)
    src = row + warp * 2 * HD;
    nw = a.p.q_norm;
    dst = a.q_buf + (size_t(t) * nq + warp) * HD;
  } else if (warp < nq + nkv) {
    const int kh = warp - nq;
    src = row + nq * 2 * HD + kh * HD;
    nw = a.p.k_norm;
    dst = a.k_buf + (size_t(t) * nkv + kh) * HD;
    if (save) pool_dst = a.k_pool + (size_t(kv0 + j) * nkv + kh) * HD;
  } else {
    const int vh = warp - nq - nkv;
    src = row + nq * 2 * HD + nkv * HD + vh * HD;
    dst = a.v_buf + (size_t(t) * nkv + vh) * HD;
    if (save) pool_dst = a.v_pool + (size_t(kv0 + j) * nkv + vh) * HD;
  }
  // the lane's PER consecutive elements as 16-byte loads (row and head offsets are multiples of
  // 4 floats) and, below, one 16-byte bf16 store per 8 elements
  static_assert(PER % 4 == 0 || PER == 2, "head_dim / 32 elements per lane");
  constexpr int VW = PER % 4 == 0 ? 4 : 2;  // floats per vector load
  float x[PER];
#pragma unroll
  for (int e = 0; e < PER; e += VW) {
    if constexpr (VW == 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + lane * PER + e);
      x[e] = v.x;
      x[e + 1] = v.y;
      x[e + 2] = v.z;
      x[e + 3] = v.w;
    } else {
      const float2 v = *reinterpret_cast<const float2*>(src + lane * PER + e);
      x[e] = v.x;
      x[e + 1] = v.y;
    }
  }
  if (nw) {
    float ss2 = 0.0f;
#pragma unroll
    for (int e = 0; e < PER; ++e) ss2 += x[e] * x[e];
    ss2 = warp_sum(ss2);
    const float r = rsqrtf(ss2 / float(HD) + a.p.eps);
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] *= r * (1.0f + __ldg(nw + lane * PER + e));
    // partial RoPE: dims [0, rope_dim) rotate as pairs (i, i + rope_dim/2)
    const int half = a.p.rope_dim / 2;
    const int xd = half / PER;  // lane distance between paired elements
    float y[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], xd);
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = lane * PER + e;
      if (i < a.p.rope_dim) {
        const int fi = i < half ? i : i - half;
        const float c = a.p.rope_cos[size_t(pos) * half + fi], s = a.p.rope_sin[size_t(pos) * half + fi];
        x[e] = i < half ? x[e] * c - y[e] * s : x[e] * c + y[e] * s;
      }
    }
  }
  if constexpr (PER % 8 == 0) {
#pragma unroll
    for (int e = 0; e < PER; e += 8) {
      const uint4 b = make_uint4(pack_bf16x2(x[e], x[e + 1]), pack_bf16x2(x[e + 2], x[e + 3]),
                                 pack_bf16x2(x[e + 4], x[e + 5]), pack_bf16x2(x[e + 6], x[e + 7]));
      *reinterpret_cast<uint4*>(dst + lane * PER + e) = b;
      if (pool_dst) *reinterpret_cast<uint4*>(pool_dst + lane * PER + e) = b;
    }
  } else {
#pragma unroll
    for (int e = 0; e < PER; e += 2) {
      const uint32_t b = pack_bf16x2(x[e], x[e + 1]);
      *reinterpret_cast<uint32_t*>(dst + lane * PER + e) = b;
      if (pool_dst) *reinterpret_cast<uint32_t*>(pool_dst + lane * PER + e) = b;
    }
  }
}

// ----------------------------------------------------------------------------- flash kernel
// Tensor-core (mma.sync m16n8k16, bf16 in, fp32 accumulate) flash attention. One CTA = 64
// queries of one sequence and one query head, 4 x FA_DG warps: warp w owns query rows
// 16*(w%4).. and value columns (w/4) * HD/FA_DG ..; the FA_DG warps of a row block each
// compute the same scores (so they agree on the softmax without talking) and a slice of P V.
// Keys stream in tiles of 32 (prefix-pool keys first, then the sequence's own), double
// buffered with cp.async; online softmax in registers; P is fed to the P V product straight
// from the score accumulators. Shared tiles are row-major with 16-byte chunks XOR-swizzled
// by row, so ldmatrix reads are conflict-free.
constexpr int FA_Q = 64;
constexpr int FA_K = 32;
// value-column groups: wide heads split P V and the output over two warp groups, which
// halves each warp's accumulators and doubles the warps that hide latency
template <int HD>
constexpr int fa_dg() { return HD >= 128 ? 2 : 1; }

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// byte offset of 16-byte chunk c of row r in a row-major tile with HD bf16 per row
template <int HD>
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return uint32_t(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(128 * fa_dg<HD>(), 2) attn_flash_kernel(const AttnArgs a) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int DG = fa_dg<HD>(), NT = 128 * DG, DW = HD / DG;  // DW: value columns per warp
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  extern __shared__ uint8_t fa_smem[];
  uint8_t* sQ = fa_smem;                          // [FA_Q][HD]
  uint8_t* sK = sQ + FA_Q * HD * 2;               // [2][FA_K][HD]
  uint8_t* sV = sK + 2 * FA_K * HD * 2;           // [2][FA_K][HD]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = blockIdx.y, h = blockIdx.z;
  const int nq = a.p.heads, nkv = a.p.kv_heads, kh = h / (nq / nkv);
  const int tok0 = a.cu[seq], len = a.cu[seq + 1] - tok0;
  const int q0 = blockIdx.x * FA_Q;
  if (q0 >= len) return;
  const int ps = a.prefix_slot ? a.prefix_slot[seq] : -1;
  bool pv = ps >= 0 && ps < a.n_slots;
  int P = pv ? a.slot_len[ps] : 0;
  if (pv && (a.slot_kv[ps] < 0 || a.slot_kv[ps] + P > a.kv_capacity)) {
    if (tid == 0) raise_fault(FAULT_BAD_INDEX);
    pv = false;
    P = 0;
  }
  const size_t pbase = pv ? size_t(a.slot_kv[ps]) : 0;
  const int n_keys = P + min(len, q0 + FA_Q);   // causal: the tile's last query sees these
  const int n_tiles = (n_keys + FA_K - 1) / FA_K;

  // Q tile (rows past the sequence are zero)
  for (int i = tid; i < FA_Q * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = q0 + r < len;
    const uint16_t* src = a.q_buf + ((size_t(tok0 + q0 + (ok ? r : 0)) * nq + h) * HD) + c * 8;
    cp_async16(sQ + sw_off<HD>(r, c), src, ok);
  }
  auto load_kv = [&](int tile, int buf) {
    for (int i = tid; i < FA_K * CH; i += NT) {
      const int r = i / CH, c = i % CH;
      const int kk = tile * FA_K + r;
      const bool ok = kk < n_keys;
      const uint16_t *ks, *vs;
      if (kk < P) {
        ks = a.k_pool + ((pbase + kk) * nkv + kh) * HD;
        vs = a.v_pool + ((pbase + kk) * nkv + kh) * HD;
      } else {
        const size_t t = size_t(tok0 + (ok ? kk - P : 0));
        ks = a.k_buf + (t * nkv + kh) * HD;
        vs = a.v_buf + (t * nkv + kh) * HD;
      }
      cp_async16(sK + buf * FA_K * HD * 2 + sw_off<HD>(r, c), ks + c * 8, ok);
      cp_async16(sV + buf * FA_K * HD * 2 + sw_off<HD>(r, c), vs + c * 8, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[DW / 8][4];
#pragma unroll
  for (int j = 0; j < DW / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  const float scale = rsqrtf(float(HD));
  const int g = lane >> 2, tq = lane & 3;
  const int qrow0 = (warp & 3) * 16;                    // warp's first row in the tile
  const int col0 = (warp >> 2) * DW;                    // warp's first value column
  const int qpos0 = P + q0 + qrow0 + g, qpos1 = qpos0 + 8;  // positions of this thread's two rows
  const uint32_t sQa = smem_addr(sQ);

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < n_tiles) load_kv(tile + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sKa = smem_addr(sK + buf * FA_K * HD * 2), sVa = smem_addr(sV + buf * FA_K * HD * 2);
    // A warp whose 16 rows are all past the sequence (short sequences), or whose queries all
    // precede this key tile (causal), would only add zeros: it keeps to the loads and barriers.
    if (q0 + qrow0 < len && tile * FA_K <= P + q0 + qrow0 + 15) {
    // ---- S = Q K^T : 16 x 32 per warp
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
    for (int kd = 0; kd < HD / 16; ++kd) {
      uint32_t qa[4];
      {
        const int r = qrow0 + (lane & 15), c = kd * 2 + (lane >> 4);
        ldsm_x4(qa, sQa + sw_off<HD>(r, c));
      }
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {  // two n-tile pairs of 8 keys
        uint32_t kb[4];
        const int r = nb * 16 + (lane & 7) + ((lane >> 4) << 3), c = kd * 2 + ((lane >> 3) & 1);
        ldsm_x4(kb, sKa + sw_off<HD>(r, c));
        mma_bf16_16816(sc[2 * nb], qa, kb[0], kb[1]);
        mma_bf16_16816(sc[2 * nb + 1], qa, kb[2], kb[3]);
      }
    }
    // ---- mask + online softmax (rows g and g+8 of the warp's 16)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = tile * FA_K + j * 8 + tq * 2 + (e & 1);
        const int qp = e < 2 ? qpos0 : qpos1;
        float v = sc[j][e] * scale;
        if (key >= n_keys || key > qp) v = -INFINITY;
        sc[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float alpha[2], rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m_run[r], mx[r]);
      alpha[r] = mn == -INFINITY ? 1.0f : __expf(m_run[r] - mn);
      m_run[r] = mn;
    }
    uint32_t pa[2][4];  // P as A fragments for two k16 steps (keys 0-15, 16-31)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mref = m_run[e >> 1];
        p[e] = mref == -INFINITY ? 0.0f : __expf(sc[j][e] - mref);
        rs[e >> 1] += p[e];
      }
      const int ks = j >> 1, hi = j & 1;
      pa[ks][hi * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[ks][hi * 2 + 1] = pack_bf16x2(p[2], p[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int j = 0; j < DW / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // ---- O += P V   (A fragment register order: rows g / g+8 x keys lo / hi)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const uint32_t a4[4] = {pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3]};
#pragma unroll
      for (int nd = 0; nd < DW / 16; ++nd) {  // 16 value dims per ldmatrix.x4.trans
        uint32_t vb[4];
        const int r = ks * 16 + (lane & 15), c = col0 / 8 + nd * 2 + (lane >> 4);
        ldsm_x4_t(vb, sVa + sw_off<HD>(r, c));
        mma_bf16_16816(o[2 * nd], a4, vb[0], vb[1]);
        mma_bf16_16816(o[2 * nd + 1], a4, vb[2], vb[3]);
      }
    }
    }
    __syncthreads();
  }

  // ---- epilogue: O / l * sigmoid(gate) -> hi/lo planes
  const float inv[2] = {l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f, l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = q0 + qrow0 + g + 8 * r;
    if (q >= len) continue;
    const size_t t = size_t(tok0 + q);
    const float* gate = a.qkv + t * a.ld_qkv + h * 2 * HD + HD;
    uint16_t* dst = a.out + (t * nq + h) * HD;
#pragma unroll
    for (int j = 0; j < DW / 8; ++j) {
      const int d = col0 + j * 8 + tq * 2;
      const float y0 = o[j][2 * r] * inv[r] * sigmoid(gate[d]);
      const float y1 = o[j][2 * r + 1] * inv[r] * sigmoid(gate[d + 1]);
      const uint32_t hp = pack_bf16x2(y0, y1);
      *reinterpret_cast<uint32_t*>(dst + d) = hp;
      if (a.lo_offset && a.lo8)
        *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(a.out + a.lo_offset) + (t * nq + h) * HD + d) =
            f32x2_to_e4m3x2((y0 - bf16x2_lo(hp)) * float(1 << B200_LO8_X_SHIFT),
                            (y1 - bf16x2_hi(hp)) * float(1 << B200_LO8_X_SHIFT));
      else if (a.lo_offset)
        *reinterpret_cast<uint32_t*>(dst + a.lo_offset + d) = lo_pair(y0, y1, hp);
    }
  }
}

// ----------------------------------------------------------------------------- tcgen05 flash kernel
// Flash attention on the 5th-generation tensor cores. One CTA = 128 query rows of one sequence
// and one kv head: the gqa query heads that share the kv head, 128 / gqa positions each (row
// r = position (r / gqa), head (r % gqa)), so a short question fills the MMA and every K / V
// tile serves all gqa heads at once.
//   warp 0      TMA: the Q tile once (a 4-D box over [token][kv head][head in group][dim]),
//               then each key tile's K into a 2-stage ring
//   warp 1      TMEM and the MMAs: S_j = Q K_j^T (M = 128, N = 64 keys, K = head_dim; both
//               operands K-major in shared memory) into one of two S buffers, then
//               O += P_j V_j (A = P_j from TMEM, B = V_j MN-major in shared memory, N = head_dim)
//   warps 2..9  softmax: two warps per TMEM lane quarter, each thread one query row (its lane)
//               and half of the tile's 64 keys; the pair exchanges its row maxima through
//               shared memory, so both take the same decisions. P_j goes to TMEM as bf16.
//               Epilogue: O / l staged in the (then idle) Q / K / V shared memory, then written
//               row by row by whole warps (coalesced gate loads and plane stores)
//   warp 10     TMA: each key tile's V into its own 2-stage ring (freed only after P V)
// Key tiles: the prefix slot's keys [0, P) in tiles of 64 (the last partial), then the
// sequence's own [P, n_keys). Columns of a partial tile and keys after a query's position are
// masked to -inf before the max; rows of a box past the keys hold finite values (the prefix
// pool's other rows, other sequences' keys, or zeros past the tensor).
// Online softmax with a lazy rescale: P = exp(s - m_ref) with m_ref raised (and O, l scaled
// by exp(m_ref_old - m_ref_new), O read from and written back to TMEM by the same threads)
// only when a tile's max exceeds m_ref by more than AT_RESCALE; otherwise P <= e^AT_RESCALE,
// and since O and l share m_ref the quotient is the same.
constexpr int AT_BK = 64;
constexpr int AT_ROWS = 128;
constexpr int AT_SOFTMAX_WARPS = 8;
constexpr int AT_THREADS = 32 * (3 + AT_SOFTMAX_WARPS);  // 352
constexpr int AT_V_WARP = 2 + AT_SOFTMAX_WARPS;          // 10
constexpr float AT_RESCALE = 8.0f;

template <int HD>
struct AtSmem {
  static constexpr int ATOMS = HD / 64;                // 64-wide head_dim atoms
  static constexpr int Q_ATOM = AT_ROWS * 128;         // 128 rows x 128 bytes
  static constexpr int Q_BYTES = ATOMS * Q_ATOM;
  static constexpr int KV_ATOM = AT_BK * 128;          // 64 keys x 128 bytes
  static constexpr int KV_BYTES = ATOMS * KV_ATOM;     // one K or V tile
  static constexpr int BARS = 1 + 2 * 8;               // q_full; k/v full/empty, s full/empty, p_full, pv_done x2
  static constexpr int O_LD = HD + 4;                   // fp32 row stride of the epilogue's staged O
  static constexpr int XCH = 2 * 2 * AT_ROWS * 4;       // row maxima of the two halves, by tile parity
  static constexpr int TOTAL = 1024 + Q_BYTES + 4 * KV_BYTES + XCH + 2 * AT_ROWS * 4 + BARS * 8 + 16;
  static_assert(AT_ROWS * O_LD * 4 <= Q_BYTES + 4 * KV_BYTES, "the staged O fits in the Q / K / V buffers");
  // TMEM columns: O [0, HD), S_b at HD + 64 b, P_b (bf16 pairs) at HD + 128 + 32 b
  static constexpr int S_COL = HD, P_COL = HD + 2 * AT_BK;
  static constexpr int TM_COLS = P_COL + AT_BK <= 256 ? 256 : 512;
  static_assert(P_COL + AT_BK <= 512, "TMEM columns");
};

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKp,
                   const __grid_constant__ CUtensorMap tmVp, const AttnArgs a) {
  using SM = AtSmem<HD>;
  extern __shared__ uint8_t at_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                         // [ATOMS][128 rows][128 B]
  uint8_t* sK = sQ + SM::Q_BYTES;             // [2][ATOMS][64 keys][128 B]
  uint8_t* sV = sK + 2 * SM::KV_BYTES;        // [2][ATOMS][64 keys][128 B]
  float* xmax = reinterpret_cast<float*>(sV + 2 * SM::KV_BYTES);  // [2 parity][2 half][128 rows]
  float* lsum = xmax + 4 * AT_ROWS;                                  // [2 half][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(lsum + 2 * AT_ROWS);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2] the S MMA read the tile
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2] the P V MMA read the tile
  uint64_t* s_full = bars + 9;   // [2] S_j in TMEM
  uint64_t* s_empty = bars + 11; // [2] the softmax warps read S_j
  uint64_t* p_full = bars + 13;  // [2] P_j in TMEM
  uint64_t* pv_done = bars + 15; // [2] O += P_j V_j complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + SM::BARS);

  pdl_wait();  // q / k / v come from the prep kernel before this one
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.y, kh = blockIdx.z;
  const int nq = a.p.heads, nkv = a.p.kv_heads, gqa = nq / nkv, QT = AT_ROWS / gqa;
  const int tok0 = a.cu[seq], len = a.cu[seq + 1] - tok0;
  const int q0 = blockIdx.x * QT;
  if (q0 >= len) {  // the whole CTA leaves before any barrier or TMEM use
    pdl_trigger();
    return;
  }
  const int ps = a.prefix_slot ? a.prefix_slot[seq] : -1;
  bool pv = ps >= 0 && ps < a.n_slots;
  int P = pv ? a.slot_len[ps] : 0;
  if (pv && (a.slot_kv[ps] < 0 || a.slot_kv[ps] + P > a.kv_capacity)) {
    if (threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
    pv = false;
    P = 0;
  }
  const int pbase = pv ? a.slot_kv[ps] : 0;
  const int n_keys = P + min(len, q0 + QT);  // causal: the tile's last position sees these
  const int npt = (P + AT_BK - 1) / AT_BK;   // prefix tiles
  const int nt = npt + (n_keys - P + AT_BK - 1) / AT_BK;
  // tile j covers keys [kk0, kk0 + valid)
  auto tile_start = [&](int j) { return j < npt ? j * AT_BK : P + (j - npt) * AT_BK; };
  auto tile_valid = [&](int j) { return j < npt ? min(AT_BK, P - j * AT_BK) : min(AT_BK, n_keys - tile_start(j)); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], AT_SOFTMAX_WARPS);  // one arrival per softmax warp
      mbar_init(&p_full[b], AT_SOFTMAX_WARPS);
      mbar_init(&pv_done[b], 1);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, SM::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ---------------- Q, then the K ring
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      mbar_arrive_expect_tx(q_full, SM::Q_BYTES);
      for (int at = 0; at < SM::ATOMS; ++at) tma_load_4d(sQ + at * SM::Q_ATOM, &tmQ, q_full, 64 * at, 0, kh, tok0 + q0);
      for (int j = 0; j < nt; ++j) {
        const int b = j & 1;
        mbar_wait_idle(&k_empty[b], ((j >> 1) & 1) ^ 1, FAULT_GEMM_WAIT_EMPTY);
        mbar_arrive_expect_tx(&k_full[b], SM::KV_BYTES);
        const bool pool = j < npt;
        const int row = pool ? pbase + j * AT_BK : tok0 + tile_start(j) - P;
        for (int at = 0; at < SM::ATOMS; ++at)
          tma_load_3d(sK + (b * SM::ATOMS + at) * SM::KV_ATOM, pool ? &tmKp : &tmK, &k_full[b], 64 * at, kh, row);
      }
    }
  } else if (warp == AT_V_WARP) {
    // ---------------- the V ring
    if (lane == 0) {
      for (int j = 0; j < nt; ++j) {
        const int b = j & 1;
        mbar_wait_idle(&v_empty[b], ((j >> 1) & 1) ^ 1, FAULT_GEMM_WAIT_EMPTY);
        mbar_arrive_expect_tx(&v_full[b], SM::KV_BYTES);
        const bool pool = j < npt;
        const int row = pool ? pbase + j * AT_BK : tok0 + tile_start(j) - P;
        for (int at = 0; at < SM::ATOMS; ++at)
          tma_load_3d(sV + (b * SM::ATOMS + at) * SM::KV_ATOM, pool ? &tmVp : &tmV, &v_full[b], 64 * at, kh, row);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMAs: S_j, then O += P_{j-1} V_{j-1} (the softmax of tile j-1 overlaps S_j)
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(AT_ROWS, AT_BK);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(AT_ROWS, HD) | (1u << 16);  // B (V) MN-major
      mbar_wait(q_full, 0, FAULT_GEMM_WAIT_FULL_A);
      for (int j = 0; j <= nt; ++j) {
        if (j < nt) {
          const int b = j & 1;
          mbar_wait(&k_full[b], (j >> 1) & 1, FAULT_GEMM_WAIT_FULL_A);
          if (j >= 2) mbar_wait(&s_empty[b], ((j - 2) >> 1) & 1, FAULT_GEMM_WAIT_EMPTY);
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {  // 16 of head_dim per MMA: atom k / 4, +32 bytes each
            const uint64_t ad = umma_desc_sw128(smem_addr(sQ + (k >> 2) * SM::Q_ATOM)) + 2 * (k & 3);
            const uint64_t bd = umma_desc_sw128(smem_addr(sK + (b * SM::ATOMS + (k >> 2)) * SM::KV_ATOM)) + 2 * (k & 3);
            umma_bf16(tmem + uint32_t(SM::S_COL + AT_BK * b), ad, bd, idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[b]);
          umma_commit(&k_empty[b]);
        }
        if (j >= 1) {
          const int jj = j - 1, b = jj & 1;
          mbar_wait(&v_full[b], (jj >> 1) & 1, FAULT_GEMM_WAIT_FULL_B);
          mbar_wait(&p_full[b], (jj >> 1) & 1, FAULT_GEMM_WAIT_FULL_B);
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < AT_BK / 16; ++k) {  // 16 keys per MMA: 8 TMEM columns of P, 2048 bytes of V
            const uint64_t bd =
                umma_desc_sw128_mn(smem_addr(sV + b * SM::ATOMS * SM::KV_ATOM + k * 2048), SM::KV_ATOM, 1024);
            umma_bf16_ts(tmem, tmem + uint32_t(SM::P_COL + (AT_BK / 2) * b + 8 * k), bd, idesc_pv,
                         (jj > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&v_empty[b]);
          umma_commit(&pv_done[b]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax (warps 2..9: TMEM lane quarter warp % 4, key half hf), then the epilogue
    const int qd = warp & 3, hf = (warp - 2) >> 2, r = 32 * qd + lane;
    const int qloc = r / gqa;
    const int qpos = P + q0 + qloc;  // keys at or before this position are visible
    const uint32_t tl = tmem + (uint32_t(32 * qd) << 16);
    const float scale = rsqrtf(float(HD));
    constexpr int HK = AT_BK / 2;   // keys per thread per tile
    constexpr int HO = HD / 2;      // O columns this warp rescales
    float m_ref = -INFINITY, l = 0.0f;
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1;
      mbar_wait(&s_full[b], (j >> 1) & 1, FAULT_GEMM_WAIT_ACCUM);
      tc_fence_after();
      float x[HK];
      {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tl + uint32_t(SM::S_COL + AT_BK * b + HK * hf), v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < HK; ++c) x[c] = __uint_as_float(v[c]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      const int kk0 = tile_start(j) + HK * hf, valid = tile_valid(j) - HK * hf;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < HK; ++c) {
        const bool vis = c < valid && kk0 + c <= qpos;
        x[c] = vis ? x[c] * scale : -INFINITY;
        mx4[c & 3] = fmaxf(mx4[c & 3], x[c]);
      }
      // the row's max over both halves: through shared memory, by tile parity
      float* xm = xmax + b * 2 * AT_ROWS;
      xm[hf * AT_ROWS + r] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      asm volatile("bar.sync %0, 64;" ::"r"(1 + qd) : "memory");
      const float mt = fmaxf(xm[r], xm[AT_ROWS + r]);
      // lazy rescale (the pair decides alike); warp-wide, since TMEM loads and stores are
      // warp-collective
      const bool raise = mt > m_ref + AT_RESCALE;
      if (__any_sync(0xffffffffu, raise)) {
        // a raised row's old terms shrink by exp(m_old - m_new) (none to keep at m_old = -inf)
        const float m_new = raise ? mt : m_ref;
        float alpha = 1.0f;
        if (raise) alpha = m_ref == -INFINITY ? 0.0f : __expf(m_ref - m_new);
        l *= alpha;
        if (j >= 1) {  // O holds tiles < j: scale this warp's half once their P V products are done
          mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, FAULT_GEMM_WAIT_ACCUM);
          tc_fence_after();
#pragma unroll 1
          for (int c0 = HO * hf; c0 < HO * hf + HO; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tl + uint32_t(c0), v);
            tmem_ld_wait();
            uint4 w[4], w2[4];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              reinterpret_cast<uint32_t*>(w)[c] = __float_as_uint(__uint_as_float(v[c]) * alpha);
              reinterpret_cast<uint32_t*>(w2)[c] = __float_as_uint(__uint_as_float(v[16 + c]) * alpha);
            }
            tmem_st_32x32b_x16(tl + uint32_t(c0), w);
            tmem_st_32x32b_x16(tl + uint32_t(c0 + 16), w2);
          }
          tmem_st_wait();
        }
        m_ref = m_new;
      }
      // P_j into TMEM buffer b (this thread's 32 keys: 16 columns), once P_{j-2} V_{j-2} read it
      if (j >= 2) mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, FAULT_GEMM_WAIT_ACCUM);
      tc_fence_after();
      float rs4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint4 pw[4];
      // masked keys hold -inf, so exp gives 0; a row still at m_ref = -inf has only masked keys
      const float mb = m_ref == -INFINITY ? 0.0f : m_ref;
#pragma unroll
      for (int c = 0; c < HK; c += 2) {
        const float p0 = __expf(x[c] - mb);
        const float p1 = __expf(x[c + 1] - mb);
        rs4[(c >> 1) & 3] += p0 + p1;
        reinterpret_cast<uint32_t*>(pw)[c / 2] = pack_bf16x2(p0, p1);
      }
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      tmem_st_32x32b_x16(tl + uint32_t(SM::P_COL + (AT_BK / 2) * b + (HK / 2) * hf), pw);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    // ---- epilogue 1: O / l (this warp's half of the columns) staged in shared memory
    lsum[hf * AT_ROWS + r] = l;
    mbar_wait(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, FAULT_GEMM_WAIT_ACCUM);
    tc_fence_after();
    float* sO = reinterpret_cast<float*>(sQ);  // Q, K and V are all consumed by now
#pragma unroll 1
    for (int c0 = HO * hf; c0 < HO * hf + HO; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tl + uint32_t(c0), v);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<float4*>(sO + r * SM::O_LD + c0 + c) = make_float4(
            __uint_as_float(v[c]), __uint_as_float(v[c + 1]), __uint_as_float(v[c + 2]), __uint_as_float(v[c + 3]));
    }
    asm volatile("bar.sync 5, %0;" ::"n"(32 * AT_SOFTMAX_WARPS) : "memory");
    // ---- epilogue 2: rows by whole warps: O / l * sigmoid(gate) -> hi / lo planes. A batch of
    // ER rows is loaded (gates read-only, O from shared memory) before any of it is stored, so
    // the loads of a batch overlap rather than wait behind the previous row's stores.
    constexpr int CPL = HD / 32;  // columns per lane
    constexpr int ER = 4;         // rows per batch and warp
    const int sw = warp - 2;
#pragma unroll 1
    for (int rb = sw; rb < AT_ROWS; rb += ER * AT_SOFTMAX_WARPS) {
      float g[ER][CPL], o[ER][CPL], inv[ER];
      bool ok[ER];
#pragma unroll
      for (int e = 0; e < ER; ++e) {
        const int rr = rb + e * AT_SOFTMAX_WARPS, ql = rr / gqa;
        ok[e] = rr < AT_ROWS && q0 + ql < len;
        const float lt = ok[e] ? lsum[rr] + lsum[AT_ROWS + rr] : 0.0f;
        inv[e] = lt > 0.0f ? 1.0f / lt : 0.0f;
        const size_t t = size_t(tok0 + q0 + (ok[e] ? ql : 0));
        const int h = kh * gqa + rr % gqa;
        const float* gate = a.qkv + t * a.ld_qkv + size_t(h) * 2 * HD + HD + CPL * lane;
        const float* orow = sO + (ok[e] ? rr : 0) * SM::O_LD + CPL * lane;
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          const float2 gv = ok[e] ? __ldg(reinterpret_cast<const float2*>(gate + c)) : make_float2(0.f, 0.f);
          const float2 ov = *reinterpret_cast<const float2*>(orow + c);
          g[e][c] = gv.x;
          g[e][c + 1] = gv.y;
          o[e][c] = ov.x;
          o[e][c + 1] = ov.y;
        }
      }
#pragma unroll
      for (int e = 0; e < ER; ++e) {
        if (!ok[e]) continue;
        const int rr = rb + e * AT_SOFTMAX_WARPS, ql = rr / gqa;
        const size_t t = size_t(tok0 + q0 + ql);
        const int h = kh * gqa + rr % gqa;
        float y[CPL];
#pragma unroll
        for (int c = 0; c < CPL; ++c) y[c] = o[e][c] * inv[e] * sigmoid_approx(g[e][c]);
        uint32_t hw[CPL / 2], lw[CPL / 2];
#pragma unroll
        for (int c = 0; c < CPL; c += 2) hw[c / 2] = pack_bf16x2(y[c], y[c + 1]);
        uint16_t* dst = a.out + (t * nq + h) * HD + CPL * lane;
        if constexpr (CPL == 8) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        } else if constexpr (CPL == 4) {
          *reinterpret_cast<uint2*>(dst) = make_uint2(hw[0], hw[1]);
        } else {
          *reinterpret_cast<uint32_t*>(dst) = hw[0];
        }
        if (a.lo_offset) {
          if (a.lo8) {
            constexpr float S8 = float(1 << B200_LO8_X_SHIFT);
            uint8_t* d8 = reinterpret_cast<uint8_t*>(a.out + a.lo_offset) + (t * nq + h) * HD + CPL * lane;
#pragma unroll
            for (int c = 0; c < CPL; c += 2)
              reinterpret_cast<uint16_t*>(d8)[c / 2] = f32x2_to_e4m3x2((y[c] - bf16x2_lo(hw[c / 2])) * S8,
                                                                       (y[c + 1] - bf16x2_hi(hw[c / 2])) * S8);
          } else {
#pragma unroll
            for (int c = 0; c < CPL; c += 2) lw[c / 2] = lo_pair(y[c], y[c + 1], hw[c / 2]);
            uint16_t* dl = dst + a.lo_offset;
            if constexpr (CPL == 8) {
              *reinterpret_cast<uint4*>(dl) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            } else if constexpr (CPL == 4) {
              *reinterpret_cast<uint2*>(dl) = make_uint2(lw[0], lw[1]);
            } else {
              *reinterpret_cast<uint32_t*>(dl) = lw[0];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SM::TM_COLS);
  }
}

// Q [tokens][q heads][head_dim] as 4-D (dim, head in group, kv head, token); K / V scratch and
// the layer's pool as 3-D (dim, kv head, row). Boxes: 64 dims x gqa x 1 x 128/gqa rows for Q,
// 64 dims x 1 x 64 rows for K and V.
template <int HD>
static int launch_attn_tc(const AttnArgs& a, int n_tokens, int n_seqs, int max_len, cudaStream_t st) {
  using SM = AtSmem<HD>;
  const int nq = a.p.heads, nkv = a.p.kv_heads, gqa = nq / nkv, QT = AT_ROWS / gqa;
  CUtensorMap mq, mk, mv, mkp, mvp;
  {
    const uint64_t dims[4] = {uint64_t(HD), uint64_t(gqa), uint64_t(nkv), uint64_t(n_tokens)};
    const uint64_t str[3] = {uint64_t(HD) * 2, uint64_t(gqa) * HD * 2, uint64_t(nq) * HD * 2};
    const uint32_t box[4] = {64, uint32_t(gqa), 1, uint32_t(QT)};
    if (int rc = encode_bf16_sw128(&mq, a.q_buf, 4, dims, str, box)) return rc;
  }
  {
    const uint64_t dims[3] = {uint64_t(HD), uint64_t(nkv), uint64_t(n_tokens)};
    const uint64_t str[2] = {uint64_t(HD) * 2, uint64_t(nkv) * HD * 2};
    const uint32_t box[3] = {64, 1, AT_BK};
    if (int rc = encode_bf16_sw128(&mk, a.k_buf, 3, dims, str, box)) return rc;
    if (int rc = encode_bf16_sw128(&mv, a.v_buf, 3, dims, str, box)) return rc;
    if (a.k_pool) {
      const uint64_t pdims[3] = {uint64_t(HD), uint64_t(nkv), uint64_t(a.kv_capacity)};
      if (int rc = encode_bf16_sw128(&mkp, a.k_pool, 3, pdims, str, box)) return rc;
      if (int rc = encode_bf16_sw128(&mvp, a.v_pool, 3, pdims, str, box)) return rc;
    } else {  // no prefix keys: never read
      mkp = mk;
      mvp = mv;
    }
  }
  static DeviceOnce attr;
  const int r = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL));
    return B200_OK;
  });
  if (r != B200_OK) return r;
  dim3 grid((max_len + QT - 1) / QT, n_seqs, nkv);
  SDB_CUDA(launch_pdl(attn_tc_kernel<HD>, grid, dim3(AT_THREADS), SM::TOTAL, st, mq, mk, mv, mkp, mvp, a));
  return B200_OK;
}

// The tcgen05 kernel takes query groups of 1, 2, 4 or 8 heads per kv head.
static bool attn_tc_ok(const AttnArgs& a) {
  const int gqa = a.p.heads / a.p.kv_heads;
  return gqa == 1 || gqa == 2 || gqa == 4 || gqa == 8;
}

template <int HD>
static int launch_attn(const AttnArgs& a, int n_tokens, int n_seqs, int max_len, cudaStream_t st) {
  const int warps = a.p.heads + 2 * a.p.kv_heads;
  SDB_CUDA(launch_pdl(attn_prep_kernel<HD>, dim3(n_tokens), dim3(32 * warps), 0, st, a));
  if (attn_tc_ok(a)) return launch_attn_tc<HD>(a, n_tokens, n_seqs, max_len, st);
  constexpr int smem = FA_Q * HD * 2 + 4 * FA_K * HD * 2;
  static DeviceOnce attr;  // per head_dim and device
  const int r = once_per_device(attr, [](int) -> int {
    SDB_CUDA(cudaFuncSetAttribute(attn_flash_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    return B200_OK;
  });
  if (r != B200_OK) return r;
  dim3 grid((max_len + FA_Q - 1) / FA_Q, n_seqs, a.p.heads);
  SDB_CUDA(launch_pdl(attn_flash_kernel<HD>, grid, dim3(128 * fa_dg<HD>()), smem, st, a));
  return B200_OK;
}

}  // namespace sdb

using namespace sdb;

int sdb_attention(const b200_attn_params* p, const b200_seqs* s, const float* qkv, int32_t ld_qkv, uint16_t* q_buf,
                  uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool,
                  int32_t layer, int lo8, cudaStream_t st) {
  if (!p || !s || !qkv || !q_buf || !k_buf || !v_buf || !out) return sdb_fail(B200_ERR_ARG, "b200_attention: null pointer");
  if (!p->q_norm || !p->k_norm || !p->rope_cos || !p->rope_sin) return sdb_fail(B200_ERR_ARG, "b200_attention: null param");
  if (p->heads <= 0 || p->kv_heads <= 0 || p->heads % p->kv_heads != 0 || p->heads + 2 * p->kv_heads > 32)
    return sdb_fail(B200_ERR_SHAPE, "b200_attention: bad head counts");
  const int per = p->head_dim / 32;
  const int xd = per ? (p->rope_dim / 2) / per : 0;
  if (p->rope_dim <= 0 || p->rope_dim > p->head_dim || (p->rope_dim / 2) % per != 0 || xd <= 0 || (xd & (xd - 1)))
    return sdb_fail(B200_ERR_SHAPE, "b200_attention: rope_dim/2 / (head_dim/32) must be a power of two");
  if (s->n_seqs <= 0 || s->n_tokens <= 0 || !s->cu_seqlens) return sdb_fail(B200_ERR_SHAPE, "b200_attention: empty batch");
  const bool uses_pool = s->prefix_slot || s->save_slot;
  if (uses_pool && (!pool || !pool->k_cache || !pool->v_cache || !pool->slot_len || !pool->slot_kv))
    return sdb_fail(B200_ERR_ARG, "b200_attention: prefix/save slots need a pool");
  AttnArgs a;
  a.p = *p;
  a.cu = s->cu_seqlens;
  a.prefix_slot = s->prefix_slot;
  a.save_slot = s->save_slot;
  a.n_seqs = s->n_seqs;
  a.qkv = qkv;
  a.ld_qkv = ld_qkv;
  // the prep kernel reads each lane's elements and writes q / k / v as whole vectors
  if (ld_qkv % 4 != 0 || ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q_buf) |
                           reinterpret_cast<uintptr_t>(k_buf) | reinterpret_cast<uintptr_t>(v_buf)) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_attention: qkv and the q/k/v buffers must be 16-byte aligned, ld_qkv % 4 == 0");
  a.q_buf = q_buf;
  a.k_buf = k_buf;
  a.v_buf = v_buf;
  a.out = out;
  a.lo_offset = lo_offset;
  a.lo8 = lo8;
  a.n_slots = uses_pool ? pool->n_slots : 0;
  a.kv_capacity = uses_pool ? pool->kv_capacity : 0;
  a.slot_len = uses_pool ? pool->slot_len : nullptr;
  a.slot_kv = uses_pool ? pool->slot_kv : nullptr;
  const size_t per_layer = uses_pool ? size_t(pool->kv_capacity) * p->kv_heads * p->head_dim : 0;
  a.k_pool = uses_pool ? pool->k_cache + size_t(layer) * per_layer : nullptr;
  a.v_pool = uses_pool ? pool->v_cache + size_t(layer) * per_layer : nullptr;
  if (s->max_len <= 0) return sdb_fail(B200_ERR_SHAPE, "b200_attention: max_len must bound the sequence lengths");
  switch (p->head_dim) {
    case 64: return launch_attn<64>(a, s->n_tokens, s->n_seqs, s->max_len, st);
    case 128: return launch_attn<128>(a, s->n_tokens, s->n_seqs, s->max_len, st);
    case 256: return launch_attn<256>(a, s->n_tokens, s->n_seqs, s->max_len, st);
    default: return sdb_fail(B200_ERR_UNSUPPORTED, "b200_attention: head_dim must be 64, 128 or 256");
  }
}

extern "C" int b200_attention(const b200_attn_params* p, const b200_seqs* seqs, const float* qkv, int32_t ld_qkv,
                              uint16_t* q_buf, uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset,
                              const b200_prefix_pool* pool, int32_t attn_layer, b200_stream stream) {
  return sdb_attention(p, seqs, qkv, ld_qkv, q_buf, k_buf, v_buf, out, lo_offset, pool, attn_layer, 0,
                       reinterpret_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------------------------------- no-allocation variant
// Scratch for b200_attention_noalloc: the post-norm, post-RoPE q / k / v of one call, in a
// file-scope device array that every GPU loading this library holds until the process exits.
// Host code must not pass the symbol itself to a kernel (on the host it names a host-side
// stand-in); it looks the device address up once per device with cudaGetSymbolAddress.
constexpr size_t kAttnNoAllocBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) uint16_t g_attn_noalloc_scratch[kAttnNoAllocBytes / 2];

namespace {
std::mutex g_noalloc_mu;
uint16_t* g_noalloc_ptr[sdb::kMaxDevices] = {};
}  // namespace

extern "C" int b200_attention_noalloc(const b200_attn_params* p, const b200_seqs* seqs, const float* qkv,
                                      int32_t ld_qkv, uint16_t* out, int64_t lo_offset,
                                      const b200_prefix_pool* pool, int32_t attn_layer, b200_stream stream) {
  if (!p || !seqs) return sdb_fail(B200_ERR_ARG, "b200_attention_noalloc: null pointer");
  const size_t per_token = size_t(p->heads + 2 * p->kv_heads) * size_t(p->head_dim);
  if (seqs->n_tokens <= 0 || p->heads <= 0 || p->kv_heads < 0 || p->head_dim <= 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_attention_noalloc: bad shape");
  if (size_t(seqs->n_tokens) * per_token * 2 > kAttnNoAllocBytes)
    return sdb_fail(B200_ERR_SHAPE,
                    "b200_attention_noalloc: tokens x (heads + 2 kv_heads) x head_dim x 2 bytes exceeds the "
                    "8 MiB static scratch; use b200_attention with a caller-allocated scratch");
  int dev = 0;
  SDB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return sdb_fail(B200_ERR_UNSUPPORTED, "b200_attention_noalloc: device id");
  uint16_t* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* ptr = nullptr;
      // the current device is `dev`, so this returns that device's copy of the array
      SDB_CUDA(cudaGetSymbolAddress(&ptr, g_attn_noalloc_scratch));
      g_noalloc_ptr[dev] = static_cast<uint16_t*>(ptr);
    }
    base = g_noalloc_ptr[dev];
  }
  const size_t T = size_t(seqs->n_tokens);
  uint16_t* q_buf = base;
  uint16_t* k_buf = q_buf + T * p->heads * p->head_dim;
  uint16_t* v_buf = k_buf + T * p->kv_heads * p->head_dim;
  const int r = sdb_attention(p, seqs, qkv, ld_qkv, q_buf, k_buf, v_buf, out, lo_offset, pool, attn_layer, 0,
                              reinterpret_cast<cudaStream_t>(stream));
  if (r != B200_OK) sdb_rename_error("b200_attention:", "b200_attention_noalloc:");  // the caller's entry point
  return r;
}
