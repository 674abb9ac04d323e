// Gated GQA attention for the full-attention layers (TF:647-690).
//
// attn_prep_kernel: one block per token. Warps 0..heads-1 normalise (RMSNorm (1+w),
//   TF:644-645, 663-664) and rotate (partial RoPE on the first rope_dim dims, TF:544-579)
//   one query head each; the next kv_heads warps do the same for the keys, and the last
//   kv_heads warps copy the values. Keys and values go to the batch scratch, and, for a
//   sequence that saves its cache, to the prefix pool as well.
// attn_flash_kernel: tensor-core flash attention over the prefix slot's keys (positions
//   0..P-1) then the sequence's own keys (P..P+j), causal, times sigmoid(gate).
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

template <int HD>
static int launch_attn(const AttnArgs& a, int n_tokens, int n_seqs, int max_len, cudaStream_t st) {
  const int warps = a.p.heads + 2 * a.p.kv_heads;
  SDB_CUDA(launch_pdl(attn_prep_kernel<HD>, dim3(n_tokens), dim3(32 * warps), 0, st, a));
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
