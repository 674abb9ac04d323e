// Gated GQA attention for the full-attention layers (TF:647-690).
//
// attn_prep_kernel: one block per token. Warps 0..heads-1 normalise (RMSNorm (1+w),
//   TF:644-645, 663-664) and rotate (partial RoPE on the first rope_dim dims, TF:544-579)
//   one query head each; the next kv_heads warps do the same for the keys, and the last
//   kv_heads warps copy the values. Keys and values go to the batch scratch, and, for a
//   sequence that saves its cache, to the prefix pool as well.
// attn_kernel: one warp per (token, query head): online softmax over the prefix slot's
//   keys (positions 0..P-1) then the sequence's own keys (P..P+j), times sigmoid(gate).
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
  bool save = ss >= 0 && ss < a.n_slots && a.k_pool;
  if (save && (a.slot_kv[ss] < 0 || a.slot_kv[ss] + j >= a.kv_capacity)) {
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
    if (save) pool_dst = a.k_pool + (size_t(a.slot_kv[ss] + j) * nkv + kh) * HD;
  } else {
    const int vh = warp - nq - nkv;
    src = row + nq * 2 * HD + nkv * HD + vh * HD;
    dst = a.v_buf + (size_t(t) * nkv + vh) * HD;
    if (save) pool_dst = a.v_pool + (size_t(a.slot_kv[ss] + j) * nkv + vh) * HD;
  }
  float x[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) x[e] = src[lane * PER + e];
  if (nw) {
    float ss2 = 0.0f;
#pragma unroll
    for (int e = 0; e < PER; ++e) ss2 += x[e] * x[e];
    ss2 = warp_sum(ss2);
    const float r = rsqrtf(ss2 / float(HD) + a.p.eps);
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = x[e] * r * (1.0f + nw[lane * PER + e]);
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
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const uint16_t b = f32_to_bf16_rn(x[e]);
    dst[lane * PER + e] = b;
    if (pool_dst) pool_dst[lane * PER + e] = b;
  }
}

template <int HD>
__global__ void attn_kernel(const AttnArgs a, int n_tokens) {
  constexpr int PER = HD / 32;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nq = a.p.heads, nkv = a.p.kv_heads;
  const int t = gw / nq, h = gw % nq;
  if (t >= n_tokens) return;
  const int kh = h / (nq / nkv);
  const int seq = find_seq(a.cu, a.n_seqs, t);
  const int tok0 = a.cu[seq], j = t - tok0;
  const int ps = a.prefix_slot ? a.prefix_slot[seq] : -1;
  bool pv = ps >= 0 && ps < a.n_slots;
  int P = pv ? a.slot_len[ps] : 0;
  if (pv && (a.slot_kv[ps] < 0 || a.slot_kv[ps] + P > a.kv_capacity)) {
    if (lane == 0) raise_fault(FAULT_BAD_INDEX);
    pv = false;
    P = 0;
  }
  const float scale = rsqrtf(float(HD));
  float q[PER], acc[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    q[e] = bf16_to_f32(a.q_buf[(size_t(t) * nq + h) * HD + lane * PER + e]) * scale;
    acc[e] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  auto step = [&](const uint16_t* kp, const uint16_t* vp) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < PER; ++e) s = fmaf(q[e], bf16_to_f32(kp[lane * PER + e]), s);
    s = warp_sum(s);
    const float mn = fmaxf(m, s);
    const float alpha = __expf(m - mn), pr = __expf(s - mn);
    l = l * alpha + pr;
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = fmaf(pr, bf16_to_f32(vp[lane * PER + e]), acc[e] * alpha);
    m = mn;
  };
  if (pv) {
    const size_t base = size_t(a.slot_kv[ps]);
    for (int i = 0; i < P; ++i)
      step(a.k_pool + ((base + i) * nkv + kh) * HD, a.v_pool + ((base + i) * nkv + kh) * HD);
  }
  for (int i = 0; i <= j; ++i)
    step(a.k_buf + (size_t(tok0 + i) * nkv + kh) * HD, a.v_buf + (size_t(tok0 + i) * nkv + kh) * HD);
  const float* gate = a.qkv + size_t(t) * a.ld_qkv + h * 2 * HD + HD;
  const float inv = 1.0f / l;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const float y = acc[e] * inv * sigmoid(gate[lane * PER + e]);
    const size_t o = (size_t(t) * nq + h) * HD + lane * PER + e;
    const uint16_t hb = f32_to_bf16_rn(y);
    a.out[o] = hb;
    if (a.lo_offset) a.out[a.lo_offset + o] = f32_to_bf16_rn(y - bf16_to_f32(hb));
  }
}

template <int HD>
static int launch_attn(const AttnArgs& a, int n_tokens, cudaStream_t st) {
  const int warps = a.p.heads + 2 * a.p.kv_heads;
  attn_prep_kernel<HD><<<n_tokens, 32 * warps, 0, st>>>(a);
  SDB_LAUNCH_CHECK();
  const long total = long(n_tokens) * a.p.heads;
  attn_kernel<HD><<<int((total + 7) / 8), 256, 0, st>>>(a, n_tokens);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace sdb

using namespace sdb;

int sdb_attention(const b200_attn_params* p, const b200_seqs* s, const float* qkv, int32_t ld_qkv, uint16_t* q_buf,
                  uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool,
                  int32_t layer, cudaStream_t st) {
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
  a.q_buf = q_buf;
  a.k_buf = k_buf;
  a.v_buf = v_buf;
  a.out = out;
  a.lo_offset = lo_offset;
  a.n_slots = uses_pool ? pool->n_slots : 0;
  a.kv_capacity = uses_pool ? pool->kv_capacity : 0;
  a.slot_len = uses_pool ? pool->slot_len : nullptr;
  a.slot_kv = uses_pool ? pool->slot_kv : nullptr;
  const size_t per_layer = uses_pool ? size_t(pool->kv_capacity) * p->kv_heads * p->head_dim : 0;
  a.k_pool = uses_pool ? pool->k_cache + size_t(layer) * per_layer : nullptr;
  a.v_pool = uses_pool ? pool->v_cache + size_t(layer) * per_layer : nullptr;
  switch (p->head_dim) {
    case 64: return launch_attn<64>(a, s->n_tokens, st);
    case 128: return launch_attn<128>(a, s->n_tokens, st);
    case 256: return launch_attn<256>(a, s->n_tokens, st);
    default: return sdb_fail(B200_ERR_UNSUPPORTED, "b200_attention: head_dim must be 64, 128 or 256");
  }
}

extern "C" int b200_attention(const b200_attn_params* p, const b200_seqs* seqs, const float* qkv, int32_t ld_qkv,
                              uint16_t* q_buf, uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset,
                              const b200_prefix_pool* pool, int32_t attn_layer, b200_stream stream) {
  return sdb_attention(p, seqs, qkv, ld_qkv, q_buf, k_buf, v_buf, out, lo_offset, pool, attn_layer,
                       reinterpret_cast<cudaStream_t>(stream));
}
