// Gated-DeltaNet token mixer (after the in-projection GEMM), one CTA per (sequence, head).
//
// Per chunk of GC tokens (TF:234-311, with TF:462-530 fused around it):
//   1. causal depthwise conv (width 4) + SiLU over the head's q, k, v channels, reading the
//      3 previous raw inputs from the previous chunk, the prefix slot, or zeros
//   2. l2norm(q), l2norm(k), q *= dk^-1/2; beta = sigmoid(b); g = -exp(A_log)*softplus(a+dt)
//   3. G = cumsum(g); A = strictly-lower(beta_i k_i.k_j e^{G_i-G_j}); P = lower(q_i.k_j e^{G_i-G_j})
//   4. solve (I + A) [U | W] = [beta v | beta k e^G] by forward substitution (one column per thread)
//   5. Vn = U - W S;  O = (q e^G) S + P Vn;  S = e^{G_last} S + (k e^{G_last - G})^T Vn
//   6. gated RMSNorm: out = norm_w * O * rsqrt(mean O^2 + eps) * silu(z)
// The state S [dk, dv] lives in shared memory in fp32 for the whole sequence; it starts
// from the prefix slot (or zero) and is written back to the save slot at the end.
#include "common.cuh"

namespace sdb {

constexpr int GC = 32;     // chunk length
constexpr int GDK = 128;   // key head dim
constexpr int GDV = 128;   // value head dim
constexpr int GQKV = GDK + GDK + GDV;
constexpr int GPAD = GDK + 1;
constexpr int GDN_THREADS = 256;

struct GdnArgs {
  b200_gdn_params p;
  const int32_t* cu;
  const int32_t* prefix_slot;
  const int32_t* save_slot;
  const float* mix;      // [T, ld_mix]: q | k | v | z | b | a
  int ld_mix;
  uint16_t* out;         // hi plane [T, value_dim]; lo plane at out + lo_offset
  long long lo_offset;
  int32_t* slot_len;
  float* state_pool;     // this layer's [n_slots][heads][dk][dv]
  float* conv_pool;      // this layer's [n_slots][conv_width-1][conv_dim]
  int n_slots;
};

struct GdnSmem {
  float q[GC][GPAD];
  float k[GC][GPAD];
  float v[GC][GDV];   // v, then U, then Vn
  float w[GC][GDK];   // W, then O
  float A[GC][GC + 1];
  float P[GC][GC + 1];
  float S[GDK][GDV];
  float hist[3][GQKV];
  float G[GC], beta[GC], eG[GC];
};

__global__ void __launch_bounds__(GDN_THREADS, 1) gdn_mixer_kernel(const GdnArgs a) {
  extern __shared__ uint8_t gdn_smem_raw[];
  GdnSmem& sm = *reinterpret_cast<GdnSmem*>(gdn_smem_raw);
  const int h = blockIdx.x, seq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.p.heads;
  const int key_dim = H * GDK, value_dim = H * GDV, conv_dim = 2 * key_dim + value_dim;
  const int tok0 = a.cu[seq], len = a.cu[seq + 1] - tok0;
  const int pslot = a.prefix_slot ? a.prefix_slot[seq] : -1;
  const int sslot = a.save_slot ? a.save_slot[seq] : -1;
  const bool pvalid = pslot >= 0 && pslot < a.n_slots;
  const bool svalid = sslot >= 0 && sslot < a.n_slots;
  if ((pslot >= a.n_slots || sslot >= a.n_slots) && tid == 0) raise_fault(FAULT_BAD_INDEX);

  // channel of head-local index c in 0..383 (q, k, v)
  auto chan = [&](int c) { return c < GDK ? h * GDK + c : c < 2 * GDK ? key_dim + h * GDK + (c - GDK) : 2 * key_dim + h * GDV + (c - 2 * GDK); };

  // initial state and conv history
  for (int i = tid; i < GDK * GDV; i += GDN_THREADS)
    (&sm.S[0][0])[i] = pvalid ? a.state_pool[(size_t(pslot) * H + h) * GDK * GDV + i] : 0.0f;
  for (int i = tid; i < 3 * GQKV; i += GDN_THREADS) {
    const int r = i / GQKV, c = i % GQKV;
    sm.hist[r][c] = pvalid ? a.conv_pool[(size_t(pslot) * 3 + r) * conv_dim + chan(c)] : 0.0f;
  }
  const float A_exp = __expf(a.p.a_log[h]);
  const float dtb = a.p.dt_bias[h];
  __syncthreads();

  for (int c0 = 0; c0 < len; c0 += GC) {
    const int L = min(GC, len - c0);
    // ---- 1. conv + SiLU
    for (int i = tid; i < L * GQKV; i += GDN_THREADS) {
      const int j = i / GQKV, c = i % GQKV, ch = chan(c);
      float acc = 0.0f;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int jj = j - 3 + t;
        const float xv = jj < 0 ? sm.hist[3 + jj][c] : a.mix[size_t(tok0 + c0 + jj) * a.ld_mix + ch];
        acc = fmaf(a.p.conv_w[ch * 4 + t], xv, acc);
      }
      acc = silu(acc);
      if (c < GDK) sm.q[j][c] = acc;
      else if (c < 2 * GDK) sm.k[j][c - GDK] = acc;
      else sm.v[j][c - 2 * GDK] = acc;
    }
    __syncthreads();
    // new history = last 3 raw inputs of (history ++ chunk)
    {
      float keep[5];
      int n = 0;
      for (int i = tid; i < 3 * GQKV; i += GDN_THREADS, ++n) {
        const int r = i / GQKV, c = i % GQKV;
        const int jj = L - 3 + r;
        keep[n] = jj < 0 ? sm.hist[3 + jj][c] : a.mix[size_t(tok0 + c0 + jj) * a.ld_mix + chan(c)];
      }
      __syncthreads();
      n = 0;
      for (int i = tid; i < 3 * GQKV; i += GDN_THREADS, ++n) sm.hist[i / GQKV][i % GQKV] = keep[n];
    }
    // ---- 2. l2norm q, k; gating
    for (int j = warp; j < L; j += GDN_THREADS / 32) {
      float sq = 0.0f, sk = 0.0f;
      for (int d = lane; d < GDK; d += 32) {
        sq += sm.q[j][d] * sm.q[j][d];
        sk += sm.k[j][d] * sm.k[j][d];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      const float rq = rsqrtf(sq + 1e-6f) * rsqrtf(float(GDK)), rk = rsqrtf(sk + 1e-6f);
      for (int d = lane; d < GDK; d += 32) {
        sm.q[j][d] *= rq;
        sm.k[j][d] *= rk;
      }
    }
    if (tid < L) {
      const size_t t = size_t(tok0 + c0 + tid);
      const float* ab = a.mix + t * a.ld_mix + conv_dim + value_dim;
      sm.beta[tid] = sigmoid(ab[h]);
      sm.G[tid] = -A_exp * softplus(ab[H + h] + dtb);
    }
    __syncthreads();
    if (tid == 0) {
      float acc = 0.0f;
      for (int j = 0; j < L; ++j) {
        acc += sm.G[j];
        sm.G[j] = acc;
        sm.eG[j] = __expf(acc);
      }
    }
    __syncthreads();
    // ---- 3. A (strictly lower) and P (lower incl. diagonal); lane = column j
    for (int i = warp; i < L; i += GDN_THREADS / 32) {
      const int j = lane;
      float kk = 0.0f, qk = 0.0f;
      if (j <= i && j < L) {
        for (int d = 0; d < GDK; ++d) {
          kk = fmaf(sm.k[i][d], sm.k[j][d], kk);
          qk = fmaf(sm.q[i][d], sm.k[j][d], qk);
        }
        const float dec = __expf(sm.G[i] - sm.G[j]);
        sm.A[i][j] = j < i ? sm.beta[i] * kk * dec : 0.0f;
        sm.P[i][j] = qk * dec;
      }
    }
    __syncthreads();
    // ---- 4. forward substitution, one column per thread (columns 0..127 U, 128..255 W)
    {
      const int c = tid;
      float x[GC];
#pragma unroll
      for (int i = 0; i < GC; ++i) {
        if (i < L) {
          float r = c < GDV ? sm.beta[i] * sm.v[i][c] : sm.beta[i] * sm.k[i][c - GDV] * sm.eG[i];
#pragma unroll
          for (int j = 0; j < i; ++j) r = fmaf(-sm.A[i][j], x[j], r);
          x[i] = r;
        } else {
          x[i] = 0.0f;
        }
      }
      __syncthreads();  // everyone has read v before U overwrites it
      for (int i = 0; i < L; ++i) {
        if (c < GDV) sm.v[i][c] = x[i];
        else sm.w[i][c - GDV] = x[i];
      }
    }
    __syncthreads();
    // ---- 5a. Vn = U - W S   (thread: column c, 16 rows)
    const int c = tid & (GDV - 1), half = tid >> 7;
    {
      float acc[GC / 2];
#pragma unroll
      for (int ii = 0; ii < GC / 2; ++ii) acc[ii] = 0.0f;
      for (int r = 0; r < GDK; ++r) {
        const float s = sm.S[r][c];
#pragma unroll
        for (int ii = 0; ii < GC / 2; ++ii) acc[ii] = fmaf(sm.w[half * (GC / 2) + ii][r], s, acc[ii]);
      }
#pragma unroll
      for (int ii = 0; ii < GC / 2; ++ii) {
        const int i = half * (GC / 2) + ii;
        if (i < L) sm.v[i][c] -= acc[ii];
      }
    }
    __syncthreads();
    // ---- 5b. O = e^G (q S) + P Vn  -> stored in w
    {
      float acc[GC / 2];
#pragma unroll
      for (int ii = 0; ii < GC / 2; ++ii) acc[ii] = 0.0f;
      for (int r = 0; r < GDK; ++r) {
        const float s = sm.S[r][c];
#pragma unroll
        for (int ii = 0; ii < GC / 2; ++ii) acc[ii] = fmaf(sm.q[half * (GC / 2) + ii][r], s, acc[ii]);
      }
#pragma unroll
      for (int ii = 0; ii < GC / 2; ++ii) {
        const int i = half * (GC / 2) + ii;
        if (i < L) {
          float o = acc[ii] * sm.eG[i];
          for (int j = 0; j <= i; ++j) o = fmaf(sm.P[i][j], sm.v[j][c], o);
          acc[ii] = o;
        }
      }
      __syncthreads();  // all reads of w (as W) are done
#pragma unroll
      for (int ii = 0; ii < GC / 2; ++ii) {
        const int i = half * (GC / 2) + ii;
        if (i < L) sm.w[i][c] = acc[ii];
      }
    }
    __syncthreads();
    // ---- 5c. S = e^{G_last} S + (k e^{G_last - G})^T Vn   (thread: column c, 64 rows)
    {
      const float gl = sm.G[L - 1], el = sm.eG[L - 1];
      float kd[GC];
#pragma unroll
      for (int i = 0; i < GC; ++i) kd[i] = i < L ? __expf(gl - sm.G[i]) : 0.0f;
      for (int rr = 0; rr < GDK / 2; ++rr) {
        const int r = half * (GDK / 2) + rr;
        float s = sm.S[r][c] * el;
        for (int i = 0; i < L; ++i) s = fmaf(sm.k[i][r] * kd[i], sm.v[i][c], s);
        sm.S[r][c] = s;
      }
    }
    // ---- 6. gated RMSNorm of O rows -> out
    for (int j = warp; j < L; j += GDN_THREADS / 32) {
      float ss = 0.0f;
      for (int d = lane; d < GDV; d += 32) ss += sm.w[j][d] * sm.w[j][d];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / float(GDV) + a.p.eps);
      const size_t t = size_t(tok0 + c0 + j);
      for (int d = lane; d < GDV; d += 32) {
        const float z = a.mix[t * a.ld_mix + conv_dim + h * GDV + d];
        const float y = a.p.norm_w[d] * (sm.w[j][d] * r) * silu(z);
        const uint16_t hb = f32_to_bf16_rn(y);
        a.out[t * value_dim + h * GDV + d] = hb;
        if (a.lo_offset) a.out[a.lo_offset + t * value_dim + h * GDV + d] = f32_to_bf16_rn(y - bf16_to_f32(hb));
      }
    }
    __syncthreads();
  }

  if (svalid) {
    for (int i = tid; i < GDK * GDV; i += GDN_THREADS)
      a.state_pool[(size_t(sslot) * H + h) * GDK * GDV + i] = (&sm.S[0][0])[i];
    for (int i = tid; i < 3 * GQKV; i += GDN_THREADS) {
      const int r = i / GQKV, cc = i % GQKV;
      a.conv_pool[(size_t(sslot) * 3 + r) * conv_dim + chan(cc)] = sm.hist[r][cc];
    }
    if (h == 0 && tid == 0) a.slot_len[sslot] = (pvalid ? a.slot_len[pslot] : 0) + len;
  }
}

}  // namespace sdb

using namespace sdb;

int sdb_gdn_mixer(const b200_gdn_params* p, const b200_seqs* s, const float* mix, int32_t ld_mix, uint16_t* out,
                  int64_t lo_offset, const b200_prefix_pool* pool, int32_t layer, cudaStream_t st) {
  if (!p || !s || !mix || !out) return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: null pointer");
  if (p->dk != GDK || p->dv != GDV || p->conv_width != 4)
    return sdb_fail(B200_ERR_UNSUPPORTED, "b200_gdn_mixer: only dk = dv = 128 and conv width 4 are built");
  if (!p->conv_w || !p->a_log || !p->dt_bias || !p->norm_w) return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: null param");
  if (s->n_seqs <= 0 || !s->cu_seqlens) return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: empty batch");
  const bool uses_pool = s->prefix_slot || s->save_slot;
  if (uses_pool && (!pool || !pool->gdn_state || !pool->conv_hist || !pool->slot_len))
    return sdb_fail(B200_ERR_ARG, "b200_gdn_mixer: prefix/save slots need a pool");
  GdnArgs a;
  a.p = *p;
  a.cu = s->cu_seqlens;
  a.prefix_slot = s->prefix_slot;
  a.save_slot = s->save_slot;
  a.mix = mix;
  a.ld_mix = ld_mix;
  a.out = out;
  a.lo_offset = lo_offset;
  const int conv_dim = 2 * p->heads * GDK + p->heads * GDV;
  if (ld_mix < conv_dim + p->heads * GDV + 2 * p->heads)
    return sdb_fail(B200_ERR_SHAPE, "b200_gdn_mixer: ld_mix is narrower than [q|k|v|z|b|a]");
  a.n_slots = uses_pool ? pool->n_slots : 0;
  a.slot_len = uses_pool ? pool->slot_len : nullptr;
  a.state_pool = uses_pool ? pool->gdn_state + size_t(layer) * pool->n_slots * p->heads * GDK * GDV : nullptr;
  a.conv_pool = uses_pool ? pool->conv_hist + size_t(layer) * pool->n_slots * 3 * conv_dim : nullptr;
  static bool attr = false;
  if (!attr) {
    SDB_CUDA(cudaFuncSetAttribute(gdn_mixer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GdnSmem))));
    attr = true;
  }
  gdn_mixer_kernel<<<dim3(p->heads, s->n_seqs), GDN_THREADS, sizeof(GdnSmem), st>>>(a);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

extern "C" int b200_gdn_mixer(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix, int32_t ld_mix,
                              uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t gdn_layer,
                              b200_stream stream) {
  return sdb_gdn_mixer(p, seqs, mix, ld_mix, out, lo_offset, pool, gdn_layer, reinterpret_cast<cudaStream_t>(stream));
}
