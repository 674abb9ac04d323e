// Embedding lookup, RMSNorm, and the fused option-token decision head.
#include <algorithm>

#include "common.cuh"

namespace sdb {

// x[t, :] = float(table[ids[t], :]); one block per token, 8 bf16 per thread per step.
__global__ void embed_kernel(const int32_t* __restrict__ ids, const uint16_t* __restrict__ table, int hidden,
                             float* __restrict__ x, int vocab) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    raise_fault(FAULT_BAD_INDEX);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + size_t(id) * hidden);
  float4* dst = reinterpret_cast<float4*>(x + size_t(t) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) {
    uint4 v = __ldg(src + i);
    dst[2 * i] = make_float4(bf16_to_f32(v.x & 0xFFFF), bf16_to_f32(v.x >> 16), bf16_to_f32(v.y & 0xFFFF),
                             bf16_to_f32(v.y >> 16));
    dst[2 * i + 1] = make_float4(bf16_to_f32(v.z & 0xFFFF), bf16_to_f32(v.z >> 16), bf16_to_f32(v.w & 0xFFFF),
                                 bf16_to_f32(v.w >> 16));
  }
}


// One warp per row: y = x * rsqrt(mean(x^2) + eps) * (1 + w) as hi/lo planes (lo in bf16, or
// e4m3 with lo8). hidden % 128 == 0.
__global__ void rmsnorm_kernel(const float* __restrict__ x, int rows, int hidden, const float* __restrict__ w,
                               float eps, uint16_t* __restrict__ out, long long lo_offset, int lo8) {
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + size_t(row) * hidden);
  float ss = 0.0f;
  for (int i = lane; i < hidden / 4; i += 32) {
    float4 v = xr[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(hidden) + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  for (int i = lane; i < hidden / 4; i += 32) {
    float4 v = xr[i], g = __ldg(wr + i);
    store_planes4(out, lo_offset, lo8, size_t(row) * hidden + 4 * i, v.x * r * (1.0f + g.x), v.y * r * (1.0f + g.y),
                  v.z * r * (1.0f + g.z), v.w * r * (1.0f + g.w));
  }
}

// Few rows (a latency-bound batch): one 256-thread block per row, the row held in registers
// (hidden <= 4096, hidden % 1024 == 0), so each row costs one load round trip. With `zero`,
// each block also clears row `row` of that fp32 [rows, zero_ld] buffer (zero_n floats, a
// multiple of 4): the next GEMM's split-K accumulator, so that it needs no clearing launch.
__global__ void __launch_bounds__(256) rmsnorm_block_kernel(const float* __restrict__ x, int hidden,
                                                            const float* __restrict__ w, float eps,
                                                            uint16_t* __restrict__ out, long long lo_offset,
                                                            int lo8, float* __restrict__ zero, int zero_ld,
                                                            int zero_n) {
  __shared__ float part[8];
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int row = blockIdx.x, tid = threadIdx.x;
  if (zero) {
    float4* z = reinterpret_cast<float4*>(zero + size_t(row) * zero_ld);
    for (int i = tid; i < zero_n / 4; i += 256) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int n4 = hidden / 1024;  // float4 per thread
  const float4* xr = reinterpret_cast<const float4*>(x + size_t(row) * hidden);
  float4 v[4];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < n4) {
      v[i] = xr[tid + 256 * i];
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float r = rsqrtf(tot / float(hidden) + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < n4) {
      const int j = tid + 256 * i;
      const float4 g = __ldg(wr + j);
      store_planes4(out, lo_offset, lo8, size_t(row) * hidden + 4 * j, v[i].x * r * (1.0f + g.x),
                    v[i].y * r * (1.0f + g.y), v[i].z * r * (1.0f + g.z), v[i].w * r * (1.0f + g.w));
    }
  }
}

// Decision head: one CTA of DECIDE_THREADS per decision row. Gathers the row's last token from
// the fp32 residual stream, applies the final RMSNorm (1 + w), dots it with the option tokens'
// tied-embedding rows, divides by the row's temperature (clamped at 1e-6), takes the masked
// softmax and derives the answer numbers. Each thread holds 8-element chunks c = tid, tid + 256
// of the row (hidden <= 4096, a multiple of 32), so every load of the row, the norm weight and
// the option rows is in flight at once (a single-request forward waits on this kernel's
// latency, not its bytes). kmax <= 16.
constexpr int DECIDE_THREADS = 256;
constexpr int DECIDE_CHUNKS = 4096 / 8 / DECIDE_THREADS;  // 8-element chunks per thread

__global__ void __launch_bounds__(DECIDE_THREADS)
    decide_kernel(const float* __restrict__ x, int hidden, const float* __restrict__ fnorm, float eps,
                  const uint16_t* __restrict__ table, b200_decide_args d, int vocab, int n_tokens) {
  __shared__ float red[17][DECIDE_THREADS / 32];  // [0]: sum of squares, [1 + k]: option k's dot
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int tok = d.last_tok[row];
  if (tok < 0 || tok >= n_tokens) {
    if (threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
    tok = 0;
  }
  const int n = d.n_opts[row];
  const int nk = min(min(n, d.kmax), 16);
  const int n8 = hidden / 8;
  int ids[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    ids[k] = 0;
    if (k < nk) {
      const int id = d.opt_ids[row * d.kmax + k];
      if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
      } else {
        ids[k] = id;
      }
    }
  }
  const float4* xr = reinterpret_cast<const float4*>(x + size_t(tok) * hidden);
  const float4* wr = reinterpret_cast<const float4*>(fnorm);
  float h[DECIDE_CHUNKS][8];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < DECIDE_CHUNKS; ++c) {
    const int j = threadIdx.x + c * DECIDE_THREADS;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (j < n8) {
      a = xr[2 * j];
      b = xr[2 * j + 1];
    }
    h[c][0] = a.x, h[c][1] = a.y, h[c][2] = a.z, h[c][3] = a.w;
    h[c][4] = b.x, h[c][5] = b.y, h[c][6] = b.z, h[c][7] = b.w;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += h[c][e] * h[c][e];
  }
  ss = warp_sum(ss);
  if (lane == 0) red[0][warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < DECIDE_THREADS / 32; ++w) tot += red[0][w];
  const float r = rsqrtf(tot / float(hidden) + eps);
#pragma unroll
  for (int c = 0; c < DECIDE_CHUNKS; ++c) {
    const int j = threadIdx.x + c * DECIDE_THREADS;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (j < n8) {
      a = __ldg(wr + 2 * j);
      b = __ldg(wr + 2 * j + 1);
    }
    const float g[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) h[c][e] = h[c][e] * r * (1.0f + g[e]);
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (k < nk) {
      const uint4* er = reinterpret_cast<const uint4*>(table + size_t(ids[k]) * hidden);
      float acc = 0.0f;
#pragma unroll
      for (int c = 0; c < DECIDE_CHUNKS; ++c) {
        const int j = threadIdx.x + c * DECIDE_THREADS;
        if (j < n8) {
          const uint4 e = __ldg(er + j);
          const uint32_t w4[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc = fmaf(h[c][2 * i], bf16x2_lo(w4[i]), acc);
            acc = fmaf(h[c][2 * i + 1], bf16x2_hi(w4[i]), acc);
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) red[1 + k][warp] = acc;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  const float temp = fmaxf(d.temperature[row], 1e-6f);
  float logit[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    logit[k] = -1e4f;  // MASK_VALUE for slots past n (modeling.py:39, 210-221)
    if (k < nk) {
      float dot = 0.0f;
#pragma unroll
      for (int w = 0; w < DECIDE_THREADS / 32; ++w) dot += red[1 + k][w];
      logit[k] = dot / temp;
    }
  }
  // masked softmax over the first n slots
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < n && k < d.kmax) mx = fmaxf(mx, logit[k]);
  float p[16], sum = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    p[k] = (k < n && k < d.kmax) ? __expf(logit[k] - mx) : 0.0f;
    sum += p[k];
  }
  int best = 0;
  float pmax = -1.0f, mean = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    p[k] /= sum;
    if (k < n && p[k] > pmax) {
      pmax = p[k];
      best = k;
    }
    mean += float(k) * p[k];
  }
  if (lane == 0) {
    for (int k = 0; k < d.kmax; ++k) d.probs[row * d.kmax + k] = p[k];
    float conf, score;
    const int kind = d.kinds[row];
    if (kind == 0) {  // noul: P(true) is slot 1 (prompting.py:27, 153-156)
      score = n > 1 ? p[1] : 0.0f;
      conf = fabsf(2.0f * score - 1.0f);
    } else if (kind == 1) {  // choice: schema.py:185-198
      score = float(best);
      conf = n <= 1 ? 1.0f : fminf(1.0f, fmaxf(0.0f, (float(n) * pmax - 1.0f) / float(n - 1)));
    } else {  // score: expected level and schema.py:141-182
      float tot = 0.0f, m2 = 0.0f, var = 0.0f;
      for (int k = 0; k < n && k < 16; ++k) tot += p[k];
      for (int k = 0; k < n && k < 16; ++k) m2 += float(k) * (p[k] / tot);
      for (int k = 0; k < n && k < 16; ++k) var += (p[k] / tot) * (float(k) - m2) * (float(k) - m2);
      score = mean;
      const float sigma = sqrtf(var), smax = float(n - 1) * 0.5f;
      const float floor_ = d.ordinal_smoothing > 0.0f ? sqrtf(d.ordinal_smoothing) : 0.0f;
      if (n <= 1)
        conf = 1.0f;
      else if (tot <= 0.0f)
        conf = 0.0f;
      else if (smax <= floor_)
        conf = sigma <= floor_ ? 1.0f : 0.0f;
      else
        conf = fminf(1.0f, fmaxf(0.0f, (smax - sigma) / (smax - floor_)));
    }
    d.argmax[row] = best;
    d.confidence[row] = conf;
    d.score[row] = score;
  }
}

// ----------------------------------------------------------------------------- trained readouts
constexpr int HEAD_THREADS = 256;
constexpr int HEAD_KMAX = 32;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < HEAD_THREADS / 32; ++i) t += red[i];
  return t;
}

// v = LayerNorm(RMSNorm_final(x[t])) into shared memory (SlotHead / PointerHead norm of the
// torso's final hidden state, modeling.py:120-121, 154-157); every thread returns after v is
// complete.
__device__ void head_input(const float* __restrict__ x, int hidden, const float* __restrict__ fnorm, float eps,
                           const b200_readout& hd, int t, float* v, float* red) {
  const float* xr = x + size_t(t) * hidden;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += HEAD_THREADS) {
    const float xv = xr[i];
    v[i] = xv;
    ss += xv * xv;
  }
  const float r = rsqrtf(block_sum(ss, red) / float(hidden) + eps);
  float s1 = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += HEAD_THREADS) {
    const float hv = v[i] * r * (1.0f + fnorm[i]);
    v[i] = hv;
    s1 += hv;
  }
  const float mean = block_sum(s1, red) / float(hidden);
  float s2 = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += HEAD_THREADS) {
    const float dv = v[i] - mean;
    s2 += dv * dv;
  }
  const float rs = rsqrtf(block_sum(s2, red) / float(hidden) + hd.ln_eps);
  for (int i = threadIdx.x; i < hidden; i += HEAD_THREADS) v[i] = (v[i] - mean) * rs * hd.ln_w[i] + hd.ln_b[i];
  __syncthreads();
}

// y[o] = b[o] + W[o, :] . v for o < n_out (W [n_out][n_in], nn.Linear layout): warp per
// output row, lanes across the input; gelu applies the exact-erf GELU (nn.GELU default).
__device__ void head_linear(const float* __restrict__ w, const float* __restrict__ b, const float* v, int n_in,
                           int n_out, float* y, bool gelu) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int o = warp; o < n_out; o += HEAD_THREADS / 32) {
    const float* wr = w + size_t(o) * n_in;
    float acc = 0.0f;
    for (int i = lane; i < n_in; i += 32) acc = fmaf(wr[i], v[i], acc);
    acc = warp_sum(acc);
    if (lane == 0) {
      float yv = acc + b[o];
      if (gelu) yv = 0.5f * yv * (1.0f + erff(yv * 0.70710678118654752f));
      y[o] = yv;
    }
  }
  __syncthreads();
}

// temperature, masked softmax over the first n of kmax slots, per-kind answers (the same
// read-back as decide_kernel); run by one thread.
__device__ void head_answers(const b200_decide_args& d, int row, const float* logit, int n) {
  const float temp = fmaxf(d.temperature[row], 1e-6f);
  float mx = -INFINITY;
  for (int k = 0; k < n; ++k) mx = fmaxf(mx, logit[k] / temp);
  float p[HEAD_KMAX], sum = 0.0f;
  for (int k = 0; k < HEAD_KMAX; ++k) {
    p[k] = k < n ? __expf(logit[k] / temp - mx) : 0.0f;
    sum += p[k];
  }
  int best = 0;
  float pmax = -1.0f, mean = 0.0f;
  for (int k = 0; k < HEAD_KMAX; ++k) {
    p[k] = sum > 0.0f ? p[k] / sum : 0.0f;
    if (k < n && p[k] > pmax) {
      pmax = p[k];
      best = k;
    }
    mean += float(k) * p[k];
  }
  for (int k = 0; k < d.kmax; ++k) d.probs[row * d.kmax + k] = p[k];
  float conf, score;
  const int kind = d.kinds[row];
  if (kind == 0) {  // noul: P(true) is slot 1 (prompting.py:27, 153-156)
    score = n > 1 ? p[1] : 0.0f;
    conf = fabsf(2.0f * score - 1.0f);
  } else if (kind == 1) {  // choice: schema.py:185-198
    score = float(best);
    conf = n <= 1 ? 1.0f : fminf(1.0f, fmaxf(0.0f, (float(n) * pmax - 1.0f) / float(n - 1)));
  } else {  // score: expected level and schema.py:141-182
    float tot = 0.0f, m2 = 0.0f, var = 0.0f;
    for (int k = 0; k < n; ++k) tot += p[k];
    for (int k = 0; k < n; ++k) m2 += float(k) * (p[k] / tot);
    for (int k = 0; k < n; ++k) var += (p[k] / tot) * (float(k) - m2) * (float(k) - m2);
    score = mean;
    const float sigma = sqrtf(var), smax = float(n - 1) * 0.5f;
    const float floor_ = d.ordinal_smoothing > 0.0f ? sqrtf(d.ordinal_smoothing) : 0.0f;
    if (n <= 1)
      conf = 1.0f;
    else if (tot <= 0.0f)
      conf = 0.0f;
    else if (smax <= floor_)
      conf = sigma <= floor_ ? 1.0f : 0.0f;
    else
      conf = fminf(1.0f, fmaxf(0.0f, (smax - sigma) / (smax - floor_)));
  }
  d.argmax[row] = best;
  d.confidence[row] = conf;
  d.score[row] = score;
}

// One CTA per decision row. Shared memory: v [hidden] | y [max(out, mlp_hidden)] | q [out] |
// logits [32] | reduction scratch [8].
__global__ void __launch_bounds__(HEAD_THREADS) head_decide_kernel(const float* __restrict__ x, int hidden,
                                                                    const float* __restrict__ fnorm, float eps,
                                                                    b200_readout hd, b200_decide_args d, int n_tokens,
                                                                    int ybuf) {
  extern __shared__ float hsm[];
  pdl_wait();  // inputs come from the kernel before this one (programmatic dependent launch)
  pdl_trigger();
  float* v = hsm;
  float* y = v + hidden;
  float* q = y + ybuf;
  float* logit = q + hd.out;
  float* red = logit + HEAD_KMAX;
  const int row = blockIdx.x;
  int tok = d.last_tok[row];
  if (tok < 0 || tok >= n_tokens) {
    if (threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
    tok = 0;
  }
  const int n = min(min(d.n_opts[row], d.kmax), hd.kind == B200_HEAD_SLOT ? hd.out : HEAD_KMAX);
  head_input(x, hidden, fnorm, eps, hd, tok, v, red);
  if (hd.kind == B200_HEAD_SLOT) {
    if (hd.mlp_hidden > 0) {
      head_linear(hd.w1, hd.b1, v, hidden, hd.mlp_hidden, y, true);
      head_linear(hd.w2, hd.b2, y, hd.mlp_hidden, min(hd.out, d.kmax), logit, false);
    } else {
      head_linear(hd.w1, hd.b1, v, hidden, min(hd.out, d.kmax), logit, false);
    }
  } else {  // pointer
    head_linear(hd.w1, hd.b1, v, hidden, hd.out, q, false);
    const float scale = rsqrtf(float(hd.out));
    for (int k = 0; k < n; ++k) {
      int t = d.opt_tok[row * d.kmax + k];
      if (t < 0 || t >= n_tokens) {
        if (threadIdx.x == 0) raise_fault(FAULT_BAD_INDEX);
        t = 0;
      }
      head_input(x, hidden, fnorm, eps, hd, t, v, red);
      head_linear(hd.w2, hd.b2, v, hidden, hd.out, y, false);
      float part = 0.0f;
      for (int i = threadIdx.x; i < hd.out; i += HEAD_THREADS) part = fmaf(y[i], q[i], part);
      const float dot = block_sum(part, red);
      if (threadIdx.x == 0) logit[k] = dot * scale;
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) head_answers(d, row, logit, n);
}

int sdb_check_readout(const b200_readout* hd, int hidden) {
  if (!hd || !hd->ln_w || !hd->ln_b || !hd->w1 || !hd->b1) return sdb_fail(B200_ERR_ARG, "readout: null weight");
  if (hd->kind != B200_HEAD_SLOT && hd->kind != B200_HEAD_POINTER)
    return sdb_fail(B200_ERR_ARG, "readout: kind must be B200_HEAD_SLOT or B200_HEAD_POINTER");
  if (hd->hidden != hidden || hidden > 4096 || hidden % 32 != 0)
    return sdb_fail(B200_ERR_SHAPE, "readout: hidden must match the torso (<= 4096, a multiple of 32)");
  if (hd->out <= 0 || hd->out > 1024 || hd->mlp_hidden < 0 || hd->mlp_hidden > 4096)
    return sdb_fail(B200_ERR_SHAPE, "readout: out must be 1..1024 and mlp_hidden 0..4096");
  if (hd->kind == B200_HEAD_POINTER && (!hd->w2 || !hd->b2 || hd->mlp_hidden != 0))
    return sdb_fail(B200_ERR_ARG, "readout: a pointer head needs k weights and no mlp_hidden");
  if (hd->kind == B200_HEAD_SLOT && hd->mlp_hidden > 0 && (!hd->w2 || !hd->b2))
    return sdb_fail(B200_ERR_ARG, "readout: a slot head with mlp_hidden needs its second layer");
  return B200_OK;
}

int sdb_decide_readout(const float* x, int32_t hidden, const float* final_norm, float eps, const b200_readout* hd,
                       const b200_decide_args* d, int n_tokens, cudaStream_t st) {
  if (!x || !final_norm || !d) return sdb_fail(B200_ERR_ARG, "b200_decide_readout: null pointer");
  if (int rc = sdb_check_readout(hd, hidden)) return rc;
  if (d->n_rows <= 0) return B200_OK;
  if (d->kmax < 1 || d->kmax > HEAD_KMAX) return sdb_fail(B200_ERR_SHAPE, "b200_decide_readout: kmax must be 1..32");
  if (!d->last_tok || !d->n_opts || !d->kinds || !d->temperature || !d->probs || !d->argmax || !d->confidence ||
      !d->score)
    return sdb_fail(B200_ERR_ARG, "b200_decide_readout: null array");
  if (hd->kind == B200_HEAD_POINTER && !d->opt_tok)
    return sdb_fail(B200_ERR_ARG, "b200_decide_readout: a pointer head needs opt_tok (option token positions)");
  const int ybuf = std::max(hd->out, hd->mlp_hidden);
  const size_t smem = size_t(hidden + ybuf + hd->out + HEAD_KMAX + 8) * 4;  // <= 37 KB by the checks above
  SDB_CUDA(launch_pdl(head_decide_kernel, dim3(d->n_rows), dim3(HEAD_THREADS), smem, st, x, hidden, final_norm, eps,
                      *hd, *d, n_tokens, ybuf));
  return B200_OK;
}

}  // namespace sdb

using namespace sdb;

extern "C" int b200_decide_readout(const float* x, int32_t hidden, const float* final_norm, float eps,
                                   const b200_readout* head, const b200_decide_args* d, int32_t n_tokens,
                                   b200_stream stream) {
  if (n_tokens <= 0) return sdb_fail(B200_ERR_SHAPE, "b200_decide_readout: n_tokens must be positive");
  return sdb_decide_readout(x, hidden, final_norm, eps, head, d, n_tokens, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b200_embed(const int32_t* ids, int32_t n_tokens, const uint16_t* table, int32_t hidden, float* x,
                          b200_stream stream) {
  if (!ids || !table || !x) return sdb_fail(B200_ERR_ARG, "b200_embed: null pointer");
  if (n_tokens <= 0 || hidden % 8 != 0) return sdb_fail(B200_ERR_SHAPE, "b200_embed: bad shape");
  embed_kernel<<<n_tokens, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ids, table, hidden, x, 1 << 30);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

int sdb_embed_vocab(const int32_t* ids, int32_t n_tokens, const uint16_t* table, int32_t hidden, float* x, int vocab,
                    cudaStream_t st) {
  embed_kernel<<<n_tokens, 128, 0, st>>>(ids, table, hidden, x, vocab);
  SDB_LAUNCH_CHECK();
  return B200_OK;
}

// `zero` (optional, fp32 [rows, zero_ld], zero_n floats per row cleared): only with the
// one-block-per-row form, which rmsnorm_folds_zero() tells the caller in advance.
bool rmsnorm_folds_zero(int32_t rows, int32_t hidden) { return rows <= 1024 && hidden % 1024 == 0 && hidden <= 4096; }

int sdb_rmsnorm(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                int64_t lo_offset, int lo8, cudaStream_t st, float* zero, int32_t zero_ld, int32_t zero_n) {
  if (!x || !w || !out) return sdb_fail(B200_ERR_ARG, "b200_rmsnorm: null pointer");
  if (rows <= 0 || hidden % 128 != 0 || lo_offset % 8 != 0 || (reinterpret_cast<uintptr_t>(out) & 15))
    return sdb_fail(B200_ERR_SHAPE, "b200_rmsnorm: hidden % 128 and lo_offset % 8 must be 0, out 16-byte aligned");
  if (zero && (!rmsnorm_folds_zero(rows, hidden) || zero_n % 4 != 0 || zero_ld % 4 != 0 || zero_n > zero_ld ||
               (reinterpret_cast<uintptr_t>(zero) & 15)))
    return sdb_fail(B200_ERR_SHAPE, "b200_rmsnorm: bad region to clear");
  if (rmsnorm_folds_zero(rows, hidden))
    SDB_CUDA(launch_pdl(rmsnorm_block_kernel, dim3(rows), dim3(256), 0, st, x, hidden, w, eps, out, lo_offset, lo8,
                        zero, zero_ld, zero_n));
  else
    SDB_CUDA(launch_pdl(rmsnorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, st, x, rows, hidden, w, eps, out,
                        lo_offset, lo8));
  return B200_OK;
}

extern "C" int b200_rmsnorm(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                            int64_t lo_offset, b200_stream stream) {
  return sdb_rmsnorm(x, rows, hidden, w, eps, out, lo_offset, 0, reinterpret_cast<cudaStream_t>(stream), nullptr, 0, 0);
}

extern "C" int b200_rmsnorm_lo8(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                                int64_t lo_offset, b200_stream stream) {
  if (!lo_offset) return sdb_fail(B200_ERR_ARG, "b200_rmsnorm_lo8: lo_offset must locate the e4m3 plane");
  return sdb_rmsnorm(x, rows, hidden, w, eps, out, lo_offset, 1, reinterpret_cast<cudaStream_t>(stream), nullptr, 0, 0);
}

int sdb_decide_vocab(const float* x, int32_t hidden, const float* final_norm, float eps, const uint16_t* table,
                     const b200_decide_args* d, int vocab, int n_tokens, cudaStream_t st) {
  if (!x || !final_norm || !table || !d) return sdb_fail(B200_ERR_ARG, "b200_decide: null pointer");
  if (d->n_rows <= 0) return B200_OK;
  if (d->kmax < 1 || d->kmax > 16 || hidden > 4096 || hidden % 32 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_decide: kmax must be 1..16 and hidden <= 4096");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(final_norm) | reinterpret_cast<uintptr_t>(table)) & 15)
    return sdb_fail(B200_ERR_SHAPE, "b200_decide: x, final_norm and table must be 16-byte aligned");
  if (!d->last_tok || !d->opt_ids || !d->n_opts || !d->kinds || !d->temperature || !d->probs || !d->argmax ||
      !d->confidence || !d->score)
    return sdb_fail(B200_ERR_ARG, "b200_decide: null array");
  SDB_CUDA(launch_pdl(decide_kernel, dim3(d->n_rows), dim3(DECIDE_THREADS), 0, st, x, hidden, final_norm, eps, table,
                      *d, vocab, n_tokens));
  return B200_OK;
}

extern "C" int b200_decide(const float* x, int32_t hidden, const float* final_norm, float eps, const uint16_t* table,
                           const b200_decide_args* d, b200_stream stream) {
  return sdb_decide_vocab(x, hidden, final_norm, eps, table, d, 1 << 30, 1 << 30,
                          reinterpret_cast<cudaStream_t>(stream));
}
