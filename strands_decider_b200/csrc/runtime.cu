// Model context and the whole-torso prefill (TF:1227-1290) as a native layer loop.
#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"

// error reporting ---------------------------------------------------------------------
static thread_local std::string g_last_error;

void sdb_set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
int sdb_fail(int status, const char* msg) {
  sdb_set_last_error(msg);
  return status;
}
void sdb_rename_error(const char* from, const char* to) {
  const size_t n = std::char_traits<char>::length(from);
  if (g_last_error.compare(0, n, from) == 0) g_last_error = std::string(to) + g_last_error.substr(n);
}

namespace sdb {
__device__ unsigned int g_fault = 0;

int sm_count() {
  static std::mutex mu;
  static int n_sm[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (!n_sm[dev]) {
    int v = 0;
    n_sm[dev] = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
  }
  return n_sm[dev];
}
}  // namespace sdb

// kernels' internal entry points (other translation units)
int sdb_embed_vocab(const int32_t* ids, int32_t n_tokens, const uint16_t* table, int32_t hidden, float* x, int vocab,
                    cudaStream_t st);
int sdb_decide_vocab(const float* x, int32_t hidden, const float* final_norm, float eps, const uint16_t* table,
                     const b200_decide_args* d, int vocab, int n_tokens, cudaStream_t st);
int sdb_gdn_mixer(const b200_gdn_params* p, const b200_seqs* s, const float* mix, int32_t ld_mix, uint16_t* out,
                  int64_t lo_offset, const b200_prefix_pool* pool, int32_t layer, float* prep, int lo8,
                  cudaStream_t st);
int sdb_gdn_prep_floats(int heads, int n_tokens);
namespace sdb {
int sdb_check_readout(const b200_readout* hd, int hidden);
int sdb_decide_readout(const float* x, int32_t hidden, const float* final_norm, float eps, const b200_readout* hd,
                       const b200_decide_args* d, int n_tokens, cudaStream_t st);
}  // namespace sdb
int sdb_attention(const b200_attn_params* p, const b200_seqs* s, const float* qkv, int32_t ld_qkv, uint16_t* q_buf,
                  uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool,
                  int32_t layer, int lo8, cudaStream_t st);
int sdb_rmsnorm(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                int64_t lo_offset, int lo8, cudaStream_t st, float* zero = nullptr, int32_t zero_ld = 0,
                int32_t zero_n = 0);
bool rmsnorm_folds_zero(int32_t rows, int32_t hidden);
namespace sdb {
bool linear_small_m(int32_t m, int32_t format);
}  // namespace sdb

extern "C" const char* b200_last_error(void) { return g_last_error.c_str(); }
extern "C" int b200_version(void) { return 100; }

extern "C" int b200_read_fault(unsigned int* fault_out) {
  if (!fault_out) return sdb_fail(B200_ERR_ARG, "b200_read_fault: null pointer");
  unsigned int v = 0, zero = 0;
  SDB_CUDA(cudaMemcpyFromSymbol(&v, sdb::g_fault, sizeof(v)));
  SDB_CUDA(cudaMemcpyToSymbol(sdb::g_fault, &zero, sizeof(zero)));
  *fault_out = v;
  return B200_OK;
}

// model -------------------------------------------------------------------------------
struct b200_model {
  b200_model_config cfg;
  std::vector<b200_layer_weights> layers;
  std::vector<int> kind_index;  // index among layers of the same kind
  std::vector<bool> layer_set;
  const uint16_t* embed = nullptr;
  const float* final_norm = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  b200_readout readout{};  // kind B200_HEAD_OPTION_TOKEN (0): the option-token logits

  int key_dim() const { return cfg.gdn_heads * cfg.gdn_dk; }
  int value_dim() const { return cfg.gdn_heads * cfg.gdn_dv; }
  int conv_dim() const { return 2 * key_dim() + value_dim(); }
  int gdn_split() const { return conv_dim() + value_dim(); }
  // columns the GDN in-projection writes: [q|k|v|z|b|a] rounded up to a multiple of 32
  // (the padding columns come from zero weight rows)
  int gdn_in_cols() const { return (gdn_split() + 2 * cfg.gdn_heads + 31) / 32 * 32; }
  int attn_qkv() const { return 2 * cfg.attn_heads * cfg.head_dim + 2 * cfg.attn_kv_heads * cfg.head_dim; }
  int attn_o_in() const { return cfg.attn_heads * cfg.head_dim; }
  bool has_gdn() const {
    for (int i = 0; i < cfg.n_layers; ++i)
      if (cfg.layer_kind[i] == B200_LAYER_GDN) return true;
    return false;
  }
  bool dequant_at(int T) const {
    const int from = cfg.dequant_min_tokens == 0 ? 4096 : cfg.dequant_min_tokens;
    return from > 0 && T >= from;
  }
  // GEMMs of this batch run on e4m3 low planes (b200_linear_lo8)
  bool lo8_at(int T) const { return cfg.lo_format == B200_LO_E4M3 && dequant_at(T); }
  bool has_attn() const {
    for (int i = 0; i < cfg.n_layers; ++i)
      if (cfg.layer_kind[i] == B200_LAYER_ATTN) return true;
    return false;
  }
};

namespace {

// Workspace (all offsets 256-byte aligned), for T tokens:
//   x    fp32 [T, hidden]            residual stream (first, so callers can read it back)
//   xn   2 x bf16 [T, hidden]        normed activations as hi/lo planes (GEMM input)
//   mix  fp32 [T, mix_cols]          in-projection outputs (GDN [q|k|v|z|b|a], attention [q,gate|k|v])
//   act  2 x bf16 [T, act_cols]      mixer outputs / SwiGLU outputs as hi/lo planes (GEMM input)
//   q, k, v  bf16                    attention scratch (post norm + RoPE)
//   prep fp32                        GDN scratch (conv / l2norm / gating outputs)
//   wdq  bf16 [N, K]                 one dequantised weight (batches of >= dequant_min_tokens)
//   wdq8 e4m3 [N, K]                 its e4m3 copy (lo_format B200_LO_E4M3)
// With e4m3 low planes the xn / act lo planes hold one byte per element in the same space.
struct WsLayout {
  size_t x, xn, mix, act, q, k, v, prep, wdq, wdq8, total;
  int mix_cols, act_cols;
  long long xn_lo, act_lo;  // element offsets of the lo planes
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

WsLayout layout(const b200_model& m, int T) {
  WsLayout L{};
  const auto& c = m.cfg;
  L.mix_cols = 32;
  if (m.has_gdn()) L.mix_cols = std::max(L.mix_cols, m.gdn_in_cols());
  if (m.has_attn()) L.mix_cols = std::max(L.mix_cols, m.attn_qkv());
  L.act_cols = std::max({c.inter, m.has_gdn() ? m.value_dim() : 0, m.has_attn() ? m.attn_o_in() : 0});
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  L.x = take(size_t(T) * c.hidden * 4);
  const size_t xn_plane = align256(size_t(T) * c.hidden * 2);
  L.xn = take(2 * xn_plane);
  L.xn_lo = (long long)(xn_plane / 2);
  L.mix = take(size_t(T) * L.mix_cols * 4);
  const size_t act_plane = align256(size_t(T) * L.act_cols * 2);
  L.act = take(2 * act_plane);
  L.act_lo = (long long)(act_plane / 2);
  const size_t kvb = size_t(T) * std::max(c.attn_kv_heads * c.head_dim, 8) * 2;
  L.q = take(size_t(T) * std::max(m.attn_o_in(), 8) * 2);
  L.k = take(kvb);
  L.v = take(kvb);
  L.prep = take(m.has_gdn() ? size_t(sdb_gdn_prep_floats(c.gdn_heads, T)) * 4 : 16);
  L.wdq = 0;
  if (m.dequant_at(T)) {
    size_t most = 0;
    for (int i = 0; i < c.n_layers; ++i) {
      const b200_layer_weights& w = m.layers[i];
      for (const b200_qweight* q : {&w.mix_in, &w.mix_out, &w.gate_up, &w.down})
        most = std::max(most, size_t(q->n) * size_t(q->k));
    }
    L.wdq = take(most * 2);
    if (m.lo8_at(T)) L.wdq8 = take(most);
  }
  L.total = off;
  return L;
}

// One linear layer: for large batches the packed weight is first dequantised into the bf16
// buffer (bit-exact with the GEMM's own unpack), then the GEMM streams it by TMA. With e4m3
// low planes (wdq8) the dequantiser writes the two copies b200_linear_lo8 reads.
int run_linear(const b200_model& m, const uint16_t* x, const uint16_t* x_lo, int T, int k, const b200_qweight& w,
               const b200_linear_out& o, uint16_t* wdq, uint8_t* wdq8, b200_stream stream) {
  if (wdq8) {
    if (int rc = b200_dequantize_lo8(&w, wdq, wdq8, stream)) return rc;
    return b200_linear_lo8(x, reinterpret_cast<const uint8_t*>(x_lo), T, k, k, wdq, wdq8, w.n, &o, stream);
  }
  if (wdq && m.dequant_at(T) && w.format != B200_W_BF16) {
    if (int rc = b200_dequantize(&w, wdq, stream)) return rc;
    b200_qweight wb{};
    wb.format = B200_W_BF16;
    wb.n = w.n;
    wb.k = w.k;
    wb.data = wdq;
    return b200_linear(x, x_lo, T, k, k, &wb, &o, stream);
  }
  return b200_linear(x, x_lo, T, k, k, &w, &o, stream);
}

int check_qw(const b200_qweight& w, int n_min, int k, const char* what) {
  if (!w.data || w.n < n_min || w.k != k || w.n % 256 != 0) {
    std::string msg = std::string("b200_model_set_layer: bad weight ") + what;
    return sdb_fail(B200_ERR_SHAPE, msg.c_str());
  }
  return B200_OK;
}

}  // namespace

extern "C" int b200_model_create(const b200_model_config* cfg, b200_model** out) {
  if (!cfg || !out) return sdb_fail(B200_ERR_ARG, "b200_model_create: null pointer");
  if (cfg->n_layers <= 0 || cfg->n_layers > 64 || cfg->hidden % 128 != 0 || cfg->inter % 128 != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_model_create: bad layer count or hidden/inter not a multiple of 128");
  if (cfg->weight_format < 0 || cfg->weight_format > 3) return sdb_fail(B200_ERR_FORMAT, "b200_model_create: format");
  if (cfg->lo_format != B200_LO_BF16 && cfg->lo_format != B200_LO_E4M3)
    return sdb_fail(B200_ERR_ARG, "b200_model_create: unknown lo_format");
  auto* m = new b200_model();
  m->cfg = *cfg;
  m->layers.resize(cfg->n_layers);
  m->layer_set.assign(cfg->n_layers, false);
  m->kind_index.resize(cfg->n_layers);
  int ng = 0, na = 0;
  for (int i = 0; i < cfg->n_layers; ++i) {
    if (cfg->layer_kind[i] == B200_LAYER_GDN) m->kind_index[i] = ng++;
    else if (cfg->layer_kind[i] == B200_LAYER_ATTN) m->kind_index[i] = na++;
    else {
      delete m;
      return sdb_fail(B200_ERR_ARG, "b200_model_create: unknown layer kind");
    }
  }
  if (ng && (cfg->gdn_dk != 128 || cfg->gdn_dv != 128 || cfg->conv_width != 4)) {
    delete m;
    return sdb_fail(B200_ERR_UNSUPPORTED, "b200_model_create: GDN layers need dk = dv = 128, conv width 4");
  }
  *out = m;
  return B200_OK;
}

extern "C" int b200_model_destroy(b200_model* m) {
  delete m;
  return B200_OK;
}

extern "C" int b200_model_set_layer(b200_model* m, int32_t layer, const b200_layer_weights* w) {
  if (!m || !w) return sdb_fail(B200_ERR_ARG, "b200_model_set_layer: null pointer");
  if (layer < 0 || layer >= m->cfg.n_layers) return sdb_fail(B200_ERR_ARG, "b200_model_set_layer: layer out of range");
  const auto& c = m->cfg;
  if (!w->input_norm || !w->post_norm) return sdb_fail(B200_ERR_ARG, "b200_model_set_layer: null norm");
  const bool gdn = c.layer_kind[layer] == B200_LAYER_GDN;
  int rc;
  if (gdn) {
    if ((rc = check_qw(w->mix_in, m->gdn_split() + 2 * c.gdn_heads, c.hidden, "mix_in"))) return rc;
    if ((rc = check_qw(w->mix_out, c.hidden, m->value_dim(), "mix_out"))) return rc;
    if (!w->gdn.conv_w || !w->gdn.a_log || !w->gdn.dt_bias || !w->gdn.norm_w)
      return sdb_fail(B200_ERR_ARG, "b200_model_set_layer: null GDN parameter");
  } else {
    if ((rc = check_qw(w->mix_in, m->attn_qkv(), c.hidden, "mix_in"))) return rc;
    if ((rc = check_qw(w->mix_out, c.hidden, m->attn_o_in(), "mix_out"))) return rc;
    if (!w->q_norm || !w->k_norm) return sdb_fail(B200_ERR_ARG, "b200_model_set_layer: null q/k norm");
  }
  if ((rc = check_qw(w->gate_up, 2 * c.inter, c.hidden, "gate_up"))) return rc;
  if ((rc = check_qw(w->down, c.hidden, c.inter, "down"))) return rc;
  m->layers[layer] = *w;
  if (gdn) {
    m->layers[layer].gdn.heads = c.gdn_heads;
    m->layers[layer].gdn.dk = c.gdn_dk;
    m->layers[layer].gdn.dv = c.gdn_dv;
    m->layers[layer].gdn.conv_width = c.conv_width;
    m->layers[layer].gdn.eps = c.eps;
  }
  m->layer_set[layer] = true;
  return B200_OK;
}

extern "C" int b200_model_set_globals(b200_model* m, const uint16_t* embed, const float* final_norm,
                                      const float* rope_cos, const float* rope_sin) {
  if (!m || !embed || !final_norm) return sdb_fail(B200_ERR_ARG, "b200_model_set_globals: null pointer");
  if (m->has_attn() && (!rope_cos || !rope_sin)) return sdb_fail(B200_ERR_ARG, "b200_model_set_globals: rope tables");
  m->embed = embed;
  m->final_norm = final_norm;
  m->rope_cos = rope_cos;
  m->rope_sin = rope_sin;
  return B200_OK;
}

// After a forward that saved states: each saving sequence's slot holds its prefix's tokens
// (when it appended to its own slot) plus its own. Updated once, after every layer has read
// the old lengths.
__global__ void slot_len_kernel(const int32_t* cu, int n_seqs, const int32_t* prefix_slot, const int32_t* save_slot,
                                int32_t* slot_len, int n_slots) {
  sdb::pdl_wait();  // slot lengths are read by every layer's kernels before this one
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seqs) return;
  const int ss = save_slot[s];
  if (ss < 0 || ss >= n_slots) return;
  const int ps = prefix_slot ? prefix_slot[s] : -1;
  const int base = (ps >= 0 && ps < n_slots) ? slot_len[ps] : 0;
  slot_len[ss] = base + cu[s + 1] - cu[s];
}

extern "C" int b200_model_set_readout(b200_model* m, const b200_readout* head) {
  if (!m) return sdb_fail(B200_ERR_ARG, "b200_model_set_readout: null model");
  if (!head) {
    m->readout = b200_readout{};
    return B200_OK;
  }
  if (int rc = sdb::sdb_check_readout(head, m->cfg.hidden)) return rc;
  m->readout = *head;
  return B200_OK;
}

extern "C" int b200_model_workspace_bytes(const b200_model* m, int32_t max_tokens, size_t* bytes) {
  if (!m || !bytes || max_tokens <= 0) return sdb_fail(B200_ERR_ARG, "b200_model_workspace_bytes: bad argument");
  *bytes = layout(*m, max_tokens).total;
  return B200_OK;
}

extern "C" int b200_model_forward(b200_model* m, const int32_t* ids, const b200_seqs* seqs, const b200_prefix_pool* pool,
                                  const b200_decide_args* decide, void* workspace, size_t workspace_bytes,
                                  b200_stream stream) {
  if (!m || !ids || !seqs || !workspace) return sdb_fail(B200_ERR_ARG, "b200_model_forward: null pointer");
  if (!m->embed || !m->final_norm) return sdb_fail(B200_ERR_ARG, "b200_model_forward: globals not set");
  for (int i = 0; i < m->cfg.n_layers; ++i)
    if (!m->layer_set[i]) return sdb_fail(B200_ERR_ARG, "b200_model_forward: a layer has no weights");
  const int T = seqs->n_tokens;
  if (T <= 0 || seqs->n_seqs <= 0) return sdb_fail(B200_ERR_SHAPE, "b200_model_forward: empty batch");
  const WsLayout L = layout(*m, T);
  if (workspace_bytes < L.total) return sdb_fail(B200_ERR_WORKSPACE, "b200_model_forward: workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return sdb_fail(B200_ERR_SHAPE, "b200_model_forward: workspace must be 256-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto& c = m->cfg;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* x = reinterpret_cast<float*>(ws + L.x);
  uint16_t* xn = reinterpret_cast<uint16_t*>(ws + L.xn);
  float* mix = reinterpret_cast<float*>(ws + L.mix);
  uint16_t* act = reinterpret_cast<uint16_t*>(ws + L.act);
  uint16_t* qb = reinterpret_cast<uint16_t*>(ws + L.q);
  uint16_t* kb = reinterpret_cast<uint16_t*>(ws + L.k);
  uint16_t* vb = reinterpret_cast<uint16_t*>(ws + L.v);
  float* prep = reinterpret_cast<float*>(ws + L.prep);
  uint16_t* wdq = L.wdq ? reinterpret_cast<uint16_t*>(ws + L.wdq) : nullptr;
  uint8_t* wdq8 = L.wdq8 ? ws + L.wdq8 : nullptr;
  const int lo8 = wdq8 ? 1 : 0;
  const uint16_t* xn_lo = xn + L.xn_lo;

  int rc;
  if ((rc = sdb_embed_vocab(ids, T, m->embed, c.hidden, x, c.vocab, st))) return rc;
  for (int li = 0; li < c.n_layers; ++li) {
    const b200_layer_weights& w = m->layers[li];
    // A small batch's in-projection splits K and accumulates its partials into `mix`: the
    // norm before it clears `mix` and the GEMM adds into it (no clearing launch of its own).
    const int n_in = c.layer_kind[li] == B200_LAYER_GDN ? m->gdn_in_cols() : m->attn_qkv();
    const bool fold = !wdq8 && !m->dequant_at(T) && sdb::linear_small_m(T, w.mix_in.format) &&
                      rmsnorm_folds_zero(T, c.hidden);
    if ((rc = sdb_rmsnorm(x, T, c.hidden, w.input_norm, c.eps, xn, L.xn_lo, lo8, st, fold ? mix : nullptr, n_in,
                          n_in)))
      return rc;
    const int in_ep = fold ? B200_EP_RESID_ADD : B200_EP_STORE;
    int mix_in_dim;
    if (c.layer_kind[li] == B200_LAYER_GDN) {
      const int n = m->gdn_in_cols();
      b200_linear_out o{in_ep, n, mix, n, 0};
      if ((rc = run_linear(*m, xn, xn_lo, T, c.hidden, w.mix_in, o, wdq, wdq8, stream))) return rc;
      if ((rc = sdb_gdn_mixer(&w.gdn, seqs, mix, n, act, L.act_lo, pool, m->kind_index[li], prep, lo8, st)))
        return rc;
      mix_in_dim = m->value_dim();
    } else {
      const int n = m->attn_qkv();
      b200_linear_out o{in_ep, n, mix, n, 0};
      if ((rc = run_linear(*m, xn, xn_lo, T, c.hidden, w.mix_in, o, wdq, wdq8, stream))) return rc;
      b200_attn_params ap{c.attn_heads, c.attn_kv_heads, c.head_dim, c.rope_dim, c.max_pos, c.eps,
                          w.q_norm, w.k_norm, m->rope_cos, m->rope_sin};
      if ((rc = sdb_attention(&ap, seqs, mix, n, qb, kb, vb, act, L.act_lo, pool, m->kind_index[li], lo8, st)))
        return rc;
      mix_in_dim = m->attn_o_in();
    }
    b200_linear_out r{B200_EP_RESID_ADD, c.hidden, x, c.hidden, 0};
    if ((rc = run_linear(*m, act, act + L.act_lo, T, mix_in_dim, w.mix_out, r, wdq, wdq8, stream))) return rc;
    if ((rc = sdb_rmsnorm(x, T, c.hidden, w.post_norm, c.eps, xn, L.xn_lo, lo8, st))) return rc;
    b200_linear_out g{B200_EP_SWIGLU, 2 * c.inter, act, c.inter, L.act_lo, lo8 ? B200_LO_E4M3 : B200_LO_BF16};
    if ((rc = run_linear(*m, xn, xn_lo, T, c.hidden, w.gate_up, g, wdq, wdq8, stream))) return rc;
    b200_linear_out d{B200_EP_RESID_ADD, c.hidden, x, c.hidden, 0};
    if ((rc = run_linear(*m, act, act + L.act_lo, T, c.inter, w.down, d, wdq, wdq8, stream))) return rc;
  }
  if (seqs->save_slot) {
    if (!pool || !pool->slot_len) return sdb_fail(B200_ERR_ARG, "b200_model_forward: save slots need a pool");
    SDB_CUDA(sdb::launch_pdl(slot_len_kernel, dim3((seqs->n_seqs + 127) / 128), dim3(128), 0, st, seqs->cu_seqlens,
                        seqs->n_seqs, seqs->prefix_slot, seqs->save_slot, pool->slot_len, pool->n_slots));
  }
  if (decide && decide->n_rows > 0) {
    if (m->readout.kind != B200_HEAD_OPTION_TOKEN) {
      if ((rc = sdb::sdb_decide_readout(x, c.hidden, m->final_norm, c.eps, &m->readout, decide, T, st))) return rc;
    } else if ((rc = sdb_decide_vocab(x, c.hidden, m->final_norm, c.eps, m->embed, decide, c.vocab, T, st))) {
      return rc;
    }
  }
  return B200_OK;
}
