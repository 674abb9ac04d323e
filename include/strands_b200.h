/*
 * strands_b200.h -- C ABI of the B200 (sm_100a) scoring-prefill backend for strands-decider.
 *
 * The reference runs its scoring prefill in Python: `SystemOneEngine._slot_probs_batched`
 * and `_slot_probs_shared_prefix` (src/strands_decider/infer.py:253-337) call the
 * transformers Qwen3.5 torso (models/qwen3_5/modeling_qwen3_5.py, cited TF:line) and then
 * the readout in src/strands_decider/modeling.py. This library replaces everything below
 * those two methods: the torso forward, the prefix-cache fork, and the readout.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless its comment says otherwise;
 *     the caller (torch) allocates and owns all memory. Nothing here calls cudaMalloc.
 *   - Every call is asynchronous on the given stream (a cudaStream_t) and returns an
 *     int status (B200_OK == 0). A non-zero status leaves the stream usable;
 *     b200_last_error() returns a message for the calling thread.
 *   - Token batches are ragged and packed: sequence i owns tokens
 *     [cu_seqlens[i], cu_seqlens[i+1]) of every [tokens, ...] activation array.
 *   - bf16 tensors are passed as uint16_t bit patterns.
 */
#ifndef STRANDS_B200_H
#define STRANDS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* b200_stream; /* cudaStream_t */

/* ---------------------------------------------------------------- status codes */
enum b200_status {
  B200_OK = 0,
  B200_ERR_ARG = 1,         /* null pointer, negative size, unknown enum */
  B200_ERR_SHAPE = 2,       /* a size the kernels do not support (alignment, limits) */
  B200_ERR_FORMAT = 3,      /* unknown or mismatched weight format */
  B200_ERR_CUDA = 4,        /* a CUDA runtime call or launch failed */
  B200_ERR_WORKSPACE = 5,   /* the caller's workspace is smaller than required */
  B200_ERR_TIMEOUT = 6,     /* a device-side bounded wait gave up (see b200_read_fault) */
  B200_ERR_UNSUPPORTED = 7, /* a combination this build does not implement */
};

/* Message for the last non-zero status returned on this thread. */
const char* b200_last_error(void);
/* Library ABI version (major * 100 + minor). */
int b200_version(void);
/* Reads and clears the device fault word of the current device (0 = no fault). Blocking. */
int b200_read_fault(unsigned int* fault_out);

/* ---------------------------------------------------------------- packed weights
 * Replaces the bf16 `nn.Linear` weights of TF:417-420, TF:403, TF:632-643, TF:701-703.
 * Formats (each element dequantises to bf16_rn(code value x its scale); the quantisation
 * rules are b200_quantize's):
 *   B200_W_BF16     data uint16 [n, k]
 *   B200_W_INT4G128 data int32 [n, k/8] (8 nibbles per word, element k at bits 4*(k%8)),
 *                   scales bf16 [n, k/128]
 *   B200_W_NVFP4    data uint8 [n, k/2] (element k: low nibble if k even, high if odd),
 *                   scales e4m3 uint8 [n, k/16], row_scale fp32 [n] (the per-tensor scale
 *                   of the logical tensor each row belongs to)
 *   B200_W_TERNARY  data uint8 [n, k/4] (2 bits per element: 00=0, 01=+1, 11=-1),
 *                   scales bf16 [n]
 */
enum b200_wfmt { B200_W_BF16 = 0, B200_W_INT4G128 = 1, B200_W_NVFP4 = 2, B200_W_TERNARY = 3 };

typedef struct b200_qweight {
  int32_t format;
  int32_t n; /* rows (output features), a multiple of 256 for b200_linear */
  int32_t k; /* columns (input features), a multiple of 128 */
  const void* data;
  const void* scales;
  const float* row_scale; /* NVFP4 only, else NULL */
  /* The GEMM's streaming copy of data/scales (b200_tile_weights): one contiguous chunk per
   * (256-row tile, 64-column stage), so each stage is one bulk copy. Required by
   * b200_linear for the packed formats; NULL for bf16 (read through a tensor map). */
  const void* tiles;
  const void* tile_scales;
} b200_qweight;

/* Quantise an fp32 weight w[n, k] (one logical nn.Linear) into `format`; writes data,
 * scales and (NVFP4) row_scale[n]. Bit-exact to oracle/quant.py. */
int b200_quantize(int32_t format, const float* w, int32_t n, int32_t k, void* data, void* scales,
                  float* row_scale, b200_stream stream);
/* Unpack a packed weight to bf16 out[n, k], exactly as the GEMM's shared-memory unpacker. */
int b200_dequantize(const b200_qweight* w, uint16_t* out, b200_stream stream);
/* The two weight copies b200_linear_lo8 reads, from a packed (or bf16) weight: w_hi bf16
 * [n, k] = dequant(W) * 2^B200_LO8_SHIFT (exact: a power-of-two rescale of b200_dequantize's
 * output) and w_lo8 e4m3 [n, k] = e4m3_rn_satfinite(dequant(W) * 2^B200_LO8_W_SHIFT). */
int b200_dequantize_lo8(const b200_qweight* w, uint16_t* w_hi, uint8_t* w_lo8, b200_stream stream);
/* Bytes of the streaming copy of a packed [n, k] weight (n % 256 == 0, k % 128 == 0). */
int b200_tile_bytes(int32_t format, int32_t n, int32_t k, size_t* tile_bytes, size_t* tile_scale_bytes);
/* Write the streaming copy: tiles[n/256][k/64][256 rows][row bytes of 64 columns] and, for
 * int4 / NVFP4, tile_scales[n/256][k/64][256 rows][scale bytes of 64 columns]. */
int b200_tile_weights(const b200_qweight* w, void* tiles, void* tile_scales, b200_stream stream);

/* ---------------------------------------------------------------- linear (GEMM)
 * y = x @ dequant(W)^T with a fused epilogue, fp32 accumulation in tensor memory (tcgen05
 * on sm_100a); batches of at most 16 rows on packed weights stream the weights through
 * registers into mma.sync instead (fp32 accumulation in registers; the weight-read-bound
 * case). Activations carry fp32-level precision as two bf16 planes, x = x_hi + x_lo
 * (x_hi = bf16_rn(x), x_lo = bf16_rn(x - x_hi)); the tensor cores run one bf16 MMA per
 * plane into the same accumulator. Each plane is bf16 [m, ldx] row-major (ldx a multiple of
 * 8, 16-byte aligned). x_lo may be NULL for a single bf16 pass.
 * Replaces one or several `nn.Linear` calls plus the elementwise op that follows them:
 *   B200_EP_STORE     out fp32 [m, ldo] = y  (the in-projections TF:442-449, TF:658-665)
 *   B200_EP_RESID_ADD out fp32 [m, ldo] += y (the residual adds of TF:775 and TF:781)
 *   B200_EP_SWIGLU    W rows interleaved in blocks of 64 (gate, up); h[:, 64b+i] =
 *                     silu(y[:, 128b+i]) * y[:, 128b+64+i] (TF:707), written as the two bf16
 *                     planes of the next GEMM's input: hi at out [m, ldo], lo at
 *                     out + lo_offset (lo_offset 0: hi plane only)
 * Only columns < n_valid are written (n_valid a multiple of 32; of 128 for SwiGLU). */
enum b200_epilogue { B200_EP_STORE = 0, B200_EP_RESID_ADD = 1, B200_EP_SWIGLU = 2 };

/* Format of a low activation plane (lo = x - bf16_rn(x), same element index as the hi plane):
 *   B200_LO_BF16  bf16_rn(lo), 2 bytes per element
 *   B200_LO_E4M3  e4m3_rn_satfinite(lo * 2^B200_LO8_X_SHIFT), 1 byte per element (a row of
 *                 ldx elements is ldx bytes); read by b200_linear_lo8 */
enum b200_lo_format { B200_LO_BF16 = 0, B200_LO_E4M3 = 1 };
#define B200_LO8_X_SHIFT 6
#define B200_LO8_W_SHIFT 6
#define B200_LO8_SHIFT (B200_LO8_X_SHIFT + B200_LO8_W_SHIFT)

typedef struct b200_linear_out {
  int32_t epilogue;
  int32_t n_valid;
  void* out;
  int32_t ldo;
  int64_t lo_offset;
  int32_t lo_format; /* SwiGLU: format of the lo plane written at out + lo_offset (b200_lo_format) */
} b200_linear_out;

int b200_linear(const uint16_t* x_hi, const uint16_t* x_lo, int32_t m, int32_t k, int32_t ldx,
                const b200_qweight* w, const b200_linear_out* out, b200_stream stream);
/* The e4m3-low-plane GEMM: y = (x_hi . w_hi + x_lo8 . w_lo8) * 2^-B200_LO8_SHIFT, i.e. x @ W^T
 * with the low plane at e4m3 precision, for the weight copies of b200_dequantize_lo8 ([n, k],
 * n % 256 == 0, k % 128 == 0). x_hi bf16 [m, ldx]; x_lo8 the B200_LO_E4M3 plane [m, ldx] bytes
 * (ldx a multiple of 16). Per 64 k the tensor cores run four bf16 MMAs (K = 16) for the hi plane
 * and two e4m3 MMAs (K = 32, twice the rate) for the low plane into one fp32 accumulator: 3/4 of
 * the tensor work of two bf16 planes. Same epilogues and n_valid rules as b200_linear. */
int b200_linear_lo8(const uint16_t* x_hi, const uint8_t* x_lo8, int32_t m, int32_t k, int32_t ldx,
                    const uint16_t* w_hi, const uint8_t* w_lo8, int32_t n, const b200_linear_out* out,
                    b200_stream stream);
/* Same contract on plain CUDA cores (fp32 FMA), used by the tests to cross-check b200_linear. */
int b200_linear_simt(const uint16_t* x_hi, const uint16_t* x_lo, int32_t m, int32_t k, int32_t ldx,
                     const b200_qweight* w, const b200_linear_out* out, b200_stream stream);

/* ---------------------------------------------------------------- native NVFP4 (W4A4)
 * The block-scaled tensor-core path (tcgen05.mma kind::mxf4nvf4): activations AND weights in
 * NVFP4, y[t, n] = row_scale[n] * sum over 16-blocks b of sa[t, b] * sw[n, b] * sum e2m1 a * e2m1 w.
 * Replaces the same `nn.Linear` calls as b200_linear (TF:417-420, TF:632-643, TF:701-703), at
 * four times the bf16 tensor rate, but with 4-bit activations: on the 2B-shape decider that
 * moves option probabilities by up to 0.5 against the fp32 reference, far outside the 2e-3
 * bar, so the model runtime does not use it; it is offered for callers that accept W4A4.
 * Scale factors travel in 512-byte atoms per 128 rows and 64 k: byte 16*(r%32) + 4*((r%128)/32)
 * + (b%4) of atom [r/128][b/4] holds the unsigned-e4m3 scale of row r, 16-block b. */
/* Bytes of scale atoms for a [rows, k] NVFP4 matrix (rows rounded up to 128; k % 64 == 0). */
int b200_nvfp4_sf_atom_bytes(int32_t rows, int32_t k, size_t* bytes);
/* Activation quantiser: x fp32 [m, ldx] -> codes uint8 [m, k/2] (element k in the low nibble of
 * byte k/2 when k is even) and scale atoms (rows m .. round_up(m, 128) written as zeros).
 * Per 16-block: scale byte = e4m3_rn_sat(amax / 6), code = e2m1_rn_sat(x / scale), 0 for a zero
 * scale. No tensor scale (block maxima from about 3e-3 to 2688 are representable). */
int b200_quantize_act_nvfp4(const float* x, int32_t m, int32_t k, int32_t ldx, uint8_t* codes, uint8_t* sf_atoms,
                            b200_stream stream);
/* A packed NVFP4 weight's scales [rows][k/16] (rows % 128 == 0) -> scale atoms. */
int b200_nvfp4_sf_atoms(const uint8_t* scales, int32_t rows, int32_t k, uint8_t* sf_atoms, b200_stream stream);
/* y = x @ W^T on the block-scaled MMA: x as b200_quantize_act_nvfp4 left it, W a B200_W_NVFP4
 * weight (data, row_scale) with its scale atoms w_sf; k % 256 == 0, n % 128 == 0. Epilogues and
 * n_valid rules as b200_linear (SwiGLU writes bf16 planes). */
int b200_linear_nvfp4_native(const uint8_t* x_codes, const uint8_t* x_sf, int32_t m, int32_t k, const b200_qweight* w,
                             const uint8_t* w_sf, const b200_linear_out* out, b200_stream stream);

/* ---------------------------------------------------------------- ragged batches, prefix cache */
typedef struct b200_seqs {
  int32_t n_seqs;
  int32_t n_tokens;
  int32_t max_len;             /* host-side upper bound on any sequence's length */
  const int32_t* cu_seqlens;   /* [n_seqs + 1] */
  const int32_t* prefix_slot;  /* [n_seqs]: prefix-pool slot this sequence continues, -1 none; may be NULL */
  const int32_t* save_slot;    /* [n_seqs]: slot to write this sequence's cache into, -1 none; may be NULL */
} b200_seqs;

/* The prefix-state pool that replaces the reference's cache fork (infer.py:79-124,
 * _expand_cache): question suffixes read a state's cache in place by slot index, so the
 * `expand(n).contiguous()` copies of infer.py:103,107 never happen. One pool per model;
 * arrays are indexed [layer of that kind][slot]. A saving sequence (save_slot >= 0) either
 * has no prefix and fills the slot from position 0, or continues its own slot
 * (prefix_slot == save_slot) and appends: the GDN state and conv history are replaced by the
 * continued ones and its keys / values go after the slot's existing ones, so the slot's
 * region in k_cache / v_cache (from slot_kv[slot]) must have room for the grown length.
 * Saving into a slot other than the prefix slot is refused (fault word, nothing saved).
 * b200_model_forward sets slot_len[save_slot] after the whole forward; the kernel-level
 * entry points leave slot_len to the caller. k_cache / v_cache must hold finite values
 * everywhere (allocate them zeroed): attention reads whole 64-key tiles, and the keys past a
 * slot's length are masked out of the softmax but still meet zero probabilities in P V. */
typedef struct b200_prefix_pool {
  int32_t n_slots;
  int32_t kv_capacity;     /* tokens per attention layer in k_cache / v_cache */
  int32_t* slot_len;       /* [n_slots]: cached length (positions); set by b200_model_forward for saved slots */
  const int32_t* slot_kv;  /* [n_slots]: token offset of the slot's keys in k_cache / v_cache (host-assigned) */
  float* gdn_state;        /* [n_gdn_layers][n_slots][heads][dk][dv] fp32 (TF:285-305 state) */
  float* conv_hist;        /* [n_gdn_layers][n_slots][conv_width-1][conv_dim] fp32 (TF:462-464) */
  uint16_t* k_cache;       /* [n_attn_layers][kv_capacity][kv_heads][head_dim] bf16, post norm+RoPE */
  uint16_t* v_cache;       /* [n_attn_layers][kv_capacity][kv_heads][head_dim] bf16 */
} b200_prefix_pool;

/* ---------------------------------------------------------------- torso building blocks */

/* x[t, :] = float(table[ids[t], :]) (the embedding lookup, TF:1241). */
int b200_embed(const int32_t* ids, int32_t n_tokens, const uint16_t* table, int32_t hidden, float* x,
               b200_stream stream);

/* y = x * rsqrt(mean(x^2) + eps) * (1 + w) per row (Qwen3_5RMSNorm, TF:711-728), written
 * as the two bf16 planes of a GEMM input: hi at out [rows, hidden], lo at out + lo_offset. */
int b200_rmsnorm(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                 int64_t lo_offset, b200_stream stream);
/* Same, with the lo plane in B200_LO_E4M3 form at (uint8_t*)(out + lo_offset) [rows, hidden]. */
int b200_rmsnorm_lo8(const float* x, int32_t rows, int32_t hidden, const float* w, float eps, uint16_t* out,
                     int64_t lo_offset, b200_stream stream);

/* One Gated-DeltaNet token mixer after its in-projection (TF:462-530): depthwise causal
 * conv (width conv_width) + SiLU, q/k l2norm, beta = sigmoid(b), g = -exp(A_log) *
 * softplus(a + dt_bias), the chunked gated delta rule (TF:234-311) from the prefix slot's
 * state, and the gated RMSNorm (TF:175-190). mix: fp32 [tokens, ld_mix] holding the
 * in-projection's [q | k | v | z | b | a] columns; out: the two bf16 planes of the
 * out-projection's input, hi [tokens, heads*dv] and lo at out + lo_offset. gdn_layer
 * indexes the pool's GDN arrays. scratch: fp32, b200_gdn_scratch_floats(heads, tokens)
 * floats (the conv / l2norm / gating outputs the chunk kernel reads). */
typedef struct b200_gdn_params {
  int32_t heads, dk, dv, conv_width;
  float eps;
  const float* conv_w;   /* [conv_dim][conv_width] */
  const float* a_log;    /* [heads] */
  const float* dt_bias;  /* [heads] */
  const float* norm_w;   /* [dv] */
} b200_gdn_params;

int b200_gdn_mixer(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix, int32_t ld_mix,
                   uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t gdn_layer,
                   float* scratch, b200_stream stream);
/* b200_gdn_mixer picks its scan by the batch: the token-by-token recurrent form
 * (torch_recurrent_gated_delta_rule, TF:314-353) when n_tokens <= n_seqs (single-token
 * appends to cached states), the chunked rule otherwise. These two force one of them, with
 * the same arguments and results (the state after the last token, outputs per token); the
 * recurrent one needs norm_w, scratch and the pool's gdn_state 16-byte aligned. */
int b200_gdn_mixer_recurrent(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix, int32_t ld_mix,
                             uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t gdn_layer,
                             float* scratch, b200_stream stream);
int b200_gdn_mixer_chunked(const b200_gdn_params* p, const b200_seqs* seqs, const float* mix, int32_t ld_mix,
                           uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t gdn_layer,
                           float* scratch, b200_stream stream);
/* fp32 scratch floats b200_gdn_mixer needs for a batch of n_tokens. */
int b200_gdn_scratch_floats(int32_t heads, int32_t n_tokens);

/* Gated GQA attention after its qkv projection (TF:647-690): per-head q/k RMSNorm(1+w),
 * partial RoPE on the first rope_dim dims (cos/sin tables [max_pos][rope_dim/2]), causal
 * softmax attention over the prefix slot's keys and the sequence's own, times
 * sigmoid(gate). qkv: fp32 [tokens, ld_qkv] = [per q head (query, gate) | k | v]
 * (TF:658-665); q_buf, k_buf, v_buf: scratch bf16 [tokens][heads][head_dim]; out: the two
 * bf16 planes of o_proj's input, hi [tokens, heads*head_dim] and lo at out + lo_offset. */
typedef struct b200_attn_params {
  int32_t heads, kv_heads, head_dim, rope_dim, max_pos;
  float eps;
  const float* q_norm;   /* [head_dim] */
  const float* k_norm;   /* [head_dim] */
  const float* rope_cos; /* [max_pos][rope_dim/2] */
  const float* rope_sin;
} b200_attn_params;

int b200_attention(const b200_attn_params* p, const b200_seqs* seqs, const float* qkv, int32_t ld_qkv,
                   uint16_t* q_buf, uint16_t* k_buf, uint16_t* v_buf, uint16_t* out, int64_t lo_offset,
                   const b200_prefix_pool* pool, int32_t attn_layer, b200_stream stream);

/* Same as b200_attention, but it allocates nothing and takes no scratch argument: the
 * q / k / v scratch lives in a static 8 MiB device array inside this library (one per GPU
 * that loads it, held until the process exits). It has no counterpart in the reference.
 * It is for callers that cannot call cudaMalloc: a host runtime whose device memory is owned
 * by its own arena or caching allocator (an embedding server that preallocated its pool, a
 * Go or Java host that hands the library only its request buffers) cannot allocate or free
 * mid-request, because cudaFree synchronises the device and a fresh cudaMalloc can fail on a
 * full pool. Limits: tokens * (heads + 2*kv_heads) * head_dim * 2 bytes <= 8 MiB, else
 * B200_ERR_SHAPE. The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) with that device current. Every call shares the array and it keeps
 * the last call's contents (each call overwrites all the scratch it reads, so nothing needs
 * clearing); calls that can overlap on the GPU (different streams, or different host threads)
 * race on it and must be serialised by the caller. */
int b200_attention_noalloc(const b200_attn_params* p, const b200_seqs* seqs, const float* qkv, int32_t ld_qkv,
                           uint16_t* out, int64_t lo_offset, const b200_prefix_pool* pool, int32_t attn_layer,
                           b200_stream stream);

/* ---------------------------------------------------------------- decision head
 * Replaces pool_last_token -> final RMSNorm -> option-token logits over the tied
 * embedding rows -> apply_temperature -> masked_log_softmax -> exp (modeling.py:193-238,
 * 412-438) and the per-kind read-back of infer.py:444-472 / schema.py:141-198, for rows
 * whose last token is x[last_tok[i]]. The full-vocabulary logits are never formed.
 * kinds: 0 noul, 1 choice, 2 score. Outputs per row: probs[i][kmax] (masked slots 0),
 * argmax[i], confidence[i] (choice: (n p_max - 1)/(n - 1); score: normalised-sigma
 * confidence with ordinal_smoothing; noul: |2p - 1|) and score[i] (score: expected level;
 * noul: P(true) = probs[i][1]; choice: argmax). kmax <= 16. */
typedef struct b200_decide_args {
  int32_t n_rows, kmax;
  const int32_t* last_tok;   /* [n_rows] */
  const int32_t* opt_ids;    /* [n_rows][kmax] */
  const int32_t* n_opts;     /* [n_rows] */
  const int32_t* kinds;      /* [n_rows] */
  const float* temperature;  /* [n_rows] */
  float ordinal_smoothing;
  float* probs;              /* [n_rows][kmax] */
  int32_t* argmax;
  float* confidence;
  float* score;
  const int32_t* opt_tok;    /* pointer readout only: [n_rows][kmax] token index (into x) of the last
                                token of each option's line, -1 past the row's options; else NULL */
} b200_decide_args;

int b200_decide(const float* x, int32_t hidden, const float* final_norm, float eps, const uint16_t* table,
                const b200_decide_args* d, b200_stream stream);

/* Trained readouts (modeling.py:99-158, build_head 161-180), used instead of the option-token
 * logits by checkpoints whose head_type is "slot" or "pointer". Both start from the final
 * hidden state (the torso's final RMSNorm applied to x) and a LayerNorm(hidden):
 *   slot:    logits = Linear(hidden -> out)(LN(h_last)), or with mlp_hidden > 0
 *            Linear(mlp_hidden -> out)(GELU(Linear(hidden -> mlp_hidden)(LN(h_last))))
 *            (SlotHead.forward, modeling.py:120-121; out = num_slots)
 *   pointer: logits[k] = k(LN(h_opt_k)) . q(LN(h_last)) * out^-1/2 with q, k: hidden -> out
 *            and h_opt_k the hidden state at opt_tok[i][k] (PointerHead.forward,
 *            modeling.py:154-158; gather_options 183-190; out = pointer_dim)
 * then apply_temperature / masked_log_softmax / the per-kind answers as b200_decide.
 * Weights are fp32 in nn.Linear layout ([out_features][in_features]). kmax <= 32; slot
 * heads need out <= 32 (logits past kmax are dropped). */
enum b200_head_kind { B200_HEAD_OPTION_TOKEN = 0, B200_HEAD_SLOT = 1, B200_HEAD_POINTER = 2 };
typedef struct b200_readout {
  int32_t kind;        /* B200_HEAD_SLOT or B200_HEAD_POINTER */
  int32_t hidden;      /* torso hidden size, <= 4096, a multiple of 32 */
  int32_t out;         /* slot: number of slots; pointer: the q / k dimension (<= 1024) */
  int32_t mlp_hidden;  /* slot: width of the GELU layer, 0 for a single linear layer (<= 4096) */
  float ln_eps;        /* the LayerNorm's eps (nn.LayerNorm default 1e-5) */
  const float* ln_w;   /* [hidden] */
  const float* ln_b;   /* [hidden] */
  const float* w1;     /* slot: [mlp_hidden or out][hidden]; pointer: q.weight [out][hidden] */
  const float* b1;     /* its bias */
  const float* w2;     /* slot with mlp_hidden > 0: [out][mlp_hidden]; pointer: k.weight [out][hidden] */
  const float* b2;     /* its bias */
} b200_readout;

int b200_decide_readout(const float* x, int32_t hidden, const float* final_norm, float eps, const b200_readout* head,
                        const b200_decide_args* d, int32_t n_tokens, b200_stream stream);

/* ---------------------------------------------------------------- whole-torso runtime
 * A model context holds the configuration and the device pointers of every weight
 * (registered once, owned by the caller). b200_model_forward runs the full torso prefill
 * (TF:1227-1290) over a ragged batch -- reading and/or filling the prefix pool -- and,
 * when `decide` is non-NULL, the decision head: one call covers the reference's
 * `self.model(...)` of infer.py:272-279 or the two torso calls of infer.py:298-335. */
enum b200_layer_kind { B200_LAYER_GDN = 0, B200_LAYER_ATTN = 1 };

typedef struct b200_model_config {
  int32_t vocab, hidden, inter, n_layers;
  int32_t layer_kind[64];
  int32_t gdn_heads, gdn_dk, gdn_dv, conv_width;
  int32_t attn_heads, attn_kv_heads, head_dim, rope_dim, max_pos;
  float eps;
  int32_t weight_format;
  /* Batches of at least this many tokens dequantise each packed weight once per GEMM into a
   * bf16 [N, K] workspace buffer and run the GEMM on it (the in-kernel unpack would repeat for
   * every 128-token tile); smaller batches stream the packed tiles. 0 = the library default
   * (4096), < 0 = never. */
  int32_t dequant_min_tokens;
  /* Low activation plane of the GEMMs on the dequantised path (b200_lo_format): B200_LO_BF16
   * keeps two bf16 planes everywhere; B200_LO_E4M3 stores it as e4m3 and runs those GEMMs
   * as b200_linear_lo8 (3/4 of the tensor work). Streamed-tile GEMMs always use bf16 planes. */
  int32_t lo_format;
} b200_model_config;

typedef struct b200_layer_weights {
  const float* input_norm;   /* [hidden] */
  const float* post_norm;    /* [hidden] */
  b200_qweight mix_in;       /* GDN: [qkv|z|b|a] rows; attention: [q(+gate)|k|v] rows */
  b200_qweight mix_out;      /* GDN out_proj / attention o_proj */
  b200_qweight gate_up;      /* interleaved blocks of 64 */
  b200_qweight down;
  b200_gdn_params gdn;       /* GDN layers */
  const float* q_norm;       /* attention layers */
  const float* k_norm;
} b200_layer_weights;

typedef struct b200_model b200_model;

int b200_model_create(const b200_model_config* cfg, b200_model** out);
int b200_model_destroy(b200_model* m);
int b200_model_set_layer(b200_model* m, int32_t layer, const b200_layer_weights* w);
int b200_model_set_globals(b200_model* m, const uint16_t* embed, const float* final_norm, const float* rope_cos,
                           const float* rope_sin);
/* A trained readout for the forward's decision head (NULL: the option-token logits). The
 * struct is copied; its weight pointers must stay valid. */
int b200_model_set_readout(b200_model* m, const b200_readout* head);
/* Bytes of workspace b200_model_forward needs for batches up to max_tokens tokens. */
int b200_model_workspace_bytes(const b200_model* m, int32_t max_tokens, size_t* bytes);
int b200_model_forward(b200_model* m, const int32_t* ids, const b200_seqs* seqs, const b200_prefix_pool* pool,
                       const b200_decide_args* decide, void* workspace, size_t workspace_bytes,
                       b200_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* STRANDS_B200_H */
