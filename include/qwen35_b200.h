/*
 * qwen35_b200.h — C ABI of the B200 (sm_100a) Qwen3.5 fused inference hot path.
 *
 * Drop-in boundary for the reference project's fused operator layer,
 * qwen35_fused/kernels.py, and for the decode/prefill loop its integration patches into the
 * Hugging Face model (qwen35_fused/integration.py, qwen35_fused/graph.py). Each entry point
 * names the reference interface it replaces as `file:line`.
 *
 * Conventions (mirroring kernels.py:16-21 and the wrappers):
 *   - every tensor argument is a device pointer to a contiguous row-major buffer;
 *     "bf16" means IEEE bfloat16 stored as uint16_t;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); work is enqueued on it,
 *     nothing synchronises the host, and no entry point allocates device memory:
 *     scratch ("workspace") is caller-provided, sized by the matching *_workspace_size();
 *   - lengths and positions that change from step to step are read from device int64
 *     scalars, so a captured CUDA graph stays valid across steps (graph.py:50-79);
 *   - return value: Q35_OK, or an error code with a message from q35_last_error().
 *     Q35_EINVAL is what the reference reports as ValueError (bad shape / layout).
 */
#ifndef QWEN35_B200_H
#define QWEN35_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  Q35_OK = 0,
  Q35_EINVAL = 1,   /* invalid argument (reference: ValueError) */
  Q35_ECUDA = 2,    /* CUDA launch / runtime error */
  Q35_ETIMEOUT = 3, /* a bounded device-side wait gave up */
  Q35_ENOTSUP = 4   /* shape outside what the kernels are built for */
};

/* Message of the last failing call on this host thread. */
const char* q35_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int q35_abi_version(void);

/* ---------------------------------------------------------------- norms & activations */

/* kernels.py:44 rms_norm — out = bf16(x * rsqrt(mean(x^2) + eps) * (1 + w)), per row. */
int q35_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t width,
                 float eps, void* stream);

/* kernels.py:85 residual_add_rms_norm — r' = bf16(r + u); n = rms_norm(r'). */
int q35_residual_add_rms_norm(const void* residual, const void* update, const void* weight,
                              void* residual_out, void* norm_out, int64_t rows, int64_t width,
                              float eps, void* stream);

/* kernels.py:139 gated_rms_norm — bf16(bf16(bf16(norm(x)) * w) * silu(gate)), plain weight. */
int q35_gated_rms_norm(const void* x, const void* gate, const void* weight, void* out,
                       int64_t rows, int64_t width, float eps, void* stream);

/* kernels.py:170 silu_and_mul — packed [rows, 2*width] -> [rows, width]. */
int q35_silu_and_mul(const void* packed, void* out, int64_t rows, int64_t width, void* stream);

/* kernels.py:276 sigmoid_mul — bf16(x * bf16(sigmoid(gate))). */
int q35_sigmoid_mul(const void* x, const void* gate, void* out, int64_t n, void* stream);

/* kernels.py:312 attention_gate_mul — x [rows, hidden] times sigmoid of the gate half of each
 * packed Q|gate head block (packed row stride `packed_stride`). */
int q35_attention_gate_mul(const void* x, const void* packed, void* out, int64_t rows,
                           int64_t hidden, int64_t packed_stride, int64_t head_dim, void* stream);

/* Embedding gather (integration.py:402-403, embed_tokens): out[i] = table[ids[i]]. */
int q35_embedding(const int64_t* ids, const void* table, void* out, int64_t n, int64_t vocab,
                  int64_t width, void* stream);

/* ---------------------------------------------------------------- decode GEMVs */

/* kernels.py:232 ppu_swiglu_gemv — x [k] times packed [gate; up] weight [2*n_out, k]:
 * out[n] = bf16(bf16(silu(bf16(g_n))) * bf16(u_n)). */
int q35_swiglu_gemv(const void* x, const void* packed_weight, void* out, int64_t n_out,
                    int64_t k, void* stream);

/* Fused batch-1 decode GEMV used by the decoder loop (integration.py:245, 298, 183-185, 272,
 * 359 as F.linear / ppu_swiglu_gemv, with the residual_add_rms_norm of :478-499 folded in).
 * Prologue builds the input vector in shared memory; epilogue writes the result. */
enum {
  Q35_PRO_PLAIN = 0, /* x = input[k] */
  Q35_PRO_NORM = 1,  /* x = rms_norm(input[k], norm_weight) */
  Q35_PRO_EMBED = 2  /* x = rms_norm(embed[token[0]], norm_weight); the raw row -> resid_out */
};
enum {
  Q35_EPI_STORE = 0,    /* out[n] = bf16(y_n) */
  Q35_EPI_RESIDUAL = 1, /* resid_out[n] = bf16(resid_out[n] + bf16(y_n)) (in place) */
  Q35_EPI_SWIGLU = 2,   /* rows n and n + n_out are gate/up: out[n] = SwiGLU */
  /* tensor-core GEMM only (the vision tower's biased linears, q35_gemm_tc_bias): */
  Q35_EPI_BIAS = 3,           /* out[n] = bf16(y_n + bias[n]) */
  Q35_EPI_BIAS_GELU_TANH = 4, /* out[n] = bf16(gelu_tanh(bf16(y_n + bias[n]))) */
  Q35_EPI_BIAS_GELU = 5       /* out[n] = bf16(gelu_erf(bf16(y_n + bias[n]))) */
};
typedef struct {
  const void* weight;       /* bf16 [rows, k], or int8 [rows, k] when int8 != 0 */
  const float* w_scale;     /* int8 only: fp32 per-row scale [rows] */
  const void* input;        /* bf16 [k] (PLAIN / NORM) */
  const void* norm_weight;  /* bf16 [k] (NORM / EMBED) */
  const int64_t* token;     /* EMBED: device token id */
  const void* embed;        /* EMBED: bf16 [vocab, k] */
  void* resid_out;          /* EMBED: receives the raw embedding row; RESIDUAL: updated in place */
  void* out;                /* bf16 [n_out] (STORE / SWIGLU) */
  int64_t n_out;            /* outputs (rows, or rows/2 for SWIGLU) */
  int64_t k;                /* reduction length (fast paths for 2048 and 6144) */
  int64_t vocab;            /* EMBED: rows of embed; token ids are clamped into [0, vocab) */
  int32_t prologue;
  int32_t epilogue;
  int32_t int8;             /* 1 = A8W8: per-token int8 activation, int32 accumulation */
  float eps;
} q35_gemv_desc;
int q35_gemv(const q35_gemv_desc* d, void* stream);

/* Weight-streaming strategy of the K = 2048 / 6144 decode GEMVs (process-wide, default REGISTERS):
 * BULK stages weights through shared memory with bulk asynchronous copies issued before the
 * programmatic-dependent-launch wait; REGISTERS streams 16-byte loads into registers. */
enum { Q35_GEMV_BULK = 0, Q35_GEMV_REGISTERS = 1 };
int q35_set_gemv_variant(int variant);
/* Grid cap of the REGISTERS decode GEMVs in CTAs per SM (process-wide; 0 = as many as fit). A cap
 * leaves registers for the next kernel's CTAs, which then start and issue their weight loads
 * while this kernel drains (programmatic dependent launch). */
int q35_set_gemv_ctas_per_sm(int ctas);
/* Error word of the bulk GEMV (non-zero when a bounded copy wait gave up); reading clears it. */
int q35_gemv_error(void);

/* kernels.py:1146 lm_head_argmax — token[b] = argmax_v bf16(hidden[b] . weight[v]), lowest v on
 * ties, in one launch. With norm_weight != NULL the hidden row is rms_norm'ed first (the final
 * norm of integration.py:494-499 fused in). Workspace: q35_lm_head_workspace_size(batch) bytes,
 * zeroed once by the caller; every call leaves it zeroed again. */
size_t q35_lm_head_workspace_size(int64_t batch);
int q35_lm_head_argmax(const void* hidden, const void* norm_weight, const void* weight,
                       int64_t* token_out, int64_t batch, int64_t vocab, int64_t hidden_size,
                       float eps, void* workspace, size_t workspace_bytes, void* stream);

/* Vocab-sharded top-1 (no reference counterpart: the multi-GPU split of kernels.py:1093-1185 for
 * lock-step decode of `batch` requests, one per rank). For each of the `batch` hiddens (rows of
 * [batch, hidden_size], rms_norm'ed first when norm_weight != NULL) and the shard of rows
 * [row_offset, row_offset + shard_rows) of the [vocab, hidden_size] table (weight_shard points at
 * its first row), writes keys_out[b] = ((order(bf16 logit) << 32) | (0xFFFFFFFF - global index))
 * - 2^63 as int64, INT64_MIN for an empty shard. The maximum of a request's keys over all shards
 * (an int64 MAX all-reduce) encodes q35_lm_head_argmax's token: logits are bit-identical to it,
 * and ties go to the lowest index. batch <= 8, hidden_size 2048. Workspace:
 * q35_lm_shard_workspace_size() bytes, zeroed once; every call leaves it zeroed again. */
size_t q35_lm_shard_workspace_size(void);
int q35_lm_head_shard_keys(const void* hidden, int64_t batch, const void* norm_weight,
                           const void* weight_shard, int64_t row_offset, int64_t shard_rows,
                           int64_t vocab, int64_t hidden_size, float eps, int64_t* keys_out,
                           void* workspace, size_t workspace_bytes, void* stream);
/* tokens_out[b] = the token a reduced key encodes (0 for INT64_MIN), b < n (<= 1024). */
int q35_lm_keys_to_tokens(const int64_t* keys, int64_t n, int64_t* tokens_out, void* stream);

/* ---------------------------------------------------------------- A8W8 */

/* Weight side, explore_runtime_quantization.py:143-155 (PPUA8W8Linear.__init__): per-row
 * symmetric int8, scale = amax|x| / 127 (1 for an all-zero row), q = clamp(rne(x / s), +-127). */
int q35_quantize_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                      void* stream);

/* Activation side, explore_runtime_quantization.py:167-172 (vllm scaled_int8_quant(x, scale=None,
 * azp=None, symmetric=True), dynamic per token): scale = amax|x| / 127 (0 for an all-zero row),
 * q = saturate_int8(rne(x * (127 / amax))) (0 for an all-zero row). */
int q35_quantize_tokens(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                        void* stream);

/* explore_runtime_quantization.py:161-181 (PPUA8W8Linear.forward with acext int8_gemm):
 * out = bf16((float(qx @ qw^T) * s_x) * s_w), qx/s_x from q35_quantize_tokens(x).
 * Workspace: q35_a8w8_linear_workspace_size(m, k) bytes. */
size_t q35_a8w8_linear_workspace_size(int64_t m, int64_t k);
int q35_a8w8_linear(const void* x, const int8_t* qw, const float* w_scale, void* out, int64_t m,
                    int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream);

/* Exact int32 accumulation of an int8 GEMM, acc = qx [m,k] @ qw [n,k]^T (bit-exactness probe). */
int q35_int8_gemm_i32(const int8_t* qx, const int8_t* qw, int32_t* acc, int64_t m, int64_t n,
                      int64_t k, void* stream);

/* ---------------------------------------------------------------- prefill GEMM */

/* Dense prefill projection C = A [m,k] @ W [n,k]^T, bf16 in, fp32 accumulate (integration.py:183,
 * 245, 298 F.linear; :185, 272, 359 down/out/o proj). Epilogues as the decode GEMV:
 * STORE -> out [m,n]; RESIDUAL -> resid [m,n] += (bf16 rounding both); SWIGLU -> W rows
 * [0,n) are gate and [n,2n) up, out [m,n] = SwiGLU. */
int q35_gemm_bf16(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k,
                  int32_t epilogue, void* stream);

/* The same projection on the 5th-generation tensor cores: persistent, TMA-fed output tiles
 * accumulated by tcgen05.mma in TMEM (kind::f16), by default on pairs of SMs (256-row tiles,
 * cta_group::2). k must be a multiple of 64, n of 8. */
int q35_gemm_tc(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k,
                int32_t epilogue, void* stream);

/* Biased bf16 projection on tcgen05 for the vision tower (HF Qwen3_5Vision* nn.Linear with bias
 * and the activations that follow them: integration.py:509-736 runs them through F.linear):
 * out [m,n] = epilogue(A [m,k] @ W [n,k]^T + bias [n]) with epilogue Q35_EPI_BIAS,
 * Q35_EPI_BIAS_GELU_TANH (gelu_pytorch_tanh, the vision MLP) or Q35_EPI_BIAS_GELU (nn.GELU, the
 * patch merger). k must be a multiple of 64, n of 8. */
int q35_gemm_tc_bias(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n,
                     int64_t k, int32_t epilogue, void* stream);

/* A8W8 prefill projection on tcgen05 (kind::i8, exact int32 accumulation in TMEM) with the
 * dequantisation bf16((float(acc) * sx[m]) * sw[n]) and the epilogue fused (k multiple of 128).
 * qa/sx come from q35_quantize_tokens (explore_runtime_quantization.py:161-181). */
int q35_gemm_tc_a8w8(const int8_t* qa, const float* sx, const int8_t* qw, const float* sw, void* out,
                     int64_t m, int64_t n, int64_t k, int32_t epilogue, void* stream);

/* Error word of the tensor-core kernels: non-zero when a bounded pipeline wait gave up (the
 * kernel then finished without hanging). Reading it synchronises and clears it. */
int q35_tc_error(void);
/* Process-wide: 1 (default) runs the tensor-core projections on CTA pairs (thread-block clusters
 * of 2, tcgen05 cta_group::2, 256-row tiles), 0 on single CTAs (128-row tiles). */
int q35_set_gemm_tc_pairs(int on);

/* ---------------------------------------------------------------- attention */

/* kernels.py:507 qgkv_norm_rope — packed [B, L, 2*Hq*D + 2*Hkv*D] -> q [B,Hq,L,D] and K/V written
 * to k_out/v_out [B, Hkv, kv_len, D] at row offset *cache_start (NULL = 0). cos/sin [B,L,rot]. */
int q35_qgkv_norm_rope(const void* packed, const void* q_weight, const void* k_weight,
                       const void* cos, const void* sin, void* q_out, void* k_out, void* v_out,
                       const int64_t* cache_start, int64_t batch, int64_t seq_len,
                       int64_t q_heads, int64_t kv_heads, int64_t dim, int64_t rotary_dim,
                       int64_t kv_len, float eps, void* stream);

/* kernels.py:1031 gqa_decode_attention — q [B,H,1,D] over cache [B,Hkv,cache_len,D] with the
 * valid prefix *valid_length (device, includes the current token) -> out [B,1,H*D] bf16.
 * FP32 online softmax, split-KV with an in-kernel combine. Batch >= 1 (reference: batch 1). */
size_t q35_gqa_decode_workspace_size(int64_t batch, int64_t heads, int64_t kv_heads,
                                     int64_t head_dim, int64_t cache_len);
int q35_gqa_decode_attention(const void* q, const void* cache_k, const void* cache_v,
                             const int64_t* valid_length, float scale, void* out, int64_t batch,
                             int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cache_len,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free q35_gqa_decode_attention (no counterpart in the reference). For callers that
 * cannot allocate device memory when they call in (a locked or pool-only allocator, a thread that
 * must not touch the CUDA allocator, a runtime that passes only inputs and outputs): the scratch
 * lives in a static device array of q35_gqa_decode_noalloc_max_bytes() bytes (2 MiB) that every
 * GPU loading this library keeps until exit. Shapes whose scratch exceeds it, or that need more
 * than 256 split-ticket words (batch x kv_heads, plus one per group of 16 splits when a (batch,
 * KV head) has more than 16), are rejected with Q35_EINVAL before anything is queued on
 * the stream. The first call on a device looks up the array's device address (make it before any
 * stream capture); every call clears the ticket words and shares the array, so calls that overlap
 * on the GPU (other streams, other threads) race with each other. Calls no allocator. */
size_t q35_gqa_decode_noalloc_max_bytes(void);
int q35_gqa_decode_attention_noalloc(const void* q, const void* cache_k, const void* cache_v,
                                     const int64_t* valid_length, float scale, void* out,
                                     int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                     int64_t cache_len, void* stream);

/* Fused decode attention layer step (integration.py:298-359 for L == 1): from the packed QGKV
 * projection output [B, 5120] it does Q/K RMSNorm + partial RoPE at position *rope_pos, writes
 * K/V at row *cache_len, attends over rows [0, *cache_len] and multiplies by sigmoid(gate):
 * out [B, Hq*D]. Does not advance *cache_len (the decoder does once per step). */
size_t q35_attn_decode_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                      int64_t head_dim, int64_t cache_len);
int q35_attn_decode(const void* packed, const void* q_weight, const void* k_weight,
                    const float* inv_freq, void* cache_k, void* cache_v, const int64_t* cache_len,
                    const int64_t* rope_pos, void* out, int64_t batch, int64_t q_heads,
                    int64_t kv_heads, int64_t head_dim, int64_t rotary_dim, int64_t max_len,
                    float eps, void* workspace, size_t workspace_bytes, void* stream);

/* Causal prefill attention (integration.py:360-372, SDPA with a causal mask): q [B,Hq,L,D],
 * keys/values [B,Hkv,kv_len,D] (rows [0, q_offset + L) valid) -> out [B, L, Hq*D] bf16, FP32
 * softmax. Query i attends keys j <= q_offset + i. */
int q35_prefill_attention(const void* q, const void* k, const void* v, void* out, int64_t batch,
                          int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                          int64_t q_offset, int64_t head_dim, float scale, void* stream);

/* The same causal attention on tcgen05 (the decoder's prefill path; replaces the SDPA call of
 * integration.py:360-372 for 4 query heads per KV head, head dim 256, queries at rows 0 .. L-1 of
 * the cache): q [B,Hq,L,256], k [B,Hkv,kv_len,256], vt = V transposed [B,Hkv,256,vt_stride] with
 * vt_stride a multiple of 64 >= L whose columns past L hold finite values -> out [B, L, Hq*256].
 * FP32 softmax; P enters the P.V product as a bf16 high part plus a bf16 remainder. The
 * workspace (256-byte aligned, zeroed before first use; the kernel leaves it zeroed) holds the
 * partials of query blocks whose keys are split over two CTAs.
 * q35_prefill_attention_tc_error returns (and clears) the kernel's bounded-wait error word: 0, or
 * 1 + the shared-memory barrier slot whose wait gave up first. */
size_t q35_prefill_attention_tc_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq_len);
int q35_prefill_attention_tc(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                             int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                             int64_t vt_stride, float scale, void* workspace, size_t workspace_bytes,
                             void* stream);
int q35_prefill_attention_tc_error(void);

/* ---------------------------------------------------------------- Gated DeltaNet */

/* kernels.py:659 causal_conv1d_fused — x [B,L,in_stride] (first `channels` columns), weight
 * [channels, K], state [B, channels, K] updated in place; out [B, L, channels] = SiLU(conv). */
int q35_causal_conv1d(const void* x, const void* weight, void* state, void* out, int64_t batch,
                      int64_t seq_len, int64_t in_stride, int64_t channels, int64_t kernel_size,
                      void* stream);

/* kernels.py:854 delta_recurrent_fused — sequential gated delta rule over L tokens.
 * qkv [B,L,3*H*D] (conv output), packed [B,L,packed_stride] holding [qkv|z|a|b],
 * state [B,H,D,D] fp32 in place; out [B,L,H,D] bf16. */
int q35_delta_recurrent(const void* qkv, const void* packed, const void* a_log,
                        const void* dt_bias, float* state, void* out, int64_t batch,
                        int64_t seq_len, int64_t heads, int64_t dim, int64_t packed_stride,
                        void* stream);

/* The same recurrence in chunked (WY / UT-transform) form, chunk 64, FP32 throughout — the
 * algorithm of HF torch_chunk_gated_delta_rule — used for prefill: chunk-local factors for all
 * chunks in parallel, one pass over the chunks per (head, 16 value columns) for the state, then
 * the outputs of all chunks in parallel on tcgen05 (3xTF32, TMEM accumulator). Same inputs,
 * outputs and in-place state update as q35_delta_recurrent; workspace from
 * q35_delta_chunked_workspace_size. */
size_t q35_delta_chunked_workspace_size(int64_t batch, int64_t heads, int64_t seq_len);
/* Error word of the chunked DeltaNet output kernel (0 = its bounded TMEM wait completed; read and
 * cleared). */
int q35_delta_chunk_error(void);
int q35_delta_chunked(const void* qkv, const void* packed, const void* a_log, const void* dt_bias,
                      float* state, void* out, int64_t batch, int64_t seq_len, int64_t heads,
                      int64_t dim, int64_t packed_stride, void* workspace, size_t workspace_bytes,
                      void* stream);
/* The same with the causal conv folded in (kernels.py:659 causal_conv1d_fused on the [q k v]
 * columns of packed, 4 taps, starting from a zero history, then the chunked rule): reads the
 * raw projection `packed` [B, L, packed_stride] instead of a conv output, writes conv_state
 * [B, 3*H*D, 4] (the last 4 raw inputs); seq_len >= 4. Workspace as for q35_delta_chunked. */
int q35_delta_chunked_conv(const void* packed, const void* conv_weight, void* conv_state, const void* a_log,
                           const void* dt_bias, float* state, void* out, int64_t batch, int64_t seq_len,
                           int64_t heads, int64_t dim, int64_t packed_stride, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Fused DeltaNet decode step (integration.py:245-272 for L == 1): conv update + SiLU, q/k L2
 * norm, gated delta step on the fp32 state, gated RMSNorm with z. packed [B, packed_stride]
 * -> out [B, H*D] bf16 (input of out_proj). */
int q35_delta_decode(const void* packed, const void* conv_weight, void* conv_state,
                     const void* a_log, const void* dt_bias, const void* norm_weight,
                     float* state, void* out, int64_t batch, int64_t heads, int64_t dim,
                     int64_t packed_stride, float eps, void* stream);

/* ---------------------------------------------------------------- decoder loop */

/* One layer of the text model as packed device tensors (integration.py:69-140 packing). */
typedef struct {
  int32_t kind;              /* 0 = Gated DeltaNet, 1 = full attention */
  const void* in_ln;         /* bf16 [H] input_layernorm (1 + w) */
  const void* post_ln;       /* bf16 [H] post_attention_layernorm */
  const void* mix_in;        /* packed [qkv|z|a|b] [delta_rows, H] or [Q|G..|K|V] [qgkv_rows, H] */
  const float* mix_in_scale; /* A8W8 per-row scales (NULL for bf16) */
  const void* mix_out;       /* out_proj / o_proj [H, 2048] */
  const float* mix_out_scale;
  const void* gate_up;       /* [2I, H] */
  const float* gate_up_scale;
  const void* down;          /* [H, I] */
  const float* down_scale;
  const void* conv_w;        /* DeltaNet: bf16 [conv_dim, K] */
  const void* a_log;         /* bf16 [heads] */
  const void* dt_bias;       /* bf16 [heads] */
  const void* gnorm;         /* bf16 [dv] gated norm weight */
  void* conv_state;          /* bf16 [B, conv_dim, K] */
  float* rec_state;          /* fp32 [B, heads, dk, dv] */
  const void* q_norm;        /* attention: bf16 [D] */
  const void* k_norm;
  void* k_cache;             /* bf16 [B, Hkv, max_len, D] */
  void* v_cache;
} q35_layer_desc;

typedef struct {
  int32_t n_layers, hidden, intermediate, vocab;
  int32_t q_heads, kv_heads, head_dim, rotary_dim;
  int32_t lin_heads, lin_dk, lin_dv, conv_kernel, delta_rows;
  int32_t max_len;        /* KV cache rows */
  int32_t max_prefill;    /* longest prefill the workspace is sized for */
  int32_t a8w8;
  float eps;
  const q35_layer_desc* layers;
  const void* embed;      /* bf16 [vocab, H], tied LM head */
  const void* final_norm; /* bf16 [H] */
  const float* inv_freq;  /* fp32 [rotary_dim / 2] RoPE inverse frequencies */
  int64_t* token;         /* device [1]: token fed to the next decode step / last greedy token */
  int64_t* cache_len;     /* device: rows already in the KV cache */
  int64_t* rope_pos;      /* device: RoPE position of the next token */
  int64_t* token_log;     /* optional device ring [log_len]: decode tokens by step (may be NULL) */
  int64_t* log_pos;       /* device counter into token_log */
  int32_t log_len;
  int32_t use_pdl;        /* launch decode kernels with programmatic dependent launch */
  int32_t prefill_tc;     /* prefill projections on tcgen05 (1) or warp-level MMA (0) */
  int32_t prefill_delta;  /* prefill DeltaNet scan: 0 = chunked WY form, 1 = sequential */
  int32_t mrope_section[3]; /* interleaved M-RoPE sections (t, h, w) in frequency pairs, e.g.
                               {11, 11, 10}; used by multimodal prefills with 3-axis positions */
  int32_t batch;          /* requests decoded in lock step (1..8; 0 means 1). With batch > 1 every
                             state / cache tensor has a leading batch dimension, token[] holds one
                             token per request, and all requests share cache_len / rope_pos (equal
                             prompt lengths); bf16 weights only */
  void* workspace;
  size_t workspace_bytes;
} q35_decoder_desc;

typedef struct q35_decoder q35_decoder;

size_t q35_decoder_workspace_size(const q35_decoder_desc* desc);
int q35_decoder_create(const q35_decoder_desc* desc, q35_decoder** out);
void q35_decoder_destroy(q35_decoder* dec);
/* Prefill `length` token ids (device int64) from an empty cache (evaluation_wrapper.py:354-363):
 * all layers, caches/states filled, greedy first token -> *token; cache_len = rope_pos = length. */
int q35_decoder_prefill(q35_decoder* dec, const int64_t* ids, int64_t length, void* stream);
/* Multimodal prefill (the text-model forward of a Qwen3.5 image + text request, integration.py:
 * 390-504 with inputs_embeds from the vision tower): as q35_decoder_prefill, but the rows
 * image_rows[i] (device int64 [n_image], each in [0, length)) of the input sequence take
 * image_embeds[i] (bf16 [n_image, hidden]) instead of the embedding of their id, and the rotary
 * positions are the 3-axis M-RoPE positions positions3 (device int64 [3, length]: temporal,
 * height, width; interleaved per mrope_section) instead of 0..length-1. Afterwards
 * cache_len = length and rope_pos = rope_next (the text position after the prompt, max + 1). */
int q35_decoder_prefill_mm(q35_decoder* dec, const int64_t* ids, int64_t length, const void* image_embeds,
                           const int64_t* image_rows, int64_t n_image, const int64_t* positions3,
                           int64_t rope_next, int64_t slot, void* stream);
/* Batched decoders: prefill request slot `slot` (0 <= slot < batch) -- its states, caches and
 * token[slot]; cache_len / rope_pos are set to `length`, so every slot of a batch is prefilled
 * with the same length before the batch decodes (evaluation_wrapper.py:338-341 pads a batch to
 * one cache bucket the same way). q35_decoder_prefill is slot 0. */
int q35_decoder_prefill_slot(q35_decoder* dec, const int64_t* ids, int64_t length, int64_t slot, void* stream);
/* Batched decoders: prefill `nseq` requests of `length` tokens each (ids [nseq * length]) into slots
 * [slot, slot + nseq) in one pass: the projections, norms and GEMMs take all nseq * length rows,
 * the DeltaNet scans, causal attention and cache writes run per request, and one LM-head pass
 * over the tied table gives every request's first token. image_rows index the nseq * length
 * rows; positions3 (optional) is int64 [3, nseq, length]; rope_next = -1 leaves rope_pos =
 * length. nseq * length <= max_prefill. */
int q35_decoder_prefill_batch(q35_decoder* dec, const int64_t* ids, int64_t length, int64_t nseq,
                              const void* image_embeds, const int64_t* image_rows, int64_t n_image,
                              const int64_t* positions3, int64_t rope_next, int64_t slot, void* stream);
/* The decoder's batched projection (no counterpart in the reference, whose decode is batch 1):
 * q35_gemv for `batch` <= 8 input vectors [batch, k] / outputs [batch, n_out] at once, the weights
 * streamed once; bf16, k 2048 (NORM / EMBED + STORE, NORM + SWIGLU, PLAIN + RESIDUAL) or 6144
 * (PLAIN + RESIDUAL). */
int q35_gemv_batch(const q35_gemv_desc* desc, int64_t batch, void* stream);
/* One greedy decode step (graph.py:51-79 body): consumes *token, appends to caches, writes the
 * next greedy token to *token (and token_log), advances cache_len / rope_pos. */
int q35_decoder_decode_step(q35_decoder* dec, void* stream);
/* The decode step split for a vocab-sharded LM head (lock-step decode across ranks):
 * q35_decoder_decode_layers runs every layer and leaves the final residual (pre final norm,
 * [hidden] bf16) at q35_decoder_hidden(dec) without writing a token or advancing the counters;
 * after the caller has reduced the shard keys of q35_lm_head_shard_keys over ranks,
 * q35_decoder_finish_step writes the token keys[index] encodes to *token (and token_log) and
 * advances cache_len / rope_pos, exactly as q35_decoder_decode_step's LM head does. */
int q35_decoder_decode_layers(q35_decoder* dec, void* stream);
void* q35_decoder_hidden(const q35_decoder* dec);
int q35_decoder_finish_step(q35_decoder* dec, const int64_t* keys, int64_t index, void* stream);
/* Number of kernels one decode step launches (for launch accounting). */
int q35_decoder_kernels_per_step(const q35_decoder* dec);

/* The same greedy decode step as ONE cooperative kernel (graph.py:51-79 in one launch, plus a
 * 4-byte memset of its barrier counter): one CTA per SM streams its share of every weight matrix
 * through a shared-memory ring without stopping at op boundaries; dependent ops meet at bounded
 * grid barriers. bf16 weights and the Qwen3.5-2B shapes only (Q35_ENOTSUP otherwise, with the
 * reason; the per-op q35_decoder_decode_step covers the rest). Results match the per-op step up
 * to FP32 summation order. */
int q35_decoder_decode_step_persistent(q35_decoder* dec, void* stream);
int q35_decoder_has_persistent(const q35_decoder* dec);
/* Step tracing of the persistent step (no counterpart in the reference: a profiling aid). With a
 * device buffer of >= (ops + 1) * 148 * 2 int64 entries, thread 0 of every CTA writes the
 * %globaltimer (ns) on arriving at and leaving grid barrier j to [(j * 148 + cta) * 2 + {0, 1}];
 * row `ops` holds each CTA's step start and end. NULL turns tracing off. `ops` is
 * q35_decoder_trace_ops() (0 without a persistent step). */
int q35_decoder_set_trace(q35_decoder* dec, int64_t* trace, int64_t entries);
int q35_decoder_trace_ops(const q35_decoder* dec);
/* A8W8 parity probe (no counterpart in the reference: a diagnostic). With a device buffer set,
 * every A8W8 prefill projection appends its input's per-token int8 codes [length x k] and FP32
 * scales [length] to the buffer, in call order (per layer: in-projection, out-projection, gate/up,
 * down), as far as the buffer holds; q35_decoder_probe_bytes() gives the bytes the last prefill
 * needed. NULL / 0 turns it off. */
int q35_decoder_set_probe(q35_decoder* dec, void* buf, size_t bytes);
size_t q35_decoder_probe_bytes(const q35_decoder* dec);
/* Non-zero when a bounded wait of the persistent step gave up (1 grid barrier, 2 ring slot,
 * 3 ring data); reading clears it. */
int q35_decoder_persistent_error(void);

/* ---------------------------------------------------------------- vision tower */

/* kernels.py:1188-1222 layer_norm: out = LayerNorm(x; weight, bias, eps) over the last dim,
 * FP32 mean / centred variance, bf16 out. x, out [rows, width] bf16. */
int q35_layer_norm(const void* x, const void* weight, const void* bias, void* out, int64_t rows,
                   int64_t width, float eps, void* stream);
/* kernels.py:1225-1287 residual_add_layer_norm: residual_out = bf16(residual + update);
 * norm_out = LayerNorm(residual_out). residual_out may alias residual. */
int q35_residual_add_layer_norm(const void* residual, const void* update, const void* weight,
                                const void* bias, void* residual_out, void* norm_out, int64_t rows,
                                int64_t width, float eps, void* stream);
/* kernels.py:1290-1336 position_embed_add: out[r] = bf16(hidden[r] + bf16(sum_k weights[r,k] *
 * table[indices[r,k]])) (FP32 accumulation); indices int64 / weights fp32 [rows, neighbors]. */
int q35_position_embed_add(const void* hidden, const void* table, const int64_t* indices,
                           const float* weights, void* out, int64_t rows, int64_t width,
                           int64_t neighbors, void* stream);
/* kernels.py:336-416 vision_qkv_rope: packed [tokens, 3*heads*dim] -> q, k, v [heads, tokens, dim]
 * (batch 1) with RoPE on q, k: x*cos + rotate_half(x)*sin in FP32 without fused multiply-adds;
 * cos / sin fp32 [tokens, dim]. dim 64. */
int q35_vision_qkv_rope(const void* packed, const float* cos, const float* sin, void* q_out,
                        void* k_out, void* v_out, int64_t tokens, int64_t heads, int64_t dim,
                        void* stream);
/* Bidirectional attention over one image (integration.py:616-700 with cu_seqlens = [0, tokens]):
 * q, k, v [heads, tokens, dim] bf16 -> out [tokens, heads*dim] bf16, FP32 softmax. dim 64. */
int q35_vision_attention(const void* q, const void* k, const void* v, void* out, int64_t tokens,
                         int64_t heads, int64_t dim, float scale, void* stream);
/* 2-D rotary tables of HF Qwen3_5VisionModel.rot_pos_emb for a grid_h x grid_w patch grid in
 * merge-block order: cos/sin fp32 [grid_h*grid_w, 64] from inv_freq fp32 [16]. */
int q35_vision_rope_table(const float* inv_freq, float* cos_out, float* sin_out, int64_t grid_h,
                          int64_t grid_w, int64_t merge, void* stream);
/* Processor-side patch extraction (Qwen2-VL image processor order, a single frame repeated over
 * temporal_patch): pixels fp32 [channels, height, width] (rescaled to [0,1)) -> bf16
 * [(height/patch)*(width/patch), channels*temporal_patch*patch*patch], normalised (x-mean)/std. */
int q35_vision_patchify(const float* pixels, void* out, int64_t channels, int64_t height,
                        int64_t width, int64_t patch, int64_t temporal_patch, int64_t merge,
                        float mean, float std, void* stream);

/* One ViT block (HF Qwen3_5VisionBlock): pre-norm attention and GELU(tanh) MLP, biased linears. */
typedef struct {
  const void* norm1_w; const void* norm1_b;   /* bf16 [width] */
  const void* qkv_w; const void* qkv_b;       /* [3*width, width], [3*width] */
  const void* proj_w; const void* proj_b;     /* [width, width], [width] */
  const void* norm2_w; const void* norm2_b;
  const void* fc1_w; const void* fc1_b;       /* [intermediate, width] */
  const void* fc2_w; const void* fc2_b;       /* [width, intermediate] */
} q35_vit_block_desc;

typedef struct {
  int32_t depth, width, heads, intermediate;
  int32_t in_channels, patch, temporal_patch, merge;
  int32_t out_width;        /* merger output (the text model's hidden size) */
  int32_t pos_side;         /* learned position table is pos_side x pos_side */
  int32_t max_patches;      /* largest patch count the workspace is sized for */
  float eps;                /* LayerNorm epsilon (1e-6) */
  float pixel_mean, pixel_std;
  const q35_vit_block_desc* blocks;
  const void* patch_w;      /* Conv3d weight flattened [width, in_channels*temporal_patch*patch^2] */
  const void* patch_b;
  const void* pos_table;    /* [pos_side^2, width] */
  const float* rope_inv_freq; /* fp32 [16] */
  const void* merger_norm_w; const void* merger_norm_b;
  const void* merger_fc1_w; const void* merger_fc1_b;   /* [merge^2*width, merge^2*width] */
  const void* merger_fc2_w; const void* merger_fc2_b;   /* [out_width, merge^2*width] */
  void* workspace;
  size_t workspace_bytes;
} q35_vit_desc;

typedef struct q35_vit q35_vit;
size_t q35_vit_workspace_size(const q35_vit_desc* desc);
int q35_vit_create(const q35_vit_desc* desc, q35_vit** out);
void q35_vit_destroy(q35_vit* vit);
/* The vision forward of integration.py:509-736 for one image: patchify, patch embedding (tcgen05
 * GEMM + bias), bilinear position embedding + norm1, `depth` blocks (8 launches each: QKV GEMM,
 * QKV RoPE, attention, projection GEMM, residual + norm2, fc1 GEMM + GELU(tanh), fc2 GEMM,
 * residual + next norm1 / merger norm), then the 2x2 merger (fc1 + GELU, fc2): out bf16
 * [(height/patch/merge)*(width/patch/merge), out_width]. */
int q35_vit_encode(q35_vit* vit, const float* pixels, int64_t height, int64_t width, void* out,
                   void* stream);
/* The same forward for `images` images of one size, fp32 [images, C, height, width]: every launch
 * covers the whole batch (the GEMMs take images * patches rows; attention runs per image), out
 * bf16 [images * merged tokens, out_width] in image order. images * patches <= max_patches. */
int q35_vit_encode_batch(q35_vit* vit, const float* pixels, int64_t images, int64_t height, int64_t width,
                         void* out, void* stream);
/* The same forward from the processor's patches (Transformers' pixel_values for one image,
 * fp32 [grid_h*grid_w, in_channels*temporal_patch*patch^2] in merge-block order, the input of
 * Qwen3_5VisionModel.forward that integration.py:576-637 patches). */
int q35_vit_encode_patches(q35_vit* vit, const float* patches, int64_t grid_h, int64_t grid_w, void* out,
                           void* stream);
/* Device address of the final patch states [patches, width] of the last encode (pre-merger). */
void* q35_vit_hidden(const q35_vit* vit);

#ifdef __cplusplus
}
#endif

#endif /* QWEN35_B200_H */
