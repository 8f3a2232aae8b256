// The Qwen3.5 text-decoder loop on the device (reference: the patched text-model forward,
// qwen35_fused/integration.py:390-504; the greedy step of qwen35_fused/graph.py:51-79; the
// prefill + first token of evaluation_wrapper.py:354-365).
//
// Decode step (batch 1), per layer five launches:
//   in-projection GEMV   (prologue: RMSNorm of the residual, or embedding gather at layer 0)
//   mixer                (DeltaNet: conv + recurrent step + gated norm | attention: norm/RoPE/
//                         cache write/split-KV attention/gate), one kernel each
//   out-projection GEMV  (epilogue: residual add in place)
//   gate/up GEMV         (prologue: post-attention RMSNorm; epilogue: SwiGLU)
//   down GEMV            (epilogue: residual add)
// then the LM head with the final norm fused in, greedy top-1, and the step counters advanced
// by its last CTA: 5 * layers + 1 kernels, all on one stream, optionally chained with
// programmatic dependent launch so each kernel's weight prefetch overlaps its predecessor.
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

int q35_gemv_launch(const q35_gemv_desc* d, cudaStream_t s, bool pdl);
int q35_gemv_batch_launch(const q35_gemv_desc* d, int64_t batch, cudaStream_t s, bool pdl, void* split_ws = nullptr);
size_t q35_gemv_batch_split_bytes(int64_t n_out);
int q35_lm_head_batch_launch(const void* hidden, int64_t batch, const void* norm_weight, const void* weight,
                             int64_t vocab, float eps, int64_t* keys_out, void* workspace, cudaStream_t s, bool pdl);
extern "C" size_t q35_lm_shard_workspace_size(void);
int q35_lm_head_launch(const void* hidden, const void* norm_weight, const void* weight, int64_t* token_out,
                       int64_t vocab, int64_t k, float eps, void* ws, cudaStream_t s, bool pdl,
                       const q35_step_counters* adv, bool ring);
int q35_lm_keys_finish_launch(const int64_t* keys, int64_t n, int64_t* tokens, cudaStream_t s, bool pdl,
                              const q35_step_counters* adv);
int q35_attn_decode_launch(const void* packed, const void* q_weight, const void* k_weight, const float* inv_freq,
                           void* cache_k, void* cache_v, const int64_t* cache_len, const int64_t* rope_pos,
                           void* out, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t rotary_dim,
                           int64_t max_len, float eps, void* workspace, cudaStream_t stream, bool pdl);
int q35_delta_decode_launch(const void* packed, const void* conv_weight, void* conv_state, const void* a_log,
                            const void* dt_bias, const void* norm_weight, float* state, void* out, int64_t batch,
                            int64_t heads, int64_t packed_stride, float eps, cudaStream_t stream, bool pdl,
                            bool qk_regs);
int q35_gemm_launch(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k, int epi, bool int8,
                    const float* sx, const float* sw, cudaStream_t s, bool pdl);
int q35_gemm_tc_launch(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k, int epi, bool int8,
                       const float* sx, const float* sw, cudaStream_t s, const void* bias, bool pdl);
int q35_quantize_tokens_launch(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                               cudaStream_t s, bool pdl);
int q35_rms_norm_launch(const void* x, const void* weight, void* out, int64_t rows, int64_t width, float eps,
                        cudaStream_t stream, bool pdl);
int q35_embedding_launch(const int64_t* ids, const void* table, void* out, int64_t n, int64_t vocab, int64_t width,
                         cudaStream_t stream, bool pdl);
int q35_attention_gate_launch(const void* x, const void* packed, void* out, int64_t rows, int64_t hidden,
                              int64_t packed_stride, int64_t head_dim, cudaStream_t stream, bool pdl);
int q35_prefill_attention_launch(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                 int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len, int64_t q_offset,
                                 int64_t head_dim, float scale, cudaStream_t stream, bool pdl);
int q35_qgkv_rope_positions_launch(const void* packed, const void* q_weight, const void* k_weight,
                                   const float* inv_freq, void* q_out, void* k_out, void* v_out,
                                   const int64_t* cache_start, int64_t batch, int64_t seq_len, int64_t q_heads,
                                   int64_t kv_heads, int64_t rotary_dim, int64_t kv_len, float eps,
                                   cudaStream_t stream, const int64_t* pos3, int sec_h, int sec_w, bool pdl,
                                   void* vt_out, int64_t vt_stride);
int q35_prefill_attention_tc_launch(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                                    int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                    int64_t vt_stride, float scale, void* ws, size_t ws_bytes, cudaStream_t stream,
                                    bool pdl);
size_t q35_prefill_attention_tc_ws_bytes(int64_t batch, int64_t kv_heads, int64_t seq_len);
int q35_gated_rms_strided_launch(const void* x, const void* gate, int gate_group, int64_t gate_stride,
                                 const void* weight, void* out, int64_t rows, int64_t width, float eps,
                                 cudaStream_t stream, bool pdl);
int q35_set_counters_launch(int64_t* a, int64_t* b, int64_t value, cudaStream_t stream, bool pdl);
size_t q35_delta_chunk_workspace_bytes(int64_t batch, int64_t heads, int64_t max_len);
int q35_delta_chunked_launch(const void* qkv, const void* packed, const void* a_log, const void* dt_bias, float* state,
                             void* out, int64_t batch, int64_t seq_len, int64_t heads, int64_t packed_stride,
                             float* ws, cudaStream_t s, const void* conv_weight, void* conv_state, bool pdl);
size_t q35_attn_decode_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                      int64_t cache_len);
struct q35_pk_plan;
size_t q35_pk_workspace_bytes(const q35_decoder_desc& d);
const char* q35_pk_unsupported(const q35_decoder_desc& d);
int q35_pk_create(const q35_decoder_desc& d, const q35_layer_desc* layers, bf16* resid, bf16* proj, bf16* act,
                  void* ws, q35_pk_plan** out);
void q35_pk_destroy(q35_pk_plan* plan);
int q35_pk_launch(const q35_pk_plan* plan, cudaStream_t s);
int q35_pk_set_trace(q35_pk_plan* plan, int64_t* trace, int64_t entries);
int q35_pk_ops(const q35_pk_plan* plan);

namespace {

struct Carve {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~(size_t)255;
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
};

struct Buffers {
  // decode
  bf16* resid;
  bf16* mix_in_out;   // projection output [max(delta_rows, qgkv_rows)]
  bf16* mix_out;      // mixer output [max(value_dim, q_heads*head_dim)]
  bf16* act;          // SwiGLU output [intermediate]
  void* attn_ws;
  void* lm_ws;
  void* lm_keys_ws;   // batched decode: the shard top-1 workspace (keys reduced over the vocabulary)
  void* split_ws;     // batched decode: split-K parts + tickets of the narrow projections (zeroed)
  int64_t* lm_keys;   // batched decode: [batch] reduced keys
  void* pk_ws;        // persistent decode step: op table, attention partials, barrier words
  // prefill
  bf16* p_resid;      // [L, H]
  bf16* p_norm;       // [L, H]
  bf16* p_packed;     // [L, max rows]
  bf16* p_conv;       // [L, conv_dim]
  bf16* p_core;       // [L, value_dim] / q [Hq, L, D]
  bf16* p_attn;       // [L, Hq*D]
  bf16* p_mix;        // [L, max(value_dim, Hq*D)]
  bf16* p_act;        // [L, I]
  int8_t* p_q8;       // [L, max(H, I, mix width)]
  float* p_sx;        // [L]
  float* p_chunk;     // chunked DeltaNet factors for one layer
  bf16* p_vt;         // V^T [seq][kv heads][head dim][keys padded to 64] (tcgen05 prefill attention;
                      // the workspace starts zeroed, so padding columns are finite)
  void* p_attn_ws;    // its key-split partials and tickets (zeroed, left zeroed)
  size_t p_attn_ws_bytes;
};

Buffers carve(const q35_decoder_desc& d, void* base, size_t* total) {
  Carve c{static_cast<char*>(base)};
  Buffers b;
  const int64_t rows_in = d.delta_rows > 2 * d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim
                              ? d.delta_rows
                              : 2 * d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim;
  const int64_t mixw = (int64_t)d.lin_heads * d.lin_dv > (int64_t)d.q_heads * d.head_dim
                           ? (int64_t)d.lin_heads * d.lin_dv
                           : (int64_t)d.q_heads * d.head_dim;
  const int64_t conv_dim = (int64_t)d.lin_heads * (2 * d.lin_dk + d.lin_dv);
  const int64_t L = d.max_prefill;
  const int64_t nb = d.batch > 1 ? d.batch : 1;
  b.lm_ws = c.take<char>(256);  // LM head ticket + key (must start zeroed)
  b.lm_keys_ws = c.take<char>(128);  // batched LM head: 8 keys + count (zeroed, left zeroed)
  b.lm_keys = c.take<int64_t>(8);
  b.split_ws = c.take<char>(nb > 1 ? q35_gemv_batch_split_bytes(d.hidden) : 0);
  b.resid = c.take<bf16>(nb * d.hidden);
  b.mix_in_out = c.take<bf16>(nb * rows_in);
  b.mix_out = c.take<bf16>(nb * mixw);
  b.act = c.take<bf16>(nb * d.intermediate);
  b.attn_ws = c.take<char>(q35_attn_decode_workspace_size(nb, d.q_heads, d.kv_heads, d.head_dim, d.max_len));
  b.pk_ws = c.take<char>(q35_pk_workspace_bytes(d));
  b.p_resid = c.take<bf16>(L * d.hidden);
  b.p_norm = c.take<bf16>(L * d.hidden);
  b.p_packed = c.take<bf16>(L * rows_in);
  b.p_conv = c.take<bf16>(L * conv_dim);
  b.p_core = c.take<bf16>(L * mixw);
  b.p_attn = c.take<bf16>(L * mixw);
  b.p_mix = c.take<bf16>(L * mixw);
  b.p_act = c.take<bf16>(L * d.intermediate);
  int64_t qw = d.hidden > d.intermediate ? d.hidden : d.intermediate;
  if (mixw > qw) qw = mixw;
  b.p_q8 = c.take<int8_t>(L * qw);
  b.p_sx = c.take<float>(L);
  // batched prefill: up to `nb` sequences sharing the L rows, each padded to whole chunks
  b.p_chunk = c.take<float>(q35_delta_chunk_workspace_bytes(1, d.lin_heads, L + 64 * nb) / sizeof(float));
  b.p_vt = c.take<bf16>((size_t)d.kv_heads * d.head_dim * (L + 64 * nb));
  // the key-split workspace for nb sequences whose lengths add up to L: bounded by L / 32 + nb
  // query blocks (the size function counts ceil(L / 32) blocks per sequence)
  b.p_attn_ws_bytes = q35_prefill_attention_tc_ws_bytes(1, d.kv_heads, L + 32 * nb);
  b.p_attn_ws = c.take<char>(b.p_attn_ws_bytes);
  *total = c.off + 256;
  return b;
}

}  // namespace

struct q35_decoder {
  q35_decoder_desc d;
  std::vector<q35_layer_desc> layers;
  Buffers buf;
  q35_pk_plan* pk = nullptr;  // persistent decode step, when the model fits its built-in shapes
  std::string pk_why;         // otherwise the reason
  char* probe = nullptr;      // A8W8 prefill probe: int8 codes + scales of every projection input
  size_t probe_bytes = 0;
  size_t probe_want = 0;      // bytes the last prefill had to record
};

extern "C" int q35_decoder_set_probe(q35_decoder* dec, void* buf, size_t bytes) {
  Q35_REQUIRE(dec, "set_probe: null decoder");
  Q35_REQUIRE(buf || bytes == 0, "set_probe: null buffer with a size");
  dec->probe = static_cast<char*>(buf);
  dec->probe_bytes = bytes;
  return Q35_OK;
}

extern "C" size_t q35_decoder_probe_bytes(const q35_decoder* dec) { return dec ? dec->probe_want : 0; }

extern "C" size_t q35_decoder_workspace_size(const q35_decoder_desc* desc) {
  if (!desc) return 0;
  size_t total = 0;
  carve(*desc, nullptr, &total);
  return total;
}

extern "C" int q35_decoder_create(const q35_decoder_desc* desc, q35_decoder** out) {
  Q35_REQUIRE(desc && out && desc->layers && desc->n_layers > 0, "decoder_create: bad descriptor");
  const q35_decoder_desc& d = *desc;
  Q35_REQUIRE(d.embed && d.final_norm && d.inv_freq && d.token && d.cache_len && d.rope_pos,
              "decoder_create: missing model/state pointer");
  Q35_REQUIRE(d.head_dim == 256 && d.lin_dk == 128 && d.lin_dv == 128 && d.conv_kernel == 4,
              "decoder_create: kernels are built for head dims 256 / 128 and conv kernel 4");
  Q35_REQUIRE(d.hidden % 16 == 0 && d.intermediate % 16 == 0 && d.max_len > 0 && d.max_prefill > 0,
              "decoder_create: bad sizes");
  Q35_REQUIRE(d.batch >= 0 && d.batch <= 8, "decoder_create: batch %d outside [1, 8]", d.batch);
  Q35_REQUIRE(d.batch <= 1 || (!d.a8w8 && d.hidden == 2048 && d.intermediate % 2 == 0),
              "decoder_create: batched decode is built for bf16 weights and hidden 2048");
  Q35_REQUIRE(d.workspace && d.workspace_bytes >= q35_decoder_workspace_size(desc),
              "decoder_create: workspace too small (%zu < %zu)", d.workspace_bytes, q35_decoder_workspace_size(desc));
  for (int i = 0; i < d.n_layers; ++i) {
    const q35_layer_desc& L = d.layers[i];
    Q35_REQUIRE(L.in_ln && L.post_ln && L.mix_in && L.mix_out && L.gate_up && L.down, "layer %d: missing weight", i);
    Q35_REQUIRE(!d.a8w8 || (L.mix_in_scale && L.mix_out_scale && L.gate_up_scale && L.down_scale),
                "layer %d: A8W8 scales missing", i);
    if (L.kind == 0)
      Q35_REQUIRE(L.conv_w && L.a_log && L.dt_bias && L.gnorm && L.conv_state && L.rec_state,
                  "layer %d: DeltaNet tensors missing", i);
    else
      Q35_REQUIRE(L.q_norm && L.k_norm && L.k_cache && L.v_cache, "layer %d: attention tensors missing", i);
  }
  q35_decoder* dec = new q35_decoder();
  dec->d = d;
  dec->layers.assign(d.layers, d.layers + d.n_layers);
  dec->d.layers = dec->layers.data();
  size_t total = 0;
  dec->buf = carve(d, d.workspace, &total);
  const char* why = q35_pk_unsupported(dec->d);
  if (why[0]) {
    dec->pk_why = why;
  } else if (q35_pk_create(dec->d, dec->layers.data(), dec->buf.resid, dec->buf.mix_in_out, dec->buf.act,
                           dec->buf.pk_ws, &dec->pk) != Q35_OK) {
    dec->pk_why = q35_last_error();
    dec->pk = nullptr;
  }
  *out = dec;
  return Q35_OK;
}

extern "C" void q35_decoder_destroy(q35_decoder* dec) {
  if (dec && dec->pk) q35_pk_destroy(dec->pk);
  delete dec;
}

extern "C" int q35_decoder_decode_step_persistent(q35_decoder* dec, void* stream) {
  Q35_REQUIRE(dec, "decode_step_persistent: null decoder");
  if (!dec->pk) return q35_fail(Q35_ENOTSUP, "persistent decode unavailable: %s", dec->pk_why.c_str());
  return q35_pk_launch(dec->pk, (cudaStream_t)stream);
}

extern "C" int q35_decoder_has_persistent(const q35_decoder* dec) { return dec && dec->pk ? 1 : 0; }

extern "C" int q35_decoder_set_trace(q35_decoder* dec, int64_t* trace, int64_t entries) {
  Q35_REQUIRE(dec, "set_trace: null decoder");
  if (!dec->pk) return q35_fail(Q35_ENOTSUP, "persistent decode unavailable: %s", dec->pk_why.c_str());
  return q35_pk_set_trace(dec->pk, trace, entries);
}

extern "C" int q35_decoder_trace_ops(const q35_decoder* dec) { return dec && dec->pk ? q35_pk_ops(dec->pk) : 0; }

extern "C" int q35_decoder_kernels_per_step(const q35_decoder* dec) {
  return dec ? 5 * dec->d.n_layers + (dec->d.batch > 1 ? 2 : 1) : 0;
}

#define Q35_TRY(x)          \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

// The decode step's layers: leaves the final residual in B.resid (pre final norm); the LM head
// that follows writes the token and advances the step counters.
static int decode_layers(q35_decoder* dec, cudaStream_t s) {
  const q35_decoder_desc& d = dec->d;
  const Buffers& B = dec->buf;
  const bool pdl = d.use_pdl != 0;
  const bool q8 = d.a8w8 != 0;
  const int64_t nb = d.batch > 1 ? d.batch : 1;
  auto gemv = [&](const q35_gemv_desc* g) -> int {
    return nb > 1 ? q35_gemv_batch_launch(g, nb, s, pdl, B.split_ws) : q35_gemv_launch(g, s, pdl);
  };
  const int qgkv_rows = 2 * d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim;
  for (int i = 0; i < d.n_layers; ++i) {
    const q35_layer_desc& L = dec->layers[i];
    const bool delta = L.kind == 0;
    q35_gemv_desc g = {};
    // in-projection (+ residual norm / embedding)
    g.weight = L.mix_in;
    g.w_scale = L.mix_in_scale;
    g.input = B.resid;
    g.norm_weight = L.in_ln;
    g.token = d.token;
    g.embed = d.embed;
    g.vocab = d.vocab;
    g.resid_out = B.resid;
    g.out = B.mix_in_out;
    g.n_out = delta ? d.delta_rows : qgkv_rows;
    g.k = d.hidden;
    g.prologue = (i == 0) ? Q35_PRO_EMBED : Q35_PRO_NORM;
    g.epilogue = Q35_EPI_STORE;
    g.int8 = q8;
    g.eps = d.eps;
    Q35_TRY(gemv(&g));
    // mixer
    if (delta) {
      Q35_TRY(q35_delta_decode_launch(B.mix_in_out, L.conv_w, L.conv_state, L.a_log, L.dt_bias, L.gnorm,
                                      L.rec_state, B.mix_out, nb, d.lin_heads, d.delta_rows, d.eps, s, pdl, q8));
    } else {
      Q35_TRY(q35_attn_decode_launch(B.mix_in_out, L.q_norm, L.k_norm, d.inv_freq, L.k_cache, L.v_cache,
                                     d.cache_len, d.rope_pos, B.mix_out, nb, d.q_heads, d.kv_heads, d.rotary_dim,
                                     d.max_len, d.eps, B.attn_ws, s, pdl));
    }
    // out-projection + residual
    g = q35_gemv_desc{};
    g.weight = L.mix_out;
    g.w_scale = L.mix_out_scale;
    g.input = B.mix_out;
    g.resid_out = B.resid;
    g.n_out = d.hidden;
    g.k = delta ? d.lin_heads * d.lin_dv : d.q_heads * d.head_dim;
    g.prologue = Q35_PRO_PLAIN;
    g.epilogue = Q35_EPI_RESIDUAL;
    g.int8 = q8;
    g.eps = d.eps;
    Q35_TRY(gemv(&g));
    // gate/up + SwiGLU
    g = q35_gemv_desc{};
    g.weight = L.gate_up;
    g.w_scale = L.gate_up_scale;
    g.input = B.resid;
    g.norm_weight = L.post_ln;
    g.out = B.act;
    g.n_out = d.intermediate;
    g.k = d.hidden;
    g.prologue = Q35_PRO_NORM;
    g.epilogue = Q35_EPI_SWIGLU;
    g.int8 = q8;
    g.eps = d.eps;
    Q35_TRY(gemv(&g));
    // down + residual
    g = q35_gemv_desc{};
    g.weight = L.down;
    g.w_scale = L.down_scale;
    g.input = B.act;
    g.resid_out = B.resid;
    g.n_out = d.hidden;
    g.k = d.intermediate;
    g.prologue = Q35_PRO_PLAIN;
    g.epilogue = Q35_EPI_RESIDUAL;
    g.int8 = q8;
    g.eps = d.eps;
    Q35_TRY(gemv(&g));
  }
  return Q35_OK;
}

extern "C" int q35_decoder_decode_step(q35_decoder* dec, void* stream) {
  Q35_REQUIRE(dec, "decode_step: null decoder");
  const q35_decoder_desc& d = dec->d;
  cudaStream_t s = (cudaStream_t)stream;
  Q35_TRY(decode_layers(dec, s));
  q35_step_counters adv = {d.cache_len, d.rope_pos, d.token_log, d.log_pos, d.log_len};
  if (d.batch > 1) {  // one pass over the tied table for every request: keys, then tokens + counters
    Q35_TRY(q35_lm_head_batch_launch(dec->buf.resid, d.batch, d.final_norm, d.embed, d.vocab, d.eps,
                                     dec->buf.lm_keys, dec->buf.lm_keys_ws, s, d.use_pdl != 0));
    return q35_lm_keys_finish_launch(dec->buf.lm_keys, d.batch, d.token, s, false, &adv);
  }
  return q35_lm_head_launch(dec->buf.resid, d.final_norm, d.embed, d.token, d.vocab, d.hidden, d.eps, dec->buf.lm_ws,
                            s, d.use_pdl != 0, &adv, d.a8w8 == 0);
}

extern "C" int q35_decoder_decode_layers(q35_decoder* dec, void* stream) {
  Q35_REQUIRE(dec, "decode_layers: null decoder");
  return decode_layers(dec, (cudaStream_t)stream);
}

extern "C" void* q35_decoder_hidden(const q35_decoder* dec) { return dec ? dec->buf.resid : nullptr; }

extern "C" int q35_decoder_finish_step(q35_decoder* dec, const int64_t* keys, int64_t index, void* stream) {
  Q35_REQUIRE(dec && keys, "finish_step: null pointer");
  Q35_REQUIRE(index >= 0 && index < 1024, "finish_step: key index %lld outside [0, 1024)", (long long)index);
  const q35_decoder_desc& d = dec->d;
  q35_step_counters adv = {d.cache_len, d.rope_pos, d.token_log, d.log_pos, d.log_len};
  return q35_lm_keys_finish_launch(keys + index, 1, d.token, (cudaStream_t)stream, false, &adv);
}

// Multimodal input rows: image_embeds[i] -> resid[rows[i]] (rows outside [0, L) are skipped).
__global__ void image_rows_kernel(const bf16* __restrict__ embeds, const int64_t* __restrict__ rows,
                                  bf16* __restrict__ resid, int64_t L, int64_t width) {
  q35::pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  q35::pdl_launch_dependents();
  const int64_t r = rows[blockIdx.x];
  if (r < 0 || r >= L) return;
  const uint4* src = reinterpret_cast<const uint4*>(embeds + (int64_t)blockIdx.x * width);
  uint4* dst = reinterpret_cast<uint4*>(resid + r * width);
  for (int64_t c = threadIdx.x; c < width / 8; c += blockDim.x) dst[c] = src[c];
}

struct MmInputs {
  const void* image_embeds = nullptr;
  const int64_t* image_rows = nullptr;
  int64_t n_image = 0;
  const int64_t* pos3 = nullptr;
  int64_t rope_next = -1;
};

static int prefill_impl(q35_decoder* dec, const int64_t* ids, int64_t length, const MmInputs& mm, int64_t slot,
                        int64_t nseq, cudaStream_t s);

extern "C" int q35_decoder_prefill(q35_decoder* dec, const int64_t* ids, int64_t length, void* stream) {
  Q35_REQUIRE(dec && ids, "prefill: null argument");
  return prefill_impl(dec, ids, length, MmInputs{}, 0, 1, (cudaStream_t)stream);
}

extern "C" int q35_decoder_prefill_slot(q35_decoder* dec, const int64_t* ids, int64_t length, int64_t slot,
                                        void* stream) {
  Q35_REQUIRE(dec && ids, "prefill_slot: null argument");
  return prefill_impl(dec, ids, length, MmInputs{}, slot, 1, (cudaStream_t)stream);
}

extern "C" int q35_decoder_prefill_batch(q35_decoder* dec, const int64_t* ids, int64_t length, int64_t nseq,
                                         const void* image_embeds, const int64_t* image_rows, int64_t n_image,
                                         const int64_t* positions3, int64_t rope_next, int64_t slot, void* stream) {
  Q35_REQUIRE(dec && ids, "prefill_batch: null argument");
  Q35_REQUIRE(nseq >= 1 && length >= 1 && n_image >= 0 && n_image <= nseq * length &&
                  (n_image == 0 || (image_embeds && image_rows)),
              "prefill_batch: %lld sequences of %lld tokens, %lld image rows (embeddings and row indices needed)",
              (long long)nseq, (long long)length, (long long)n_image);
  Q35_REQUIRE(!image_embeds || Q35_ALIGNED(image_embeds, 16), "prefill_mm: image embeddings 16-byte aligned");
  Q35_REQUIRE(!positions3 || dec->d.mrope_section[1] + dec->d.mrope_section[2] > 0,
              "prefill_mm: 3-axis positions need the decoder's mrope_section");
  Q35_REQUIRE(rope_next >= -1, "prefill_mm: rope_next must be non-negative (or -1: the prompt length)");
  MmInputs mm;
  mm.image_embeds = image_embeds;
  mm.image_rows = image_rows;
  mm.n_image = n_image;
  mm.pos3 = positions3;
  mm.rope_next = rope_next;
  return prefill_impl(dec, ids, length, mm, slot, nseq, (cudaStream_t)stream);
}

extern "C" int q35_decoder_prefill_mm(q35_decoder* dec, const int64_t* ids, int64_t length, const void* image_embeds,
                                      const int64_t* image_rows, int64_t n_image, const int64_t* positions3,
                                      int64_t rope_next, int64_t slot, void* stream) {
  Q35_REQUIRE(rope_next >= 0, "prefill_mm: rope_next must be non-negative");
  return q35_decoder_prefill_batch(dec, ids, length, 1, image_embeds, image_rows, n_image, positions3, rope_next, slot,
                                   stream);
}

// `nseq` sequences of `length` tokens each (ids [nseq * length]) into request slots
// [slot, slot + nseq): every projection, norm and GEMM runs over all nseq * length rows at once;
// the DeltaNet scan, the causal attention and the KV-cache writes run per sequence; the LM head
// reads each sequence's last row.
static int prefill_impl(q35_decoder* dec, const int64_t* ids, int64_t length, const MmInputs& mm, int64_t slot,
                        int64_t nseq, cudaStream_t s) {
  const q35_decoder_desc& d = dec->d;
  const int64_t nb = d.batch > 1 ? d.batch : 1;
  Q35_REQUIRE(length >= 1 && nseq >= 1 && nseq * length <= d.max_prefill && length < d.max_len,
              "prefill: %lld x %lld tokens outside [1, %d] (cache %d)", (long long)nseq, (long long)length,
              d.max_prefill, d.max_len);
  Q35_REQUIRE(slot >= 0 && slot + nseq <= nb, "prefill: slots [%lld, %lld) outside the batch of %lld",
              (long long)slot, (long long)(slot + nseq), (long long)nb);
  // this slot's states and caches: the layers' tensors have a leading batch dimension
  const int64_t conv_elems = (int64_t)d.lin_heads * (2 * d.lin_dk + d.lin_dv) * d.conv_kernel;
  const int64_t rec_elems = (int64_t)d.lin_heads * d.lin_dk * d.lin_dv;
  const int64_t kv_elems = (int64_t)d.kv_heads * d.max_len * d.head_dim;
  std::vector<q35_layer_desc> slot_layers(dec->layers);
  for (q35_layer_desc& L : slot_layers) {
    if (L.conv_state) L.conv_state = static_cast<bf16*>(L.conv_state) + slot * conv_elems;
    if (L.rec_state) L.rec_state += slot * rec_elems;
    if (L.k_cache) L.k_cache = static_cast<bf16*>(L.k_cache) + slot * kv_elems;
    if (L.v_cache) L.v_cache = static_cast<bf16*>(L.v_cache) + slot * kv_elems;
  }
  int64_t* token_out = d.token + slot;
  const Buffers& B = dec->buf;
  const bool q8 = d.a8w8 != 0;
  const int64_t H = d.hidden, I = d.intermediate, Lt = length, R = nseq * length;  // R rows in all
  const int64_t qgkv_rows = 2 * d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim;
  const int64_t conv_dim = (int64_t)d.lin_heads * (2 * d.lin_dk + d.lin_dv);
  const int64_t vdim = (int64_t)d.lin_heads * d.lin_dv;
  const int64_t adim = (int64_t)d.q_heads * d.head_dim;
  // Every prefill kernel waits on its predecessor (griddepcontrol.wait) before touching memory,
  // so chaining them with programmatic dependent launch only overlaps launch and prologue.
  const bool pdl = d.use_pdl != 0;
  dec->probe_want = 0;

  // Projection helper: bf16 GEMM, or per-token int8 quantisation + int8 GEMM for A8W8; tcgen05
  // tiles when enabled (K must fill the 128-byte slabs), warp-level MMA otherwise.
  auto proj = [&](const bf16* x, int64_t k, const void* w, const float* sw, void* out, int64_t n, int epi) -> int {
    const bool tc = d.prefill_tc && (k * (q8 ? 1 : 2)) % 128 == 0 && n % 8 == 0;
    if (!q8)
      return tc ? q35_gemm_tc_launch(x, w, out, R, n, k, epi, false, nullptr, nullptr, s, nullptr, pdl)
                : q35_gemm_launch(x, w, out, R, n, k, epi, false, nullptr, nullptr, s, pdl);
    int rc = q35_quantize_tokens_launch(x, B.p_q8, B.p_sx, R, k, s, pdl);
    if (rc) return rc;
    if (dec->probe) {  // record [codes R x k][scales R] of this projection's input
      const size_t codes = (size_t)R * k, need = codes + (size_t)R * sizeof(float);
      if (dec->probe_want + need <= dec->probe_bytes &&
          (cudaMemcpyAsync(dec->probe + dec->probe_want, B.p_q8, codes, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
           cudaMemcpyAsync(dec->probe + dec->probe_want + codes, B.p_sx, (size_t)R * sizeof(float),
                           cudaMemcpyDeviceToDevice, s) != cudaSuccess))
        return q35_fail(Q35_ECUDA, "prefill: probe copy failed");
      dec->probe_want += need;
    }
    return tc ? q35_gemm_tc_launch(B.p_q8, w, out, R, n, k, epi, true, B.p_sx, sw, s, nullptr, pdl)
              : q35_gemm_launch(B.p_q8, w, out, R, n, k, epi, true, B.p_sx, sw, s, pdl);
  };

  // fresh cache: zero the recurrent/conv states (the KV rows past `length` are never read)
  for (int i = 0; i < d.n_layers; ++i) {
    const q35_layer_desc& L = slot_layers[i];
    if (L.kind == 0) {
      if (cudaMemsetAsync(L.rec_state, 0, (size_t)(nseq * rec_elems) * sizeof(float), s) != cudaSuccess ||
          cudaMemsetAsync(L.conv_state, 0, (size_t)(nseq * conv_elems) * sizeof(bf16), s) != cudaSuccess)
        return q35_fail(Q35_ECUDA, "prefill: state reset failed");
    }
  }
  Q35_TRY(q35_set_counters_launch(d.cache_len, d.rope_pos, 0, s, false));
  Q35_TRY(q35_embedding_launch(ids, d.embed, B.p_resid, R, d.vocab, H, s, pdl));
  if (mm.n_image > 0) {
    const cudaError_t e = q35_launch(image_rows_kernel, dim3((unsigned)mm.n_image), dim3(128), 0, s, pdl,
                                     (const bf16*)mm.image_embeds, mm.image_rows, B.p_resid, R, H);
    if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "prefill_mm image rows launch: %s", cudaGetErrorString(e));
  }
  for (int i = 0; i < d.n_layers; ++i) {
    const q35_layer_desc& L = slot_layers[i];
    Q35_TRY(q35_rms_norm_launch(B.p_resid, L.in_ln, B.p_norm, R, H, d.eps, s, pdl));
    if (L.kind == 0) {
      Q35_TRY(proj(B.p_norm, H, L.mix_in, L.mix_in_scale, B.p_packed, d.delta_rows, Q35_EPI_STORE));
      if (d.prefill_delta == 0 && d.conv_kernel == 4 && Lt >= 4) {
        // causal conv folded into the chunk prep (reads the raw [q k v] columns of the projection)
        Q35_TRY(q35_delta_chunked_launch(nullptr, B.p_packed, L.a_log, L.dt_bias, L.rec_state, B.p_core, nseq, Lt,
                                         d.lin_heads, d.delta_rows, B.p_chunk, s, L.conv_w, L.conv_state, pdl));
      } else {
        Q35_TRY(q35_causal_conv1d(B.p_packed, L.conv_w, L.conv_state, B.p_conv, nseq, Lt, d.delta_rows, conv_dim,
                                  d.conv_kernel, s));
        if (d.prefill_delta == 0)
          Q35_TRY(q35_delta_chunked_launch(B.p_conv, B.p_packed, L.a_log, L.dt_bias, L.rec_state, B.p_core, nseq,
                                           Lt, d.lin_heads, d.delta_rows, B.p_chunk, s, nullptr, nullptr, false));
        else
          Q35_TRY(q35_delta_recurrent(B.p_conv, B.p_packed, L.a_log, L.dt_bias, L.rec_state, B.p_core, nseq, Lt,
                                      d.lin_heads, d.lin_dk, d.delta_rows, s));
      }
      Q35_TRY(q35_gated_rms_strided_launch(B.p_core, B.p_packed + conv_dim, d.lin_heads, d.delta_rows, L.gnorm,
                                           B.p_mix, R * d.lin_heads, d.lin_dv, d.eps, s, pdl));
      Q35_TRY(proj(B.p_mix, vdim, L.mix_out, L.mix_out_scale, B.p_resid, H, Q35_EPI_RESIDUAL));
    } else {
      Q35_TRY(proj(B.p_norm, H, L.mix_in, L.mix_in_scale, B.p_packed, qgkv_rows, Q35_EPI_STORE));
      // tcgen05 attention (4 query heads per KV head, head dim 256) reads V transposed, written by
      // the norm + RoPE kernel beside the cache rows; else the warp-MMA kernel reads the cache
      const bool tc_attn = d.prefill_tc && d.q_heads == 4 * d.kv_heads && d.head_dim == 256;
      const int64_t vt_stride = (Lt + 63) / 64 * 64;
      const float scale = 1.0f / sqrtf((float)d.head_dim);
      Q35_TRY(q35_qgkv_rope_positions_launch(B.p_packed, L.q_norm, L.k_norm, d.inv_freq, B.p_core, L.k_cache,
                                             L.v_cache, nullptr, nseq, Lt, d.q_heads, d.kv_heads, d.rotary_dim,
                                             d.max_len, d.eps, s, mm.pos3, d.mrope_section[1], d.mrope_section[2],
                                             pdl, tc_attn ? B.p_vt : nullptr, vt_stride));
      if (tc_attn)
        Q35_TRY(q35_prefill_attention_tc_launch(B.p_core, L.k_cache, B.p_vt, B.p_attn, nseq, d.q_heads, d.kv_heads, Lt,
                                                d.max_len, vt_stride, scale, B.p_attn_ws, B.p_attn_ws_bytes, s, pdl));
      else
        Q35_TRY(q35_prefill_attention_launch(B.p_core, L.k_cache, L.v_cache, B.p_attn, nseq, d.q_heads, d.kv_heads,
                                             Lt, d.max_len, 0, d.head_dim, scale, s, pdl));
      Q35_TRY(q35_attention_gate_launch(B.p_attn, B.p_packed, B.p_mix, R, adim, qgkv_rows, d.head_dim, s, pdl));
      Q35_TRY(proj(B.p_mix, adim, L.mix_out, L.mix_out_scale, B.p_resid, H, Q35_EPI_RESIDUAL));
    }
    Q35_TRY(q35_rms_norm_launch(B.p_resid, L.post_ln, B.p_norm, R, H, d.eps, s, pdl));
    Q35_TRY(proj(B.p_norm, H, L.gate_up, L.gate_up_scale, B.p_act, I, Q35_EPI_SWIGLU));
    Q35_TRY(proj(B.p_act, I, L.down, L.down_scale, B.p_resid, H, Q35_EPI_RESIDUAL));
  }
  if (nseq == 1) {
    Q35_TRY(q35_lm_head_launch(B.p_resid + (Lt - 1) * H, d.final_norm, d.embed, token_out, d.vocab, H, d.eps,
                               B.lm_ws, s, pdl, nullptr, d.a8w8 == 0));
  } else {  // each sequence's last row -> the decode rows, one pass over the tied table for all
    if (cudaMemcpy2DAsync(B.resid, (size_t)H * sizeof(bf16), B.p_resid + (Lt - 1) * H, (size_t)(Lt * H) * sizeof(bf16),
                          (size_t)H * sizeof(bf16), (size_t)nseq, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return q35_fail(Q35_ECUDA, "prefill: last-row gather failed");
    Q35_TRY(q35_lm_head_batch_launch(B.resid, nseq, d.final_norm, d.embed, d.vocab, d.eps, B.lm_keys, B.lm_keys_ws,
                                     s, false));
    Q35_TRY(q35_lm_keys_finish_launch(B.lm_keys, nseq, token_out, s, false, nullptr));
  }
  Q35_TRY(q35_set_counters_launch(d.cache_len, d.rope_pos, Lt, s, pdl));
  if (mm.rope_next >= 0) Q35_TRY(q35_set_counters_launch(d.rope_pos, d.rope_pos, mm.rope_next, s, pdl));
  return Q35_OK;
}
