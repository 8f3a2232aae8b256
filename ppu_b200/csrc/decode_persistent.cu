// Persistent decode step: the whole batch-1 greedy decode step (reference: the patched text-model
// forward, qwen35_fused/integration.py:390-504, one step of qwen35_fused/graph.py:51-79) as ONE
// cooperative kernel with one CTA per SM.
//
// Why: the per-op decode path streams each weight matrix at copy bandwidth but pays a fixed
// ~3 us per launch (launch, first-byte latency, tail) over 121 launches a token. Here the weight
// stream never stops at op boundaries:
//  * a producer warp walks the step's GEMV ops and copies this CTA's rows of every weight matrix
//    (rows [b*n/148, (b+1)*n/148), gate and up rows together for SwiGLU) into a 6-stage x 32 KB
//    shared-memory ring with 1-D bulk async copies (cp.async.bulk, no tensor map, no multicast),
//    each completing on a per-stage mbarrier; it runs ahead across op boundaries, grid barriers and
//    the mixers, limited only by free ring stages;
//  * 16 consumer warps run the ops in order. Between dependent ops all CTAs meet at a grid barrier
//    (atomic counter, acquire polling, bounded wait that sets an error word instead of hanging;
//    the cooperative launch guarantees co-residency). A GEMV op builds its input vector in shared
//    memory (plain / RMSNorm / embedding gather + RMSNorm / gated RMSNorm of the DeltaNet output),
//    then consumes its stages (8 weight rows x 2048 k each) with groups of 4 warps: each warp
//    covers a quarter of the k range with FP32 FMAs on the CUDA cores (vectorised 16-byte reads;
//    no tensor cores on the decode path), releases the stage itself and reduces per row at the end
//    of the tile; the group's first warp adds the four partials in a fixed order and applies the
//    epilogue (store; store + causal-conv update of that channel; residual add in place; SwiGLU;
//    running greedy top-1);
//  * mixers use all CTAs: the DeltaNet step is 128 items (head x 16 value columns, state slice
//    prefetched before the barrier), attention is split-KV partials over 2 x 74 items and a
//    combine over 128 (head x 16 dims) items; the conv update rides the in-projection epilogue
//    (each channel has one owner CTA) and the gated RMSNorm the out-projection prologue.
// The LM head streams the tied embedding through the same ring; the CTA maxima meet in a 64-bit
// (value, ~index) atomicMax and CTA 0 writes the token and advances the step counters.
//
// Numerics follow the per-op kernels (BF16 rounding points of the eager path); FP32 summation
// orders differ, which the parity tests bound.
#include <cfloat>
#include <cstddef>
#include <vector>

#include "common.cuh"

using namespace q35;

__device__ int q35_pk_error_word = 0;

namespace {

constexpr int kPkCWarps = 16;
constexpr int kPkCThreads = kPkCWarps * 32;
constexpr int kPkThreads = kPkCThreads + 32;  // + one producer warp
constexpr int kPkStages = 6;
constexpr int kPkKChunk = 2048;                  // k values of one stage row (4 KB of bf16)
constexpr int kPkTileRows = 8;                   // weight rows per stage
constexpr int kPkRowPad = 0;                     // lanes read consecutive 16-byte chunks: no bank padding
constexpr int kPkRowStride = kPkKChunk * 2 + kPkRowPad;
constexpr int kPkStageStride = (kPkTileRows * kPkRowStride + 127) / 128 * 128;
constexpr int kPkGroups = 4;                     // consumer warp groups, one stage each at a time
constexpr int kPkGroupWarps = kPkCWarps / kPkGroups;  // warps splitting a stage's k range
constexpr int kPkMaxK = 6144;
constexpr int kPkSplits = 74;                    // attention splits per KV head
constexpr int kPkMaxRows = 256;                  // cache rows per attention item
constexpr long long kPkWaitBudget = 4000000000LL;  // ~2 s at 1.9 GHz, then report and stop

enum : int { OP_GEMV = 0, OP_DELTA = 1, OP_ATTN_PART = 2, OP_ATTN_COMBINE = 3 };
enum : int { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED = 2, PRO_GATED = 3 };
enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_CONV = 3, EPI_TOP1 = 4 };

struct PkOp {
  int kind, pro, epi, rpu;
  int n_out, k;
  const bf16* weight;   // GEMV: [rpu * n_out, k]
  const bf16* input;    // prologue input [k] (NORM: residual; GATED: DeltaNet output)
  const bf16* norm_w;   // NORM/EMBED: [k]; GATED: [head_dim]
  const bf16* gate;     // GATED: z [k]
  bf16* out;            // STORE/CONV/SWIGLU: output; RESID: residual updated in place
  const bf16* conv_w;   // CONV: [conv_ch, 4]
  bf16* conv_state;     // CONV: [conv_ch, 4]
  bf16* conv_out;       // CONV: post-SiLU conv output [conv_ch]
  int conv_ch;
  // mixers
  const bf16* packed;   // projection output of this layer
  const bf16* a_log;
  const bf16* dt_bias;
  float* rec_state;     // [heads, 128, 128]
  const bf16* q_norm;
  const bf16* k_norm;
  bf16* k_cache;        // [Hkv, max_len, 256]
  bf16* v_cache;
};

struct PkParams {
  const PkOp* ops;
  int n_ops;
  const int64_t* token;  // read at the start, written at the end
  const bf16* embed;
  int vocab;
  bf16* resid;
  const float* inv_freq;
  int64_t* cache_len;
  int64_t* rope_pos;
  int64_t* token_log;
  int64_t* log_pos;
  int log_len;
  int max_len, q_heads, kv_heads, rot, lin_heads;
  float eps, attn_scale;
  bf16* conv_out;
  bf16* delta_out;
  bf16* attn_out;
  float* attn_part;           // [Hkv * kPkSplits * G][256]
  float* attn_ml;             // [Hkv * kPkSplits * G][2]
  unsigned* bar_counter;      // zeroed before each launch
  unsigned long long* top1;   // zero between launches (the finisher re-zeroes it)
  int64_t* trace;             // optional: [n_ops + 1][CTAs][2] globaltimer ns (see q35_decoder_set_trace)
};

struct __align__(16) PkShared {
  uint64_t full[kPkStages];
  uint64_t empty[kPkStages];
  uint32_t issued[kPkStages];  // stage number whose copies the producer last armed in each slot
  float gpart[kPkGroups][2][kPkGroupWarps][kPkTileRows];  // per-warp tile partials, by tile parity
  float red[kPkCWarps * 4];
  int red_i[kPkCWarps];
  int abort;
  union __align__(16) {  // xs is read and written as 16-byte vectors
    bf16 xs[kPkMaxK];
    struct {
      float qhat[128], khat[128], vv[16];
      float part[kPkCWarps][16];
      float gates[2];
    } dl;
    struct {
      float qf[4][256];
      float nrm[5][256];
      float kn[256], vn[256];
      float sc[kPkMaxRows][4];
      float m[4], l[4];
    } at;
    struct {
      float es[kPkSplits];
      float lsum;
    } cb;
  } u;
};

constexpr size_t kPkSmemBytes = (size_t)kPkStages * kPkStageStride + sizeof(PkShared);
static_assert(offsetof(PkShared, u) % 16 == 0 && sizeof(PkShared) % 16 == 0, "vector access alignment");
static_assert(kPkStageStride % 128 == 0, "ring stages keep bulk-copy alignment");
static_assert(kPkSmemBytes <= 227 * 1024, "persistent decode shared memory over budget");

// ------------------------------------------------------------------------------ primitives
Q35_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

Q35_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kPkCThreads) : "memory"); }

// Consumer barrier that also ORs a per-thread flag: every consumer thread gets the same answer,
// so a decision to stop is taken by all of them at the same barrier.
// Named barrier of one consumer warp group (ids 2..), with the same OR-reduction.
Q35_DEV bool gbar_any(int group, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(2 + group), "n"(kPkGroupWarps * 32)
      : "memory");
  return r != 0;
}

Q35_DEV bool cbar_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kPkCThreads)
      : "memory");
  return r != 0;
}

Q35_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kPkWaitBudget) return false;
  }
}

// Consumers take stages out of order (each warp its own tiles), so a warp may ask for stage s
// while its slot still holds stage s - kPkStages: wait until the producer has armed stage s in
// the slot before waiting on the slot's phase parity (which would alias stage s - 2 * kPkStages).
Q35_DEV bool wait_issued(const uint32_t* issued, uint32_t stage) {
  const long long t0 = clock64();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(issued)) : "memory");
    if (v == stage) return true;
    if (clock64() - t0 > kPkWaitBudget) return false;
    __nanosleep(128);  // most waiting warps are several stages early: stay off the issue ports
  }
}

Q35_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

Q35_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

Q35_DEV int64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return (int64_t)t;
}

// Thread 0 records (arrival, release) of grid barrier `j`; row n_ops holds (start, end) of the step.
Q35_DEV void trace_mark(const PkParams& p, int j, int which) {
  if (p.trace && threadIdx.x == 0) p.trace[((int64_t)j * gridDim.x + blockIdx.x) * 2 + which] = globaltimer_ns();
}

Q35_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

Q35_DEV float ldcg_bf(const bf16* p) {
  return __uint_as_float(((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p))) << 16);
}

// All CTAs meet; returns false (and sets the error word) if the wait runs out.
Q35_DEV bool grid_barrier(const PkParams& p, unsigned target, PkShared& S) {
  cbar();
  bool fail = false;
  const int j = (int)(target / gridDim.x) - 1;
  trace_mark(p, j, 0);
  if (threadIdx.x == 0) {
    // release: the CTA's writes (ordered before this thread by the consumer barrier) become
    // visible before the count; acquire on the polled count makes the other CTAs' writes visible
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar_counter) : "memory");
    const long long t0 = clock64();
    while (ld_acquire(p.bar_counter) < target) {
      if (clock64() - t0 > kPkWaitBudget) {
        atomicCAS(&q35_pk_error_word, 0, 1);
        fail = true;
        break;
      }
      __nanosleep(32);
    }
  }
  trace_mark(p, j, 1);
  if (cbar_any(fail)) {
    if (threadIdx.x == 0) *(volatile int*)&S.abort = 1;  // tells the producer to stop issuing
    return false;
  }
  return true;
}

Q35_DEV float cblock_sum(float v, PkShared& S) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) S.red[warp] = v;
  cbar();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kPkCWarps; ++w) t += S.red[w];
  cbar();
  return t;
}

Q35_DEV unsigned long long top1_key(float v, int idx) {
  return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

Q35_DEV void unit_range(int n, int& u0, int& u1) {
  u0 = (int)((int64_t)blockIdx.x * n / gridDim.x);
  u1 = (int)((int64_t)(blockIdx.x + 1) * n / gridDim.x);
}

// A GEMV op's work on one CTA: tiles of 8 weight rows (8 units, or 4 units' gate + up rows for
// SwiGLU) over K, each tile K / 2048 stages (k-chunks) of 8 x 4 KB.
struct TilePlan {
  int u0, u1, upt, ntiles, spt;
};
Q35_DEV TilePlan tile_plan(const PkOp& op) {
  TilePlan t;
  unit_range(op.n_out, t.u0, t.u1);
  t.upt = kPkTileRows / op.rpu;
  t.ntiles = (t.u1 - t.u0 + t.upt - 1) / t.upt;
  t.spt = op.k / kPkKChunk;
  return t;
}

// ------------------------------------------------------------------------------ producer
Q35_DEV void producer(const PkParams& p, PkShared& S, unsigned char* ring) {
  uint32_t st = 0;
  bool stop = false;
  for (int i = 0; i < p.n_ops && !stop && !*(volatile int*)&S.abort; ++i) {
    if (p.ops[i].kind != OP_GEMV) continue;
    // the fields this loop needs, in registers (each copy instruction clobbers memory, which
    // would otherwise reload them from the op table)
    const int n_out = p.ops[i].n_out, k = p.ops[i].k, rpu = p.ops[i].rpu;
    const char* w = reinterpret_cast<const char*>(p.ops[i].weight);
    int u0, u1;
    unit_range(n_out, u0, u1);
    const int upt = kPkTileRows / rpu, spt = k / kPkKChunk;
    const int64_t rb = (int64_t)k * 2;
    for (int ua = u0; ua < u1 && !stop; ua += upt) {
      const int nu = min(upt, u1 - ua);
      const char* gate = w + ua * rb;
      const char* up = w + ((int64_t)n_out + ua) * rb;
      for (int j = 0; j < spt; ++j, ++st) {
        const int slot = st % kPkStages;
        if (!mbar_wait(&S.empty[slot], ((st / kPkStages) & 1) ^ 1)) {
          atomicCAS(&q35_pk_error_word, 0, 2);
          stop = true;  // the consumers time out on the stage this would have filled
          break;
        }
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.full[slot])),
                     "r"((uint32_t)(nu * rpu * kPkKChunk * 2))
                     : "memory");
        asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(&S.issued[slot])), "r"(st) : "memory");
        unsigned char* dst = ring + (size_t)slot * kPkStageStride;
        const int64_t koff = (int64_t)j * kPkKChunk * 2;
        // stage rows: units' (gate) rows 0..nu-1, then for SwiGLU their up rows at upt..upt+nu-1
        for (int r = 0; r < nu; ++r)
          bulk_g2s(dst + r * kPkRowStride, gate + r * rb + koff, kPkKChunk * 2, &S.full[slot]);
        if (rpu == 2)
          for (int r = 0; r < nu; ++r)
            bulk_g2s(dst + (upt + r) * kPkRowStride, up + r * rb + koff, kPkKChunk * 2, &S.full[slot]);
      }
    }
  }
  // copies still in flight (only after an abort) must land before the CTA's memory goes away
  for (uint32_t j = (st > kPkStages ? st - kPkStages : 0); j < st; ++j)
    mbar_wait(&S.full[j % kPkStages], (j / kPkStages) & 1);
}

// ------------------------------------------------------------------------------ GEMV op
Q35_DEV void build_input(const PkParams& p, const PkOp& op, PkShared& S) {
  const int t = threadIdx.x;
  const int nv = op.k >> 3;
  bf16* xs = S.u.xs;
  if (op.pro == PRO_GATED) {  // per 128-wide head: bf16(bf16(bf16(o * rstd) * w) * silu(z))
    const int warp = t >> 5, lane = t & 31;
    for (int h = warp; h < op.k / 128; h += kPkCWarps) {
      float o[4], ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[j] = ldcg_bf(op.input + h * 128 + lane + 32 * j);
        ss += o[j] * o[j];
      }
      ss = warp_sum(ss);
      const float rstd = rsqrt_ieee(ss / 128.0f + p.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        const float nrm = rbf(o[j] * rstd);
        const float wt = rbf(nrm * bf2f(op.norm_w[d]));
        xs[h * 128 + d] = f2bf(wt * silu_f(ldcg_bf(op.gate + h * 128 + d)));
      }
    }
    cbar();
    return;
  }
  const uint4* src;
  if (op.pro == PRO_EMBED) {
    int64_t tok = *p.token;
    tok = tok < 0 ? 0 : (tok >= p.vocab ? p.vocab - 1 : tok);
    src = reinterpret_cast<const uint4*>(p.embed + tok * (int64_t)op.k);
  } else {
    src = reinterpret_cast<const uint4*>(op.input);
  }
  float ss = 0.f;
  for (int i = t; i < nv; i += kPkCThreads) {
    const uint4 v = (op.pro == PRO_EMBED) ? src[i] : __ldcg(src + i);
    if (op.pro == PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid)[i] = v;
    reinterpret_cast<uint4*>(xs)[i] = v;
    if (op.pro != PRO_PLAIN) {
      float f[8];
      unpack_bf16x8(v, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  if (op.pro != PRO_PLAIN) {
    const float var = cblock_sum(ss, S) / (float)op.k;
    const float r = rsqrt_ieee(var + p.eps);
    for (int i = t; i < nv; i += kPkCThreads) {
      float f[8], w[8];
      unpack_bf16x8(reinterpret_cast<const uint4*>(xs)[i], f);
      unpack_bf16x8(reinterpret_cast<const uint4*>(op.norm_w)[i], w);
      __align__(16) bf16 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = f2bf(f[j] * r * (1.0f + w[j]));
      reinterpret_cast<uint4*>(xs)[i] = *reinterpret_cast<const uint4*>(o);
    }
  }
  cbar();
}

Q35_DEV void gemv_epilogue(const PkOp& op, int unit, float y0, float y1, float& best_v, int& best_i) {
  switch (op.epi) {
    case EPI_STORE: op.out[unit] = f2bf(y0); break;
    case EPI_RESID: op.out[unit] = f2bf(ldcg_bf(op.out + unit) + rbf(y0)); break;
    case EPI_SWIGLU: op.out[unit] = f2bf(rbf(silu_f(rbf(y0))) * rbf(y1)); break;
    case EPI_CONV: {
      const bf16 yb = f2bf(y0);
      op.out[unit] = yb;
      if (unit < op.conv_ch) {  // causal conv update of this channel (kernels.py:622-656)
        bf16* st = op.conv_state + (int64_t)unit * 4;
        const float s1 = bf2f(st[1]), s2 = bf2f(st[2]), s3 = bf2f(st[3]);
        const bf16* w = op.conv_w + (int64_t)unit * 4;
        float acc = s1 * bf2f(w[0]);
        acc += s2 * bf2f(w[1]);
        acc += s3 * bf2f(w[2]);
        acc += bf2f(yb) * bf2f(w[3]);
        op.conv_out[unit] = f2bf(silu_f(rbf(acc)));
        st[0] = st[1];
        st[1] = st[2];
        st[2] = st[3];
        st[3] = yb;
      }
      break;
    }
    case EPI_TOP1: {
      const float v = rbf(y0);  // eager materialises BF16 logits (kernels.py:1119-1121)
      if (v > best_v || (v == best_v && unit < best_i)) {
        best_v = v;
        best_i = unit;
      }
      break;
    }
  }
}

// Returns false on abort. `st` is the ring stage counter shared (by construction) with the producer.
// Warp group g (4 warps) takes tiles g, g + 4, ...; warp w of the group covers k values
// [512 w, 512 w + 512) of every stage: lane l dots 16-byte chunks (l and l + 32 of that range) of
// the tile's 8 rows with the matching input-vector chunks, FP32 FMAs on the CUDA cores. Each warp
// releases the stage itself; at the end of the tile the warp reduces its 8 row sums, the group
// meets at its own named barrier, and its first warp adds the four partials in a fixed order and
// applies the epilogue from lanes 0-7.
Q35_DEV bool gemv_op(const PkParams& p, const PkOp& op, PkShared& S, const unsigned char* ring, uint32_t& st,
                     float& best_v, int& best_i) {
  build_input(p, op, S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = warp / kPkGroupWarps, wig = warp % kPkGroupWarps;
  constexpr int kq = kPkKChunk / kPkGroupWarps;  // k values per warp per stage (512)
  const TilePlan tp = tile_plan(op);
  const uint4* xs = reinterpret_cast<const uint4*>(S.u.xs);
  bool fail = false;
  int par = 0;
  for (int t = group; t < tp.ntiles; t += kPkGroups, par ^= 1) {
    if (op.epi == EPI_CONV && wig == 0 && lane == 0) {  // the epilogue's conv lines, ahead of the math
      const int unit0 = tp.u0 + t * kPkTileRows;
      if (unit0 < op.conv_ch) {
        asm volatile("prefetch.global.L1 [%0];" ::"l"(op.conv_state + (int64_t)unit0 * 4));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(op.conv_w + (int64_t)unit0 * 4));
      }
    }
    float acc[kPkTileRows];
#pragma unroll
    for (int r = 0; r < kPkTileRows; ++r) acc[r] = 0.f;
    for (int j = 0; j < tp.spt && !fail; ++j) {
      const uint32_t sj = st + (uint32_t)(t * tp.spt + j);
      const int slot = sj % kPkStages;
      if (!wait_issued(&S.issued[slot], sj) || !mbar_wait(&S.full[slot], (sj / kPkStages) & 1)) {
        atomicCAS(&q35_pk_error_word, 0, 3);
        fail = true;
        break;
      }
      // 16-byte chunk index (within a stage row) of this lane's two chunks
      const int c0 = (wig * kq) / 8 + lane, c1 = c0 + 32;
      const uint4 xa = xs[(j * kPkKChunk) / 8 + c0], xb = xs[(j * kPkKChunk) / 8 + c1];
      const unsigned char* base = ring + (size_t)slot * kPkStageStride;
#pragma unroll
      for (int r = 0; r < kPkTileRows; ++r) {
        const uint4* rowp = reinterpret_cast<const uint4*>(base + r * kPkRowStride);
        acc[r] = dot_bf16x8(rowp[c1], xb, dot_bf16x8(rowp[c0], xa, acc[r]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[slot]);
    }
    // warp sums of the 8 rows (rows past the CTA's units hold stale data and are dropped below)
#pragma unroll
    for (int r = 0; r < kPkTileRows; ++r) acc[r] = warp_sum(acc[r]);
    float* gp = S.gpart[group][par][wig];
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kPkTileRows; ++r) gp[r] = acc[r];
    }
    if (gbar_any(group, fail)) {
      fail = true;
      break;
    }
    if (wig == 0 && lane < kPkTileRows) {  // lane r owns tile row r
      float y = 0.f;
#pragma unroll
      for (int w = 0; w < kPkGroupWarps; ++w) y += S.gpart[group][par][w][lane];
      if (op.rpu == 1) {
        const int unit = tp.u0 + t * kPkTileRows + lane;
        if (unit < tp.u1) gemv_epilogue(op, unit, y, 0.f, best_v, best_i);
      } else if (lane < tp.upt) {  // gate row `lane`, up row `lane + upt`
        float up = 0.f;
#pragma unroll
        for (int w = 0; w < kPkGroupWarps; ++w) up += S.gpart[group][par][w][lane + tp.upt];
        const int unit = tp.u0 + t * tp.upt + lane;
        if (unit < tp.u1) gemv_epilogue(op, unit, y, up, best_v, best_i);
      }
    }
  }
  st += (uint32_t)(tp.ntiles * tp.spt);
  if (cbar_any(fail)) {
    if (threadIdx.x == 0) *(volatile int*)&S.abort = 1;
    return false;
  }
  return true;
}

// ------------------------------------------------------------------------------ DeltaNet step
// Item = (head h, 16 value columns). Thread t: column v = t & 15, key rows 4 * (t >> 4) .. +3.
Q35_DEV void delta_prefetch(const PkParams& p, const PkOp& op, float s[4]) {
  const int item = blockIdx.x;
  if (item >= p.lin_heads * 8) return;
  const int h = item >> 3, v0 = (item & 7) * 16;
  const int t = threadIdx.x, v = t & 15, kg = t >> 4;
  const float* S = op.rec_state + (int64_t)h * 128 * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] = S[(kg * 4 + i) * 128 + v0 + v];
}

Q35_DEV void delta_op(const PkParams& p, const PkOp& op, PkShared& S, float s[4]) {
  const int item = blockIdx.x;
  if (item >= p.lin_heads * 8) return;
  const int H = p.lin_heads;
  const int h = item >> 3, v0 = (item & 7) * 16;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, v = t & 15, kg = t >> 4;
  auto& D = S.u.dl;
  // L2 norms of q_h (warps 0-3) and k_h (warps 4-7) of the post-SiLU conv output
  float val = 0.f;
  if (t < 256) {
    const int ch = (t < 128) ? h * 128 + t : H * 128 + h * 128 + (t - 128);
    val = ldcg_bf(p.conv_out + ch);
    const float ws = warp_sum(val * val);
    if (lane == 0) S.red[warp] = ws;
  } else if (t < 256 + 16) {
    D.vv[t - 256] = ldcg_bf(p.conv_out + 2 * H * 128 + h * 128 + v0 + (t - 256));
  } else if (t == 288) {
    // packed row layout (integration.py:81-93): [q | k | v] (3*H*128) | z (H*128) | a (H) | b (H)
    const float a = ldcg_bf(op.packed + 4 * H * 128 + h) + bf2f(op.dt_bias[h]);
    const float sp = a > 20.0f ? a : log1pf(expf(a));
    D.gates[0] = expf(-expf(bf2f(op.a_log[h])) * sp);
    D.gates[1] = 1.0f / (1.0f + expf(-ldcg_bf(op.packed + 4 * H * 128 + H + h)));
  }
  cbar();
  if (t < 256) {
    const int g0 = (t < 128) ? 0 : 4;
    const float ss = S.red[g0] + S.red[g0 + 1] + S.red[g0 + 2] + S.red[g0 + 3];
    const float inv = rsqrt_ieee(ss + 1e-6f);
    if (t < 128)
      D.qhat[t] = (val * inv) * (1.0f / sqrtf(128.0f));
    else
      D.khat[t - 128] = val * inv;
  }
  cbar();
  const float alpha = D.gates[0], beta = D.gates[1];
  // mem = s^T k over the 128 key rows (4 per thread, 2 key groups per warp, 16 warps)
  float pm = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s[i] *= alpha;
    pm = fmaf(s[i], D.khat[kg * 4 + i], pm);
  }
  pm += __shfl_xor_sync(0xffffffffu, pm, 16);
  if (lane < 16) D.part[warp][lane] = pm;
  cbar();
  float mem = 0.f;
#pragma unroll
  for (int w = 0; w < kPkCWarps; ++w) mem += D.part[w][v];
  cbar();
  const float delta = beta * (D.vv[v] - mem);
  float po = 0.f;
  float* Sg = op.rec_state + (int64_t)h * 128 * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s[i] = fmaf(D.khat[kg * 4 + i], delta, s[i]);
    po = fmaf(s[i], D.qhat[kg * 4 + i], po);
    Sg[(kg * 4 + i) * 128 + v0 + v] = s[i];
  }
  po += __shfl_xor_sync(0xffffffffu, po, 16);
  if (lane < 16) D.part[warp][lane] = po;
  cbar();
  if (t < 16) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kPkCWarps; ++w) o += D.part[w][t];
    p.delta_out[h * 128 + v0 + t] = f2bf(o);  // the recurrent output is materialised in BF16
  }
}

// ------------------------------------------------------------------------------ attention
// Cached K/V rows of this item do not depend on the step: pull them into L2 before the barrier.
Q35_DEV void attn_prefetch(const PkParams& p, const PkOp& op) {
  const int g = blockIdx.x / kPkSplits, s = blockIdx.x % kPkSplits;
  if (g >= p.kv_heads) return;
  const int64_t len = *p.cache_len;
  const int n = (int)(len < 0 ? 0 : (len > p.max_len ? p.max_len : len));
  const int chunk = (n + kPkSplits - 1) / kPkSplits;
  const int r0 = min(s * chunk, n), r1 = min(r0 + chunk, n);
  const int lines = (r1 - r0) * 4;  // 128-byte lines per row of 256 bf16
  for (int i = threadIdx.x; i < 2 * lines; i += kPkCThreads) {
    const bf16* base = (i < lines ? op.k_cache : op.v_cache) + ((int64_t)g * p.max_len + r0) * 256;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (i % lines) * 64));
  }
}

// Item = (KV head g, split s of the cached rows); the last split also attends the current token.
Q35_DEV void attn_part_op(const PkParams& p, const PkOp& op, PkShared& S) {
  constexpr int G = 4, D = 256;
  const int g = blockIdx.x / kPkSplits, s = blockIdx.x % kPkSplits;
  if (g >= p.kv_heads) return;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  auto& A = S.u.at;
  const int Hq = p.q_heads, Hkv = p.kv_heads;
  const int64_t len = *p.cache_len;
  const int n = (int)(len < 0 ? 0 : (len > p.max_len ? p.max_len : len));
  const int chunk = (n + kPkSplits - 1) / kPkSplits;
  const int r0 = min(s * chunk, n), r1 = min(r0 + chunk, n);
  const bool last = (s == kPkSplits - 1);
  const int nr = r1 - r0 + (last ? 1 : 0);
  // Q/K RMSNorm(1+w) and partial RoPE of the current token (threads 0-255: one dim each)
  const int d = t & 255;
  float x[G + 1], v_raw = 0.f, c = 1.f, sn = 0.f;
  if (t < 256) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) x[hh] = ldcg_bf(op.packed + (g * G + hh) * 2 * D + d);
    x[G] = ldcg_bf(op.packed + 2 * Hq * D + g * D + d);
    v_raw = ldcg_bf(op.packed + 2 * Hq * D + Hkv * D + g * D + d);
#pragma unroll
    for (int i = 0; i <= G; ++i) {
      const float ws = warp_sum(x[i] * x[i]);
      if (lane == 0) S.red[warp * (G + 1) + i] = ws;
    }
    if (d < p.rot) rope_cs(d, p.rot / 2, (float)(*p.rope_pos), p.inv_freq, c, sn);
  }
  cbar();
  if (t < 256) {
    const float wq = bf2f(op.q_norm[d]), wk = bf2f(op.k_norm[d]);
#pragma unroll
    for (int i = 0; i <= G; ++i) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += S.red[w * (G + 1) + i];
      const float r = rsqrt_ieee(tot / (float)D + p.eps);
      A.nrm[i][d] = rbf(x[i] * r * (1.0f + (i < G ? wq : wk)));
    }
  }
  cbar();
  if (t < 256) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) A.qf[hh][d] = rope_apply(A.nrm[hh], d, p.rot, c, sn) * p.attn_scale;
    const float kr = rope_apply(A.nrm[G], d, p.rot, c, sn);
    A.kn[d] = kr;
    A.vn[d] = v_raw;
    if (s == 0 && len >= 0 && len < p.max_len) {
      const int64_t base = ((int64_t)g * p.max_len + len) * D;
      op.k_cache[base + d] = f2bf(kr);
      op.v_cache[base + d] = f2bf(v_raw);
    }
  }
  cbar();
  // pass 1: scores (warp per row)
  const bf16* Kb = op.k_cache + (int64_t)g * p.max_len * D;
  const bf16* Vb = op.v_cache + (int64_t)g * p.max_len * D;
  for (int j = warp; j < nr; j += kPkCWarps) {
    float kf[8];
    if (r0 + j < r1) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(Kb + (int64_t)(r0 + j) * D + lane * 8), kf);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) kf[e] = A.kn[lane * 8 + e];
    }
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) a = fmaf(A.qf[hh][lane * 8 + e], kf[e], a);
      a = warp_sum(a);
      if (lane == 0) A.sc[j][hh] = a;
    }
  }
  cbar();
  // pass 2: per-head max and weights
  if (warp < G) {
    float m = -FLT_MAX;
    for (int j = lane; j < nr; j += 32) m = fmaxf(m, A.sc[j][warp]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < nr; j += 32) {
      const float e = expf(A.sc[j][warp] - m);
      A.sc[j][warp] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      A.m[warp] = m;
      A.l[warp] = l;
    }
  }
  cbar();
  // pass 3: un-normalised output, thread = (head, two dims)
  {
    const int hh = t >> 7, dp = (t & 127) * 2;
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < nr; ++j) {
      const float w = A.sc[j][hh];
      float v0, v1;
      if (r0 + j < r1) {
        const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(Vb + (int64_t)(r0 + j) * D + dp);
        v0 = __low2float(vv);
        v1 = __high2float(vv);
      } else {
        v0 = A.vn[dp];
        v1 = A.vn[dp + 1];
      }
      a0 = fmaf(w, v0, a0);
      a1 = fmaf(w, v1, a1);
    }
    const int slot = (g * kPkSplits + s) * G + hh;
    p.attn_part[(int64_t)slot * D + dp] = a0;
    p.attn_part[(int64_t)slot * D + dp + 1] = a1;
    if ((t & 127) == 0) {
      p.attn_ml[2 * slot] = nr > 0 ? A.m[hh] : -FLT_MAX;
      p.attn_ml[2 * slot + 1] = nr > 0 ? A.l[hh] : 0.f;
    }
  }
}

// Item = (query head, 16 dims): merge the splits, normalise, round, times BF16(sigmoid(gate)).
Q35_DEV void attn_combine_op(const PkParams& p, const PkOp& op, PkShared& S) {
  constexpr int G = 4, D = 256;
  const int h = blockIdx.x >> 4, d0 = (blockIdx.x & 15) * 16;
  if (h >= p.q_heads) return;
  const int g = h / G, hh = h % G;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  auto& C = S.u.cb;
  const int base = g * kPkSplits * G + hh;  // slot of split j: base + j * G
  if (warp == 0) {
    float M = -FLT_MAX;
    for (int j = lane; j < kPkSplits; j += 32) {
      const float l = __ldcg(p.attn_ml + 2 * (base + j * G) + 1);
      if (l > 0.f) M = fmaxf(M, __ldcg(p.attn_ml + 2 * (base + j * G)));
    }
    M = warp_max(M);
    float L = 0.f;
    for (int j = lane; j < kPkSplits; j += 32) {
      const float l = __ldcg(p.attn_ml + 2 * (base + j * G) + 1);
      const float e = l > 0.f ? expf(__ldcg(p.attn_ml + 2 * (base + j * G)) - M) : 0.f;
      C.es[j] = e;
      L += l * e;
    }
    L = warp_sum(L);
    if (lane == 0) C.lsum = L;
  }
  cbar();
  const int dd = d0 + warp;  // 16 warps x 16 dims
  float a = 0.f;
  for (int j = lane; j < kPkSplits; j += 32) a += C.es[j] * __ldcg(p.attn_part + (int64_t)(base + j * G) * D + dd);
  a = warp_sum(a);
  if (lane == 0) {
    const float o = C.lsum > 0.f ? rbf(a / C.lsum) : 0.f;
    const float gate = ldcg_bf(op.packed + h * 2 * D + D + dd);
    p.attn_out[h * D + dd] = f2bf(o * rbf(sigmoid_f(gate)));
  }
}

// ------------------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kPkThreads, 1) pk_decode_kernel(const __grid_constant__ PkParams p) {
  extern __shared__ __align__(128) unsigned char pk_smem[];
  unsigned char* ring = pk_smem;
  PkShared& S = *reinterpret_cast<PkShared*>(pk_smem + (size_t)kPkStages * kPkStageStride);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPkStages; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&S.empty[i])), "n"(kPkGroupWarps)
                   : "memory");
      S.issued[i] = 0xFFFFFFFFu;
    }
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();  // the only full-CTA barrier: the producer warp leaves the consumers' barriers after this
  if (warp == kPkCWarps) {
    if (lane == 0) producer(p, S, ring);
    return;
  }

  trace_mark(p, p.n_ops, 0);
  uint32_t st = 0;
  unsigned target = 0;
  float best_v = -FLT_MAX;
  int best_i = 0x7fffffff;
  float dstate[4] = {0.f, 0.f, 0.f, 0.f};
  bool ok = true;
  for (int i = 0; i < p.n_ops && ok; ++i) {
    const PkOp& op = p.ops[i];
    if (op.kind == OP_DELTA) delta_prefetch(p, op, dstate);  // independent of the ops before it
    if (op.kind == OP_ATTN_PART) attn_prefetch(p, op);
    if (op.kind == OP_GEMV && op.norm_w && op.pro != PRO_PLAIN)  // constants: warm L2 before the barrier
      for (int q = threadIdx.x; q < (op.pro == PRO_GATED ? 2 : op.k / 64); q += kPkCThreads)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(op.norm_w + 64 * q));
    if (i > 0) {
      target += gridDim.x;
      ok = grid_barrier(p, target, S);
      if (!ok) break;
    }
    switch (op.kind) {
      case OP_GEMV: ok = gemv_op(p, op, S, ring, st, best_v, best_i); break;
      case OP_DELTA: delta_op(p, op, S, dstate); break;
      case OP_ATTN_PART: attn_part_op(p, op, S); break;
      case OP_ATTN_COMBINE: attn_combine_op(p, op, S); break;
    }
  }
  if (!ok) return;
  // greedy top-1 across the CTA, then across CTAs
  {
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best_v || (ov == best_v && oi < best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      S.red[warp] = best_v;
      S.red_i[warp] = best_i;
    }
    cbar();
    if (threadIdx.x == 0) {
      float bv = S.red[0];
      int bi = S.red_i[0];
      for (int w = 1; w < kPkCWarps; ++w)
        if (S.red[w] > bv || (S.red[w] == bv && S.red_i[w] < bi)) {
          bv = S.red[w];
          bi = S.red_i[w];
        }
      if (bi != 0x7fffffff) atomicMax(p.top1, top1_key(bv, bi));
    }
  }
  target += gridDim.x;
  if (!grid_barrier(p, target, S)) return;
  trace_mark(p, p.n_ops, 1);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long key = atomicExch(p.top1, 0ull);
    const int64_t tok = (key == 0ull) ? 0 : (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
    *const_cast<int64_t*>(p.token) = tok;
    *p.cache_len += 1;
    *p.rope_pos += 1;
    if (p.token_log && p.log_pos && p.log_len > 0) {
      const int64_t pos = *p.log_pos;
      p.token_log[pos % p.log_len] = tok;
      *p.log_pos = pos + 1;
    }
  }
}

}  // namespace

// ------------------------------------------------------------------------------ host side
struct q35_pk_plan {
  PkParams params;
};

namespace {
size_t pk_round(size_t b) { return (b + 255) & ~(size_t)255; }
int pk_max_ops(const q35_decoder_desc& d) { return d.n_layers * 6 + 1; }
}  // namespace

size_t q35_pk_workspace_bytes(const q35_decoder_desc& d) {
  const int G = d.kv_heads ? d.q_heads / d.kv_heads : 1;
  const size_t slots = (size_t)d.kv_heads * kPkSplits * G;
  return pk_round((size_t)pk_max_ops(d) * sizeof(PkOp)) + pk_round(slots * 256 * 4) + pk_round(slots * 2 * 4) +
         pk_round((size_t)d.lin_heads * 3 * 128 * 2) + pk_round((size_t)d.lin_heads * 128 * 2) +
         pk_round((size_t)d.q_heads * 256 * 2) + pk_round(16) + pk_round(16);
}

// Empty when the model fits the persistent kernel's built-in shapes, else the reason.
const char* q35_pk_unsupported(const q35_decoder_desc& d) {
  if (d.a8w8) return "A8W8 weights use the per-op decode path";
  if (d.batch > 1) return "batched decoding uses the per-op decode path";
  if (d.hidden != 2048 || d.intermediate != 6144) return "built for hidden 2048 / intermediate 6144";
  if (d.head_dim != 256 || d.q_heads != 8 || d.kv_heads != 2 || d.rotary_dim > 256)
    return "built for 8 query / 2 KV heads of 256";
  if (d.lin_heads != 16 || d.lin_dk != 128 || d.lin_dv != 128 || d.conv_kernel != 4)
    return "built for 16 DeltaNet heads of 128 and conv kernel 4";
  if (d.delta_rows < 4 * 16 * 128 + 32) return "DeltaNet projection rows too few";
  if (d.max_len > kPkSplits * (kPkMaxRows - 1)) return "cache longer than the persistent attention splits cover";
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms < kNumSMs)
    return "needs 148 SMs";
  return "";
}

int q35_pk_create(const q35_decoder_desc& d, const q35_layer_desc* layers, bf16* resid, bf16* proj, bf16* act,
                  void* ws, q35_pk_plan** out) {
  const char* why = q35_pk_unsupported(d);
  if (why[0]) return q35_fail(Q35_ENOTSUP, "persistent decode: %s", why);
  char* base = static_cast<char*>(ws);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* q = base + off;
    off += pk_round(bytes);
    return q;
  };
  const int G = d.q_heads / d.kv_heads;
  const size_t slots = (size_t)d.kv_heads * kPkSplits * G;
  PkOp* dev_ops = reinterpret_cast<PkOp*>(take((size_t)pk_max_ops(d) * sizeof(PkOp)));
  PkParams P = {};
  P.attn_part = reinterpret_cast<float*>(take(slots * 256 * 4));
  P.attn_ml = reinterpret_cast<float*>(take(slots * 2 * 4));
  P.conv_out = reinterpret_cast<bf16*>(take((size_t)d.lin_heads * 3 * 128 * 2));
  P.delta_out = reinterpret_cast<bf16*>(take((size_t)d.lin_heads * 128 * 2));
  P.attn_out = reinterpret_cast<bf16*>(take((size_t)d.q_heads * 256 * 2));
  P.bar_counter = reinterpret_cast<unsigned*>(take(16));
  P.top1 = reinterpret_cast<unsigned long long*>(take(16));

  const int H = d.lin_heads;
  const int qgkv_rows = 2 * d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim;
  std::vector<PkOp> ops;
  auto gemv = [](int pro, int epi, int rpu, int n_out, int k, const void* w, const void* in, const void* nw,
                 void* o) {
    PkOp op = {};
    op.kind = OP_GEMV;
    op.pro = pro;
    op.epi = epi;
    op.rpu = rpu;
    op.n_out = n_out;
    op.k = k;
    op.weight = static_cast<const bf16*>(w);
    op.input = static_cast<const bf16*>(in);
    op.norm_w = static_cast<const bf16*>(nw);
    op.out = static_cast<bf16*>(o);
    return op;
  };
  for (int i = 0; i < d.n_layers; ++i) {
    const q35_layer_desc& L = layers[i];
    const bool delta = L.kind == 0;
    PkOp in = gemv(i == 0 ? PRO_EMBED : PRO_NORM, delta ? EPI_CONV : EPI_STORE, 1, delta ? d.delta_rows : qgkv_rows,
                   d.hidden, L.mix_in, resid, L.in_ln, proj);
    if (delta) {
      in.conv_w = static_cast<const bf16*>(L.conv_w);
      in.conv_state = static_cast<bf16*>(L.conv_state);
      in.conv_out = P.conv_out;
      in.conv_ch = 3 * H * 128;
    }
    ops.push_back(in);
    if (delta) {
      PkOp m = {};
      m.kind = OP_DELTA;
      m.packed = proj;
      m.a_log = static_cast<const bf16*>(L.a_log);
      m.dt_bias = static_cast<const bf16*>(L.dt_bias);
      m.rec_state = L.rec_state;
      ops.push_back(m);
      PkOp o = gemv(PRO_GATED, EPI_RESID, 1, d.hidden, H * 128, L.mix_out, P.delta_out, L.gnorm, resid);
      o.gate = proj + 3 * H * 128;
      ops.push_back(o);
    } else {
      PkOp m = {};
      m.kind = OP_ATTN_PART;
      m.packed = proj;
      m.q_norm = static_cast<const bf16*>(L.q_norm);
      m.k_norm = static_cast<const bf16*>(L.k_norm);
      m.k_cache = static_cast<bf16*>(L.k_cache);
      m.v_cache = static_cast<bf16*>(L.v_cache);
      ops.push_back(m);
      m.kind = OP_ATTN_COMBINE;
      ops.push_back(m);
      ops.push_back(gemv(PRO_PLAIN, EPI_RESID, 1, d.hidden, d.q_heads * d.head_dim, L.mix_out, P.attn_out, nullptr,
                         resid));
    }
    ops.push_back(gemv(PRO_NORM, EPI_SWIGLU, 2, d.intermediate, d.hidden, L.gate_up, resid, L.post_ln, act));
    ops.push_back(gemv(PRO_PLAIN, EPI_RESID, 1, d.hidden, d.intermediate, L.down, act, nullptr, resid));
  }
  ops.push_back(gemv(PRO_NORM, EPI_TOP1, 1, d.vocab, d.hidden, d.embed, resid, d.final_norm, nullptr));
  if ((int)ops.size() > pk_max_ops(d)) return q35_fail(Q35_ENOTSUP, "persistent decode: op table overflow");
  // every pointer the kernel reads or writes as 16-byte vectors
  bool aligned = Q35_ALIGNED(resid, 16) && Q35_ALIGNED(d.embed, 16) && Q35_ALIGNED(d.final_norm, 16);
  for (const PkOp& op : ops) {
    if (op.kind != OP_GEMV) continue;
    aligned = aligned && Q35_ALIGNED(op.input, 16) && (!op.norm_w || op.pro == PRO_GATED || Q35_ALIGNED(op.norm_w, 16));
  }
  for (int i = 0; i < d.n_layers; ++i)
    if (layers[i].kind != 0) aligned = aligned && Q35_ALIGNED(layers[i].k_cache, 16) && Q35_ALIGNED(layers[i].v_cache, 16);
  if (!aligned) return q35_fail(Q35_ENOTSUP, "persistent decode: a buffer is not 16-byte aligned");
  for (const PkOp& op : ops)
    if (op.kind == OP_GEMV && (!op.weight || op.k % kPkKChunk != 0 || op.k > kPkMaxK || op.n_out < kNumSMs ||
                               !Q35_ALIGNED(op.weight, 16)))
      return q35_fail(Q35_ENOTSUP, "persistent decode: GEMV shape n=%d k=%d unsupported", op.n_out, op.k);
  if (cudaMemcpy(dev_ops, ops.data(), ops.size() * sizeof(PkOp), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(P.top1, 0, 16) != cudaSuccess)
    return q35_fail(Q35_ECUDA, "persistent decode: op table upload failed");

  P.ops = dev_ops;
  P.n_ops = (int)ops.size();
  P.token = d.token;
  P.embed = static_cast<const bf16*>(d.embed);
  P.vocab = (int)d.vocab;
  P.resid = resid;
  P.inv_freq = d.inv_freq;
  P.cache_len = d.cache_len;
  P.rope_pos = d.rope_pos;
  P.token_log = d.token_log;
  P.log_pos = d.log_pos;
  P.log_len = d.log_len;
  P.max_len = d.max_len;
  P.q_heads = d.q_heads;
  P.kv_heads = d.kv_heads;
  P.rot = d.rotary_dim;
  P.lin_heads = H;
  P.eps = d.eps;
  P.attn_scale = 1.0f / sqrtf((float)d.head_dim);
  if (cudaFuncSetAttribute(pk_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPkSmemBytes) !=
      cudaSuccess)
    return q35_fail(Q35_ECUDA, "persistent decode: shared memory attribute refused");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pk_decode_kernel, kPkThreads, kPkSmemBytes) !=
          cudaSuccess ||
      per_sm < 1)
    return q35_fail(Q35_ENOTSUP, "persistent decode: one CTA per SM does not fit");
  q35_pk_plan* plan = new q35_pk_plan();
  plan->params = P;
  *out = plan;
  return Q35_OK;
}

void q35_pk_destroy(q35_pk_plan* plan) { delete plan; }

int q35_pk_launch(const q35_pk_plan* plan, cudaStream_t s) {
  if (cudaMemsetAsync(plan->params.bar_counter, 0, sizeof(unsigned), s) != cudaSuccess)
    return q35_fail(Q35_ECUDA, "persistent decode: barrier reset failed");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kNumSMs);
  cfg.blockDim = dim3(kPkThreads);
  cfg.dynamicSmemBytes = kPkSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident, or the launch fails
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, pk_decode_kernel, plan->params);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "persistent decode launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

int q35_pk_set_trace(q35_pk_plan* plan, int64_t* trace, int64_t entries) {
  const int64_t need = ((int64_t)plan->params.n_ops + 1) * kNumSMs * 2;
  Q35_REQUIRE(!trace || entries >= need, "trace buffer needs %lld entries", (long long)need);
  plan->params.trace = trace;
  return Q35_OK;
}

int q35_pk_ops(const q35_pk_plan* plan) { return plan->params.n_ops; }

extern "C" int q35_decoder_persistent_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_pk_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_pk_error_word, &zero, sizeof(int));
  return v;
}
