// Causal GQA prefill attention on tcgen05 (the decoder's prefill path; reference: the SDPA call
// that integration.py:360-372 makes for the full-attention layers, causal, 8 query / 2 KV heads,
// head dim 256).
//
// One CTA per (batch, KV head, 32-query block): the 4 query heads of the KV head are stacked into
// the 128 rows of one MMA tile (row r = head 4 g + r / 32, query q0 + r % 32), so every K / V
// tile in shared memory serves all four. Keys stream in tiles of 64:
//   S = Q K^T            M = 128, N = 64, K = 256  (bf16 operands, FP32 accumulator in TMEM,
//                                                   two S buffers: tile t + 1's product runs
//                                                   while tile t's softmax does)
//   softmax              threads r and r + 128 own row r, 32 keys each (the row maximum is
//                        exchanged through shared memory): scale, causal mask, FP32 sums (log2 units, ex2),
//                        P = exp2(x - m) against a reference maximum m that moves only when a
//                        score exceeds it by more than 8 (so P <= 256 and O needs rescaling
//                        rarely; O / l is the same quotient for any reference)
//   O += P V             M = 128, N = 256, K = 64 with P split into a bf16 high part and a bf16
//                        remainder (two MMAs), which keeps the probabilities to ~16 bits, as the
//                        warp-MMA kernel does; O lives in TMEM and is rescaled in place (TMEM
//                        load / store of the row) when a warp's reference maximum moved
// V is read transposed (V^T [dim][key], written by the Q/K-norm + RoPE kernel next to the cache
// rows) so that both MMA operands are K-major with the 128-byte swizzle. Operands arrive by
// cp.async: Q once, K and V^T double-buffered a tile ahead. Warps 0-7 load and run the softmax; a
// ninth warp only issues the MMAs (an issuing thread stalls about as long as its MMAs run, which
// would hold back its own softmax row), handed off through two mbarriers the 256 softmax threads
// arrive on (operands ready for S, for P.V). Every wait is bounded; a timeout sets
// q35_attn_tc_error_word.
#include <cfloat>

#include "common.cuh"
#include "tcgen05.cuh"

using namespace q35;

__device__ int q35_attn_tc_error_word = 0;

namespace {

constexpr int kAD = 256;         // head dim
constexpr int kAG = 4;           // query heads stacked per KV head
constexpr int kAQ = 32;          // queries per head in a tile
constexpr int kAM = kAG * kAQ;   // 128 MMA rows
constexpr int kAK = 64;          // keys per tile
constexpr int kASoft = 256;      // softmax threads: two per row r = tid % 128 (TMEM lane r), key / O column halves
constexpr int kAThreads = kASoft + 32;  // + the MMA warp
constexpr uint32_t kQBytes = 4 * kAM * 128;  // Q: 4 slabs (64 dims) x 128 rows x 128 B
constexpr uint32_t kKBytes = 4 * kAK * 128;  // K tile: 4 slabs x 64 keys x 128 B
constexpr uint32_t kVBytes = kAD * 128;      // V^T tile: 256 dim rows x 64 keys (128 B)
constexpr uint32_t kPBytes = kAM * 128;      // P part: 128 rows x 64 keys (128 B)
constexpr uint32_t kOffK = kQBytes, kOffV = kOffK + 2 * kKBytes, kOffP = kOffV + 2 * kVBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
constexpr size_t kAttnTcSmem = kOffBar + 64 + 1024;  // barriers + TMEM slot, 1024-byte alignment slack
static_assert(kAttnTcSmem + 2 * kAM * sizeof(float) <= 232448, "dynamic + static shared memory of one CTA");
constexpr uint32_t kTmemCols = 512;                 // S buffers at columns 0 / 64, O at 256
constexpr uint32_t kColO = 256;
constexpr long long kAttnWaitBudget = 2000000000LL;

struct AttnTcParams {
  const bf16* q;   // [B, Hq, L, 256]
  const bf16* k;   // [B, Hkv, kv_len, 256]
  const bf16* vt;  // [B, Hkv, 256, vt_stride]: V transposed; columns L .. vt_stride - 1 finite
  bf16* out;       // [B, L, Hq, 256]
  int Hq, Hkv, L, kv_len, vt_stride;
  float scale_log2;  // softmax scale x log2(e)
};

Q35_DEV void cp16z(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
Q35_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
Q35_DEV uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(kAThreads, 1) prefill_attn_tc_kernel(AttnTcParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char attn_smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)attn_smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sQ = tc::smem_u32(sm), sK = sQ + kOffK, sV = sQ + kOffV, sP = sQ + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);  // S[0], S[1], PV, ready-S, ready-PV
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  const int qb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = qb * kAQ;
  const int L = p.L;
  const int nkeys = min(q0 + kAQ, L);  // keys any row of the block may see (causal)
  const int nt = (nkeys + kAK - 1) / kAK;
  const bf16* kbase = p.k + ((int64_t)b * p.Hkv + g) * p.kv_len * kAD;
  const bf16* vbase = p.vt + ((int64_t)b * p.Hkv + g) * kAD * p.vt_stride;

  const bool mma_warp = warp == kASoft / 32;
  if (mma_warp) tc::tmem_alloc(tmem_slot, kTmemCols);
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 3; ++i) tc::mbar_init(tc::smem_u32(&bars[i]), 1);
    tc::mbar_init(tc::smem_u32(&bars[3]), kASoft);
    tc::mbar_init(tc::smem_u32(&bars[4]), kASoft);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // ---- operand loads (every thread): 16-byte chunks into their 128-byte-swizzled positions
  auto load_q = [&]() {  // 128 rows x 32 chunks
    for (int i = tid; i < kAM * (kAD / 8); i += kASoft) {
      const int r = i >> 5, c = i & 31;
      const int qi = q0 + (r & (kAQ - 1)), hh = g * kAG + (r >> 5);
      const bool ok = qi < L;
      const bf16* src = p.q + (((int64_t)b * p.Hq + hh) * L + (ok ? qi : 0)) * kAD + c * 8;
      cp16z(sQ + (c >> 3) * (kAM * 128) + tc::sw128_offset(r, c & 7), src, ok);
    }
  };
  auto load_k = [&](int t, int buf) {  // 64 keys x 32 chunks
    for (int i = tid; i < kAK * (kAD / 8); i += kASoft) {
      const int r = i >> 5, c = i & 31, key = t * kAK + r;
      const bool ok = key < p.kv_len;
      const bf16* src = kbase + (int64_t)(ok ? key : 0) * kAD + c * 8;
      cp16z(sK + buf * kKBytes + (c >> 3) * (kAK * 128) + tc::sw128_offset(r, c & 7), src, ok);
    }
  };
  auto load_v = [&](int t, int buf) {  // 256 dim rows x 8 chunks of 8 keys
    for (int i = tid; i < kAD * (kAK / 8); i += kASoft) {
      const int d = i >> 3, c = i & 7, key = t * kAK + c * 8;
      const bool ok = key + 8 <= p.vt_stride;
      const bf16* src = vbase + (int64_t)d * p.vt_stride + (ok ? key : 0);
      cp16z(sV + buf * kVBytes + tc::sw128_offset(d, c), src, ok);
    }
  };
  auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };

  const uint32_t idesc_s = tc::idesc_f32acc(1, kAM, kAK);  // bf16 x bf16 -> FP32, M 128, N 64
  const uint32_t idesc_o = tc::idesc_f32acc(1, kAM, kAD);  // M 128, N 256
  auto issue_s = [&](uint32_t tmem, int t) {  // S[t & 1] = Q K_t^T
    const uint32_t d = tmem + (uint32_t)((t & 1) * kAK);
    const uint32_t kb = sK + (t & 1) * kKBytes;
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc::mma_bf16(d, tc::desc_sw128(sQ + s * (kAM * 128) + kk * 32), tc::desc_sw128(kb + s * (kAK * 128) + kk * 32),
                     idesc_s, (s | kk) ? 1u : 0u);
    tc::commit(tc::smem_u32(&bars[t & 1]));
  };
  auto issue_pv = [&](uint32_t tmem, int t) {  // O += P_hi V_t + P_lo V_t
    const uint32_t vb = sV + (t & 1) * kVBytes;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int part = 0; part < 2; ++part)
        tc::mma_bf16(tmem + kColO, tc::desc_sw128(sP + part * kPBytes + kk * 32), tc::desc_sw128(vb + kk * 32), idesc_o,
                     (t > 0 || kk > 0 || part > 0) ? 1u : 0u);
    tc::commit(tc::smem_u32(&bars[2]));
  };
  bool ok = true;
  auto wait_bar = [&](int i, uint32_t parity) {
    if (ok && !tc::mbar_wait_bounded(tc::smem_u32(&bars[i]), parity, kAttnWaitBudget)) {
      ok = false;
      atomicCAS(&q35_attn_tc_error_word, 0, 1);
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  };

  __syncthreads();  // barriers initialised, TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // arrive (release) once this thread's operand writes are complete and its TMEM accesses done
  auto ready = [&](int i) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&bars[i])) : "memory");
  };

  if (mma_warp) {
    // ---- MMA issue: S_0, then per tile S_{t+1} (operands ready) and P.V_t (P and V_t ready)
    if ((tid & 31) == 0) {
      wait_bar(3, 0);
      issue_s(tmem, 0);
      for (int t = 0; t < nt; ++t) {
        if (t + 1 < nt) {
          wait_bar(3, (uint32_t)(t + 1) & 1u);
          issue_s(tmem, t + 1);
        }
        wait_bar(4, (uint32_t)t & 1u);
        issue_pv(tmem, t);
      }
    }
    __syncwarp();
  } else {
  // prologue: {Q, K_0}, {K_1}, {V_0}
  load_q();
  load_k(0, 0);
  commit();
  if (nt > 1) load_k(1, 1);
  commit();
  load_v(0, 0);
  commit();
  asm volatile("cp.async.wait_group 2;" ::: "memory");
  ready(3);  // S_0's operands
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter

  const int row = tid & (kAM - 1), half = tid >> 7;  // row r = head 4 g + r / 32, query q0 + r % 32
  const int qi = q0 + (row & (kAQ - 1));
  // per-tile row maxima, then (after the last tile) the row sums of the two halves; only the two
  // threads of a row touch its entries
  __shared__ float xmax[2][kAM];
  float(&xsum)[2][kAM] = xmax;
  // warps w and w + 4 hold the two halves of the same 32 rows
  auto pair_sync = [&] { asm volatile("bar.sync %0, 64;" ::"r"(1 + (warp & 3)) : "memory"); };
  float m_run = -INFINITY, l_run = 0.f;
  for (int t = 0; t < nt; ++t) {
    // (a) S_t -> registers (frees its TMEM buffer for S_{t+2})
    wait_bar(t & 1, (uint32_t)(t >> 1) & 1u);
    uint32_t sv[32];
    tc::tmem_ld32_async(trow + (uint32_t)((t & 1) * kAK + half * 32), sv);
    tc::tmem_wait_ld();
    // (b) K_{t+1} present (pending: V_t's group): S_{t+1} may run during this tile's softmax
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    ready(3);
    // (c) K_{t+2} into the buffer S_t has finished reading
    if (t + 2 < nt) load_k(t + 2, t & 1);
    commit();
    // (d) softmax of this row over the tile's 64 keys: this thread's 32, the partner's maximum
    const int k0 = t * kAK + half * 32;
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int key = k0 + j;
      x[j] = (key <= qi && key < L) ? __uint_as_float(sv[j]) * p.scale_log2 : -INFINITY;
    }
    float mx[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) mx[j] = fmaxf(x[j], x[j + 16]);
#pragma unroll
    for (int w = 8; w > 0; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) mx[j] = fmaxf(mx[j], mx[j + w]);
    xmax[half][row] = mx[0];
    pair_sync();
    const float mt = fmaxf(mx[0], xmax[half ^ 1][row]);
    pair_sync();  // both halves have read before either writes the next tile's maximum
    // the reference maximum moves only past a margin of 8 (and on the first finite score); both
    // threads of the row take the same decision
    const float m_new = (mt > m_run + 8.f) ? mt : m_run;
    const float alpha = (m_new == m_run) ? 1.f : ex2(m_run - m_new);
    uint32_t ph[16], pl[16];
    float ps[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float p0 = (x[j] == -INFINITY) ? 0.f : ex2(x[j] - m_new);
      const float p1 = (x[j + 1] == -INFINITY) ? 0.f : ex2(x[j + 1] - m_new);
      ps[j / 2] = p0 + p1;
      const uint32_t hi = pack_bf16(p0, p1);
      ph[j / 2] = hi;
      pl[j / 2] = pack_bf16(p0 - __uint_as_float(hi << 16), p1 - __uint_as_float(hi & 0xffff0000u));
    }
#pragma unroll
    for (int w = 8; w > 0; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) ps[j] += ps[j + w];
    l_run = l_run * alpha + ps[0];  // this thread's half of the row sum
    m_run = m_new;
    // (e) PV_{t-1} done: O is stable, P and V_{t-1}'s buffer are free
    if (t > 0) wait_bar(2, (uint32_t)(t - 1) & 1u);
    // (f) V_{t+1} into the freed buffer
    if (t + 1 < nt) load_v(t + 1, (t + 1) & 1);
    commit();
    // (g) rescale O rows whose maximum moved (whole warps: TMEM access is warp-collective)
    if (t > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
      for (int c = half * (kAD / 2); c < (half + 1) * (kAD / 2); c += 64) {
        uint32_t o[2][32];
        tc::tmem_ld32_async(trow + kColO + c, o[0]);
        tc::tmem_ld32_async(trow + kColO + c + 32, o[1]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 32; ++j) o[h][j] = __float_as_uint(__uint_as_float(o[h][j]) * alpha);
        tc::tmem_st32(trow + kColO + c, o[0]);
        tc::tmem_st32(trow + kColO + c + 32, o[1]);
      }
      tc::tmem_wait_st();
    }
    // (h) P high / low parts: row `row`, this thread's 4 chunks of 8 keys
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t off = tc::sw128_offset(row, half * 4 + c);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sP + off), "r"(ph[4 * c]), "r"(ph[4 * c + 1]),
                   "r"(ph[4 * c + 2]), "r"(ph[4 * c + 3])
                   : "memory");
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sP + kPBytes + off), "r"(pl[4 * c]),
                   "r"(pl[4 * c + 1]), "r"(pl[4 * c + 2]), "r"(pl[4 * c + 3])
                   : "memory");
    }
    // (i) V_t present (pending: K_{t+2}, V_{t+1}): P.V_t may run
    asm volatile("cp.async.wait_group 2;" ::: "memory");
    ready(4);
  }
  // ---- epilogue: O / l for rows of real queries
  if (nt > 0) wait_bar(2, (uint32_t)(nt - 1) & 1u);
  xsum[half][row] = l_run;
  pair_sync();
  const float l_row = half ? xsum[0][row] + l_run : l_run + xsum[1][row];  // same order in both threads
  const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
  const int hh = g * kAG + (row >> 5);
#pragma unroll 1
  for (int c = half * (kAD / 2); c < (half + 1) * (kAD / 2); c += 32) {
    uint32_t o[32];
    tc::tmem_ld32(trow + kColO + c, o);
    if (ok && qi < L) {
      bf16* dst = p.out + (((int64_t)b * L + qi) * p.Hq + hh) * kAD + c;
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 v;
        v.x = pack_bf16(__uint_as_float(o[j]) * inv, __uint_as_float(o[j + 1]) * inv);
        v.y = pack_bf16(__uint_as_float(o[j + 2]) * inv, __uint_as_float(o[j + 3]) * inv);
        v.z = pack_bf16(__uint_as_float(o[j + 4]) * inv, __uint_as_float(o[j + 5]) * inv);
        v.w = pack_bf16(__uint_as_float(o[j + 6]) * inv, __uint_as_float(o[j + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + j) = v;
      }
    }
  }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (mma_warp) tc::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

// The decoder's causal prefill attention on tcgen05. q [B, Hq, L, 256], k the cache
// [B, Hkv, kv_len, 256], vt = V^T [B, Hkv, 256, vt_stride] with vt_stride a multiple of 64 that
// is >= L (columns past L hold finite values), out [B, L, Hq, 256]; Hq = 4 Hkv.
int q35_prefill_attention_tc_launch(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                                    int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                    int64_t vt_stride, float scale, cudaStream_t stream, bool pdl) {
  Q35_REQUIRE(q && k && vt && out, "prefill_attention_tc: null pointer");
  Q35_REQUIRE(q_heads == kAG * kv_heads, "prefill_attention_tc: %lld query heads for %lld KV heads (needs 4 per KV head)",
              (long long)q_heads, (long long)kv_heads);
  Q35_REQUIRE(seq_len >= 0 && kv_len >= seq_len && vt_stride % kAK == 0 && vt_stride >= seq_len,
              "prefill_attention_tc: bad shape (L %lld, kv_len %lld, vt_stride %lld)", (long long)seq_len,
              (long long)kv_len, (long long)vt_stride);
  Q35_REQUIRE(Q35_ALIGNED(q, 16) && Q35_ALIGNED(k, 16) && Q35_ALIGNED(vt, 16) && Q35_ALIGNED(out, 16),
              "prefill_attention_tc: 16-byte alignment");
  if (batch * seq_len == 0) return Q35_OK;
  static Q35PerDevice<bool> attr;
  attr.get([] {
    cudaFuncSetAttribute(prefill_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnTcSmem);
    return true;
  });
  AttnTcParams prm{(const bf16*)q, (const bf16*)k, (const bf16*)vt, (bf16*)out, (int)q_heads, (int)kv_heads,
                   (int)seq_len, (int)kv_len, (int)vt_stride, scale * 1.4426950408889634f};
  const dim3 grid((unsigned)((seq_len + kAQ - 1) / kAQ), (unsigned)kv_heads, (unsigned)batch);
  const cudaError_t e = q35_launch(prefill_attn_tc_kernel, grid, dim3(kAThreads), kAttnTcSmem, stream, pdl, prm);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "prefill_attention_tc launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_prefill_attention_tc(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                                        int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                        int64_t vt_stride, float scale, void* stream) {
  return q35_prefill_attention_tc_launch(q, k, vt, out, batch, q_heads, kv_heads, seq_len, kv_len, vt_stride, scale,
                                         (cudaStream_t)stream, false);
}

extern "C" int q35_prefill_attention_tc_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_attn_tc_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_attn_tc_error_word, &zero, sizeof(int));
  return v;
}
