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
// rows) so that both MMA operands are K-major with the 128-byte swizzle. Warps 0-7 run the
// softmax; warp 8 issues the MMAs (an issuing thread stalls about as long as its MMAs run, which
// would hold back a softmax row); warp 9 brings the operands in by TMA (Q once, K and V^T tiles
// double-buffered). They hand off through mbarriers: TMA arrivals, MMA commits, and barriers the
// 256 softmax threads arrive on (S read, P written); wherever one side can run a tile ahead of
// its waiter the barrier is per buffer, so no wait can see a later phase of the same parity.
// Every wait is bounded; a timeout sets q35_attn_tc_error_word.
#include <cuda.h>
#include <cudaTypedefs.h>

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
constexpr int kAThreads = kASoft + 64;  // + the MMA warp + the TMA warp
constexpr uint32_t kQBytes = 4 * kAM * 128;  // Q: 4 slabs (64 dims) x 128 rows x 128 B
constexpr uint32_t kKBytes = 4 * kAK * 128;  // K tile: 4 slabs x 64 keys x 128 B
constexpr uint32_t kVBytes = kAD * 128;      // V^T tile: 256 dim rows x 64 keys (128 B)
constexpr uint32_t kPBytes = kAM * 128;      // P part: 128 rows x 64 keys (128 B)
constexpr uint32_t kOffK = kQBytes, kOffV = kOffK + 2 * kKBytes, kOffP = kOffV + 2 * kVBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
constexpr size_t kAttnTcSmem = kOffBar + 128 + 1024;  // barriers + TMEM slot, 1024-byte alignment slack
static_assert(kAttnTcSmem + 2 * kAM * sizeof(float) <= 232448, "dynamic + static shared memory of one CTA");
constexpr uint32_t kTmemCols = 512;                 // S buffers at columns 0 / 64, O at 256
constexpr uint32_t kColO = 256;
constexpr long long kAttnWaitBudget = 2000000000LL;

struct AttnTcParams {
  bf16* out;  // [B, L, Hq, 256]
  int Hq, Hkv, L, kv_len, vt_stride;
  float scale_log2;  // softmax scale x log2(e)
  // key split: a block with more than `half_tiles` key tiles runs as two CTAs (tiles below /
  // from half_tiles) whose partial O, maximum and sum meet in part / ml; the later one merges
  int nqb, half_tiles;
  float* part;        // [B * Hkv][nqb][2][256 dims][128 rows] (a warp's 32 rows are contiguous)
  float* ml;          // [B * Hkv][nqb][2][128 rows][2]
  unsigned* tickets;  // [B * Hkv][nqb], zero at rest (the merger resets its word)
};
// barrier slots in shared memory
// barrier slots: TMA arrivals (Q, K[2], V[2]), MMA commits (S[2], P.V, V buffer free[2]), softmax
// arrivals (S[2] read, P written)
enum { kBarQ = 0, kBarK = 1, kBarV = 3, kBarS = 5, kBarPV = 7, kBarVFree = 8, kBarRdyS = 10, kBarRdyPV = 12, kBars = 13 };

Q35_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
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

__global__ void __launch_bounds__(kAThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, AttnTcParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char attn_smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)attn_smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sQ = tc::smem_u32(sm), sK = sQ + kOffK, sV = sQ + kOffV, sP = sQ + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  auto bar = [&](int i) { return tc::smem_u32(&bars[i]); };
  const int qb = blockIdx.x % p.nqb, split = blockIdx.x / p.nqb, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = qb * kAQ;
  const int L = p.L;
  const int nkeys = min(q0 + kAQ, L);  // keys any row of the block may see (causal)
  const int nt_all = (nkeys + kAK - 1) / kAK;
  const bool two = nt_all > p.half_tiles;  // this block runs as two CTAs
  if (split == 1 && !two) return;        // (whole CTA: before any barrier or TMEM)
  const int t0 = split ? p.half_tiles : 0;                    // first key tile of this CTA
  const int nt = (two && split == 0) ? p.half_tiles : nt_all - t0;  // its tile count

  const bool mma_warp = warp == kASoft / 32, tma_warp = warp == kASoft / 32 + 1;
  if (mma_warp) tc::tmem_alloc(tmem_slot, kTmemCols);
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < kBarRdyS; ++i) tc::mbar_init(bar(i), 1);
    tc::mbar_init(bar(kBarVFree), 1);
    tc::mbar_init(bar(kBarVFree + 1), 1);
    tc::mbar_init(bar(kBarRdyS), kASoft);
    tc::mbar_init(bar(kBarRdyS + 1), kASoft);
    tc::mbar_init(bar(kBarRdyPV), kASoft);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  bool ok = true;
  auto wait_bar = [&](int i, uint32_t parity) {
    if (ok && !tc::mbar_test(bar(i), parity) && !tc::mbar_wait_bounded(bar(i), parity, kAttnWaitBudget)) {
      ok = false;
      atomicCAS(&q35_attn_tc_error_word, 0, 1 + i);  // 1 + the barrier slot that timed out
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  };
  __syncthreads();  // barriers initialised, TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (mma_warp || tma_warp) {
    if ((tid & 31) == 0) {
      const uint32_t idesc_s = tc::idesc_f32acc(1, kAM, kAK);  // bf16 x bf16 -> FP32, M 128, N 64
      const uint32_t idesc_o = tc::idesc_f32acc(1, kAM, kAD);  // M 128, N 256
      const int krow0 = (b * p.Hkv + g) * p.kv_len, vrow0 = (b * p.Hkv + g) * kAD;
      auto load_k = [&](int t) {  // 4 boxes of 64 keys x 64 dims into buffer t & 1
        const int i = t & 1;
        tc::mbar_expect_tx(bar(kBarK + i), kKBytes);
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
          tma_load_2d(sK + i * kKBytes + sl * (kAK * 128), &tmK, sl * 64, krow0 + (t0 + t) * kAK, bar(kBarK + i));
      };
      auto load_v = [&](int t) {  // one box of 256 dims x 64 keys into buffer t & 1
        const int i = t & 1;
        tc::mbar_expect_tx(bar(kBarV + i), kVBytes);
        tma_load_2d(sV + i * kVBytes, &tmV, (t0 + t) * kAK, vrow0, bar(kBarV + i));
      };
      auto issue_s = [&](int t) {  // S[t & 1] = Q K_t^T
        const uint32_t d = tmem + (uint32_t)((t & 1) * kAK);
        const uint32_t kb = sK + (t & 1) * kKBytes;
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16(d, tc::desc_sw128(sQ + sl * (kAM * 128) + kk * 32),
                         tc::desc_sw128(kb + sl * (kAK * 128) + kk * 32), idesc_s, (sl | kk) ? 1u : 0u);
        tc::commit(bar(kBarS + (t & 1)));
      };
      auto issue_pv = [&](int t) {  // O += P_hi V_t + P_lo V_t
        const uint32_t vb = sV + (t & 1) * kVBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int part = 0; part < 2; ++part)
            tc::mma_bf16(tmem + kColO, tc::desc_sw128(sP + part * kPBytes + kk * 32), tc::desc_sw128(vb + kk * 32),
                         idesc_o, (t > 0 || kk > 0 || part > 0) ? 1u : 0u);
        tc::commit(bar(kBarPV));
        tc::commit(bar(kBarVFree + (t & 1)));
      };
      if (tma_warp) {
        // Q: 4 heads x 4 dim slabs of 32 query rows; K_0, K_1, V_0, V_1; then each buffer again
        // once the MMA that read it has completed
        tc::mbar_expect_tx(bar(kBarQ), kQBytes);
#pragma unroll
        for (int hd = 0; hd < kAG; ++hd)
#pragma unroll
          for (int sl = 0; sl < 4; ++sl)
            tma_load_2d(sQ + sl * (kAM * 128) + hd * (kAQ * 128), &tmQ, sl * 64, (b * p.Hq + g * kAG + hd) * L + q0,
                        bar(kBarQ));
        load_k(0);
        load_v(0);
        if (nt > 1) {
          load_k(1);
          load_v(1);
        }
        for (int t = 0; t + 2 < nt; ++t) {
          wait_bar(kBarS + (t & 1), (uint32_t)(t >> 1) & 1u);  // S_t read K_t's buffer
          load_k(t + 2);
          wait_bar(kBarVFree + (t & 1), (uint32_t)(t >> 1) & 1u);  // P.V_t read V_t's buffer
          load_v(t + 2);
        }
      } else {
        wait_bar(kBarQ, 0);
        wait_bar(kBarK, 0);
        issue_s(0);
        for (int t = 0; t < nt; ++t) {
          if (t + 1 < nt) {  // S_{t+1}: K_{t+1} arrived and the softmax has read S_{t-1} from its buffer
            wait_bar(kBarK + ((t + 1) & 1), (uint32_t)((t + 1) >> 1) & 1u);
            if (t >= 1) wait_bar(kBarRdyS + ((t - 1) & 1), (uint32_t)((t - 1) >> 1) & 1u);
            issue_s(t + 1);
          }
          wait_bar(kBarV + (t & 1), (uint32_t)(t >> 1) & 1u);  // V_t
          wait_bar(kBarRdyPV, (uint32_t)t & 1u);               // P_t written, O rescaled
          issue_pv(t);
        }
      }
    }
    __syncwarp();
  } else {
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter
    const int row = tid & (kAM - 1), half = tid >> 7;  // row r = head 4 g + r / 32, query q0 + r % 32
    const int qi = q0 + (row & (kAQ - 1));
    // per-tile row maxima, then (after the last tile) the row sums of the two halves; only the two
    // threads of a row touch its entries
    __shared__ float xmax[2][kAM];
    float(&xsum)[2][kAM] = xmax;
    // warps w and w + 4 hold the two halves of the same 32 rows
    auto pair_sync = [&] { asm volatile("bar.sync %0, 64;" ::"r"(1 + (warp & 3)) : "memory"); };
    // arrive (release) once this thread's shared-memory writes and TMEM accesses are done
    auto ready = [&](int i) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar(i)) : "memory");
    };
    float m_run = -INFINITY, l_run = 0.f;
    for (int t = 0; t < nt; ++t) {
      // (a) S_t -> registers; its TMEM buffer is then free for S_{t+2}
      wait_bar(kBarS + (t & 1), (uint32_t)(t >> 1) & 1u);
      uint32_t sv[32];
      tc::tmem_ld32_async(trow + (uint32_t)((t & 1) * kAK + half * 32), sv);
      tc::tmem_wait_ld();
      ready(kBarRdyS + (t & 1));
      // (d) softmax of this row over the tile's 64 keys: this thread's 32, the partner's maximum
      const int k0 = (t0 + t) * kAK + half * 32;
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
      // (e) PV_{t-1} done: O is stable, P is free
      if (t > 0) wait_bar(kBarPV, (uint32_t)(t - 1) & 1u);
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
      // (i) P.V_t may run
      ready(kBarRdyPV);
    }
    // ---- epilogue: O / l for rows of real queries
    if (nt > 0) wait_bar(kBarPV, (uint32_t)(nt - 1) & 1u);
    xsum[half][row] = l_run;
    pair_sync();
    const float l_row = half ? xsum[0][row] + l_run : l_run + xsum[1][row];  // same order in both threads
    const int hh = g * kAG + (row >> 5);
    auto store_row = [&](int c, const float* o32, float scale) {  // 32 dims of this row, bf16
      if (!(ok && qi < L)) return;
      bf16* dst = p.out + (((int64_t)b * L + qi) * p.Hq + hh) * kAD + c;
  #pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 v;
        v.x = pack_bf16(o32[j] * scale, o32[j + 1] * scale);
        v.y = pack_bf16(o32[j + 2] * scale, o32[j + 3] * scale);
        v.z = pack_bf16(o32[j + 4] * scale, o32[j + 5] * scale);
        v.w = pack_bf16(o32[j + 6] * scale, o32[j + 7] * scale);
        *reinterpret_cast<uint4*>(dst + j) = v;
      }
    };
    if (!two) {
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
  #pragma unroll 1
      for (int c = half * (kAD / 2); c < (half + 1) * (kAD / 2); c += 32) {
        uint32_t o[32];
        tc::tmem_ld32(trow + kColO + c, o);
        store_row(c, reinterpret_cast<const float*>(o), inv);
      }
    } else {
      // this part's un-normalised O (its own reference maximum), maximum and sum to global
      const int64_t slot = ((int64_t)(b * p.Hkv + g) * p.nqb + qb) * 2;
      float* my = p.part + (slot + split) * kAD * kAM + row;
  #pragma unroll 1
      for (int c = half * (kAD / 2); c < (half + 1) * (kAD / 2); c += 32) {
        uint32_t o[32];
        tc::tmem_ld32(trow + kColO + c, o);
  #pragma unroll
        for (int j = 0; j < 32; ++j) my[(c + j) * kAM] = __uint_as_float(o[j]);
      }
      if (half == 0) {
        p.ml[((slot + split) * kAM + row) * 2] = m_run;
        p.ml[((slot + split) * kAM + row) * 2 + 1] = l_row;
      }
      // the second of the two CTAs to finish merges both parts in split order
      __shared__ unsigned arrival;
      __threadfence();
      asm volatile("bar.sync 5, %0;" ::"n"(kASoft) : "memory");
      if (tid == 0) arrival = atomicAdd(&p.tickets[slot / 2], 1u);
      asm volatile("bar.sync 5, %0;" ::"n"(kASoft) : "memory");
      if (arrival == 1) {
        __threadfence();
        const float* pa = p.part + slot * kAD * kAM + row;
        const float* pb = p.part + (slot + 1) * kAD * kAM + row;
        const float ma = __ldcg(p.ml + (slot * kAM + row) * 2), la = __ldcg(p.ml + (slot * kAM + row) * 2 + 1);
        const float mb = __ldcg(p.ml + ((slot + 1) * kAM + row) * 2), lb = __ldcg(p.ml + ((slot + 1) * kAM + row) * 2 + 1);
        const float m = fmaxf(ma, mb), wa = ex2(ma - m), wb = ex2(mb - m);
        const float l = la * wa + lb * wb;
        const float inv = l > 0.f ? 1.0f / l : 0.f;
  #pragma unroll 1
        for (int c = half * (kAD / 2); c < (half + 1) * (kAD / 2); c += 32) {
          float o[32];
  #pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __ldcg(pa + (c + j) * kAM) * wa + __ldcg(pb + (c + j) * kAM) * wb;
          store_row(c, o, inv);
        }
        if (tid == 0) p.tickets[slot / 2] = 0u;  // rest state for the next launch
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (mma_warp) tc::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// 2-D bf16 map over rows x cols (row-major), boxes of 64 columns (128 bytes) x box_rows, 128-byte
// swizzle; reads past the tensor fill with zeros.
bool make_map_bf16(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace {

// Key split: blocks with more than half the longest block's key tiles run as two CTAs, when the
// longest block has at least 4 tiles (256 keys).
int half_tiles_for(int64_t seq_len) {
  const int ntmax = (int)((seq_len + kAK - 1) / kAK);
  return ntmax >= 4 ? (ntmax + 1) / 2 : ntmax;
}

struct TcWs {
  size_t tickets, ml, part, total;
};
TcWs tc_ws_layout(int64_t batch, int64_t kv_heads, int64_t seq_len) {
  const int64_t slots = batch * kv_heads * ((seq_len + kAQ - 1) / kAQ);
  TcWs w;
  w.tickets = 0;
  w.ml = (slots * sizeof(unsigned) + 255) & ~(size_t)255;
  w.part = (w.ml + (size_t)slots * 2 * kAM * 2 * sizeof(float) + 255) & ~(size_t)255;
  w.total = w.part + (size_t)slots * 2 * kAM * kAD * sizeof(float);
  return w;
}

}  // namespace

size_t q35_prefill_attention_tc_ws_bytes(int64_t batch, int64_t kv_heads, int64_t seq_len) {
  return tc_ws_layout(batch, kv_heads, seq_len).total;
}

// The decoder's causal prefill attention on tcgen05. q [B, Hq, L, 256], k the cache
// [B, Hkv, kv_len, 256], vt = V^T [B, Hkv, 256, vt_stride] with vt_stride a multiple of 64 that
// is >= L (columns past L hold finite values), out [B, L, Hq, 256]; Hq = 4 Hkv. `ws` (zeroed
// before first use, left zeroed) holds the key-split partials.
int q35_prefill_attention_tc_launch(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                                    int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                    int64_t vt_stride, float scale, void* ws, size_t ws_bytes, cudaStream_t stream,
                                    bool pdl) {
  Q35_REQUIRE(q && k && vt && out, "prefill_attention_tc: null pointer");
  Q35_REQUIRE(q_heads == kAG * kv_heads, "prefill_attention_tc: %lld query heads for %lld KV heads (needs 4 per KV head)",
              (long long)q_heads, (long long)kv_heads);
  Q35_REQUIRE(seq_len >= 0 && kv_len >= seq_len && vt_stride % kAK == 0 && vt_stride >= seq_len,
              "prefill_attention_tc: bad shape (L %lld, kv_len %lld, vt_stride %lld)", (long long)seq_len,
              (long long)kv_len, (long long)vt_stride);
  Q35_REQUIRE(Q35_ALIGNED(q, 16) && Q35_ALIGNED(k, 16) && Q35_ALIGNED(vt, 16) && Q35_ALIGNED(out, 16),
              "prefill_attention_tc: 16-byte alignment");
  if (batch * seq_len == 0) return Q35_OK;
  const TcWs w = tc_ws_layout(batch, kv_heads, seq_len);
  Q35_REQUIRE(ws && Q35_ALIGNED(ws, 256) && ws_bytes >= w.total,
              "prefill_attention_tc: workspace of %zu bytes (256-byte aligned) needed", w.total);
  static Q35PerDevice<bool> attr;
  attr.get([] {
    cudaFuncSetAttribute(prefill_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnTcSmem);
    return true;
  });
  // TMA maps (bf16, 128-byte swizzle, boxes of 64 elements along the row): q rows [B*Hq*L] boxes
  // of 32 rows, k rows [B*Hkv*kv_len] boxes of 64 keys, V^T rows [B*Hkv*256] boxes of 256 dims x 64 keys
  CUtensorMap mq, mk, mv;
  if (!make_map_bf16(&mq, q, (uint64_t)batch * q_heads * seq_len, kAD, 32) ||
      !make_map_bf16(&mk, k, (uint64_t)batch * kv_heads * kv_len, kAD, kAK) ||
      !make_map_bf16(&mv, vt, (uint64_t)batch * kv_heads * kAD, (uint64_t)vt_stride, kAD))
    return q35_fail(Q35_ECUDA, "prefill_attention_tc: tensor map encoding failed");
  const int nqb = (int)((seq_len + kAQ - 1) / kAQ), half_tiles = half_tiles_for(seq_len);
  const int ntmax = (int)((seq_len + kAK - 1) / kAK);
  char* base = static_cast<char*>(ws);
  AttnTcParams prm{(bf16*)out,
                   (int)q_heads,
                   (int)kv_heads,
                   (int)seq_len,
                   (int)kv_len,
                   (int)vt_stride,
                   scale * 1.4426950408889634f,
                   nqb,
                   half_tiles,
                   reinterpret_cast<float*>(base + w.part),
                   reinterpret_cast<float*>(base + w.ml),
                   reinterpret_cast<unsigned*>(base + w.tickets)};
  const dim3 grid((unsigned)(nqb * (ntmax > half_tiles ? 2 : 1)), (unsigned)kv_heads, (unsigned)batch);
  const cudaError_t e =
      q35_launch(prefill_attn_tc_kernel, grid, dim3(kAThreads), kAttnTcSmem, stream, pdl, mq, mk, mv, prm);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "prefill_attention_tc launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" size_t q35_prefill_attention_tc_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq_len) {
  return q35_prefill_attention_tc_ws_bytes(batch, kv_heads, seq_len);
}

extern "C" int q35_prefill_attention_tc(const void* q, const void* k, const void* vt, void* out, int64_t batch,
                                        int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                        int64_t vt_stride, float scale, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  return q35_prefill_attention_tc_launch(q, k, vt, out, batch, q_heads, kv_heads, seq_len, kv_len, vt_stride, scale,
                                         workspace, workspace_bytes, (cudaStream_t)stream, false);
}

extern "C" int q35_prefill_attention_tc_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_attn_tc_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_attn_tc_error_word, &zero, sizeof(int));
  return v;
}
