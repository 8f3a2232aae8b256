// Split-KV GQA decode attention (reference: kernels.py:940-1090 gqa_decode_attention, the decode
// branch of integration.py:343-359, and kernels.py:285-333 attention_gate_mul).
//
// One CTA = one (batch, KV head, split of cache rows) with all G = Hq/Hkv query heads of that KV
// head, so each K/V row is read from HBM once per group (the reference reads it once per query
// head). Warps stride over the split's rows with an FP32 online softmax per head; the CTA merges
// its warps and writes one (max, sum, un-normalised output) partial per head. The last CTA of a
// (batch, KV head) — elected by an atomic ticket, no second launch — combines the partials with
// all 8 warps, normalises, rounds to BF16 and (fused variant) multiplies by BF16(sigmoid(gate)).
//
// The fused variant is the whole decode attention mixer: Q/K RMSNorm(1+w) and partial RoPE of the
// current token (positions from device scalars), its K/V written to the cache row *len, and the
// current token attended from registers, so nothing waits on the cache write.
#include <cfloat>

#include <cooperative_groups.h>

#include "common.cuh"

using namespace q35;

namespace {

constexpr int kD = 256;
constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kMaxSplits = 148;  // splits per (batch, KV head): two CTAs per SM at batch 1 with two KV heads
constexpr int kRowsPerSplit = 32;
constexpr int kGroup = 16;       // splits merged per first-level combine when S > kGroup
constexpr size_t kTicketBytes = 1024;  // B*Hkv final + B*Hkv*NG group tickets (<= 256 words)

struct DecodeParams {
  const bf16* packed;    // fused: [B, stride] projection output
  const bf16* qw;
  const bf16* kw;
  const float* inv_freq;
  const int64_t* rope_pos;
  const bf16* q_in;      // API: [B, Hq, D]
  bf16* cache_k;         // [B, Hkv, max_len, D]
  bf16* cache_v;
  const int64_t* len;    // fused: rows already cached (new token -> row *len); API: valid rows
  bf16* out;             // [B, Hq*D]
  float* part;           // [B*Hkv*S*G][D]
  float* part_ml;        // [B*Hkv*S*G][2]
  float* group_part;     // [B*Hkv*NG*G][D]: partials of groups of kGroup splits (S > kGroup)
  float* group_ml;       // [B*Hkv*NG*G][2]
  unsigned* tickets;     // [B*Hkv] final, then [B*Hkv*NG] per group
  int n_bg;              // B*Hkv
  int Hq, Hkv, max_len, S, rot;
  float scale, eps;
};


Q35_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

// Paired FP32 arithmetic (sm_100 f32x2): two lanes of a 64-bit register per instruction.
Q35_DEV uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
Q35_DEV void upk2(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
Q35_DEV uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
Q35_DEV uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 8 bf16 (dims 8 lane .. + 7) as 4 FP32 pairs: a bf16 is the high half of its FP32 pattern
Q35_DEV void bf16x8_pairs(uint4 u, uint64_t (&p)[4]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = pk2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
}
Q35_DEV float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

constexpr int kR = 4;    // cache rows per group (one online-softmax rescale per group)
constexpr int kNS = 3;   // ring stages per warp: 2 groups = 8 KB in flight per warp
constexpr size_t kAttnDynSmem = (size_t)kWarps * kNS * kR * 2 * kD * sizeof(bf16);  // 96 KB: two CTAs per SM
static_assert(kWarps * 4 * kD * sizeof(float) + 2 * kMaxSplits * 4 * sizeof(float) <= kAttnDynSmem,
              "the merge / combine buffers fit in the ring");

// After this CTA's results are written: count it in at `ticket`; true for the last of `n`
// arrivals (whose later reads then see every earlier CTA's writes).
template <int G>
Q35_DEV bool last_arrival(unsigned* ticket, int n) {
  __shared__ unsigned ticket_s;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket_s = atomicAdd(ticket, 1u);
  __syncthreads();
  if (ticket_s != (unsigned)(n - 1)) return false;
  __threadfence();
  return true;
}

// Merges n partials per head (ml_in [n][G][2], part_in [n][G][kD]; un-normalised outputs with
// their running max and sum) with all warps. final: normalise, round to BF16 and (fused) apply
// the sigmoid gate into p.out; else write one partial of the same form to ml_out / part_out.
// `scratch` (shared memory, >= kWarps * G * kD floats + 2 * kMaxSplits * G floats) is free.
template <int G, bool FUSED>
Q35_DEV void merge_partials(const DecodeParams& p, const float* ml_in, const float* part_in, int n, bool final, int b,
                            int g, float* ml_out, float* part_out, unsigned char* scratch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, d = threadIdx.x;
  float (*wacc)[G][kD] = reinterpret_cast<float (*)[G][kD]>(scratch);
  float (*cm)[G] = reinterpret_cast<float (*)[G]>(scratch + (size_t)kWarps * G * kD * sizeof(float));
  float (*cl)[G] = cm + kMaxSplits;
  __shared__ float cls[G], cms[G];
  for (int i = threadIdx.x; i < n * G; i += kThreads) {
    const float mi = __ldcg(ml_in + 2 * i);
    const float li = __ldcg(ml_in + 2 * i + 1);
    cm[i / G][i % G] = li > 0.f ? mi : -INFINITY;  // empty split: zero weight
    cl[i / G][i % G] = li;
  }
  __syncthreads();
  if (warp < G) {  // one warp per head: max, weights and normaliser over the n partials
    const int hh = warp;
    float M = -FLT_MAX;
    for (int j = lane; j < n; j += 32) M = fmaxf(M, cm[j][hh]);
    M = warp_max(M);
    float Ls = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = (cm[j][hh] == -INFINITY) ? 0.f : exp2f(cm[j][hh] - M);  // log2-unit maxima
      cm[j][hh] = e;
      Ls += cl[j][hh] * e;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) {
      cls[hh] = Ls;
      cms[hh] = M;
    }
  }
  __syncthreads();
  float a8[G][8];
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
#pragma unroll
    for (int j = 0; j < 8; ++j) a8[hh][j] = 0.f;
#pragma unroll 2
  for (int j = warp; j < n; j += kWarps) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      const float wgt = cm[j][hh];
      const float4* src = reinterpret_cast<const float4*>(part_in + (int64_t)(j * G + hh) * kD + lane * 8);
      const float4 u0 = __ldcg(src), u1 = __ldcg(src + 1);
      a8[hh][0] += wgt * u0.x;
      a8[hh][1] += wgt * u0.y;
      a8[hh][2] += wgt * u0.z;
      a8[hh][3] += wgt * u0.w;
      a8[hh][4] += wgt * u1.x;
      a8[hh][5] += wgt * u1.y;
      a8[hh][6] += wgt * u1.z;
      a8[hh][7] += wgt * u1.w;
    }
  }
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float4* dst = reinterpret_cast<float4*>(&wacc[warp][hh][lane * 8]);
    dst[0] = make_float4(a8[hh][0], a8[hh][1], a8[hh][2], a8[hh][3]);
    dst[1] = make_float4(a8[hh][4], a8[hh][5], a8[hh][6], a8[hh][7]);
  }
  __syncthreads();
  const int Hq = p.Hq, Hkv = p.Hkv;
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float A = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) A += wacc[w][hh][d];
    if (!final) {
      part_out[(int64_t)hh * kD + d] = A;
      if (d == 0) {
        ml_out[2 * hh] = cls[hh] > 0.f ? cms[hh] : -FLT_MAX;
        ml_out[2 * hh + 1] = cls[hh];
      }
      continue;
    }
    const float o = cls[hh] > 0.f ? rbf(A / cls[hh]) : 0.f;
    const int h = g * G + hh;
    if (FUSED) {
      const int stride = 2 * Hq * kD + 2 * Hkv * kD;
      const float gate = bf2f(p.packed[(int64_t)b * stride + h * 2 * kD + kD + d]);
      p.out[((int64_t)b * Hq + h) * kD + d] = f2bf(o * rbf(sigmoid_f(gate)));
    } else {
      p.out[((int64_t)b * Hq + h) * kD + d] = f2bf(o);
    }
  }
}

template <int G, bool FUSED>
__global__ void __launch_bounds__(kThreads, 2) attn_decode_kernel(DecodeParams p) {
  extern __shared__ __align__(16) unsigned char attn_dsmem[];
  __shared__ __align__(16) float qf[G][kD];
  __shared__ __align__(16) float nrm[FUSED ? G + 1 : 1][kD];
  __shared__ __align__(16) float kn[kD];
  __shared__ __align__(16) float vn[kD];
  __shared__ __align__(16) float wsc[kWarps][kR * G < 4 ? 4 : kR * G];  // a warp's group scores
  __shared__ float wmax[kWarps][G], wsum[kWarps][G];
  __shared__ float red[kWarps][G + 1];

  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int S = p.S, Hkv = p.Hkv, Hq = p.Hq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = threadIdx.x;  // kThreads == kD
  const int64_t kv_base = ((int64_t)b * Hkv + g) * p.max_len * kD;

  // The cached rows and their count were written by earlier decode steps (the kernel just before
  // this one only projects the new token), so this CTA's first groups of rows are requested
  // before the programmatic-dependent-launch wait.
  const int64_t len = *p.len;
  const int n_rows = (int)(len < 0 ? 0 : (len > p.max_len ? p.max_len : len));
  // ---- this CTA's rows of the cache. Every warp streams its own groups of kR rows (group i of
  // the split goes to warp i mod 8) through a private kNS-stage cp.async ring; each lane copies,
  // and later reads back, only its own 16-byte chunk (dims 8 lane .. 8 lane + 7) of every K and V
  // row, so the stream needs no block barrier: cp.async.wait_group orders a lane's own copies.
  // Per group: the kR x G dot products reduced in one butterfly, one online-softmax rescale per
  // head, P.V on the lane's 8 dims. The warps' partials merge once at the end.
  const int chunk = (n_rows + S - 1) / S;
  const int r0 = s * chunk;
  const int r1 = min(r0 + chunk, n_rows);
  const int nr = r1 > r0 ? r1 - r0 : 0;
  const int ngrp = (nr + kR - 1) / kR;
  const int nit = warp < ngrp ? (ngrp - 1 - warp) / kWarps + 1 : 0;
  constexpr int kSlot = kR * 2 * 32;  // uint4 slots of one stage of one warp: [row][K | V][lane]
  uint4* ring = reinterpret_cast<uint4*>(attn_dsmem) + warp * (kNS * kSlot) + lane;
  const bf16* Kb = p.cache_k + kv_base + lane * 8;
  const bf16* Vb = p.cache_v + kv_base + lane * 8;
  auto issue = [&](int it) {
    if (it < nit) {
      const int rg = r0 + (warp + it * kWarps) * kR;
      uint4* st = ring + (it % kNS) * kSlot;
#pragma unroll
      for (int j = 0; j < kR; ++j)
        if (rg + j < r1) {
          cp_async16(st + (2 * j) * 32, Kb + (int64_t)(rg + j) * kD);
          cp_async16(st + (2 * j + 1) * 32, Vb + (int64_t)(rg + j) * kD);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int i = 0; i < kNS - 1; ++i) issue(i);
  pdl_wait();
  pdl_launch_dependents();
  if (FUSED) {
    const int stride = 2 * Hq * kD + 2 * Hkv * kD;
    const bf16* row = p.packed + (int64_t)b * stride;
    float x[G + 1];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) x[hh] = bf2f(row[(g * G + hh) * 2 * kD + d]);
    x[G] = bf2f(row[2 * Hq * kD + g * kD + d]);
    const float v_raw = bf2f(row[2 * Hq * kD + Hkv * kD + g * kD + d]);
#pragma unroll
    for (int i = 0; i <= G; ++i) {
      const float ws = warp_sum(x[i] * x[i]);
      if (lane == 0) red[warp][i] = ws;
    }
    float c = 1.f, sn = 0.f;
    if (d < p.rot) rope_cs(d, p.rot / 2, (float)(*p.rope_pos), p.inv_freq, c, sn);
    const float wq = bf2f(p.qw[d]), wk = bf2f(p.kw[d]);
    __syncthreads();
#pragma unroll
    for (int i = 0; i <= G; ++i) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) tot += red[w][i];
      const float r = rsqrt_ieee(tot / (float)kD + p.eps);
      nrm[i][d] = rbf(x[i] * r * (1.0f + (i < G ? wq : wk)));
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < G; ++i) qf[i][d] = rope_apply(nrm[i], d, p.rot, c, sn) * p.scale;
    const float kr = rope_apply(nrm[G], d, p.rot, c, sn);
    kn[d] = kr;
    vn[d] = v_raw;
    if (s == 0 && len >= 0 && len < p.max_len) {
      p.cache_k[kv_base + len * kD + d] = f2bf(kr);
      p.cache_v[kv_base + len * kD + d] = f2bf(v_raw);
    }
  } else {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) qf[hh][d] = bf2f(p.q_in[((int64_t)b * Hq + g * G + hh) * kD + d]) * p.scale;
  }
  __syncthreads();

  // scores in log2 units (q scaled by log2 e): the softmax then runs on exp2, one MUFU op each;
  // the partials' maxima are in the same units (merge_partials uses exp2 as well). The dot
  // products and P.V run on FP32 pairs (fma.rn.f32x2), half the instructions of scalar FMAs.
  uint64_t q2[G][4];
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      q2[hh][e] = pk2(qf[hh][lane * 8 + 2 * e] * 1.4426950408889634f, qf[hh][lane * 8 + 2 * e + 1] * 1.4426950408889634f);
  float mw[G], lw[G];  // this warp's running max / sum per head
  uint64_t aw[G][4];   // and its output at the lane's 8 dims, as pairs
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    mw[hh] = -FLT_MAX;
    lw[hh] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) aw[hh][e] = 0ull;
  }
  // one group of `nv` rows: from the ring stage `st`, or (current) the new token's kn / vn
  auto absorb = [&](const uint4* st, int nv, bool current) {
    float v[kR * G];
#pragma unroll
    for (int j = 0; j < kR; ++j) {
      uint64_t k2[4];
      if (current) {
#pragma unroll
        for (int e = 0; e < 4; ++e) k2[e] = (j == 0) ? pk2(kn[lane * 8 + 2 * e], kn[lane * 8 + 2 * e + 1]) : 0ull;
      } else if (j < nv) {
        bf16x8_pairs(st[(2 * j) * 32], k2);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) k2[e] = 0ull;
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        uint64_t a2 = mul2(q2[hh][0], k2[0]);
#pragma unroll
        for (int e = 1; e < 4; ++e) a2 = fma2(q2[hh][e], k2[e], a2);
        float lo, hi;
        upk2(a2, lo, hi);
        v[j * G + hh] = lo + hi;
      }
    }
    butterfly_sum<kR * G>(v, lane);
    if (butterfly_writer<kR * G>(lane)) wsc[warp][butterfly_index<kR * G>(lane)] = v[0];
    __syncwarp();
    float sc[kR * G];
#pragma unroll
    for (int i = 0; i < kR * G; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(&wsc[warp][i]);
      sc[i] = t.x;
      sc[i + 1] = t.y;
      sc[i + 2] = t.z;
      sc[i + 3] = t.w;
    }
    __syncwarp();  // every lane has read the scores before the next group rewrites them
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float bm = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < kR; ++j)
        if (j < nv) bm = fmaxf(bm, sc[j * G + hh]);
      const float mn = fmaxf(mw[hh], bm);
      if (mn != mw[hh]) {  // a new maximum (uniform across the warp): rescale the running terms
        const float alpha = (mw[hh] == -FLT_MAX) ? 0.f : ex2_approx(mw[hh] - mn);
        lw[hh] *= alpha;
        const uint64_t a2 = pk2(alpha, alpha);
#pragma unroll
        for (int e = 0; e < 4; ++e) aw[hh][e] = mul2(aw[hh][e], a2);
        mw[hh] = mn;
      }
#pragma unroll
      for (int j = 0; j < kR; ++j) {
        const float pj = (j < nv) ? ex2_approx(sc[j * G + hh] - mn) : 0.f;
        sc[j * G + hh] = pj;
        lw[hh] += pj;
      }
    }
#pragma unroll
    for (int j = 0; j < kR; ++j) {
      if (j >= nv) break;
      uint64_t v2[4];
      if (current) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v2[e] = pk2(vn[lane * 8 + 2 * e], vn[lane * 8 + 2 * e + 1]);
      } else {
        bf16x8_pairs(st[(2 * j + 1) * 32], v2);
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        const uint64_t p2 = pk2(sc[j * G + hh], sc[j * G + hh]);
#pragma unroll
        for (int e = 0; e < 4; ++e) aw[hh][e] = fma2(v2[e], p2, aw[hh][e]);
      }
    }
  };
  for (int it = 0; it < nit; ++it) {
    issue(it + kNS - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(kNS - 1) : "memory");
    const int rg = r0 + (warp + it * kWarps) * kR;
    absorb(ring + (it % kNS) * kSlot, min(kR, r1 - rg), false);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (FUSED && s == S - 1 && warp == 0) absorb(nullptr, 1, true);  // the current token

  // ---- merge the warps (the ring memory is free once every warp is past its stream)
  __syncthreads();
  float* mrg = reinterpret_cast<float*>(attn_dsmem);  // [kWarps][G][kD]
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) upk2(aw[hh][e], o[2 * e], o[2 * e + 1]);
    float4* dst = reinterpret_cast<float4*>(mrg + (warp * G + hh) * kD + lane * 8);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
  if (lane == 0) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      wmax[warp][hh] = mw[hh];
      wsum[warp][hh] = lw[hh];
    }
  }
  __syncthreads();
  float m_run = -FLT_MAX, l_run = 0.f;  // warp hh < G: head hh's max / sum over the CTA's rows
  float acc[G];                          // thread d: un-normalised output of every head at dim d
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wmax[w][hh]);
    float A = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float e = (wmax[w][hh] == -FLT_MAX) ? 0.f : exp2f(wmax[w][hh] - M);
      A = fmaf(e, mrg[(w * G + hh) * kD + d], A);
      Ls = fmaf(e, wsum[w][hh], Ls);
    }
    acc[hh] = A;
    if (warp == hh) {
      m_run = M;
      l_run = Ls;
    }
  }
  __syncthreads();  // the merge buffer is read before the last CTA's combine reuses the memory

  // ---- this CTA's partial per head: (max, sum) from the softmax warps, the output from every dim
  const int bg = b * Hkv + g;
  const int slot0 = (bg * S + s) * G;
  if (warp < G && lane == 0) {
    p.part_ml[2 * (slot0 + warp)] = m_run;
    p.part_ml[2 * (slot0 + warp) + 1] = l_run;
  }
#pragma unroll
  for (int hh = 0; hh < G; ++hh) p.part[(int64_t)(slot0 + hh) * kD + d] = acc[hh];
  // ---- combine. S <= kGroup: the last CTA of (batch, KV head), elected by an atomic ticket,
  // merges the S partials into the output. Otherwise two levels: the last CTA of each group of
  // kGroup splits merges the group into a group partial, and the last group merger merges the
  // NG group partials (a single merger over up to 148 partials serialised their reads).
  const int NG = (S + kGroup - 1) / kGroup;
  unsigned* tk_final = p.tickets + bg;
  if (NG > 1) {
    const int grp = s / kGroup, gsz = min(kGroup, S - grp * kGroup);
    unsigned* tk = p.tickets + p.n_bg + bg * NG + grp;
    if (!last_arrival<G>(tk, gsz)) return;
    merge_partials<G, FUSED>(p, p.part_ml + 2 * (bg * S + grp * kGroup) * G, p.part + (int64_t)(bg * S + grp * kGroup) * G * kD,
                             gsz, false, b, g, p.group_ml + 2 * (bg * NG + grp) * G,
                             p.group_part + (int64_t)(bg * NG + grp) * G * kD, attn_dsmem);
    if (threadIdx.x == 0) atomicExch(tk, 0u);
    if (!last_arrival<G>(tk_final, NG)) return;
    merge_partials<G, FUSED>(p, p.group_ml + 2 * bg * NG * G, p.group_part + (int64_t)bg * NG * G * kD, NG, true, b, g,
                             nullptr, nullptr, attn_dsmem);
  } else {
    if (!last_arrival<G>(tk_final, S)) return;
    merge_partials<G, FUSED>(p, p.part_ml + 2 * bg * S * G, p.part + (int64_t)bg * S * G * kD, S, true, b, g, nullptr,
                             nullptr, attn_dsmem);
  }
  if (threadIdx.x == 0) atomicExch(tk_final, 0u);
}

// ---------------------------------------------------------------------------------------------
// Cluster variant of the fused decode mixer (decoder path, caches up to kClMaxRows rows):
// one cluster of CL (16, else 8) CTAs per (batch, KV head). Each CTA owns a contiguous slice of the
// cached rows and copies its K/V rows into shared memory with cp.async BEFORE the programmatic-
// dependent-launch wait: those rows and the row count were written by earlier steps (the kernel
// before this one is the QGKV projection), so the HBM latency overlaps the projection. After the
// wait: Q/K RMSNorm + RoPE of the current token, scores (warp per row), per-head softmax over the
// slice, un-normalised P.V; the last CTA also attends the current token from registers. The
// partials meet over distributed shared memory: CTA r merges dims [r * D / C, (r + 1) * D / C)
// of every head from all peers and writes the gated BF16 output. No global scratch, no second
// pass.
constexpr int kClMaxRows = 1280;  // cached rows the cluster variant covers (16 x 80 or 8 x 160 per CTA)
template <int CL>
constexpr int cl_rows() {
  return kClMaxRows / CL;
}
template <int CL>
constexpr size_t cl_smem_bytes() {
  return 2ull * cl_rows<CL>() * kD * sizeof(bf16);
}

template <int G, int CL>
__global__ void __launch_bounds__(kThreads, 1) attn_decode_cluster_kernel(DecodeParams p) {
  constexpr int kClusterCTAs = CL;
  constexpr int kClRows = cl_rows<CL>();
  extern __shared__ __align__(16) unsigned char cl_smem[];
  bf16* Ks = reinterpret_cast<bf16*>(cl_smem);
  bf16* Vs = Ks + kClRows * kD;
  __shared__ __align__(16) float qf[G][kD];
  __shared__ __align__(16) float nrm[G + 1][kD];
  __shared__ __align__(16) float kn[kD];
  __shared__ __align__(16) float vn[kD];
  __shared__ __align__(16) float sc[kClRows + 1][G];
  __shared__ float red[kWarps][G + 1];
  __shared__ float inbox[kClusterCTAs][G][kD / kClusterCTAs];  // peers' partial outputs for my dims
  __shared__ float inml[kClusterCTAs][G][2];                   // peers' (max, sum) per head
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank(), C = (int)cluster.num_blocks();
  const int g = blockIdx.y, b = blockIdx.z;
  const int Hq = p.Hq, Hkv = p.Hkv;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, d = t;
  const int64_t kv_base = ((int64_t)b * Hkv + g) * p.max_len * kD;

  // ---- rows of this CTA, copied before the wait (written by earlier steps)
  const int64_t len = *p.len;
  const int n = (int)(len < 0 ? 0 : (len > p.max_len ? p.max_len : len));
  const int chunk = (n + C - 1) / C;
  const int r0 = min(rank * chunk, n), r1 = min(r0 + chunk, n), nr = r1 - r0;
  for (int i = t; i < nr * (kD / 8); i += kThreads) {
    const int row = i / (kD / 8), c = i % (kD / 8);
    cp_async16(Ks + row * kD + c * 8, p.cache_k + kv_base + (int64_t)(r0 + row) * kD + c * 8);
    cp_async16(Vs + row * kD + c * 8, p.cache_v + kv_base + (int64_t)(r0 + row) * kD + c * 8);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // peers write into this CTA's shared memory later: all CTAs of the cluster must have started
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // RoPE angle and norm weights before the wait (the position counter is advanced at the end of
  // the previous token; the weights are constants)
  float c = 1.f, sn = 0.f;
  if (d < p.rot) rope_cs(d, p.rot / 2, (float)(*p.rope_pos), p.inv_freq, c, sn);
  const float wq = bf2f(p.qw[d]), wk = bf2f(p.kw[d]);
  pdl_wait();
  pdl_launch_dependents();

  // ---- Q/K RMSNorm(1+w) and partial RoPE of the current token; its K/V row goes to the cache
  const int stride = 2 * Hq * kD + 2 * Hkv * kD;
  const bf16* row = p.packed + (int64_t)b * stride;
  float x[G + 1];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) x[hh] = bf2f(row[(g * G + hh) * 2 * kD + d]);
  x[G] = bf2f(row[2 * Hq * kD + g * kD + d]);
  const float v_raw = bf2f(row[2 * Hq * kD + Hkv * kD + g * kD + d]);
  // the output gate of this thread's first merge item (dims of this rank, below), loaded with the
  // rest of the row: read after the cluster barrier it would be one more round trip to L2
  constexpr int kDper = kD / kClusterCTAs;
  const float gate0 = t < G * kDper ? bf2f(row[(g * G + t / kDper) * 2 * kD + kD + rank * kDper + t % kDper]) : 0.f;
#pragma unroll
  for (int i = 0; i <= G; ++i) {
    const float ws = warp_sum(x[i] * x[i]);
    if (lane == 0) red[warp][i] = ws;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i <= G; ++i) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += red[w][i];
    const float r = rsqrt_ieee(tot / (float)kD + p.eps);
    nrm[i][d] = rbf(x[i] * r * (1.0f + (i < G ? wq : wk)));
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < G; ++i) qf[i][d] = rope_apply(nrm[i], d, p.rot, c, sn) * p.scale;
  const float kr = rope_apply(nrm[G], d, p.rot, c, sn);
  kn[d] = kr;
  vn[d] = v_raw;
  if (rank == 0 && len >= 0 && len < p.max_len) {
    p.cache_k[kv_base + len * kD + d] = f2bf(kr);
    p.cache_v[kv_base + len * kD + d] = f2bf(v_raw);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // ---- scores: warp per row (four rows per step, one butterfly for their 4 G dot products),
  //      lanes hold 8 dims; the last CTA adds the current token as row nr
  const bool last = rank == C - 1;
  const int rows = nr + (last ? 1 : 0);
  float q8[G][8];
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[hh][j] = qf[hh][lane * 8 + j];
  auto key_row = [&](int j, float kf[8]) {
    if (j < nr) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(Ks + j * kD + lane * 8), kf);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) kf[e] = kn[lane * 8 + e];
    }
  };
  for (int j = warp; j < rows; j += 4 * kWarps) {  // rows j, j + 8, j + 16, j + 24: one butterfly
    float v[4 * G];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = j + i * kWarps;
      float kf[8];
      if (r < rows) {
        key_row(r, kf);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) kf[e] = 0.f;
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(q8[hh][e], kf[e], a);
        v[i * G + hh] = a;
      }
    }
    butterfly_sum<4 * G>(v, lane);
    if (butterfly_writer<4 * G>(lane)) {
      const int idx = butterfly_index<4 * G>(lane);
      const int r = j + (idx / G) * kWarps;
      if (r < rows) sc[r][idx % G] = v[0];
    }
  }
  __syncthreads();
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // ---- per-head max and weights over this CTA's rows; (max, sum) pushed to every peer
  if (warp < G) {
    float m = -FLT_MAX;
    for (int j = lane; j < rows; j += 32) m = fmaxf(m, sc[j][warp]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < rows; j += 32) {
      const float e = expf(sc[j][warp] - m);
      sc[j][warp] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane < C) {
      float* dst = cluster.map_shared_rank(&inml[rank][warp][0], lane);
      dst[0] = rows > 0 ? m : -FLT_MAX;
      dst[1] = rows > 0 ? l : 0.f;
    }
  }
  __syncthreads();
  // ---- un-normalised P.V (thread = dim, all heads), pushed to the peer that owns the dim
  {
    float a[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) a[hh] = 0.f;
    for (int j = 0; j < rows; ++j) {
      const float v = (j < nr) ? bf2f(Vs[j * kD + d]) : vn[d];
      if (G == 4) {  // the row's four weights in one 16-byte shared load
        const float4 w4 = *reinterpret_cast<const float4*>(&sc[j][0]);
        a[0] = fmaf(w4.x, v, a[0]);
        a[1 % G] = fmaf(w4.y, v, a[1 % G]);
        a[2 % G] = fmaf(w4.z, v, a[2 % G]);
        a[3 % G] = fmaf(w4.w, v, a[3 % G]);
      } else {
#pragma unroll
        for (int hh = 0; hh < G; ++hh) a[hh] = fmaf(sc[j][hh], v, a[hh]);
      }
    }
    const int dper = kD / kClusterCTAs;
    const int owner = d / dper;
#pragma unroll
    for (int hh = 0; hh < G; ++hh) *cluster.map_shared_rank(&inbox[rank][hh][d % dper], owner) = a[hh];
  }
  cluster.sync();  // every push has landed; from here on only this CTA's own shared memory is read
  // ---- merge the partials of dims [rank * D / C, (rank + 1) * D / C) of every head
  const int dper = kD / kClusterCTAs;
  for (int i = t; i < G * dper; i += kThreads) {
    const int hh = i / dper, di = i % dper, dd = rank * dper + di;
    float M = -FLT_MAX;
#pragma unroll
    for (int r = 0; r < kClusterCTAs; ++r)
      if (inml[r][hh][1] > 0.f) M = fmaxf(M, inml[r][hh][0]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int r = 0; r < kClusterCTAs; ++r) {
      const float lr = inml[r][hh][1];
      const float e = lr > 0.f ? expf(inml[r][hh][0] - M) : 0.f;
      L += lr * e;
      A += inbox[r][hh][di] * e;
    }
    const float o = L > 0.f ? rbf(A / L) : 0.f;
    const int h = g * G + hh;
    const float gate = i == t ? gate0 : bf2f(row[h * 2 * kD + kD + dd]);
    p.out[((int64_t)b * Hq + h) * kD + dd] = f2bf(o * rbf(sigmoid_f(gate)));
  }
}

int choose_splits(int64_t batch, int64_t kv_heads, int64_t cache_len) {
  int64_t s = (cache_len + kRowsPerSplit - 1) / kRowsPerSplit;  // >= 32 rows (a group per warp) per CTA
  // one wave of two CTAs per SM: rounding up would leave a few CTAs for a second wave
  const int64_t fill = (2 * kNumSMs) / (batch * kv_heads);
  if (s > fill) s = fill;
  if (s > kMaxSplits) s = kMaxSplits;
  return (int)(s < 1 ? 1 : s);
}

struct WsLayout {
  size_t tickets, ml, part, gml, gpart, total;
  size_t n_tickets;  // ticket words in use
};

WsLayout ws_layout(int64_t batch, int64_t heads, int64_t kv_heads, int64_t cache_len) {
  const int S = choose_splits(batch, kv_heads, cache_len);
  const int NG = (S + kGroup - 1) / kGroup;
  const size_t slots = (size_t)batch * heads * S;
  const size_t gslots = NG > 1 ? (size_t)batch * heads * NG : 0;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  WsLayout w;
  w.tickets = 0;
  w.n_tickets = (size_t)batch * kv_heads * (NG > 1 ? 1 + NG : 1);
  w.ml = kTicketBytes;
  w.part = w.ml + up(slots * 2 * sizeof(float));
  w.gml = w.part + slots * kD * sizeof(float);
  w.gpart = w.gml + up(gslots * 2 * sizeof(float));
  w.total = w.gpart + gslots * kD * sizeof(float);
  return w;
}

template <int G, int CL>
int launch_cluster(const DecodeParams& p, int64_t batch, cudaStream_t st, bool pdl) {
  constexpr int kClusterCTAs = CL;
  constexpr size_t kClSmemBytes = cl_smem_bytes<CL>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kClusterCTAs, p.Hkv, (unsigned)batch);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kClSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = kClusterCTAs;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_decode_cluster_kernel<G, CL>, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "decode attention (cluster) launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

// Sets the cluster kernels' attributes once; 16-CTA clusters (non-portable) are used when the
// device can keep one resident, else 8.
bool cluster16_ok() {
  static Q35PerDevice<int> ok;
  return ok.get([] {
    cudaFuncSetAttribute(attn_decode_cluster_kernel<4, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)cl_smem_bytes<8>());
    cudaFuncSetAttribute(attn_decode_cluster_kernel<4, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)cl_smem_bytes<16>());
    int fits = 0;
    if (cudaFuncSetAttribute(attn_decode_cluster_kernel<4, 16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16, 1, 1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = cl_smem_bytes<16>();
      cudaLaunchAttribute a;
      a.id = cudaLaunchAttributeClusterDimension;
      a.val.clusterDim.x = 16;
      a.val.clusterDim.y = 1;
      a.val.clusterDim.z = 1;
      cfg.attrs = &a;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, attn_decode_cluster_kernel<4, 16>, &cfg) == cudaSuccess && n > 0) fits = 1;
    }
    cudaGetLastError();  // a refused query leaves no sticky error
    return fits;
  }) == 1;
}

template <bool FUSED>
int launch_decode(DecodeParams p, int64_t batch, int G, void* ws, cudaStream_t st, bool pdl) {
  if (FUSED && G == 4 && p.max_len <= kClMaxRows)
    return cluster16_ok() ? launch_cluster<4, 16>(p, batch, st, pdl) : launch_cluster<4, 8>(p, batch, st, pdl);
  const WsLayout w = ws_layout(batch, p.Hq, p.Hkv, p.max_len);
  if (w.n_tickets * sizeof(unsigned) > kTicketBytes)
    return q35_fail(Q35_ENOTSUP, "decode attention: batch x KV heads too large");
  char* base = static_cast<char*>(ws);
  p.tickets = reinterpret_cast<unsigned*>(base + w.tickets);
  p.part_ml = reinterpret_cast<float*>(base + w.ml);
  p.part = reinterpret_cast<float*>(base + w.part);
  p.group_ml = reinterpret_cast<float*>(base + w.gml);
  p.group_part = reinterpret_cast<float*>(base + w.gpart);
  p.n_bg = (int)(batch * p.Hkv);
  dim3 grid(p.S, p.Hkv, (unsigned)batch);
  static Q35PerDevice<bool> attr;
  attr.get([] {  // two CTAs per SM: the full shared-memory carve-out
    auto set = [](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnDynSmem);
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    };
    set(attn_decode_kernel<1, FUSED>);
    set(attn_decode_kernel<2, FUSED>);
    set(attn_decode_kernel<4, FUSED>);
    return true;
  });
  cudaError_t e;
  switch (G) {
    case 1: e = q35_launch(attn_decode_kernel<1, FUSED>, grid, dim3(kThreads), kAttnDynSmem, st, pdl, p); break;
    case 2: e = q35_launch(attn_decode_kernel<2, FUSED>, grid, dim3(kThreads), kAttnDynSmem, st, pdl, p); break;
    case 4: e = q35_launch(attn_decode_kernel<4, FUSED>, grid, dim3(kThreads), kAttnDynSmem, st, pdl, p); break;
    default: return q35_fail(Q35_ENOTSUP, "decode attention: group size %d unsupported (1, 2, 4)", G);
  }
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "decode attention launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

}  // namespace

extern "C" size_t q35_gqa_decode_workspace_size(int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                                int64_t cache_len) {
  (void)head_dim;
  return ws_layout(batch, heads, kv_heads, cache_len).total;
}

extern "C" int q35_gqa_decode_attention(const void* q, const void* cache_k, const void* cache_v,
                                        const int64_t* valid_length, float scale, void* out, int64_t batch,
                                        int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cache_len,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(q && cache_k && cache_v && valid_length && out && workspace, "gqa_decode_attention: null pointer");
  Q35_REQUIRE(head_dim == kD, "gqa_decode_attention: head dim %lld unsupported (256)", (long long)head_dim);
  Q35_REQUIRE(batch >= 1 && batch <= 64 && kv_heads >= 1 && heads % kv_heads == 0 && cache_len >= 1,
              "gqa_decode_attention: head layout does not match cache");
  Q35_REQUIRE(workspace_bytes >= ws_layout(batch, heads, kv_heads, cache_len).total,
              "gqa_decode_attention: workspace too small");
  DecodeParams p = {};
  p.q_in = (const bf16*)q;
  p.cache_k = (bf16*)cache_k;
  p.cache_v = (bf16*)cache_v;
  p.len = valid_length;
  p.out = (bf16*)out;
  p.Hq = (int)heads;
  p.Hkv = (int)kv_heads;
  p.max_len = (int)cache_len;
  p.S = choose_splits(batch, kv_heads, cache_len);
  p.scale = scale;
  return launch_decode<false>(p, batch, (int)(heads / kv_heads), workspace, (cudaStream_t)stream, false);
}

int q35_attn_decode_launch(const void* packed, const void* q_weight, const void* k_weight, const float* inv_freq,
                           void* cache_k, void* cache_v, const int64_t* cache_len, const int64_t* rope_pos,
                           void* out, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t rotary_dim,
                           int64_t max_len, float eps, void* workspace, cudaStream_t stream, bool pdl) {
  DecodeParams p = {};
  p.packed = (const bf16*)packed;
  p.qw = (const bf16*)q_weight;
  p.kw = (const bf16*)k_weight;
  p.inv_freq = inv_freq;
  p.rope_pos = rope_pos;
  p.cache_k = (bf16*)cache_k;
  p.cache_v = (bf16*)cache_v;
  p.len = cache_len;
  p.out = (bf16*)out;
  p.Hq = (int)q_heads;
  p.Hkv = (int)kv_heads;
  p.max_len = (int)max_len;
  p.S = choose_splits(batch, kv_heads, max_len);
  p.rot = (int)rotary_dim;
  p.scale = 1.0f / sqrtf((float)kD);
  p.eps = eps;
  return launch_decode<true>(p, batch, (int)(q_heads / kv_heads), workspace, stream, pdl);
}

extern "C" size_t q35_attn_decode_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                                 int64_t cache_len) {
  (void)head_dim;
  return ws_layout(batch, q_heads, kv_heads, cache_len).total;
}

extern "C" int q35_attn_decode(const void* packed, const void* q_weight, const void* k_weight, const float* inv_freq,
                               void* cache_k, void* cache_v, const int64_t* cache_len, const int64_t* rope_pos,
                               void* out, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                               int64_t rotary_dim, int64_t max_len, float eps, void* workspace,
                               size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(packed && q_weight && k_weight && inv_freq && cache_k && cache_v && cache_len && rope_pos && out &&
                  workspace,
              "attn_decode: null pointer");
  Q35_REQUIRE(head_dim == kD, "attn_decode: head dim must be 256");
  Q35_REQUIRE(batch >= 1 && batch <= 64 && kv_heads >= 1 && q_heads % kv_heads == 0 && max_len >= 1 &&
                  rotary_dim % 2 == 0 && rotary_dim <= head_dim,
              "attn_decode: bad shape");
  Q35_REQUIRE(workspace_bytes >= ws_layout(batch, q_heads, kv_heads, max_len).total,
              "attn_decode: workspace too small");
  return q35_attn_decode_launch(packed, q_weight, k_weight, inv_freq, cache_k, cache_v, cache_len, rope_pos, out,
                                batch, q_heads, kv_heads, rotary_dim, max_len, eps, workspace, (cudaStream_t)stream,
                                false);
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant: scratch in a file-scope device array instead of a caller workspace.
//
// For callers that cannot allocate device memory at the point of the call — for example code
// running under an allocator that is locked or pool-only, a host thread that must not touch the
// CUDA allocator, or an embedding runtime that hands this library only its inputs and outputs.
// The scratch (split tickets, per-split maxima/sums and partial outputs) lives in
// `g_gqa_noalloc_scratch`, kQ35NoAllocScratchBytes bytes that every GPU loading this library
// holds until the process exits. Host code may not pass the array's name to a kernel (on the host
// it is only a stand-in symbol): its device address is looked up with cudaGetSymbolAddress once per
// device, with that device current, by the first call made on that device.
constexpr size_t kQ35NoAllocScratchBytes = 2u << 20;  // 2 MiB

static __device__ __align__(256) unsigned char g_gqa_noalloc_scratch[kQ35NoAllocScratchBytes];

#include <mutex>

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {};  // device address of the scratch array, per device ordinal
}  // namespace

extern "C" size_t q35_gqa_decode_noalloc_max_bytes(void) { return kQ35NoAllocScratchBytes; }

extern "C" int q35_gqa_decode_attention_noalloc(const void* q, const void* cache_k, const void* cache_v,
                                                const int64_t* valid_length, float scale, void* out,
                                                int64_t batch, int64_t heads, int64_t kv_heads,
                                                int64_t head_dim, int64_t cache_len, void* stream) {
  Q35_REQUIRE(q && cache_k && cache_v && valid_length && out, "gqa_decode_attention_noalloc: null pointer");
  Q35_REQUIRE(head_dim == kD, "gqa_decode_attention_noalloc: head dim %lld unsupported (256)", (long long)head_dim);
  Q35_REQUIRE(batch >= 1 && batch <= 64 && kv_heads >= 1 && heads % kv_heads == 0 && cache_len >= 1,
              "gqa_decode_attention_noalloc: head layout does not match cache");
  const WsLayout w = ws_layout(batch, heads, kv_heads, cache_len);
  Q35_REQUIRE(w.total <= kQ35NoAllocScratchBytes,
              "gqa_decode_attention_noalloc: this shape needs %zu bytes of scratch, more than the %zu-byte "
              "static maximum (use q35_gqa_decode_attention with a workspace)",
              w.total, kQ35NoAllocScratchBytes);
  Q35_REQUIRE(w.n_tickets * sizeof(unsigned) <= kTicketBytes,
              "gqa_decode_attention_noalloc: batch x kv_heads = %lld needs %zu ticket words, more than the %zu of "
              "the scratch",
              (long long)(batch * kv_heads), w.n_tickets, kTicketBytes / sizeof(unsigned));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return q35_fail(Q35_ECUDA, "gqa_decode_attention_noalloc: no current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
      const cudaError_t e = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_gqa_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_ptr[dev] = nullptr;
        return q35_fail(Q35_ECUDA, "gqa_decode_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      }
    }
    scratch = g_noalloc_ptr[dev];
  }
  // The ticket words must start at zero; the kernel leaves them zero, but a call cut short by an
  // error would not, so clear them on every call (a memset, not an allocation).
  if (cudaMemsetAsync(scratch, 0, w.ml, (cudaStream_t)stream) != cudaSuccess)
    return q35_fail(Q35_ECUDA, "gqa_decode_attention_noalloc: clearing the tickets failed");
  DecodeParams p = {};
  p.q_in = (const bf16*)q;
  p.cache_k = (bf16*)cache_k;
  p.cache_v = (bf16*)cache_v;
  p.len = valid_length;
  p.out = (bf16*)out;
  p.Hq = (int)heads;
  p.Hkv = (int)kv_heads;
  p.max_len = (int)cache_len;
  p.S = choose_splits(batch, kv_heads, cache_len);
  p.scale = scale;
  return launch_decode<false>(p, batch, (int)(heads / kv_heads), scratch, (cudaStream_t)stream, false);
}
