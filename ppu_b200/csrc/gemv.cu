// Batch-1 decode GEMVs and the fused LM-head top-1 (reference: kernels.py:183-263, 1093-1185;
// F.linear at integration.py:183-185, 245, 272, 298, 359).
//
// Design (HBM-bound weight streaming, no tensor cores):
//  * one warp owns U output units per iteration; each lane streams 16-byte chunks of the unit's
//    weight row(s) with ld.global.nc.L1::no_allocate, so a warp keeps U*rows*K*esize bytes in
//    flight; the first group's loads are issued before the prologue (and before the PDL wait),
//    later groups are prefetched before the reduction of the current one;
//  * the prologue builds the input vector in shared memory: plain copy, RMSNorm(1+w) of the
//    residual (folding the reference's residual_add_rms_norm into the consumer), or embedding
//    gather + RMSNorm; for A8W8 it also quantises the vector per token to int8;
//  * BF16 dot products accumulate in FP32; int8 dot products use dp4a with exact int32
//    accumulation and an exact integer warp reduction;
//  * epilogues: store, in-place residual add (bf16(r + bf16(y))), SwiGLU over row pairs
//    (n, n + n_out), or top-1 with a packed 64-bit (value, index) atomicMax and a last-CTA
//    finish that writes the token and re-zeroes the workspace.
#include <cfloat>

#include "common.cuh"

using namespace q35;

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct GemvParams {
  const void* weight;
  const float* w_scale;
  const bf16* input;
  const bf16* norm_w;
  const int64_t* token;
  const bf16* embed;
  bf16* resid;
  bf16* out;
  int n_out;
  int k;       // runtime K (generic kernel)
  int vocab;   // embedding rows (EMBED prologue clamp)
  float eps;
};

// ---------------------------------------------------------------------------------------------
// Prologue: x (bf16, [k]) into shared memory, optional per-token int8 quantisation.
template <int PRO, bool INT8>
Q35_DEV void build_input(const GemvParams& p, int k, bf16* xs, int8_t* xq, float* sx_out,
                         float* red) {
  const bf16* src = p.input;
  if (PRO == Q35_PRO_EMBED) {
    int64_t t = *p.token;
    t = t < 0 ? 0 : (t >= p.vocab ? p.vocab - 1 : t);
    src = p.embed + t * (int64_t)k;
  }
  const int nv = k >> 3;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    const uint4 v = reinterpret_cast<const uint4*>(src)[i];
    if (PRO == Q35_PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid)[i] = v;
    reinterpret_cast<uint4*>(xs)[i] = v;
    if (PRO != Q35_PRO_PLAIN) {
      float f[8];
      unpack_bf16x8(v, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  if (PRO != Q35_PRO_PLAIN) {
    const float var = block_sum<kWarps>(ss, red) / (float)k;
    const float r = rsqrt_ieee(var + p.eps);
    for (int i = threadIdx.x; i < nv; i += kThreads) {
      float f[8], w[8];
      unpack_bf16x8(reinterpret_cast<const uint4*>(xs)[i], f);
      unpack_bf16x8(reinterpret_cast<const uint4*>(p.norm_w)[i], w);
      __align__(16) bf16 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = f2bf(f[j] * r * (1.0f + w[j]));
      reinterpret_cast<uint4*>(xs)[i] = *reinterpret_cast<const uint4*>(o);
    }
  }
  if (INT8) {
    __syncthreads();
    float amax = 0.f;
    for (int i = threadIdx.x; i < k; i += kThreads) amax = fmaxf(amax, fabsf(bf2f(xs[i])));
    amax = block_max<kWarps>(amax, red);
    const float inv = tok_inv(amax);
    for (int i = threadIdx.x; i < k; i += kThreads) xq[i] = (int8_t)quant_i8_tok(bf2f(xs[i]), inv);
    if (threadIdx.x == 0) *sx_out = tok_scale(amax);
  }
  __syncthreads();
}

// Int8 prologue at compile-time K (fast kernels; A8W8 decode 1236 -> 1308 tok/s against the
// shared-memory passes of build_input): each thread keeps its 16-byte chunks
// (threadIdx.x + j * kThreads) in registers through the norm, the absolute maximum and the
// quantisation, so no pass re-reads shared memory and the maximum needs no barrier of its own
// beyond block_max. Values, scale and codes equal build_input's: the same expressions in the
// same order per element, and the maximum does not depend on the order it is taken in.
template <int PRO, int K>
Q35_DEV void build_input_q8(const GemvParams& p, int8_t* xq, float* sx_out, float* red,
                            const uint4 (&nwr)[(K / 8 + kThreads - 1) / kThreads]) {
  constexpr int NV = K / 8, CPT = (NV + kThreads - 1) / kThreads;
  const bf16* src = p.input;
  if (PRO == Q35_PRO_EMBED) {
    int64_t t = *p.token;
    t = t < 0 ? 0 : (t >= p.vocab ? p.vocab - 1 : t);
    src = p.embed + t * (int64_t)K;
  }
  float f[CPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < NV) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      if (PRO == Q35_PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid)[i] = v;
      unpack_bf16x8(v, f[j]);
      if (PRO != Q35_PRO_PLAIN) {
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[j][e] * f[j][e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[j][e] = 0.f;
    }
  }
  if (PRO != Q35_PRO_PLAIN) {
    const float var = block_sum<kWarps>(ss, red) / (float)K;
    const float r = rsqrt_ieee(var + p.eps);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      if (i < NV) {
        float w[8];
        unpack_bf16x8(nwr[j], w);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[j][e] = bf2f(f2bf(f[j][e] * r * (1.0f + w[e])));
      }
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[j][e]));
  amax = block_max<kWarps>(amax, red);
  const float inv = tok_inv(amax);
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < NV) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        lo |= (uint32_t)(quant_i8_tok(f[j][e], inv) & 0xff) << (8 * e);
        hi |= (uint32_t)(quant_i8_tok(f[j][4 + e], inv) & 0xff) << (8 * e);
      }
      reinterpret_cast<uint2*>(xq)[i] = make_uint2(lo, hi);
    }
  }
  if (threadIdx.x == 0) *sx_out = tok_scale(amax);
  __syncthreads();
}

// Bf16 prologue at compile-time K: the norm weights arrive in registers, loaded before the PDL
// wait (they are constants), so the only load after the wait is the input vector itself; each
// thread keeps its chunks in registers between the sum of squares and the scaling. Values equal
// build_input's: the same per-thread order of the sum, the same block_sum, the same expression.
template <int PRO, int K>
Q35_DEV void build_input_bf16(const GemvParams& p, bf16* xs, float* red, const uint4 (&nwr)[(K / 8 + kThreads - 1) / kThreads]) {
  constexpr int NV = K / 8, CPT = (NV + kThreads - 1) / kThreads;
  const bf16* src = p.input;
  if (PRO == Q35_PRO_EMBED) {
    int64_t t = *p.token;
    t = t < 0 ? 0 : (t >= p.vocab ? p.vocab - 1 : t);
    src = p.embed + t * (int64_t)K;
  }
  uint4 v[CPT];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < NV) v[j] = reinterpret_cast<const uint4*>(src)[i];
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < NV) {
      if (PRO == Q35_PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid)[i] = v[j];
      if (PRO == Q35_PRO_PLAIN) {
        reinterpret_cast<uint4*>(xs)[i] = v[j];
      } else {
        float f[8];
        unpack_bf16x8(v[j], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
    }
  }
  if (PRO != Q35_PRO_PLAIN) {
    const float var = block_sum<kWarps>(ss, red) / (float)K;
    const float r = rsqrt_ieee(var + p.eps);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      if (i < NV) {
        float f[8], w[8];
        unpack_bf16x8(v[j], f);
        unpack_bf16x8(nwr[j], w);
        __align__(16) bf16 o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = f2bf(f[e] * r * (1.0f + w[e]));
        reinterpret_cast<uint4*>(xs)[i] = *reinterpret_cast<const uint4*>(o);
      }
    }
  }
  __syncthreads();
}

Q35_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int EPI, bool INT8>
Q35_DEV void epilogue(const GemvParams& p, int unit, float y0, float y1) {
  // y0/y1: dequantised (or fp32) results for rows unit / unit + n_out.
  if (EPI == Q35_EPI_STORE) {
    p.out[unit] = f2bf(y0);
  } else if (EPI == Q35_EPI_RESIDUAL) {
    p.resid[unit] = f2bf(bf2f(p.resid[unit]) + rbf(y0));
  } else {
    const float g = rbf(y0), u = rbf(y1);
    p.out[unit] = f2bf(rbf(silu_f(g)) * u);
  }
}

// ---------------------------------------------------------------------------------------------
// Fast path: compile-time K. A warp's unit group is streamed in SEG segments of CHS 16-byte
// chunks per lane (4 or 8 chunks = 16 or 32 registers per segment buffer), double-buffered: while
// segment i is consumed, segment i+1 is in flight, and segment i+2 is issued right after.
template <int K, bool INT8, int RPU>
struct FastShape {
  static constexpr int ES = INT8 ? 1 : 2;
  static constexpr int CHT = K * ES / 512;                       // chunks per row per lane
  // 16-byte chunks per lane per segment buffer. 8 where a unit is long (bf16 K = 6144, int8
  // K = 6144, int8 gate/up pairs): two wide segments in flight, issued before the PDL wait, start
  // the stream while the previous kernel drains (bf16 decode 999 -> 1049 tok/s, A8W8 1156 -> 1240);
  // 4 elsewhere (8 spills the bf16 gate/up pair kernel and slowed it; int8 in/out projections at
  // 8, two rows per warp group, went 1242 -> 1219 tok/s)
  static constexpr int BUDGET = (K * ES >= 6144 || (INT8 && RPU == 2)) ? 8 : 4;
  static constexpr int SEG = (RPU * CHT > BUDGET) ? (RPU * CHT + BUDGET - 1) / BUDGET : 1;
  static constexpr int CHS = CHT / SEG;                          // chunks per segment
  static constexpr int U = (SEG == 1) ? ((BUDGET / (RPU * CHT)) < 1 ? 1 : BUDGET / (RPU * CHT)) : 1;
  // bf16: segments 2 .. 2 + PRE - 1 of a warp's stream are copied into shared memory with
  // cp.async before the PDL wait, next to the two register buffers: 4 KB more per warp in flight
  // while the previous kernel drains, at no register cost (decode 1052 -> 1098 tok/s; 2 KB per
  // warp gave 1077, 8 KB 1041). Not for int8, where it measured slower (A8W8 1244 -> 1128).
  static constexpr int SEG_BYTES = U * RPU * CHS * 512;          // one segment of one warp
  static constexpr int PRE = INT8 ? 0 : 4096 / SEG_BYTES;
  static_assert(K * ES % 512 == 0, "K must fill whole warp-wide 16-byte chunks");
  static_assert(CHT % SEG == 0, "segments must split a row evenly");
};

template <int K, int PRO, int EPI, bool INT8>
__global__ void __launch_bounds__(kThreads, 2) gemv_fast_kernel(GemvParams p) {
  constexpr int RPU = (EPI == Q35_EPI_SWIGLU) ? 2 : 1;
  using Sh = FastShape<K, INT8, RPU>;
  constexpr int ES = Sh::ES, SEG = Sh::SEG, CHS = Sh::CHS, U = Sh::U, PRE = Sh::PRE;
  constexpr int SEGV = U * RPU * CHS;  // 16-byte chunks per lane per segment
  __shared__ __align__(16) bf16 xs[INT8 ? 8 : K];  // int8 kernels keep only the codes
  __shared__ __align__(16) int8_t xq[INT8 ? K : 16];
  __shared__ __align__(16) uint4 pre_s[PRE > 0 ? kWarps * PRE * SEGV * 32 : 1];
  __shared__ float red[kWarps];
  __shared__ float sx_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = p.n_out;
  const int ngroups = (n_out + U - 1) / U;
  const int gstride = gridDim.x * kWarps;
  const int g0 = blockIdx.x * kWarps + warp;
  const int n_iter = (g0 < ngroups) ? ((ngroups - 1 - g0) / gstride + 1) * SEG : 0;
  const char* W = static_cast<const char*>(p.weight);

  // two segment buffers per lane: segment it + 1 is in flight while segment it is consumed, and
  // segment it + 2 is issued as soon as it's buffer frees up
  uint4 wa[U][RPU][CHS], wb[U][RPU][CHS];
  auto load = [&](uint4 (&wr)[U][RPU][CHS], int it) {
    const int grp = g0 + (it / SEG) * gstride, seg = it % SEG;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int unit = grp * U + u;
#pragma unroll
      for (int r = 0; r < RPU; ++r) {
        const int64_t row = unit + (int64_t)r * n_out;
        const char* base = W + row * (int64_t)(K * ES) + (seg * CHS * 32 + lane) * 16;
#pragma unroll
        for (int c = 0; c < CHS; ++c)
          wr[u][r][c] = (unit < n_out) ? ld_stream(base + c * 512) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  // staged segment q (stream segment 2 + q): lane-interleaved 16-byte slots, so each lane reads
  // back exactly the chunks it copied (no cross-lane dependence; a cp.async wait suffices)
  uint4* pre_w = pre_s + warp * PRE * SEGV * 32 + lane;
  auto stage = [&](int it, int q) {
    const int grp = g0 + (it / SEG) * gstride, seg = it % SEG;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int unit = grp * U + u;
      if (unit >= n_out) continue;
#pragma unroll
      for (int r = 0; r < RPU; ++r) {
        const int64_t row = unit + (int64_t)r * n_out;
        const char* base = W + row * (int64_t)(K * ES) + (seg * CHS * 32 + lane) * 16;
#pragma unroll
        for (int c = 0; c < CHS; ++c) {
          const uint32_t dst = (uint32_t)__cvta_generic_to_shared(pre_w + ((q * U + u) * RPU * CHS + r * CHS + c) * 32);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(base + c * 512) : "memory");
        }
      }
    }
  };
  auto load_staged = [&](uint4 (&wr)[U][RPU][CHS], int it, int q) {
    const int grp = g0 + (it / SEG) * gstride;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int unit = grp * U + u;
#pragma unroll
      for (int r = 0; r < RPU; ++r)
#pragma unroll
        for (int c = 0; c < CHS; ++c)
          wr[u][r][c] = (unit < n_out) ? pre_w[((q * U + u) * RPU * CHS + r * CHS + c) * 32] : make_uint4(0, 0, 0, 0);
    }
  };
  if (n_iter > 0) load(wa, 0);
  if (n_iter > 1) load(wb, 1);
#pragma unroll
  for (int q = 0; q < PRE; ++q)
    if (2 + q < n_iter) stage(2 + q, q);
  asm volatile("cp.async.commit_group;" ::: "memory");
  constexpr int NCPT = (K / 8 + kThreads - 1) / kThreads;
  uint4 nwr[NCPT];  // norm weights: constants, in registers before the wait
  if (PRO != Q35_PRO_PLAIN) {
#pragma unroll
    for (int j = 0; j < NCPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      nwr[j] = i < K / 8 ? reinterpret_cast<const uint4*>(p.norm_w)[i] : make_uint4(0, 0, 0, 0);
    }
  }
  // int8: the per-row weight scales (constants) of the warp's first SROUNDS rounds, read before
  // the wait, one per lane: lane (round * U + u) * RPU + r holds row (unit u, r) of that round.
  // Read at the tail instead, each scale was a dependent load from HBM (the token's weight
  // stream evicts it from L2) after the warp's last dot product.
  constexpr int SPR = U * RPU, SROUNDS = 32 / SPR;
  float wsc = 0.f;
  if (INT8) {
    const int rnd = lane / SPR, u = (lane % SPR) / RPU, r = lane % RPU;
    const int grp = g0 + rnd * gstride, unit = grp * U + u;
    if (rnd < SROUNDS && grp < ngroups && unit < n_out) wsc = p.w_scale[unit + (int64_t)r * n_out];
  }
  pdl_wait();
  pdl_launch_dependents();
  // residual epilogue: this warp's first-round residual values, read now (the producers are
  // done) so that the epilogue's read-modify-write does not wait on L2 at the kernel's tail
  float rpre[U];
  if (EPI == Q35_EPI_RESIDUAL && lane == 0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int unit = g0 * U + u;
      rpre[u] = (g0 < ngroups && unit < n_out) ? bf2f(p.resid[unit]) : 0.f;
    }
  }
  if constexpr (INT8)
    build_input_q8<PRO, K>(p, xq, &sx_s, red, nwr);
  else
    build_input_bf16<PRO, K>(p, xs, red, nwr);
  const float sx = INT8 ? sx_s : 1.0f;

  float accf[U][RPU];
  int acci[U][RPU];
  auto step = [&](uint4 (&wr)[U][RPU][CHS], int it) {
    const int seg = it % SEG;
    const int g = g0 + (it / SEG) * gstride;
    if (seg == 0) {
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < RPU; ++r) {
          accf[u][r] = 0.f;
          acci[u][r] = 0;
        }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < RPU; ++r) {
#pragma unroll
        for (int c = 0; c < CHS; ++c) {
          const int xi = (seg * CHS + c) * 32 + lane;
          if (INT8)
            acci[u][r] = dot_i8x16(wr[u][r][c], reinterpret_cast<const uint4*>(xq)[xi], acci[u][r]);
          else
            accf[u][r] = dot_bf16x8(wr[u][r][c], reinterpret_cast<const uint4*>(xs)[xi], accf[u][r]);
        }
      }
    if (it + 2 < n_iter) {
      if (it < PRE) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        load_staged(wr, it + 2, it);
      } else {
        load(wr, it + 2);
      }
    }
    if (seg != SEG - 1) return;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int unit = g * U + u;
      float y[RPU];
#pragma unroll
      for (int r = 0; r < RPU; ++r) {
        if (INT8) {
          const int tot = warp_sum_i(acci[u][r]);
          const int64_t row = unit + (int64_t)r * n_out;
          const int rnd = it / SEG;  // warp-uniform
          const float sc = rnd < SROUNDS ? __shfl_sync(0xffffffffu, wsc, (rnd * U + u) * RPU + r)
                                         : ((unit < n_out) ? p.w_scale[row] : 0.f);
          y[r] = ((float)tot * sx) * sc;
        } else {
          y[r] = warp_sum(accf[u][r]);
        }
      }
      if (lane == 0 && unit < n_out) {
        if (EPI == Q35_EPI_RESIDUAL && it < SEG)  // first round: the residual read before the prologue
          p.resid[unit] = f2bf(rpre[u] + rbf(y[0]));
        else
          epilogue<EPI, INT8>(p, unit, y[0], RPU > 1 ? y[RPU - 1] : 0.f);
      }
    }
  };
  for (int it = 0; it < n_iter; it += 2) {
    step(wa, it);
    if (it + 1 < n_iter) step(wb, it + 1);
  }
}

// ---------------------------------------------------------------------------------------------
// Generic path: runtime K (multiple of 8, or of 16 for int8); x in dynamic shared memory.
template <int PRO, int EPI, bool INT8>
__global__ void __launch_bounds__(kThreads) gemv_any_kernel(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[kWarps];
  __shared__ float sx_s;
  const int k = p.k;
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);
  int8_t* xq = reinterpret_cast<int8_t*>(smem_raw + ((2 * k + 15) & ~15));
  pdl_wait();
  pdl_launch_dependents();
  build_input<PRO, INT8>(p, k, xs, xq, &sx_s, red);
  const float sx = INT8 ? sx_s : 1.0f;
  constexpr int RPU = (EPI == Q35_EPI_SWIGLU) ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int unit = blockIdx.x * kWarps + warp; unit < p.n_out; unit += gridDim.x * kWarps) {
    float y[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < RPU; ++r) {
      const int64_t row = unit + (int64_t)r * p.n_out;
      if (INT8) {
        const int8_t* wrow = static_cast<const int8_t*>(p.weight) + row * k;
        int a = 0;
        for (int c = lane; c < k / 16; c += 32)
          a = dot_i8x16(ld_stream(wrow + 16 * c), reinterpret_cast<const uint4*>(xq)[c], a);
        y[r] = ((float)warp_sum_i(a) * sx) * p.w_scale[row];
      } else {
        const bf16* wrow = static_cast<const bf16*>(p.weight) + row * k;
        float a = 0.f;
        for (int c = lane; c < k / 8; c += 32)
          a = dot_bf16x8(ld_stream(wrow + 8 * c), reinterpret_cast<const uint4*>(xs)[c], a);
        y[r] = warp_sum(a);
      }
    }
    if (lane == 0) epilogue<EPI, INT8>(p, unit, y[0], y[1]);
  }
}

// ---------------------------------------------------------------------------------------------
// LM head: GEMV over the tied embedding with a fused greedy top-1 (kernels.py:1093-1185).
struct LmWorkspace {
  unsigned long long key;
  unsigned int count;
  unsigned int pad;
};

struct LmParams {
  q35_step_counters adv;  // optional: advanced by the last CTA after the token is written
  const bf16* hidden;
  const bf16* norm_w;  // nullptr: hidden is already normalised
  const bf16* weight;
  int64_t* token_out;
  LmWorkspace* ws;
  int vocab;
  int k;
  float eps;
};

Q35_DEV unsigned long long top1_key(float v, int idx) {
  return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// The step counters the finish advances, read by thread 0 before the PDL wait: only the previous
// step's finish (or the host, before the step) writes them, so the finish stores instead of three
// dependent read-modify-writes at the step's tail.
struct LmCounters {
  int64_t len = 0, pos = 0, log_pos = 0;
};
Q35_DEV LmCounters lm_counters_preload(const LmParams& p) {
  LmCounters c;
  if (threadIdx.x == 0) {
    if (p.adv.cache_len) c.len = *p.adv.cache_len;
    if (p.adv.rope_pos) c.pos = *p.adv.rope_pos;
    if (p.adv.token_log && p.adv.log_pos && p.adv.log_len > 0) c.log_pos = *p.adv.log_pos;
  }
  return c;
}

Q35_DEV void lm_finish(const LmParams& p, float best_v, int best_i, float* red_v, int* red_i, const LmCounters& pre) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_v[warp] = best_v;
    red_i[warp] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bv = red_v[0];
    int bi = red_i[0];
    for (int w = 1; w < kWarps; ++w)
      if (red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi)) {
        bv = red_v[w];
        bi = red_i[w];
      }
    if (bi != 0x7fffffff) atomicMax(&p.ws->key, top1_key(bv, bi));
    __threadfence();
    const unsigned prev = atomicAdd(&p.ws->count, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      const unsigned long long key = atomicExch(&p.ws->key, 0ull);
      atomicExch(&p.ws->count, 0u);
      const int64_t tok = (key == 0ull) ? 0 : (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
      p.token_out[0] = tok;
      if (p.adv.cache_len) *p.adv.cache_len = pre.len + 1;
      if (p.adv.rope_pos) *p.adv.rope_pos = pre.pos + 1;
      if (p.adv.token_log && p.adv.log_pos && p.adv.log_len > 0) {
        p.adv.token_log[pre.log_pos % p.adv.log_len] = tok;
        *p.adv.log_pos = pre.log_pos + 1;
      }
    }
  }
}

// RING: the weight stream goes through a per-warp ring of kLmStages row groups in dynamic shared
// memory, filled by cp.async (each lane copies, and later reads back, only its own 16-byte chunks,
// so the lane's own cp.async.wait_group orders its reads); the first kLmStages groups are
// requested before the PDL wait and each consumed stage is refilled with the group kLmStages
// ahead, so a warp keeps 24 KB in flight. Without RING a warp holds one group in registers and
// requests the next after its dot products (0.94 of the measured copy bandwidth). The arithmetic
// is the same in both forms. Measured per engine precision: the bf16 decode step 1154 -> 1163
// tok/s with the ring; the int8 engine 1524 -> 1520 (its smaller projections leave room for the
// 42-register ring kernel to start beside the last down projection and compete with its tail),
// so int8 engines keep the register form.
constexpr int kLmStages = 3;
template <int K>
constexpr size_t lm_ring_bytes() {
  return (size_t)kWarps * kLmStages * (16 / (K * 2 / 512) < 1 ? 1 : 16 / (K * 2 / 512)) * (K * 2 / 512) * 32 * 16;
}

template <int K, bool NORM, bool RING>
__global__ void __launch_bounds__(kThreads) lm_head_fast_kernel(LmParams p) {
  constexpr int CH = K * 2 / 512;
  constexpr int U = 16 / CH < 1 ? 1 : 16 / CH;  // two rows of 2048 per warp group
  constexpr int SLOTS = U * CH;                 // 16-byte chunks per lane per group
  extern __shared__ __align__(16) uint4 lm_ring[];
  __shared__ __align__(16) bf16 xs[K];
  __shared__ float red[kWarps];
  __shared__ float red_v[kWarps];
  __shared__ int red_i[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = (p.vocab + U - 1) / U;
  const int gstride = gridDim.x * kWarps;
  int g = blockIdx.x * kWarps + warp;
  const char* W = reinterpret_cast<const char*>(p.weight);
  uint4* ring = lm_ring + warp * (kLmStages * SLOTS * 32) + lane;
  uint4 wr[RING ? 1 : U][RING ? 1 : CH];  // register form: the current group
  auto load_group = [&](int grp) {
    if constexpr (!RING) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = grp * U + u;
        const char* base = W + (int64_t)row * (K * 2) + lane * 16;
#pragma unroll
        for (int c = 0; c < CH; ++c)
          wr[u][c] = (row < p.vocab) ? ld_stream(base + c * 512) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  // ring form: group grp into stage st; one commit group per call, empty past the end, so that
  // wait_group(kLmStages - 1) always means "the oldest stage has landed"
  auto issue = [&](int grp, int st) {
    if (grp < ngroups) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = grp * U + u;
        if (row >= p.vocab) continue;
        const char* base = W + (int64_t)row * (K * 2) + lane * 16;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const uint32_t dst = (uint32_t)__cvta_generic_to_shared(ring + (st * SLOTS + u * CH + c) * 32);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(base + c * 512) : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if constexpr (RING) {
#pragma unroll
    for (int st = 0; st < kLmStages; ++st) issue(g + st * gstride, st);
  } else {
    if (g < ngroups) load_group(g);
  }
  const LmCounters pre = lm_counters_preload(p);
  constexpr int NCPT = (K / 8 + kThreads - 1) / kThreads;
  uint4 nwr[NCPT];  // final-norm weights: constants, in registers before the wait
  if (NORM) {
#pragma unroll
    for (int j = 0; j < NCPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      nwr[j] = i < K / 8 ? reinterpret_cast<const uint4*>(p.norm_w)[i] : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  {
    GemvParams gp = {};
    gp.input = p.hidden;
    gp.norm_w = p.norm_w;
    gp.eps = p.eps;
    if (NORM)
      build_input_bf16<Q35_PRO_NORM, K>(gp, xs, red, nwr);
    else
      build_input_bf16<Q35_PRO_PLAIN, K>(gp, xs, red, nwr);
  }
  float best_v = -FLT_MAX;
  int best_i = 0x7fffffff;
  int st = 0;
  for (; g < ngroups; g += gstride) {
    float acc[U];
    if constexpr (RING) {
      asm volatile("cp.async.wait_group %0;" ::"n"(kLmStages - 1) : "memory");
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float a = 0.f;
#pragma unroll
        for (int c = 0; c < CH; ++c)
          a = dot_bf16x8(ring[(st * SLOTS + u * CH + c) * 32], reinterpret_cast<const uint4*>(xs)[lane + 32 * c], a);
        acc[u] = a;
      }
      issue(g + kLmStages * gstride, st);  // the stage's values are in acc: refill it
      st = st + 1 == kLmStages ? 0 : st + 1;
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float a = 0.f;
#pragma unroll
        for (int c = 0; c < CH; ++c)
          a = dot_bf16x8(wr[u][c], reinterpret_cast<const uint4*>(xs)[lane + 32 * c], a);
        acc[u] = a;
      }
      const int gn = g + gstride;
      if (gn < ngroups) load_group(gn);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float v = rbf(warp_sum(acc[u]));  // eager materialises BF16 logits (kernels.py:1119-1121)
      const int row = g * U + u;
      if (row < p.vocab && v > best_v) {
        best_v = v;
        best_i = row;
      }
    }
  }
  if constexpr (RING) asm volatile("cp.async.wait_all;" ::: "memory");
  lm_finish(p, best_v, best_i, red_v, red_i, pre);
}

template <bool NORM>
__global__ void __launch_bounds__(kThreads) lm_head_any_kernel(LmParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[kWarps];
  __shared__ float red_v[kWarps];
  __shared__ int red_i[kWarps];
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const LmCounters pre = lm_counters_preload(p);
  pdl_wait();
  pdl_launch_dependents();
  {
    GemvParams gp = {};
    gp.input = p.hidden;
    gp.norm_w = p.norm_w;
    gp.eps = p.eps;
    if (NORM)
      build_input<Q35_PRO_NORM, false>(gp, p.k, xs, nullptr, nullptr, red);
    else
      build_input<Q35_PRO_PLAIN, false>(gp, p.k, xs, nullptr, nullptr, red);
  }
  float best_v = -FLT_MAX;
  int best_i = 0x7fffffff;
  for (int row = blockIdx.x * kWarps + warp; row < p.vocab; row += gridDim.x * kWarps) {
    const bf16* wrow = p.weight + (int64_t)row * p.k;
    float a = 0.f;
    for (int c = lane; c < p.k / 8; c += 32)
      a = dot_bf16x8(ld_stream(wrow + 8 * c), reinterpret_cast<const uint4*>(xs)[c], a);
    const float v = rbf(warp_sum(a));
    if (v > best_v) {
      best_v = v;
      best_i = row;
    }
  }
  lm_finish(p, best_v, best_i, red_v, red_i, pre);
}

// ---------------------------------------------------------------------------------------------
// Vocab-sharded LM head: the top-1 of N hiddens over one contiguous shard of the tied embedding
// (rows [row_offset, row_offset + rows)), for lock-step decode of N requests with the vocabulary
// split across GPUs. Every logit is bit-identical to lm_head_fast_kernel's (same per-lane chunk
// order, same warp-sum pairing, bf16 rounding as kernels.py:1119-1121), so the reduced shard keys
// give exactly the single-GPU token. Output per request: a signed 64-bit key
//   (order(logit) << 32 | (0xFFFFFFFF - global index)) - 2^63
// whose maximum over ranks (an NCCL all-reduce with MAX on int64) is the largest logit with the
// lowest index on ties; INT64_MIN when the shard is empty.
constexpr int kShardMaxBatch = 8;

struct LmShardWorkspace {
  unsigned long long key[kShardMaxBatch];
  unsigned int count;
  unsigned int pad[3];
};

struct LmShardParams {
  const bf16* hidden;  // [n, K]: final residuals (norm_w set) or normalised hiddens
  const bf16* norm_w;
  const bf16* weight;  // the shard's first row, [rows, K]
  long long* keys_out;
  LmShardWorkspace* ws;
  int n, rows, row_offset;
  float eps;
};

template <int NB>
constexpr size_t lm_shard_smem() {
  return (size_t)NB * 2048 * 4;  // fp32 copies of NB normalised hiddens
}
// Rows a warp streams per iteration: 4 at 8 hiddens halves the shared-memory reads of the hiddens
// per weight byte, 2 otherwise (two CTAs per SM).
template <int NB>
constexpr int lm_shard_rows() {
  return NB >= 8 ? 4 : 2;
}

// Shared-memory layout of the normalised hiddens, built for packed FP32 FMAs over hidden pairs:
// plane q (0..3) of pair p holds, per 16-byte chunk i of the hidden, the float4
//   {x[2p][8i + 2q], x[2p+1][8i + 2q], x[2p][8i + 2q + 1], x[2p+1][8i + 2q + 1]},
// so a lane reads its chunk of a pair as four conflict-free 16-byte loads of ready-made operands.
template <int NB>
Q35_DEV float* lm_shard_slot(float4* xs, int b, int q, int i) {
  constexpr int NC = 2048 / 8;
  return reinterpret_cast<float*>(xs + ((q * (NB / 2) + b / 2) * NC + i)) + (b & 1);
}

// One warp normalises one hidden: lane l holds chunks l + 32 c (c < 8), i.e. lane l of the eight
// warps of build_input's block-wide pass. Per-chunk partial sums, the butterfly (the same pairing
// as those warps' warp_sum) and the in-order sum of the eight warp totals reproduce block_sum
// bit for bit, so the normalised values equal the single-GPU head's.
template <int NB, bool NORM>
Q35_DEV void lm_shard_prologue(const LmShardParams& p, float4* xs, int warp, int lane) {
  constexpr int K = 2048, NC = K / 8, CPL = NC / 32;
  const int b = warp;
  if (b >= NB) return;
  if (b >= p.n) {
#pragma unroll 1
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float* d = lm_shard_slot<NB>(xs, b, q, lane + 32 * c);
        d[0] = 0.f;
        d[2] = 0.f;
      }
    return;
  }
  // the hidden is read twice (the second time from L1 / L2) rather than held in registers next
  // to the weight rows already in flight
  const uint4* src = reinterpret_cast<const uint4*>(p.hidden + (int64_t)b * K);
  float r = 1.0f;
  if (NORM) {
    float part[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float f[8];
      unpack_bf16x8(src[lane + 32 * c], f);
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
      part[c] = ss;
    }
    const float mine = butterfly_sum<CPL>(part, lane);  // lane 4 i: the total of warp i
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) t += __shfl_sync(0xffffffffu, mine, 4 * i);
    const float var = t / (float)K;
    r = rsqrt_ieee(var + p.eps);
  }
#pragma unroll 1
  for (int c = 0; c < CPL; ++c) {
    float f[8];
    unpack_bf16x8(src[lane + 32 * c], f);
    if (NORM) {
      float w[8];
      unpack_bf16x8(reinterpret_cast<const uint4*>(p.norm_w)[lane + 32 * c], w);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = bf2f(f2bf(f[j] * r * (1.0f + w[j])));
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float* d = lm_shard_slot<NB>(xs, b, q, lane + 32 * c);
      d[0] = f[2 * q];
      d[2] = f[2 * q + 1];
    }
  }
}

template <int NB, bool NORM>
__global__ void __launch_bounds__(kThreads, NB >= 8 ? 1 : 2) lm_shard_kernel(LmShardParams p) {
  constexpr int K = 2048;
  constexpr int CH = K * 2 / 512;          // 16-byte chunks per lane per row
  constexpr int U = lm_shard_rows<NB>();   // rows per warp iteration
  constexpr int NP = NB / 2;               // hidden pairs
  constexpr int NV = U * NB;               // dot products reduced together
  constexpr int NC = K / 8;                // chunks per hidden
  static_assert(NB >= 2 && NB % 2 == 0 && NB <= kWarps, "hidden pairs, one warp per hidden in the prologue");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float4* xs = reinterpret_cast<float4*>(smem_raw);
  __shared__ float red_v[kWarps][NV];
  __shared__ int red_i[kWarps][NV];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = (p.rows + U - 1) / U;
  const int gstride = gridDim.x * kWarps;
  int g = blockIdx.x * kWarps + warp;
  const char* W = reinterpret_cast<const char*>(p.weight);
  uint4 wr[U][CH];
  auto load_group = [&](int grp) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int row = grp * U + u;
      const char* base = W + (int64_t)row * (K * 2) + lane * 16;
#pragma unroll
      for (int c = 0; c < CH; ++c)
        wr[u][c] = (row < p.rows) ? ld_stream(base + c * 512) : make_uint4(0, 0, 0, 0);
    }
  };
  if (g < ngroups) load_group(g);
  pdl_wait();
  pdl_launch_dependents();
  lm_shard_prologue<NB, NORM>(p, xs, warp, lane);
  __syncthreads();
  const int my = butterfly_index<NV>(lane);  // the (row u, hidden b) total this lane ends with
  const int my_u = my / NB;
  float best_v = -FLT_MAX;
  int best_i = 0x7fffffff;
  for (; g < ngroups; g += gstride) {
    const int gn = g + gstride;
    float2 acc2[U][NP];  // {row u . hidden 2p, row u . hidden 2p + 1}
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int q = 0; q < NP; ++q) acc2[u][q] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      float w[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) unpack_bf16x8(wr[u][c], w[u]);
      // rolling prefetch: chunk c of the next group goes into the slot just unpacked, so its
      // load overlaps the rest of this group's arithmetic (no second register buffer)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = gn * U + u;
        wr[u][c] = (gn < ngroups && row < p.rows)
                       ? ld_stream(W + (int64_t)row * (K * 2) + lane * 16 + c * 512)
                       : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int pr = 0; pr < NP; ++pr) {
        float2 x[8];  // {hidden 2 pr, hidden 2 pr + 1} at element j of the chunk
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = xs[(q * NP + pr) * NC + lane + 32 * c];
          x[2 * q] = make_float2(v.x, v.y);
          x[2 * q + 1] = make_float2(v.z, v.w);
        }
        // per accumulator the same FMA sequence (chunk by chunk, element by element) as the
        // scalar head; __ffma2_rn rounds each half as one IEEE fma
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc2[u][pr] = __ffma2_rn(make_float2(w[u][j], w[u][j]), x[j], acc2[u][pr]);
      }
      // keeps the shared-memory reads of later chunks from being hoisted here (NB x 8 floats per
      // chunk would otherwise stay live across the whole row and spill)
      asm volatile("" ::: "memory");
    }
    float acc[NV];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        acc[u * NB + 2 * q] = acc2[u][q].x;
        acc[u * NB + 2 * q + 1] = acc2[u][q].y;
      }
    const float v = rbf(butterfly_sum<NV>(acc, lane));
    const int row = g * U + my_u;
    if (row < p.rows && v > best_v) {
      best_v = v;
      best_i = row;
    }
  }
  if (butterfly_writer<NV>(lane)) {
    red_v[warp][my] = best_v;
    red_i[warp][my] = best_i;
  }
  __syncthreads();
  if (threadIdx.x < p.n) {
    const int b = threadIdx.x;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int w = 0; w < kWarps; ++w)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float v = red_v[w][u * NB + b];
        const int i = red_i[w][u * NB + b];
        if (i != 0x7fffffff && (v > bv || (v == bv && i < bi))) {
          bv = v;
          bi = i;
        }
      }
    if (bi != 0x7fffffff) atomicMax(&p.ws->key[b], top1_key(bv, p.row_offset + bi));
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&p.ws->count, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      for (int b = 0; b < p.n; ++b) {
        const unsigned long long key = atomicExch(&p.ws->key[b], 0ull);
        p.keys_out[b] = (long long)(key ^ 0x8000000000000000ull);
      }
      atomicExch(&p.ws->count, 0u);
    }
  }
}

// Token of a reduced shard key (the inverse of the packing above; INT64_MIN -> token 0, as the
// single-GPU head does when no candidate exists), optionally advancing the decoder's counters.
__global__ void lm_keys_finish_kernel(const long long* keys, int n, int64_t* tokens, q35_step_counters adv) {
  pdl_wait();
  pdl_launch_dependents();
  for (int b = threadIdx.x; b < n; b += blockDim.x) {
    const unsigned long long key = (unsigned long long)keys[b] ^ 0x8000000000000000ull;
    tokens[b] = (key == 0ull) ? 0 : (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
  }
  if (threadIdx.x == 0) {
    if (adv.cache_len) *adv.cache_len += 1;
    if (adv.rope_pos) *adv.rope_pos += 1;
    if (adv.token_log && adv.log_pos && adv.log_len > 0) {
      const int64_t pos = *adv.log_pos;
      adv.token_log[pos % adv.log_len] = tokens[0];
      *adv.log_pos = pos + 1;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Grid choice: at most `max_ctas` resident CTAs; among grids of whole-SM multiples pick the one
// whose last round of unit groups is the fullest (less tail imbalance between warps).
int choose_grid(int ngroups, int max_ctas) {
  // Every round of unit groups costs about the same, so the best grid among the resident sizes
  // (at least half of the machine) is the one with the fewest rounds, then the fullest last
  // round, then the most CTAs. E.g. 6144 groups over 296 resident CTAs: 256 CTAs -> 3 full rounds.
  const int need = (ngroups + kWarps - 1) / kWarps;
  if (need <= max_ctas) return need < 1 ? 1 : need;
  int best = max_ctas;
  long best_rounds = 1L << 40;
  double best_eff = 0.0;
  for (int ctas = max_ctas; ctas >= (max_ctas + 1) / 2; --ctas) {
    const long warps = (long)ctas * kWarps;
    const long rounds = (ngroups + warps - 1) / warps;
    const double eff = (double)ngroups / (double)(rounds * warps);
    if (rounds < best_rounds || (rounds == best_rounds && eff > best_eff + 1e-9)) {
      best_rounds = rounds;
      best_eff = eff;
      best = ctas;
    }
  }
  return best;
}

template <typename KernelT>
int resident_ctas(KernelT kernel, size_t dyn_smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, dyn_smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return per_sm * kNumSMs;
}

int g_gemv_ctas_per_sm = 0;  // 0: as many as fit; else cap (room for the next kernel's CTAs under PDL)

template <int K, int PRO, int EPI, bool INT8>
int launch_fast(const GemvParams& p, cudaStream_t s, bool pdl) {
  using Sh = FastShape<K, INT8, (EPI == Q35_EPI_SWIGLU) ? 2 : 1>;
  static Q35PerDevice<int> resident_ctas_of;
  const int resident = resident_ctas_of.get([] { return resident_ctas(gemv_fast_kernel<K, PRO, EPI, INT8>, 0); });
  const int max_ctas = g_gemv_ctas_per_sm > 0 && g_gemv_ctas_per_sm * kNumSMs < resident
                           ? g_gemv_ctas_per_sm * kNumSMs
                           : resident;
  const int ngroups = (p.n_out + Sh::U - 1) / Sh::U;
  const int grid = choose_grid(ngroups, max_ctas);
  cudaError_t e = q35_launch(gemv_fast_kernel<K, PRO, EPI, INT8>, dim3(grid), dim3(kThreads), 0, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

template <int PRO, int EPI, bool INT8>
int launch_any(const GemvParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = ((2 * (size_t)p.k + 15) & ~(size_t)15) + (INT8 ? (size_t)p.k : 0);
  if (smem > 200 * 1024) return q35_fail(Q35_ENOTSUP, "gemv: k=%d too large", p.k);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(gemv_any_kernel<PRO, EPI, INT8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int grid = choose_grid(p.n_out, 2 * kNumSMs);
  cudaError_t e = q35_launch(gemv_any_kernel<PRO, EPI, INT8>, dim3(grid), dim3(kThreads), smem, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

#include "gemv_bulk.cuh"

int g_gemv_variant = Q35_GEMV_REGISTERS;  // measured faster on B200 (see microbench)

template <int PRO, int EPI, bool INT8>
int dispatch_k(const GemvParams& p, cudaStream_t s, bool pdl) {
  const bool bulk = g_gemv_variant == Q35_GEMV_BULK;
  if (p.k == 2048)
    return bulk ? launch_bulk<2048, PRO, EPI, INT8>(p, s, pdl) : launch_fast<2048, PRO, EPI, INT8>(p, s, pdl);
  if constexpr (EPI != Q35_EPI_SWIGLU && PRO == Q35_PRO_PLAIN) {
    if (p.k == 6144)
      return bulk ? launch_bulk<6144, PRO, EPI, INT8>(p, s, pdl) : launch_fast<6144, PRO, EPI, INT8>(p, s, pdl);
  }
  return launch_any<PRO, EPI, INT8>(p, s, pdl);
}

template <int PRO, int EPI>
int dispatch_int8(const GemvParams& p, bool int8, cudaStream_t s, bool pdl) {
  return int8 ? dispatch_k<PRO, EPI, true>(p, s, pdl) : dispatch_k<PRO, EPI, false>(p, s, pdl);
}

template <int PRO>
int dispatch_epi(const GemvParams& p, int epi, bool int8, cudaStream_t s, bool pdl) {
  switch (epi) {
    case Q35_EPI_STORE: return dispatch_int8<PRO, Q35_EPI_STORE>(p, int8, s, pdl);
    case Q35_EPI_RESIDUAL: return dispatch_int8<PRO, Q35_EPI_RESIDUAL>(p, int8, s, pdl);
    case Q35_EPI_SWIGLU: return dispatch_int8<PRO, Q35_EPI_SWIGLU>(p, int8, s, pdl);
  }
  return q35_fail(Q35_EINVAL, "gemv: bad epilogue %d", epi);
}

}  // namespace

// Shared with decoder.cu.
int q35_gemv_launch(const q35_gemv_desc* d, cudaStream_t s, bool pdl) {
  Q35_REQUIRE(d && d->weight, "gemv: null descriptor / weight");
  Q35_REQUIRE(d->n_out > 0 && d->k > 0 && d->k % (d->int8 ? 16 : 8) == 0, "gemv: bad shape n=%lld k=%lld",
              (long long)d->n_out, (long long)d->k);
  Q35_REQUIRE(!d->int8 || d->w_scale, "gemv: int8 weights need w_scale");
  Q35_REQUIRE(Q35_ALIGNED(d->weight, 16), "gemv: weight must be 16-byte aligned");
  Q35_REQUIRE(d->prologue == Q35_PRO_EMBED ? (d->token && d->embed && d->resid_out && d->norm_weight)
                                           : (d->input != nullptr),
              "gemv: prologue inputs missing");
  Q35_REQUIRE(d->prologue != Q35_PRO_NORM || d->norm_weight, "gemv: norm weight missing");
  Q35_REQUIRE(d->epilogue == Q35_EPI_RESIDUAL ? d->resid_out != nullptr : d->out != nullptr,
              "gemv: output missing");
  GemvParams p = {};
  p.weight = d->weight;
  p.w_scale = d->w_scale;
  p.input = static_cast<const bf16*>(d->input);
  p.norm_w = static_cast<const bf16*>(d->norm_weight);
  p.token = d->token;
  p.embed = static_cast<const bf16*>(d->embed);
  p.resid = static_cast<bf16*>(d->resid_out);
  p.out = static_cast<bf16*>(d->out);
  p.n_out = (int)d->n_out;
  p.k = (int)d->k;
  p.vocab = d->vocab > 0 ? (int)d->vocab : (1 << 30);
  p.eps = d->eps;
  const bool int8 = d->int8 != 0;
  switch (d->prologue) {
    case Q35_PRO_PLAIN: return dispatch_epi<Q35_PRO_PLAIN>(p, d->epilogue, int8, s, pdl);
    case Q35_PRO_NORM: return dispatch_epi<Q35_PRO_NORM>(p, d->epilogue, int8, s, pdl);
    case Q35_PRO_EMBED: return dispatch_epi<Q35_PRO_EMBED>(p, d->epilogue, int8, s, pdl);
  }
  return q35_fail(Q35_EINVAL, "gemv: bad prologue %d", d->prologue);
}

int q35_lm_head_launch(const void* hidden, const void* norm_weight, const void* weight,
                       int64_t* token_out, int64_t vocab, int64_t k, float eps, void* ws,
                       cudaStream_t s, bool pdl, const q35_step_counters* adv, bool ring) {
  LmParams p = {};
  if (adv) p.adv = *adv;
  p.hidden = static_cast<const bf16*>(hidden);
  p.norm_w = static_cast<const bf16*>(norm_weight);
  p.weight = static_cast<const bf16*>(weight);
  p.token_out = token_out;
  p.ws = static_cast<LmWorkspace*>(ws);
  p.vocab = (int)vocab;
  p.k = (int)k;
  p.eps = eps;
  cudaError_t e;
  if (k == 2048) {
    const int ngroups = (int)((vocab + 1) / 2);  // two rows per warp iteration at K = 2048
    auto go = [&](auto kern, Q35PerDevice<int>& resident, size_t smem) {
      const int max_ctas = resident.get([&] {
        if (smem > 0) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        return resident_ctas(kern, smem);
      });
      return q35_launch(kern, dim3(choose_grid(ngroups, max_ctas)), dim3(kThreads), smem, s, pdl, p);
    };
    constexpr size_t rb = lm_ring_bytes<2048>();
    static Q35PerDevice<int> res_nr, res_pr, res_n, res_p;
    if (ring)
      e = norm_weight ? go(lm_head_fast_kernel<2048, true, true>, res_nr, rb)
                      : go(lm_head_fast_kernel<2048, false, true>, res_pr, rb);
    else
      e = norm_weight ? go(lm_head_fast_kernel<2048, true, false>, res_n, 0)
                      : go(lm_head_fast_kernel<2048, false, false>, res_p, 0);
  } else {
    const size_t smem = 2 * (size_t)k;
    if (smem > 200 * 1024) return q35_fail(Q35_ENOTSUP, "lm_head: hidden size %lld too large", (long long)k);
    auto kern = norm_weight ? lm_head_any_kernel<true> : lm_head_any_kernel<false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int grid = choose_grid((int)vocab, 2 * kNumSMs);
    e = q35_launch(kern, dim3(grid), dim3(kThreads), smem, s, pdl, p);
  }
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "lm_head launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_set_gemv_variant(int variant) {
  Q35_REQUIRE(variant == Q35_GEMV_BULK || variant == Q35_GEMV_REGISTERS, "gemv variant %d unknown", variant);
  g_gemv_variant = variant;
  return Q35_OK;
}

extern "C" int q35_set_gemv_ctas_per_sm(int ctas) {
  Q35_REQUIRE(ctas >= 0 && ctas <= 32, "gemv CTAs per SM %d out of range", ctas);
  g_gemv_ctas_per_sm = ctas;
  return Q35_OK;
}

extern "C" int q35_gemv_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_gemv_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_gemv_error_word, &zero, sizeof(int));
  return v;
}

extern "C" int q35_gemv(const q35_gemv_desc* d, void* stream) {
  return q35_gemv_launch(d, (cudaStream_t)stream, false);
}

extern "C" int q35_swiglu_gemv(const void* x, const void* packed_weight, void* out, int64_t n_out,
                               int64_t k, void* stream) {
  Q35_REQUIRE(x && packed_weight && out, "swiglu_gemv: null pointer");
  q35_gemv_desc d = {};
  d.weight = packed_weight;
  d.input = x;
  d.out = out;
  d.n_out = n_out;
  d.k = k;
  d.prologue = Q35_PRO_PLAIN;
  d.epilogue = Q35_EPI_SWIGLU;
  return q35_gemv_launch(&d, (cudaStream_t)stream, false);
}

extern "C" size_t q35_lm_head_workspace_size(int64_t batch) {
  return (size_t)(batch < 1 ? 1 : batch) * sizeof(LmWorkspace);
}

extern "C" int q35_lm_head_argmax(const void* hidden, const void* norm_weight, const void* weight,
                                  int64_t* token_out, int64_t batch, int64_t vocab,
                                  int64_t hidden_size, float eps, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(hidden && weight && token_out && workspace, "lm_head_argmax: null pointer");
  Q35_REQUIRE(batch == 1, "lm_head_argmax: batch %lld unsupported (batch 1, as kernels.py:1155)",
              (long long)batch);
  Q35_REQUIRE(vocab > 0 && vocab < (1ll << 31) && hidden_size > 0 && hidden_size % 8 == 0,
              "lm_head_argmax: bad shape");
  Q35_REQUIRE(workspace_bytes >= q35_lm_head_workspace_size(batch), "lm_head_argmax: workspace too small");
  Q35_REQUIRE(Q35_ALIGNED(weight, 16) && Q35_ALIGNED(hidden, 16), "lm_head_argmax: 16-byte alignment");
  return q35_lm_head_launch(hidden, norm_weight, weight, token_out, vocab, hidden_size, eps, workspace,
                            (cudaStream_t)stream, false, nullptr, false);
}

// ---------------------------------------------------------------------------------------------
// Vocab-sharded LM head entry points.
namespace {
template <int NB, bool NORM>
cudaError_t launch_lm_shard(const LmShardParams& p, cudaStream_t s, bool pdl) {
  constexpr size_t smem = lm_shard_smem<NB>();
  static Q35PerDevice<int> resident_of;
  const int resident = resident_of.get([] {
    cudaFuncSetAttribute(lm_shard_kernel<NB, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return resident_ctas(lm_shard_kernel<NB, NORM>, smem);
  });
  constexpr int U = lm_shard_rows<NB>();
  const int ngroups = (p.rows + U - 1) / U;  // U rows per warp iteration
  return q35_launch(lm_shard_kernel<NB, NORM>, dim3(choose_grid(ngroups, resident)), dim3(kThreads), smem, s,
                    pdl, p);
}

template <bool NORM>
cudaError_t dispatch_lm_shard(const LmShardParams& p, cudaStream_t s, bool pdl) {
  if (p.n <= 2) return launch_lm_shard<2, NORM>(p, s, pdl);  // one hidden runs padded to a pair
  if (p.n <= 4) return launch_lm_shard<4, NORM>(p, s, pdl);
  return launch_lm_shard<8, NORM>(p, s, pdl);
}
}  // namespace

int q35_lm_shard_launch(const void* hidden, int64_t batch, const void* norm_weight, const void* weight_shard,
                        int64_t row_offset, int64_t shard_rows, float eps, int64_t* keys_out, void* ws,
                        cudaStream_t s, bool pdl) {
  LmShardParams p = {};
  p.hidden = static_cast<const bf16*>(hidden);
  p.norm_w = static_cast<const bf16*>(norm_weight);
  p.weight = static_cast<const bf16*>(weight_shard);
  p.keys_out = reinterpret_cast<long long*>(keys_out);
  p.ws = static_cast<LmShardWorkspace*>(ws);
  p.n = (int)batch;
  p.rows = (int)shard_rows;
  p.row_offset = (int)row_offset;
  p.eps = eps;
  const cudaError_t e = norm_weight ? dispatch_lm_shard<true>(p, s, pdl) : dispatch_lm_shard<false>(p, s, pdl);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "lm_head_shard launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

int q35_lm_keys_finish_launch(const int64_t* keys, int64_t n, int64_t* tokens, cudaStream_t s, bool pdl,
                              const q35_step_counters* adv) {
  q35_step_counters a = {};
  if (adv) a = *adv;
  const cudaError_t e = q35_launch(lm_keys_finish_kernel, dim3(1), dim3(32), 0, s, pdl,
                                   reinterpret_cast<const long long*>(keys), (int)n, tokens, a);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "lm_keys_finish launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" size_t q35_lm_shard_workspace_size(void) { return sizeof(LmShardWorkspace); }

extern "C" int q35_lm_head_shard_keys(const void* hidden, int64_t batch, const void* norm_weight,
                                      const void* weight_shard, int64_t row_offset, int64_t shard_rows,
                                      int64_t vocab, int64_t hidden_size, float eps, int64_t* keys_out,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(hidden && keys_out && workspace, "lm_head_shard_keys: null pointer");
  Q35_REQUIRE(batch >= 1 && batch <= kShardMaxBatch, "lm_head_shard_keys: batch %lld outside [1, %d]",
              (long long)batch, kShardMaxBatch);
  Q35_REQUIRE(hidden_size == 2048, "lm_head_shard_keys: hidden size %lld unsupported (2048)",
              (long long)hidden_size);
  Q35_REQUIRE(vocab > 0 && vocab < (1ll << 31), "lm_head_shard_keys: bad vocab %lld", (long long)vocab);
  Q35_REQUIRE(row_offset >= 0 && shard_rows >= 0 && row_offset + shard_rows <= vocab,
              "lm_head_shard_keys: shard [%lld, %lld) outside the vocabulary of %lld", (long long)row_offset,
              (long long)(row_offset + shard_rows), (long long)vocab);
  Q35_REQUIRE(shard_rows == 0 || weight_shard, "lm_head_shard_keys: null weight");
  Q35_REQUIRE(workspace_bytes >= q35_lm_shard_workspace_size(), "lm_head_shard_keys: workspace too small");
  Q35_REQUIRE(Q35_ALIGNED(hidden, 16) && (shard_rows == 0 || Q35_ALIGNED(weight_shard, 16)) &&
                  (!norm_weight || Q35_ALIGNED(norm_weight, 16)),
              "lm_head_shard_keys: 16-byte alignment");
  return q35_lm_shard_launch(hidden, batch, norm_weight, weight_shard, row_offset, shard_rows, eps, keys_out,
                             workspace, (cudaStream_t)stream, false);
}

extern "C" int q35_lm_keys_to_tokens(const int64_t* keys, int64_t n, int64_t* tokens_out, void* stream) {
  Q35_REQUIRE(keys && tokens_out, "lm_keys_to_tokens: null pointer");
  Q35_REQUIRE(n >= 1 && n <= 1024, "lm_keys_to_tokens: n %lld outside [1, 1024]", (long long)n);
  return q35_lm_keys_finish_launch(keys, n, tokens_out, (cudaStream_t)stream, false, nullptr);
}
