// Batched decode GEMV: one decode step of up to 8 requests in lock step streams each weight
// matrix once for all of them (the decode projections of integration.py:183-185, 245, 272, 298,
// 359 with a batch of B in-flight requests instead of one).
//
// y[b, n] = W[n, :] . x_b for b < B, with the batch-1 GEMV's fused prologues (RMSNorm of the
// residual, or the embedding gather + RMSNorm at layer 0) and epilogues (store, in-place residual
// add, SwiGLU over gate / up row pairs), computed per request with the same rounding points.
// The weights stream through registers with a rolling prefetch (chunk c of the next row group is
// loaded into the slot chunk c of this group just left); the B input vectors sit in shared memory
// as FP32 pairs so that one packed FMA (__ffma2_rn, one IEEE fma per half) serves two requests.
// CUDA cores only: at B <= 8 the step is still bound by the weight stream.
#include <cfloat>

#include "common.cuh"

using namespace q35;

namespace {

constexpr int kThreads = 256, kWarps = kThreads / 32;

struct BatchGemvParams {
  const bf16* weight;     // [rows, K] (rows = n_out, or 2 n_out for SWIGLU: gate rows, then up rows)
  const bf16* input;      // PLAIN / NORM: [n, K]
  const bf16* norm_w;     // NORM / EMBED: [K] (1 + w)
  const int64_t* token;   // EMBED: [n] token ids
  const bf16* embed;      // EMBED: [vocab, K]
  bf16* resid;            // RESIDUAL: [n, n_out] updated in place; EMBED: receives the raw rows [n, K]
  bf16* out;              // STORE / SWIGLU: [n, n_out]
  int64_t vocab;
  int n, n_out;
  float eps;
};

// Plane q (0..3) of pair p holds, per 16-byte chunk i of a vector, the float4
// {x[2p][8i + 2q], x[2p+1][8i + 2q], x[2p][8i + 2q + 1], x[2p+1][8i + 2q + 1]}.
template <int K, int NB>
Q35_DEV float* slot(float4* xs, int b, int q, int i) {
  return reinterpret_cast<float*>(xs + ((q * (NB / 2) + b / 2) * (K / 8) + i)) + (b & 1);
}

// Warp b builds vector b: PLAIN copies the input row, NORM / EMBED apply RMSNorm(1 + w) with the
// batch-1 prologue's rounding (bf16(x * r * (1 + w))).
template <int K, int NB, int PRO>
Q35_DEV void build_inputs(const BatchGemvParams& p, float4* xs, int warp, int lane) {
  constexpr int CPL = K / 8 / 32;  // 16-byte chunks per lane
  for (int b = warp; b < NB; b += kWarps) {
    if (b >= p.n) {
      for (int c = 0; c < CPL; ++c)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float* d = slot<K, NB>(xs, b, q, lane + 32 * c);
          d[0] = 0.f;
          d[2] = 0.f;
        }
      continue;
    }
    const bf16* row = p.input + (int64_t)b * K;
    if (PRO == Q35_PRO_EMBED) {
      int64_t t = p.token[b];
      t = t < 0 ? 0 : (t >= p.vocab ? p.vocab - 1 : t);
      row = p.embed + t * (int64_t)K;
    }
    const uint4* src = reinterpret_cast<const uint4*>(row);
    float r = 1.f;
    if (PRO != Q35_PRO_PLAIN) {
      float ss = 0.f;
      for (int c = 0; c < CPL; ++c) {
        const uint4 v = src[lane + 32 * c];
        if (PRO == Q35_PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid + (int64_t)b * K)[lane + 32 * c] = v;
        float f[8];
        unpack_bf16x8(v, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
      }
      r = rsqrt_ieee(warp_sum(ss) / (float)K + p.eps);
    }
    for (int c = 0; c < CPL; ++c) {
      float f[8];
      unpack_bf16x8(src[lane + 32 * c], f);
      if (PRO != Q35_PRO_PLAIN) {
        float w[8];
        unpack_bf16x8(reinterpret_cast<const uint4*>(p.norm_w)[lane + 32 * c], w);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = bf2f(f2bf(f[j] * r * (1.0f + w[j])));
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float* d = slot<K, NB>(xs, b, q, lane + 32 * c);
        d[0] = f[2 * q];
        d[2] = f[2 * q + 1];
      }
    }
  }
}

// Rows a warp streams per group: SWIGLU streams a (gate, up) pair; otherwise 2 rows at K = 2048
// and 1 at K = 6144 (24 chunks per lane already).
template <int K, int EPI>
constexpr int rows_per_group() {
  return EPI == Q35_EPI_SWIGLU ? 2 : (K <= 2048 ? 2 : 1);
}

template <int K, int NB, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_batch_kernel(BatchGemvParams p) {
  constexpr int CH = K * 2 / 512;              // 16-byte chunks per lane per row
  constexpr int U = rows_per_group<K, EPI>();  // rows per warp group
  constexpr int UNITS = EPI == Q35_EPI_SWIGLU ? 1 : U;  // output units per group
  constexpr int NP = NB / 2;
  constexpr int NV = U * NB;
  constexpr int NC = K / 8;
  static_assert(NB >= 2 && NB % 2 == 0 && NB <= 8, "request pairs, at most 8 requests");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float4* xs = reinterpret_cast<float4*>(smem_raw);
  __shared__ float tot_s[kWarps][NV];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = p.n_out;
  const int ngroups = (n_out + UNITS - 1) / UNITS;
  const int gstride = gridDim.x * kWarps;
  int g = blockIdx.x * kWarps + warp;
  const char* W = reinterpret_cast<const char*>(p.weight);
  auto row_of = [&](int grp, int u) -> int64_t {
    return EPI == Q35_EPI_SWIGLU ? (int64_t)grp + (int64_t)u * n_out : (int64_t)grp * U + u;
  };
  auto unit_ok = [&](int grp, int u) -> bool {
    return EPI == Q35_EPI_SWIGLU ? grp < n_out : grp * U + u < n_out;
  };
  uint4 wr[U][CH];
  if (g < ngroups) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const char* base = W + row_of(g, u) * (K * 2) + lane * 16;
#pragma unroll
      for (int c = 0; c < CH; ++c) wr[u][c] = unit_ok(g, u) ? ld_stream(base + c * 512) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  build_inputs<K, NB, PRO>(p, xs, warp, lane);
  __syncthreads();
  const int my = butterfly_index<NV>(lane);
  for (; g < ngroups; g += gstride) {
    const int gn = g + gstride;
    float2 acc2[U][NP];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int q = 0; q < NP; ++q) acc2[u][q] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      float w[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) unpack_bf16x8(wr[u][c], w[u]);
#pragma unroll
      for (int u = 0; u < U; ++u)
        wr[u][c] = (gn < ngroups && unit_ok(gn, u)) ? ld_stream(W + row_of(gn, u) * (K * 2) + lane * 16 + c * 512)
                                                    : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int pr = 0; pr < NP; ++pr) {
        float2 x[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = xs[(q * NP + pr) * NC + lane + 32 * c];
          x[2 * q] = make_float2(v.x, v.y);
          x[2 * q + 1] = make_float2(v.z, v.w);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc2[u][pr] = __ffma2_rn(make_float2(w[u][j], w[u][j]), x[j], acc2[u][pr]);
      }
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
    const float v = butterfly_sum<NV>(acc, lane);
    if (butterfly_writer<NV>(lane)) tot_s[warp][my] = v;
    __syncwarp();
    // lane (u, b) applies the epilogue of output unit u for request b
    if (lane < UNITS * NB) {
      const int u = lane / NB, b = lane % NB;
      if (b < p.n && unit_ok(g, u)) {
        if (EPI == Q35_EPI_SWIGLU) {
          const float gt = rbf(tot_s[warp][b]), up = rbf(tot_s[warp][NB + b]);
          p.out[(int64_t)b * n_out + g] = f2bf(rbf(silu_f(gt)) * up);
        } else {
          const int64_t o = (int64_t)b * n_out + g * U + u;
          const float y = tot_s[warp][u * NB + b];
          if (EPI == Q35_EPI_RESIDUAL)
            p.resid[o] = f2bf(bf2f(p.resid[o]) + rbf(y));
          else
            p.out[o] = f2bf(y);
        }
      }
    }
    __syncwarp();
  }
}

template <int K, int NB, int PRO, int EPI>
int launch_nb(const BatchGemvParams& p, cudaStream_t s, bool pdl) {
  constexpr size_t smem = (size_t)NB * K * 4;
  static Q35PerDevice<int> ctas_of;
  const int ctas = ctas_of.get([] {
    cudaFuncSetAttribute(gemv_batch_kernel<K, NB, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_batch_kernel<K, NB, PRO, EPI>, kThreads, smem) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cudaGetLastError();
    return per_sm * kNumSMs;
  });
  constexpr int UNITS = EPI == Q35_EPI_SWIGLU ? 1 : rows_per_group<K, EPI>();
  const int ngroups = (p.n_out + UNITS - 1) / UNITS;
  int grid = (ngroups + kWarps - 1) / kWarps;
  if (grid > ctas) grid = ctas;
  const cudaError_t e = q35_launch(gemv_batch_kernel<K, NB, PRO, EPI>, dim3(grid), dim3(kThreads), smem, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "batched gemv launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

template <int K, int PRO, int EPI>
int launch_k(const BatchGemvParams& p, cudaStream_t s, bool pdl) {
  if (p.n <= 2) return launch_nb<K, 2, PRO, EPI>(p, s, pdl);
  if (p.n <= 4) return launch_nb<K, 4, PRO, EPI>(p, s, pdl);
  return launch_nb<K, 8, PRO, EPI>(p, s, pdl);
}

}  // namespace

// The decoder's batched projections (same descriptor as the batch-1 GEMV, `batch` vectors).
int q35_gemv_batch_launch(const q35_gemv_desc* d, int64_t batch, cudaStream_t s, bool pdl) {
  Q35_REQUIRE(d && d->weight, "gemv_batch: null descriptor");
  Q35_REQUIRE(batch >= 1 && batch <= 8, "gemv_batch: batch %lld outside [1, 8]", (long long)batch);
  Q35_REQUIRE(!d->int8, "gemv_batch: bf16 weights only (the A8W8 decode path is batch 1)");
  BatchGemvParams p = {};
  p.weight = static_cast<const bf16*>(d->weight);
  p.input = static_cast<const bf16*>(d->input);
  p.norm_w = static_cast<const bf16*>(d->norm_weight);
  p.token = d->token;
  p.embed = static_cast<const bf16*>(d->embed);
  p.resid = static_cast<bf16*>(d->resid_out);
  p.out = static_cast<bf16*>(d->out);
  p.vocab = d->vocab;
  p.n = (int)batch;
  p.n_out = (int)d->n_out;
  p.eps = d->eps;
  const int pro = d->prologue, epi = d->epilogue;
  Q35_REQUIRE(pro != Q35_PRO_PLAIN || p.input, "gemv_batch: PLAIN needs an input");
  Q35_REQUIRE(pro == Q35_PRO_PLAIN || p.norm_w, "gemv_batch: NORM / EMBED need the norm weight");
  Q35_REQUIRE(pro != Q35_PRO_EMBED || (p.token && p.embed && p.resid), "gemv_batch: EMBED needs tokens, table, resid");
  Q35_REQUIRE(pro != Q35_PRO_NORM || p.input, "gemv_batch: NORM needs an input");
  Q35_REQUIRE(epi == Q35_EPI_RESIDUAL ? p.resid != nullptr : p.out != nullptr, "gemv_batch: missing output");
  if (d->k == 2048) {
    if (epi == Q35_EPI_SWIGLU) {
      if (pro == Q35_PRO_NORM) return launch_k<2048, Q35_PRO_NORM, Q35_EPI_SWIGLU>(p, s, pdl);
    } else if (epi == Q35_EPI_STORE) {
      if (pro == Q35_PRO_NORM) return launch_k<2048, Q35_PRO_NORM, Q35_EPI_STORE>(p, s, pdl);
      if (pro == Q35_PRO_EMBED) return launch_k<2048, Q35_PRO_EMBED, Q35_EPI_STORE>(p, s, pdl);
    } else if (epi == Q35_EPI_RESIDUAL) {
      if (pro == Q35_PRO_PLAIN) return launch_k<2048, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL>(p, s, pdl);
    }
  } else if (d->k == 6144) {
    if (epi == Q35_EPI_RESIDUAL && pro == Q35_PRO_PLAIN) return launch_k<6144, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL>(p, s, pdl);
  }
  return q35_fail(Q35_ENOTSUP, "gemv_batch: k=%lld with prologue %d / epilogue %d is not a decoder projection",
                  (long long)d->k, pro, epi);
}

extern "C" int q35_gemv_batch(const q35_gemv_desc* desc, int64_t batch, void* stream) {
  return q35_gemv_batch_launch(desc, batch, (cudaStream_t)stream, false);
}
