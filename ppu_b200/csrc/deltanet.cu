// Gated DeltaNet (linear attention) for Qwen3.5 (reference: kernels.py:576-937;
// integration.py:228-272; HF Qwen3_5GatedDeltaNet).
//
// * causal_conv1d: elementwise over (token, channel) with the 4 taps in registers; decode is a
//   shift-and-append update of the per-channel state.
// * delta_recurrent: the reference's sequential scan (also its prefill path). One CTA per
//   (batch, head, 16 value columns); thread (v, kq) keeps 16 rows of the FP32 state column in
//   registers, so the per-token k-reductions are 3 register shuffles. Tokens are staged 32 at
//   a time into shared memory with cp.async double buffering and their q/k L2 factors are
//   computed per chunk, off the serial chain.
// * delta_decode: the whole batch-1 DeltaNet mixer between the two projections in one kernel:
//   a cluster of 4 CTAs per head, each owning 32 value columns (16 KB of state); conv update +
//   SiLU, q/k L2 norm, decay/beta, the rank-1 state update, and the gated RMSNorm whose
//   128-wide reduction crosses the 4 CTAs through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;
using namespace q35;

namespace {

// softplus as F.softplus (threshold 20) and the decay/beta factors (kernels.py:833-841).
Q35_DEV void delta_gates(float a_raw, float b_raw, float a_log, float dt_bias, float& alpha, float& beta) {
  const float a = a_raw + dt_bias;
  const float sp = a > 20.0f ? a : log1pf(expf(a));
  alpha = expf(-expf(a_log) * sp);
  beta = 1.0f / (1.0f + expf(-b_raw));
}

// ============================================================================ conv1d
__global__ void conv_prefill_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ state,
                                    bf16* __restrict__ out, int L, int in_stride, int C, int K) {
  const int64_t total = (int64_t)gridDim.y * L * C;  // gridDim.y = batch
  const int b = blockIdx.y;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)L * C;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / C), c = (int)(i - (int64_t)t * C);
    const bf16* xb = x + (int64_t)b * L * in_stride;
    float acc = 0.f;
    for (int tap = 0; tap < K; ++tap) {
      const int src = t - (K - 1 - tap);
      if (src >= 0) acc += bf2f(xb[(int64_t)src * in_stride + c]) * bf2f(w[c * K + tap]);
    }
    out[((int64_t)b * L + t) * C + c] = f2bf(silu_f(rbf(acc)));
    const int sp = t - (L - K);
    if (sp >= 0 && sp < K) state[((int64_t)b * C + c) * K + sp] = xb[(int64_t)t * in_stride + c];
  }
  (void)total;
}

// Prefill with a compile-time kernel width: thread = (channel, run of kConvRun timesteps), the
// last KT inputs held in registers as the window slides (one load per output instead of KT, and
// no per-element index division). Same tap order and rounding as conv_prefill_kernel.
constexpr int kConvRun = 32;
template <int KT>
__global__ void __launch_bounds__(256) conv_prefill_win_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                               bf16* __restrict__ state, bf16* __restrict__ out, int L,
                                                               int in_stride, int C) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * kConvRun;
  const int b = blockIdx.z;
  if (c >= C || t0 >= L) return;
  const bf16* xb = x + (int64_t)b * L * in_stride + c;
  float wk[KT], hist[KT];
#pragma unroll
  for (int tap = 0; tap < KT; ++tap) wk[tap] = bf2f(w[c * KT + tap]);
#pragma unroll
  for (int j = 0; j < KT - 1; ++j) {  // inputs before the run (the sequence starts from a zero history)
    const int src = t0 - (KT - 1) + j;
    hist[j] = src >= 0 ? bf2f(xb[(int64_t)src * in_stride]) : 0.f;
  }
  const int t1 = min(t0 + kConvRun, L);
  for (int t = t0; t < t1; ++t) {
    const bf16 xt = xb[(int64_t)t * in_stride];
    hist[KT - 1] = bf2f(xt);
    float acc = 0.f;
#pragma unroll
    for (int tap = 0; tap < KT; ++tap) acc += hist[tap] * wk[tap];
    out[((int64_t)b * L + t) * C + c] = f2bf(silu_f(rbf(acc)));
    const int sp = t - (L - KT);
    if (sp >= 0) state[((int64_t)b * C + c) * KT + sp] = xt;
#pragma unroll
    for (int j = 0; j < KT - 1; ++j) hist[j] = hist[j + 1];
  }
}

__global__ void conv_update_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ state,
                                   bf16* __restrict__ out, int batch, int in_stride, int C, int K) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)batch * C) return;
  const int b = (int)(i / C), c = (int)(i - (int64_t)b * C);
  bf16* st = state + ((int64_t)b * C + c) * K;
  float acc = 0.f;
  for (int tap = 0; tap < K - 1; ++tap) {
    const bf16 v = st[tap + 1];
    st[tap] = v;
    acc += bf2f(v) * bf2f(w[c * K + tap]);
  }
  const bf16 xv = x[(int64_t)b * in_stride + c];
  st[K - 1] = xv;
  acc += bf2f(xv) * bf2f(w[c * K + K - 1]);
  out[(int64_t)b * C + c] = f2bf(silu_f(rbf(acc)));
}

// ============================================================================ sequential scan
constexpr int kD = 128;      // key/value head dim of Qwen3.5 linear attention
constexpr int kVB = 16;      // value columns per CTA
constexpr int kT = 32;       // tokens per staged chunk
constexpr int kScanThreads = 128;

struct ScanParams {
  const bf16* qkv;     // [B, L, 3*H*D]
  const bf16* packed;  // [B, L, packed_stride] ([qkv | z | a | b])
  const bf16* a_log;
  const bf16* dt_bias;
  float* state;        // [B, H, D, D]
  bf16* out;           // [B, L, H, D]
  int L, H, packed_stride;
};

Q35_DEV void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
Q35_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
Q35_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kScanThreads) delta_scan_kernel(ScanParams p) {
  __shared__ __align__(16) bf16 qs[2][kT][kD];
  __shared__ __align__(16) bf16 ks[2][kT][kD];
  __shared__ __align__(16) bf16 vs[2][kT][kVB];
  __shared__ float fq[kT], fk[kT], fa[kT], fb[kT];
  const int nvb = kD / kVB;
  const int vb = blockIdx.x % nvb;
  const int h = (blockIdx.x / nvb) % p.H;
  const int b = blockIdx.x / (nvb * p.H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vl = lane >> 3, kq = lane & 7;
  const int v = vb * kVB + warp * 4 + vl;  // value column owned by this thread
  const int H = p.H, L = p.L;
  const int qkv_stride = 3 * H * kD;
  const int a_off = 3 * H * kD + H * kD, b_off = a_off + H;
  const float a_log = bf2f(p.a_log[h]), dt_bias = bf2f(p.dt_bias[h]);
  const float qscale = 1.0f / sqrtf((float)kD);

  float* S = p.state + (((int64_t)b * H + h) * kD) * kD;
  float s[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) s[i] = S[(int64_t)(kq * 16 + i) * kD + v];

  auto stage = [&](int buf, int t0) {
    // q and k rows of this head: 2 x kT x 256 B = 1024 16-byte pieces; v: kT x 32 B.
    for (int i = threadIdx.x; i < 2 * kT * (kD / 8); i += kScanThreads) {
      const int which = i / (kT * (kD / 8));
      const int r = (i / (kD / 8)) % kT, c = (i % (kD / 8)) * 8;
      const int t = t0 + r;
      bf16* dst = which ? &ks[buf][r][c] : &qs[buf][r][c];
      if (t < L) {
        const bf16* src = p.qkv + ((int64_t)b * L + t) * qkv_stride + which * H * kD + h * kD + c;
        cp_async16(dst, src);
      }
    }
    for (int i = threadIdx.x; i < kT * 2; i += kScanThreads) {
      const int r = i >> 1, c = (i & 1) * 8;
      const int t = t0 + r;
      if (t < L) cp_async16(&vs[buf][r][c], p.qkv + ((int64_t)b * L + t) * qkv_stride + 2 * H * kD + h * kD + vb * kVB + c);
    }
    cp_async_commit();
  };

  const int n_chunks = (L + kT - 1) / kT;
  if (n_chunks > 0) stage(0, 0);
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int buf = ch & 1;
    const int t0 = ch * kT;
    if (ch + 1 < n_chunks) {
      stage(buf ^ 1, t0 + kT);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // per-token factors of this chunk: one warp per token, lanes over the 128 dims
    for (int r = warp; r < kT; r += kScanThreads / 32) {
      const int t = t0 + r;
      float sq = 0.f, sk = 0.f;
      for (int c = lane; c < kD; c += 32) {
        const float qv = bf2f(qs[buf][r][c]), kv = bf2f(ks[buf][r][c]);
        sq += qv * qv;
        sk += kv * kv;
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      if (lane == 0) {
        fq[r] = rsqrt_ieee(sq + 1e-6f);
        fk[r] = rsqrt_ieee(sk + 1e-6f);
        float alpha = 1.f, beta = 0.f;
        if (t < L) {
          const bf16* pr = p.packed + ((int64_t)b * L + t) * p.packed_stride;
          delta_gates(bf2f(pr[a_off + h]), bf2f(pr[b_off + h]), a_log, dt_bias, alpha, beta);
        }
        fa[r] = alpha;
        fb[r] = beta;
      }
    }
    __syncthreads();
    const int nt = min(kT, L - t0);
    for (int r = 0; r < nt; ++r) {
      float qh[16], kh[16];
      const float qi = fq[r], ki = fk[r];
      {
        float qf[16], kf[16];
        const uint4* qp = reinterpret_cast<const uint4*>(&qs[buf][r][kq * 16]);
        const uint4* kp = reinterpret_cast<const uint4*>(&ks[buf][r][kq * 16]);
        unpack_bf16x8(qp[0], qf);
        unpack_bf16x8(qp[1], qf + 8);
        unpack_bf16x8(kp[0], kf);
        unpack_bf16x8(kp[1], kf + 8);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          qh[i] = (qf[i] * qi) * qscale;
          kh[i] = kf[i] * ki;
        }
      }
      const float alpha = fa[r], beta = fb[r];
      float m0 = 0.f, m1 = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        s[i] *= alpha;
        s[i + 1] *= alpha;
        m0 = fmaf(s[i], kh[i], m0);
        m1 = fmaf(s[i + 1], kh[i + 1], m1);
      }
      float mem = m0 + m1;
      mem += __shfl_xor_sync(0xffffffffu, mem, 1);
      mem += __shfl_xor_sync(0xffffffffu, mem, 2);
      mem += __shfl_xor_sync(0xffffffffu, mem, 4);
      const float delta = beta * (bf2f(vs[buf][r][warp * 4 + vl]) - mem);
      float o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        s[i] = fmaf(kh[i], delta, s[i]);
        s[i + 1] = fmaf(kh[i + 1], delta, s[i + 1]);
        o0 = fmaf(s[i], qh[i], o0);
        o1 = fmaf(s[i + 1], qh[i + 1], o1);
      }
      float o = o0 + o1;
      o += __shfl_xor_sync(0xffffffffu, o, 1);
      o += __shfl_xor_sync(0xffffffffu, o, 2);
      o += __shfl_xor_sync(0xffffffffu, o, 4);
      if (kq == 0) p.out[(((int64_t)b * L + t0 + r) * H + h) * kD + v] = f2bf(o);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) S[(int64_t)(kq * 16 + i) * kD + v] = s[i];
}

// ============================================================================ fused decode step
constexpr int kCluster = 4;
constexpr int kVS = kD / kCluster;  // 32 value columns per CTA
constexpr int kDecThreads = 256;

struct DecodeStepParams {
  const bf16* packed;     // [B, packed_stride]
  const bf16* conv_w;     // [3*H*D, 4]
  bf16* conv_state;       // [B, 3*H*D, 4]
  const bf16* a_log;
  const bf16* dt_bias;
  const bf16* norm_w;     // [D]
  float* state;           // [B, H, D, D]
  bf16* out;              // [B, H*D]
  int H, packed_stride;
  float eps;
};

// QK_REGS: the 16 scaled q and k values of the thread's state rows are computed once into
// registers (80 registers) instead of at each use from shared memory (64 registers). The values
// are the same; which form lets the neighbouring projections overlap the mixer better depends on
// the projections' own footprint, and was measured per engine precision: int8 projections
// 1494 -> 1526 tok/s with registers, bf16 1151 -> 1145 (so bf16 keeps the shared-memory form).
template <bool QK_REGS>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kDecThreads)
    delta_decode_kernel(DecodeStepParams p) {
  __shared__ float qhat[kD], khat[kD];
  __shared__ float vconv[kVS];
  __shared__ float red1[kDecThreads / 32][kVS], red2[kDecThreads / 32][kVS];
  __shared__ float nred[kDecThreads / 32];
  __shared__ float cl_parts[kCluster];  // the gated norm's partial sums, pushed by every CTA
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int bh = blockIdx.x / kCluster;
  const int H = p.H;
  const int h = bh % H, b = bh / H;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int C = 3 * H * kD;
  const int v0 = rank * kVS;

  // ---- independent of the producer kernel: state column slice, conv state and weights
  float* S = p.state + (((int64_t)b * H + h) * kD) * kD;
  float s[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) s[i] = S[(int64_t)(warp * 16 + i) * kD + v0 + lane];
  // conv channel handled by this thread: q (t < 128) / k (t >= 128); threads < 32 also a v channel
  const int cqk = (t < kD) ? h * kD + t : H * kD + h * kD + (t - kD);
  const int cv = 2 * H * kD + h * kD + v0 + lane;
  bf16* stq = p.conv_state + ((int64_t)b * C + cqk) * 4;
  bf16* stv = p.conv_state + ((int64_t)b * C + cv) * 4;
  float sq[4], sv[4], wq[4], wv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sq[j] = bf2f(stq[j]);
    wq[j] = bf2f(p.conv_w[cqk * 4 + j]);
    sv[j] = (t < kVS) ? bf2f(stv[j]) : 0.f;
    wv[j] = (t < kVS) ? bf2f(p.conv_w[cv * 4 + j]) : 0.f;
  }
  const float a_log = bf2f(p.a_log[h]), dt_bias = bf2f(p.dt_bias[h]);
  const float gw = bf2f(p.norm_w[v0 + lane]);
  // the peers write into this CTA's shared memory later: all CTAs of the cluster must have started
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  pdl_wait();
  pdl_launch_dependents();

  const bf16* row = p.packed + (int64_t)b * p.packed_stride;
  // packed row layout (integration.py:81-93): [q | k | v] (3*H*D) | z (H*D) | a (H) | b (H).
  // Every value this thread needs from the row is loaded here, at once: a load after one of the
  // barriers below would be one more dependent round trip to L2.
  const int z_off = 3 * H * kD, a_off = 4 * H * kD, b_off = 4 * H * kD + H;
  const bf16 a_raw = row[a_off + h], b_raw = row[b_off + h];
  const bf16 z_raw = warp == 0 ? row[z_off + h * kD + v0 + lane] : bf16();
  const bf16 xq_raw = row[cqk];
  const bf16 xv_raw = t < kVS ? row[cv] : bf16();
  // ---- causal conv update + SiLU (kernels.py:622-656), rounded to BF16 (conv output dtype)
  const float xq = bf2f(xq_raw);
  float acc = sq[1] * wq[0];
  acc += sq[2] * wq[1];
  acc += sq[3] * wq[2];
  acc += xq * wq[3];
  const float cqk_out = rbf(silu_f(rbf(acc)));
  float xv = 0.f;
  if (t < kVS) {
    xv = bf2f(xv_raw);
    float av = sv[1] * wv[0];
    av += sv[2] * wv[1];
    av += sv[3] * wv[2];
    av += xv * wv[3];
    vconv[t] = rbf(silu_f(rbf(av)));
  }
  // ---- L2 norms of q (warps 0-3) and k (warps 4-7): the raw conv outputs are published with
  // the norm partials, and every thread scales the 16 q / k values it uses itself after the one
  // barrier (the same expressions, so the values equal a normalise-then-publish pass)
  {
    const float ws = warp_sum(cqk_out * cqk_out);
    if (lane == 0) nred[warp] = ws;
    if (t < kD)
      qhat[t] = cqk_out;
    else
      khat[t - kD] = cqk_out;
  }
  float alpha, beta;
  delta_gates(bf2f(a_raw), bf2f(b_raw), a_log, dt_bias, alpha, beta);
  __syncthreads();
  const float inv_q = rsqrt_ieee(nred[0] + nred[1] + nred[2] + nred[3] + 1e-6f);
  const float inv_k = rsqrt_ieee(nred[4] + nred[5] + nred[6] + nred[7] + 1e-6f);
  auto kh_at = [&](int i) { return khat[warp * 16 + i] * inv_k; };
  auto qh_at = [&](int i) { return (qhat[warp * 16 + i] * inv_q) * (1.0f / sqrtf((float)kD)); };
  float khr[QK_REGS ? 16 : 1], qhr[QK_REGS ? 16 : 1];
  if constexpr (QK_REGS) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      khr[i] = kh_at(i);
      qhr[i] = qh_at(i);
    }
  }
  auto kh = [&](int i) {
    if constexpr (QK_REGS) return khr[i]; else return kh_at(i);
  };
  auto qh = [&](int i) {
    if constexpr (QK_REGS) return qhr[i]; else return qh_at(i);
  };

  // ---- state update: s = alpha*s; mem = s^T k; d = beta (v - mem); s += k d^T; o = s^T q
  float pm = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    s[i] *= alpha;
    pm = fmaf(s[i], kh(i), pm);
  }
  red1[warp][lane] = pm;
  __syncthreads();
  float mem = 0.f;
#pragma unroll
  for (int w = 0; w < kDecThreads / 32; ++w) mem += red1[w][lane];
  const float delta = beta * (vconv[lane] - mem);
  float po = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    s[i] = fmaf(kh(i), delta, s[i]);
    po = fmaf(s[i], qh(i), po);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) S[(int64_t)(warp * 16 + i) * kD + v0 + lane] = s[i];
  red2[warp][lane] = po;
  __syncthreads();
  float o = 0.f;
#pragma unroll
  for (int w = 0; w < kDecThreads / 32; ++w) o += red2[w][lane];
  o = rbf(o);  // the recurrent output is materialised in BF16 (kernels.py:849, 884)

  // ---- gated RMSNorm over the head's 128 values: each CTA pushes its partial sum into slot
  // `rank` of every CTA of the cluster, and after one cluster barrier reads only its own shared
  // memory (so no second barrier has to keep it alive for the peers' reads)
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  if (warp == 0) {
    const float ps = warp_sum(o * o);
    if (lane < kCluster) *cluster.map_shared_rank(&cl_parts[rank], lane) = ps;
  }
  cluster.sync();
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) tot += cl_parts[r];
  // conv state writes: every CTA of the cluster has read the old state before cluster.sync()
  if ((t < kD ? t : t - kD) / kVS == rank) {
    stq[0] = f2bf(sq[1]);
    stq[1] = f2bf(sq[2]);
    stq[2] = f2bf(sq[3]);
    stq[3] = xq_raw;
  }
  if (t < kVS) {
    stv[0] = f2bf(sv[1]);
    stv[1] = f2bf(sv[2]);
    stv[2] = f2bf(sv[3]);
    stv[3] = xv_raw;
  }
  if (warp == 0) {
    const float rstd = rsqrt_ieee(tot / (float)kD + p.eps);
    const float nrm = rbf(o * rstd);
    const float wt = rbf(nrm * gw);
    const float z = bf2f(z_raw);
    p.out[(int64_t)b * H * kD + h * kD + v0 + lane] = f2bf(wt * silu_f(z));
  }
  (void)xv;
}

}  // namespace

// ------------------------------------------------------------------------------------ C ABI
extern "C" int q35_causal_conv1d(const void* x, const void* weight, void* state, void* out, int64_t batch,
                                 int64_t seq_len, int64_t in_stride, int64_t channels, int64_t kernel_size,
                                 void* stream) {
  Q35_REQUIRE(x && weight && state && out, "causal_conv1d: null pointer");
  Q35_REQUIRE(batch >= 0 && seq_len >= 0 && channels > 0 && kernel_size >= 1 && kernel_size <= 16 &&
                  in_stride >= channels,
              "causal conv shapes do not match");
  if (batch * seq_len == 0) return Q35_OK;
  if (seq_len == 1) {
    const int64_t total = batch * channels;
    conv_update_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)weight, (bf16*)state, (bf16*)out, (int)batch, (int)in_stride, (int)channels,
        (int)kernel_size);
  } else if (kernel_size == 4 && seq_len >= 4) {
    const dim3 grid((unsigned)((channels + 255) / 256), (unsigned)((seq_len + kConvRun - 1) / kConvRun), (unsigned)batch);
    conv_prefill_win_kernel<4><<<grid, 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)weight, (bf16*)state, (bf16*)out, (int)seq_len, (int)in_stride, (int)channels);
  } else {
    int64_t blocks = (seq_len * channels + 255) / 256;
    if (blocks > 4 * kNumSMs) blocks = 4 * kNumSMs;
    conv_prefill_kernel<<<dim3((unsigned)blocks, (unsigned)batch), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)weight, (bf16*)state, (bf16*)out, (int)seq_len, (int)in_stride, (int)channels,
        (int)kernel_size);
  }
  return q35_check_launch("causal_conv1d");
}

extern "C" int q35_delta_recurrent(const void* qkv, const void* packed, const void* a_log, const void* dt_bias,
                                   float* state, void* out, int64_t batch, int64_t seq_len, int64_t heads,
                                   int64_t dim, int64_t packed_stride, void* stream) {
  Q35_REQUIRE(qkv && packed && a_log && dt_bias && state && out, "delta_recurrent: null pointer");
  Q35_REQUIRE(dim == kD, "delta recurrent dimensions do not match (dim %lld, built for 128)", (long long)dim);
  Q35_REQUIRE(batch >= 0 && seq_len >= 0 && heads > 0 && packed_stride >= 4 * heads * dim + 2 * heads,
              "packed projection width %lld is smaller than %lld", (long long)packed_stride,
              (long long)(4 * heads * dim + 2 * heads));
  Q35_REQUIRE(Q35_ALIGNED(qkv, 16), "delta_recurrent: qkv must be 16-byte aligned");
  if (batch * seq_len == 0) return Q35_OK;
  ScanParams p;
  p.qkv = (const bf16*)qkv;
  p.packed = (const bf16*)packed;
  p.a_log = (const bf16*)a_log;
  p.dt_bias = (const bf16*)dt_bias;
  p.state = state;
  p.out = (bf16*)out;
  p.L = (int)seq_len;
  p.H = (int)heads;
  p.packed_stride = (int)packed_stride;
  delta_scan_kernel<<<(unsigned)(batch * heads * (kD / kVB)), kScanThreads, 0, (cudaStream_t)stream>>>(p);
  return q35_check_launch("delta_recurrent");
}

int q35_delta_decode_launch(const void* packed, const void* conv_weight, void* conv_state, const void* a_log,
                            const void* dt_bias, const void* norm_weight, float* state, void* out, int64_t batch,
                            int64_t heads, int64_t packed_stride, float eps, cudaStream_t stream, bool pdl,
                            bool qk_regs) {
  DecodeStepParams p;
  p.packed = (const bf16*)packed;
  p.conv_w = (const bf16*)conv_weight;
  p.conv_state = (bf16*)conv_state;
  p.a_log = (const bf16*)a_log;
  p.dt_bias = (const bf16*)dt_bias;
  p.norm_w = (const bf16*)norm_weight;
  p.state = state;
  p.out = (bf16*)out;
  p.H = (int)heads;
  p.packed_stride = (int)packed_stride;
  p.eps = eps;
  const dim3 grid((unsigned)(batch * heads * kCluster));
  cudaError_t e = qk_regs ? q35_launch(delta_decode_kernel<true>, grid, dim3(kDecThreads), 0, stream, pdl, p)
                          : q35_launch(delta_decode_kernel<false>, grid, dim3(kDecThreads), 0, stream, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "delta_decode launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_delta_decode(const void* packed, const void* conv_weight, void* conv_state, const void* a_log,
                                const void* dt_bias, const void* norm_weight, float* state, void* out,
                                int64_t batch, int64_t heads, int64_t dim, int64_t packed_stride, float eps,
                                void* stream) {
  Q35_REQUIRE(packed && conv_weight && conv_state && a_log && dt_bias && norm_weight && state && out,
              "delta_decode: null pointer");
  Q35_REQUIRE(dim == kD && heads >= 1 && batch >= 1, "delta_decode: built for head dim 128");
  Q35_REQUIRE(packed_stride >= 4 * heads * dim + 2 * heads, "delta_decode: packed width too small");
  return q35_delta_decode_launch(packed, conv_weight, conv_state, a_log, dt_bias, norm_weight, state, out, batch,
                                 heads, packed_stride, eps, (cudaStream_t)stream, false, false);
}
