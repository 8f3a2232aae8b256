// Batched decode projections: one decode step of up to 8 requests in lock step streams each
// weight matrix once for all of them (the decode projections of integration.py:183-185, 245, 272,
// 298, 359 and the LM head top-1 of kernels.py:1093-1185, with a batch of B in-flight requests).
//
// Y[b, n] = W[n, :] . x_b for b < B as a skinny product on the warp tensor cores: a warp takes 16
// weight rows x 8 requests (mma.sync m16n8k16, bf16 in, FP32 accumulate), the rows as the M side
// and the requests as N. Each lane loads 16 contiguous bytes of rows g and g + 8 per 32-column
// block (fully used 32-byte sectors) and one 16-byte slice of request g's input from shared
// memory; the 16-column slots of the two MMAs of a block are assigned to those bytes by one
// permutation of the K order, the same for both operands, so no operand is rearranged. The K range
// of a 16-row group is split over the CTA's 8 warps and the partial tiles are summed in a fixed
// order. At batch 8 each weight element feeds 8 products: on the CUDA cores that is issue-bound
// (8 FMAs per element), on the tensor cores the step stays bound by the weight stream.
//
// Prologues as the batch-1 GEMV (input row, RMSNorm(1 + w) of it, or the embedding gather +
// RMSNorm at layer 0) with its rounding points, per request; epilogues store / in-place residual
// add / SwiGLU (the warp's 16 rows are 8 gate rows and their 8 up rows) / top-1 keys of the tied
// LM head (bf16-rounded logits, lowest index on ties, the shard-key encoding).
#include <cfloat>

#include "common.cuh"

using namespace q35;

namespace {

constexpr int kThreads = 256, kWarps = kThreads / 32;
constexpr int kBlk = 32;        // K columns per block (two MMAs)
constexpr int kBatch = 8;       // N of the MMA: requests per step
constexpr int kEpiTop1 = 100;   // epilogue: LM head top-1 keys

struct BatchGemvParams {
  const bf16* weight;     // [rows, K] (SWIGLU: gate rows [0, n_out), up rows [n_out, 2 n_out))
  const bf16* input;      // PLAIN / NORM: [n, K]
  const bf16* norm_w;     // NORM / EMBED: [K] (1 + w)
  const int64_t* token;   // EMBED: [n]
  const bf16* embed;      // EMBED: [vocab, K]
  bf16* resid;            // RESIDUAL: [n, n_out] in place; EMBED: receives the raw rows [n, K]
  bf16* out;              // STORE / SWIGLU: [n, n_out]
  unsigned long long* top1;  // TOP1: workspace keys [8] + count (zero before, zero after)
  long long* keys_out;    // TOP1: [n] reduced signed keys
  float4* part;           // split K: [groups][KSPLIT][32] partial tiles (lane layout of warp 0)
  unsigned* tickets;      // split K: [groups], zero between launches (the last part re-zeroes it)
  int64_t vocab;
  int n, n_out;
  float eps;
};

template <int K>
constexpr int xs_stride() {  // bf16 elements per request row in shared memory (+64 bytes: see load)
  return K + 32;
}

// Largest batch of per-lane 16-byte loads (<= 8) that divides a row's CPL chunks.
constexpr int load_batch(int cpl) {
  for (int b = 8; b > 1; --b)
    if (cpl % b == 0) return b;
  return 1;
}

// Split K (PLAIN prologue): columns [k0, k0 + KS) of request b's input into its row of xs.
template <int KS>
Q35_DEV void build_input_slice(const BatchGemvParams& p, int k_full, int k0, bf16* xs, int warp, int lane) {
  constexpr int CPL = KS / 8 / 32;
  constexpr int BATCH = load_batch(CPL);
  uint4* dst = reinterpret_cast<uint4*>(xs + warp * xs_stride<KS>());
  const uint4* src = reinterpret_cast<const uint4*>(p.input + (int64_t)warp * k_full + k0);
  for (int c0 = 0; c0 < CPL; c0 += BATCH) {
    uint4 v[BATCH];
#pragma unroll
    for (int i = 0; i < BATCH; ++i) v[i] = warp < p.n ? src[lane + 32 * (c0 + i)] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < BATCH; ++i) dst[lane + 32 * (c0 + i)] = v[i];
  }
}

// Warp b builds request b's input row (bf16) in shared memory. `nws`: the norm weights, already
// in shared memory (copied before the PDL wait: they are constants).
template <int K, int PRO>
Q35_DEV void build_inputs(const BatchGemvParams& p, bf16* xs, const uint4* nws, int warp, int lane) {
  constexpr int CPL = K / 8 / 32;
  const int b = warp;
  uint4* dst = reinterpret_cast<uint4*>(xs + b * xs_stride<K>());
  if (b >= p.n) {
    for (int c = 0; c < CPL; ++c) dst[lane + 32 * c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const bf16* row = p.input + (int64_t)b * K;
  if (PRO == Q35_PRO_EMBED) {
    int64_t t = p.token[b];
    t = t < 0 ? 0 : (t >= p.vocab ? p.vocab - 1 : t);
    row = p.embed + t * (int64_t)K;
  }
  const uint4* src = reinterpret_cast<const uint4*>(row);
  if (PRO == Q35_PRO_PLAIN) {  // loads in batches of up to 8 per lane, each batch before its stores
    constexpr int BATCH = load_batch(CPL);
    for (int c0 = 0; c0 < CPL; c0 += BATCH) {
      uint4 v[BATCH];
#pragma unroll
      for (int i = 0; i < BATCH; ++i) v[i] = src[lane + 32 * (c0 + i)];
#pragma unroll
      for (int i = 0; i < BATCH; ++i) dst[lane + 32 * (c0 + i)] = v[i];
    }
    return;
  }
  float ss = 0.f;
  for (int c = 0; c < CPL; ++c) {
    const uint4 v = src[lane + 32 * c];
    if (PRO == Q35_PRO_EMBED && blockIdx.x == 0) reinterpret_cast<uint4*>(p.resid + (int64_t)b * K)[lane + 32 * c] = v;
    float f[8];
    unpack_bf16x8(v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  const float r = rsqrt_ieee(warp_sum(ss) / (float)K + p.eps);
  for (int c = 0; c < CPL; ++c) {
    float f[8], w[8];
    unpack_bf16x8(src[lane + 32 * c], f);
    unpack_bf16x8(nws[lane + 32 * c], w);
    __align__(16) bf16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = f2bf(f[j] * r * (1.0f + w[j]));
    dst[lane + 32 * c] = *reinterpret_cast<const uint4*>(o);
  }
}

Q35_DEV void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}

Q35_DEV unsigned long long top1_key(float v, int idx) {
  return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// KSPLIT > 1 (PLAIN + RESIDUAL only): the K range of every 16-row group is split over KSPLIT
// CTAs (CTA i takes part i % KSPLIT of groups i / KSPLIT, i / KSPLIT + gridDim.x / KSPLIT, ...);
// each part writes its partial tile, and the last part of a group (atomic ticket) sums the parts
// in part order and applies the residual epilogue, so the result does not depend on arrival order.
template <int K, int PRO, int EPI, int KSPLIT = 1>
__global__ void __launch_bounds__(kThreads) gemv_batch_kernel(BatchGemvParams p) {
  static_assert(KSPLIT == 1 || (PRO == Q35_PRO_PLAIN && EPI == Q35_EPI_RESIDUAL), "split K: plain residual only");
  constexpr int KS = K / KSPLIT;       // K columns of this CTA's part
  constexpr int KW = KS / kWarps;      // K columns per warp
  constexpr int NBK = KW / kBlk;       // blocks per warp
  constexpr int STAGE = NBK > 8 ? 6 : NBK;  // blocks per register stage
  constexpr int NST = NBK / STAGE;     // stages per group; more than one: two register buffers
  constexpr int NBUF = NST > 1 ? 2 : 1;
  static_assert(KW % kBlk == 0 && NBK % STAGE == 0, "K must split into whole blocks per warp");
  // an even stage count keeps the buffer of each stage the same from group to group
  static_assert(NST == 1 || NST % 2 == 0, "stages per group: one, or an even count");
  constexpr int UNITS = (EPI == Q35_EPI_SWIGLU) ? 8 : 16;  // output units per 16-row group
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);  // [8][KS + 32]
  __shared__ float4 part[kWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n_out = p.n_out;
  const int ngroups = (n_out + UNITS - 1) / UNITS;
  const char* W = reinterpret_cast<const char*>(p.weight);
  const int ks = (int)blockIdx.x % KSPLIT;  // this CTA's part of K
  const int kbase = ks * KS;
  const int k0 = kbase + warp * KW;         // weight column of this warp's first block
  const int gstep = (int)gridDim.x / KSPLIT;

  // rows of lane g's two A-fragment rows in group grp (clamped in range; masked at the epilogue)
  auto rows = [&](int grp, int64_t& r0, int64_t& r1, bool& ok0, bool& ok1) {
    if (EPI == Q35_EPI_SWIGLU) {
      const int u = grp * 8 + g;
      ok0 = ok1 = u < n_out;
      r0 = ok0 ? u : 0;
      r1 = ok0 ? (int64_t)u + n_out : 0;
    } else {
      const int u0 = grp * 16 + g, u1 = u0 + 8;
      ok0 = u0 < n_out;
      ok1 = u1 < n_out;
      r0 = ok0 ? u0 : 0;
      r1 = ok1 ? u1 : 0;
    }
  };
  uint4 wa[NBUF][STAGE], wb[NBUF][STAGE];
  auto load = [&](int grp, int stage, int buf) {
    int64_t r0, r1;
    bool ok0, ok1;
    rows(grp, r0, r1, ok0, ok1);
    const char* b0 = W + r0 * (K * 2) + (k0 + stage * STAGE * kBlk + 8 * t) * 2;
    const char* b1 = W + r1 * (K * 2) + (k0 + stage * STAGE * kBlk + 8 * t) * 2;
#pragma unroll
    for (int i = 0; i < STAGE; ++i) {
      wa[buf][i] = ok0 ? ld_stream(b0 + i * kBlk * 2) : make_uint4(0, 0, 0, 0);
      wb[buf][i] = ok1 ? ld_stream(b1 + i * kBlk * 2) : make_uint4(0, 0, 0, 0);
    }
  };
  int grp = (int)blockIdx.x / KSPLIT;
  const int grp0 = grp;
  if (grp < ngroups) {
    load(grp, 0, 0);
    if (NST > 1) load(grp, 1, NBUF - 1);
  }
  // norm weights (constants) copied into shared memory before the wait: read after the sum of
  // squares, they would be a dependent load from HBM (the step's weight stream evicts them)
  constexpr bool kNormed = PRO == Q35_PRO_NORM || PRO == Q35_PRO_EMBED;
  __shared__ __align__(16) uint4 nws[kNormed ? K / 8 : 1];
  if constexpr (kNormed) {
    for (int i = threadIdx.x; i < K / 8; i += kThreads) cp_async16(&nws[i], p.norm_w + 8 * i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  pdl_wait();
  pdl_launch_dependents();
  // residual epilogue: warp 0's values for its first group, read now (the producers are done) so
  // that the epilogue's read-modify-write does not wait on L2 at the kernel's tail
  float rp[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [row h][request 2t + e]
  if (EPI == Q35_EPI_RESIDUAL && warp == 0 && grp0 < ngroups) {
    int64_t r0, r1;
    bool ok0, ok1;
    rows(grp0, r0, r1, ok0, ok1);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int b = 2 * t + e;
        if (b < p.n && (h ? ok1 : ok0)) rp[h][e] = bf2f(p.resid[(int64_t)b * n_out + (h ? r1 : r0)]);
      }
  }
  if constexpr (kNormed) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  }
  if constexpr (KSPLIT > 1)
    build_input_slice<KS>(p, K, kbase, xs, warp, lane);
  else
    build_inputs<K, PRO>(p, xs, nws, warp, lane);
  __syncthreads();

  unsigned long long best[2] = {0ull, 0ull};  // TOP1: this lane's best keys for requests 2t, 2t + 1
  const bf16* xrow = xs + g * xs_stride<KS>() + (k0 - kbase) + 8 * t;
  for (; grp < ngroups; grp += gstep) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // stage st computes from buffer st % NBUF; the buffer is refilled at once with the stage two
    // ahead (or the next group's first stages), so one stage is always in flight
#pragma unroll
    for (int st = 0; st < NST; ++st) {
      const int buf = st % NBUF;
#pragma unroll
      for (int i = 0; i < STAGE; ++i) {
        const uint4 x = *reinterpret_cast<const uint4*>(xrow + (st * STAGE + i) * kBlk);
        mma_bf16(acc, wa[buf][i].x, wb[buf][i].x, wa[buf][i].y, wb[buf][i].y, x.x, x.y);
        mma_bf16(acc, wa[buf][i].z, wb[buf][i].z, wa[buf][i].w, wb[buf][i].w, x.z, x.w);
      }
      const int nxt = st + NBUF;  // the stage this buffer holds next
      if (nxt < NST)
        load(grp, nxt, buf);
      else if (grp + gstep < ngroups)
        load(grp + gstep, nxt - NST, buf);
    }
    part[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    bool finish = true;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (warp == 0) {
      s = part[0][lane];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) {
        const float4 q = part[w][lane];
        s.x += q.x;
        s.y += q.y;
        s.z += q.z;
        s.w += q.w;
      }
      if constexpr (KSPLIT > 1) {  // this part's tile out; the group's last part sums them in order
        float4* gp = p.part + (int64_t)grp * KSPLIT * 32;
        gp[ks * 32 + lane] = s;
        __threadfence();
        __syncwarp();
        unsigned tk = 0;
        if (lane == 0) tk = atomicAdd(p.tickets + grp, 1u);
        tk = __shfl_sync(0xffffffffu, tk, 0);
        finish = tk == (unsigned)(KSPLIT - 1);
        if (finish) {
          __threadfence();
          s = __ldcg(gp + lane);
#pragma unroll
          for (int k = 1; k < KSPLIT; ++k) {
            const float4 q = __ldcg(gp + k * 32 + lane);
            s.x += q.x;
            s.y += q.y;
            s.z += q.z;
            s.w += q.w;
          }
          if (lane == 0) atomicExch(p.tickets + grp, 0u);
        }
      }
    }
    if (warp == 0 && finish) {
      // lane (g, t): rows g / g + 8 of the group, requests 2t / 2t + 1
      const float d[4] = {s.x, s.y, s.z, s.w};
      int64_t r0, r1;
      bool ok0, ok1;
      rows(grp, r0, r1, ok0, ok1);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int b = 2 * t + e;
        if (b >= p.n) continue;
        if (EPI == Q35_EPI_SWIGLU) {
          if (ok0) p.out[(int64_t)b * n_out + r0] = f2bf(rbf(silu_f(rbf(d[e]))) * rbf(d[2 + e]));
        } else if (EPI == kEpiTop1) {
          if (ok0) {
            const unsigned long long k = top1_key(rbf(d[e]), (int)r0);
            best[e] = k > best[e] ? k : best[e];
          }
          if (ok1) {
            const unsigned long long k = top1_key(rbf(d[2 + e]), (int)r1);
            best[e] = k > best[e] ? k : best[e];
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!(h ? ok1 : ok0)) continue;
            const int64_t o = (int64_t)b * n_out + (h ? r1 : r0);
            const float y = d[2 * h + e];
            if (EPI == Q35_EPI_RESIDUAL)
              p.resid[o] = f2bf((grp == grp0 ? rp[h][e] : bf2f(p.resid[o])) + rbf(y));
            else
              p.out[o] = f2bf(y);
          }
        }
      }
    }
    __syncthreads();  // part[] is rewritten by the next group
  }
  if (EPI == kEpiTop1) {
    if (warp == 0) {
      // lanes with the same t hold the same requests: reduce over g (lane bits 2-4)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[e], o);
          best[e] = other > best[e] ? other : best[e];
        }
      if (g == 0) {
        if (2 * t < p.n && best[0]) atomicMax(p.top1 + 2 * t, best[0]);
        if (2 * t + 1 < p.n && best[1]) atomicMax(p.top1 + 2 * t + 1, best[1]);
      }
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned* count = reinterpret_cast<unsigned*>(p.top1 + kBatch);
      __threadfence();
      const unsigned prev = atomicAdd(count, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        for (int b = 0; b < p.n; ++b) {
          const unsigned long long key = atomicExch(p.top1 + b, 0ull);
          p.keys_out[b] = (long long)(key ^ 0x8000000000000000ull);
        }
        atomicExch(count, 0u);
      }
    }
  }
}

template <int K, int PRO, int EPI, int KSPLIT = 1>
int launch(const BatchGemvParams& p, cudaStream_t s, bool pdl) {
  constexpr size_t smem = (size_t)kBatch * xs_stride<K / KSPLIT>() * sizeof(bf16);
  static Q35PerDevice<int> ctas_of;
  const int ctas = ctas_of.get([] {
    cudaFuncSetAttribute(gemv_batch_kernel<K, PRO, EPI, KSPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_batch_kernel<K, PRO, EPI, KSPLIT>, kThreads,
                                                      smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cudaGetLastError();
    return per_sm * kNumSMs;
  });
  constexpr int UNITS = (EPI == Q35_EPI_SWIGLU) ? 8 : 16;
  const int ngroups = (p.n_out + UNITS - 1) / UNITS;
  const int items = ngroups * KSPLIT;
  const int grid = items < ctas ? items : ctas / KSPLIT * KSPLIT;
  const cudaError_t e =
      q35_launch(gemv_batch_kernel<K, PRO, EPI, KSPLIT>, dim3(grid), dim3(kThreads), smem, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "batched gemv launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

BatchGemvParams params_of(const q35_gemv_desc* d, int64_t batch) {
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
  return p;
}

}  // namespace

// Split-K scratch of the decoder's narrow batched projections (n_out / 16 groups, 2 parts).
size_t q35_gemv_batch_split_bytes(int64_t n_out) {
  const size_t groups = (size_t)((n_out + 15) / 16);
  return groups * 2 * 32 * sizeof(float4) + ((groups * sizeof(unsigned) + 255) & ~(size_t)255);
}

// The decoder's batched projections (same descriptor as the batch-1 GEMV, `batch` vectors).
// `split_ws` (q35_gemv_batch_split_bytes(n_out), tickets zeroed once) lets the down projection
// (K = 6144, 128 row groups for 148 SMs) split K over two CTAs: batch-8 step 1.68 -> 1.20 ms.
// Measured and not used: the out-projection (K = 2048) split as well (1.26 ms), four parts for
// the down projection (1.30 ms).
int q35_gemv_batch_launch(const q35_gemv_desc* d, int64_t batch, cudaStream_t s, bool pdl, void* split_ws = nullptr) {
  Q35_REQUIRE(d && d->weight, "gemv_batch: null descriptor");
  Q35_REQUIRE(batch >= 1 && batch <= kBatch, "gemv_batch: batch %lld outside [1, 8]", (long long)batch);
  Q35_REQUIRE(!d->int8, "gemv_batch: bf16 weights only (the A8W8 decode path is batch 1)");
  Q35_REQUIRE(Q35_ALIGNED(d->weight, 16), "gemv_batch: 16-byte aligned weights");
  const BatchGemvParams p = params_of(d, batch);
  const int pro = d->prologue, epi = d->epilogue;
  Q35_REQUIRE(pro == Q35_PRO_EMBED || p.input, "gemv_batch: PLAIN / NORM need an input");
  Q35_REQUIRE(pro == Q35_PRO_PLAIN || p.norm_w, "gemv_batch: NORM / EMBED need the norm weight");
  Q35_REQUIRE(pro != Q35_PRO_EMBED || (p.token && p.embed && p.resid), "gemv_batch: EMBED needs tokens, table, resid");
  Q35_REQUIRE(epi == Q35_EPI_RESIDUAL ? p.resid != nullptr : p.out != nullptr, "gemv_batch: missing output");
  BatchGemvParams ps = p;
  const bool split = split_ws && epi == Q35_EPI_RESIDUAL && pro == Q35_PRO_PLAIN && (p.n_out + 15) / 16 < kNumSMs &&
                     d->k == 6144;
  if (split) {
    const size_t groups = (size_t)((p.n_out + 15) / 16);
    ps.part = static_cast<float4*>(split_ws);
    ps.tickets = reinterpret_cast<unsigned*>(static_cast<char*>(split_ws) + groups * 2 * 32 * sizeof(float4));
  }
  if (d->k == 2048) {
    if (epi == Q35_EPI_SWIGLU && pro == Q35_PRO_NORM) return launch<2048, Q35_PRO_NORM, Q35_EPI_SWIGLU>(p, s, pdl);
    if (epi == Q35_EPI_STORE && pro == Q35_PRO_NORM) return launch<2048, Q35_PRO_NORM, Q35_EPI_STORE>(p, s, pdl);
    if (epi == Q35_EPI_STORE && pro == Q35_PRO_EMBED) return launch<2048, Q35_PRO_EMBED, Q35_EPI_STORE>(p, s, pdl);
    if (epi == Q35_EPI_RESIDUAL && pro == Q35_PRO_PLAIN)
      return split ? launch<2048, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL, 2>(ps, s, pdl)
                   : launch<2048, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL>(p, s, pdl);
  } else if (d->k == 6144) {
    if (epi == Q35_EPI_RESIDUAL && pro == Q35_PRO_PLAIN)
      return split ? launch<6144, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL, 2>(ps, s, pdl)
                   : launch<6144, Q35_PRO_PLAIN, Q35_EPI_RESIDUAL>(p, s, pdl);
  }
  return q35_fail(Q35_ENOTSUP, "gemv_batch: k=%lld with prologue %d / epilogue %d is not a decoder projection",
                  (long long)d->k, pro, epi);
}

// Batched LM head: RMSNorm of the `batch` final residuals, logits over the whole tied table, one
// reduced top-1 key per request in keys_out (the q35_lm_head_shard_keys encoding; workspace of
// q35_lm_shard_workspace_size() bytes, zero before, left zero).
int q35_lm_head_batch_launch(const void* hidden, int64_t batch, const void* norm_weight, const void* weight,
                             int64_t vocab, float eps, int64_t* keys_out, void* workspace, cudaStream_t s, bool pdl) {
  Q35_REQUIRE(hidden && norm_weight && weight && keys_out && workspace, "lm_head_batch: null pointer");
  Q35_REQUIRE(batch >= 1 && batch <= kBatch && vocab > 0 && vocab < (1ll << 31), "lm_head_batch: bad shape");
  BatchGemvParams p = {};
  p.weight = static_cast<const bf16*>(weight);
  p.input = static_cast<const bf16*>(hidden);
  p.norm_w = static_cast<const bf16*>(norm_weight);
  p.top1 = static_cast<unsigned long long*>(workspace);
  p.keys_out = reinterpret_cast<long long*>(keys_out);
  p.n = (int)batch;
  p.n_out = (int)vocab;
  p.eps = eps;
  return launch<2048, Q35_PRO_NORM, kEpiTop1>(p, s, pdl);
}

extern "C" int q35_gemv_batch(const q35_gemv_desc* desc, int64_t batch, void* stream) {
  return q35_gemv_batch_launch(desc, batch, (cudaStream_t)stream, false);
}
