// Chunked (WY / UT-transform) Gated DeltaNet prefill, FP32 (reference semantics: the gated delta
// rule of qwen35_fused/kernels.py:768-851; chunked form of HF torch_chunk_gated_delta_rule,
// chunk 64, modeling_qwen3_5.py).
//
// Phase A (one CTA per (batch, head, 64-token chunk), all chunks in parallel):
//   q_hat = q * rsqrt(|q|^2 + 1e-6) / sqrt(D), k_hat = k * rsqrt(|k|^2 + 1e-6),
//   g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b), c = cumsum(g) in the chunk;
//   A_ij = -beta_i (k_i . k_j) exp(c_i - c_j) (i > j); T = (I - A)^-1 by forward substitution;
//   U = T diag(beta) V;  W = T diag(beta exp(c)) K;  P_ij = (q_i . k_j) exp(c_i - c_j) (i >= j);
//   Qe = q_hat exp(c);   Kd = k_hat exp(c_last - c);  gl = exp(c_last).
// Phase B (one CTA per (batch, head, 16 value columns), chunks in order):
//   Vn = U - W S;  O = Qe S + P Vn;  S <- gl S + Kd^T Vn;  out = bf16(O).
// Padded tokens (beyond L) have beta = 0 and g = 0, as the reference's zero padding.
#include "common.cuh"

using namespace q35;

namespace {

constexpr int kC = 64;      // chunk length
constexpr int kD = 128;     // key / value head dim
constexpr int kVS = 16;     // value columns per phase-B CTA
constexpr int kThreads = 256;
constexpr int kP = 129;     // padded row stride (floats) of the phase-A operand tiles
constexpr int kPW = 132;    // padded row stride of phase-B W / Qe tiles (16-byte aligned rows)

struct ChunkWs {  // per (b, h, chunk) record in the workspace, FP32
  static constexpr size_t W = 0, U = W + kC * kD, Qe = U + kC * kD, Kd = Qe + kC * kD, P = Kd + kC * kD,
                          GL = P + kC * kC, SIZE = GL + 4;
};

struct PrepParams {
  const bf16* qkv;     // [B, L, 3*H*D] conv output
  const bf16* packed;  // [B, L, stride] ([qkv | z | a | b])
  const bf16* a_log;
  const bf16* dt_bias;
  float* ws;           // [B, H, NC] x ChunkWs::SIZE
  int L, H, NC, packed_stride;
};

__global__ void __launch_bounds__(kThreads, 1) delta_chunk_prep_kernel(PrepParams p) {
  extern __shared__ __align__(16) float sm[];
  float* q = sm;                 // [64][129]
  float* k = q + kC * kP;        // [64][129]
  float* v = k + kC * kP;        // [64][129]
  float* T = v + kC * kP;        // [64][65]  A then T
  float* QK = T + kC * 65;       // [64][65]
  __shared__ float c[kC], beta[kC], qs[kC], ks[kC];
  const int ch = blockIdx.x % p.NC;
  const int h = (blockIdx.x / p.NC) % p.H;
  const int b = blockIdx.x / (p.NC * p.H);
  const int H = p.H, L = p.L;
  const int t0 = ch * kC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qkv_stride = 3 * H * kD;

  // ---- load the chunk (bf16 -> fp32), zero padding past L
  for (int i = tid; i < kC * 3 * (kD / 8); i += kThreads) {
    const int r = i / (3 * kD / 8), rem = i % (3 * kD / 8);
    const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
    const int t = t0 + r;
    float f[8];
    if (t < L) {
      const uint4 u = *reinterpret_cast<const uint4*>(p.qkv + ((int64_t)b * L + t) * qkv_stride + which * H * kD +
                                                      h * kD + col);
      unpack_bf16x8(u, f);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.f;
    }
    float* dst = (which == 0 ? q : which == 1 ? k : v) + r * kP + col;
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = f[j];
  }
  __syncthreads();
  // ---- per-token factors (one warp per token)
  const float a_log = bf2f(p.a_log[h]), dt_bias = bf2f(p.dt_bias[h]);
  const int a_off = 4 * H * kD, b_off = a_off + H;
  for (int r = warp; r < kC; r += kThreads / 32) {
    float sq = 0.f, sk = 0.f;
    for (int e = lane; e < kD; e += 32) {
      sq += q[r * kP + e] * q[r * kP + e];
      sk += k[r * kP + e] * k[r * kP + e];
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      qs[r] = rsqrt_ieee(sq + 1e-6f);
      ks[r] = rsqrt_ieee(sk + 1e-6f);
      const int t = t0 + r;
      float g = 0.f, bt = 0.f;
      if (t < L) {
        const bf16* pr = p.packed + ((int64_t)b * L + t) * p.packed_stride;
        const float a = bf2f(pr[a_off + h]) + dt_bias;
        const float sp = a > 20.0f ? a : log1pf(expf(a));
        g = -expf(a_log) * sp;
        bt = 1.0f / (1.0f + expf(-bf2f(pr[b_off + h])));
      }
      c[r] = g;
      beta[r] = bt;
    }
  }
  __syncthreads();
  if (tid == 0) {  // cumulative log decay, in token order
    float acc = 0.f;
    for (int r = 0; r < kC; ++r) {
      acc += c[r];
      c[r] = acc;
    }
  }
  // normalise q, k in place: q_hat = (q * q_inv) / sqrt(D) (kernels.py:826-827 association)
  const float qscale = 1.0f / sqrtf((float)kD);
  for (int i = tid; i < kC * kD; i += kThreads) {
    const int r = i / kD, e = i % kD;
    q[r * kP + e] = (q[r * kP + e] * qs[r]) * qscale;
    k[r * kP + e] = k[r * kP + e] * ks[r];
  }
  __syncthreads();
  // ---- KK and QK (64 x 64): thread (ti, tj) owns a 4 x 4 block
  {
    const int ti = tid / 16, tj = tid % 16;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) kk[a][bb] = qk[a][bb] = 0.f;
    for (int e = 0; e < kD; ++e) {
      float ki[4], qi[4], kj[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        ki[a] = k[(4 * ti + a) * kP + e];
        qi[a] = q[(4 * ti + a) * kP + e];
        kj[a] = k[(4 * tj + a) * kP + e];
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          kk[a][bb] = fmaf(ki[a], kj[bb], kk[a][bb]);
          qk[a][bb] = fmaf(qi[a], kj[bb], qk[a][bb]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const int i = 4 * ti + a, j = 4 * tj + bb;
        T[i * 65 + j] = (j < i) ? -(beta[i] * kk[a][bb]) * expf(c[i] - c[j]) : 0.f;
        QK[i * 65 + j] = (j <= i) ? qk[a][bb] * expf(c[i] - c[j]) : 0.f;
      }
  }
  __syncthreads();
  // ---- T = (I - A)^-1, forward substitution row by row (rows < i are final)
  for (int i = 1; i < kC; ++i) {
    float nv = 0.f;
    if (tid < i) {
      const int j = tid;
      float s = 0.f;
      for (int m = j + 1; m < i; ++m) s = fmaf(T[i * 65 + m], T[m * 65 + j], s);
      nv = T[i * 65 + j] + s;
    }
    __syncthreads();
    if (tid < i) T[i * 65 + tid] = nv;
    __syncthreads();
  }
  if (tid < kC) T[tid * 65 + tid] = 1.0f;
  __syncthreads();
  // ---- U = T diag(beta) V, W = T diag(beta exp(c)) K; thread owns column e and 32 rows
  float* out = p.ws + ((size_t)(b * H + h) * p.NC + ch) * ChunkWs::SIZE;
  {
    const int e = tid % kD, i0 = (tid / kD) * 32;
    float u[32], w[32];
#pragma unroll
    for (int a = 0; a < 32; ++a) u[a] = w[a] = 0.f;
    for (int j = 0; j < kC; ++j) {
      const float bv = beta[j] * v[j * kP + e];
      const float bk = (beta[j] * expf(c[j])) * k[j * kP + e];
#pragma unroll
      for (int a = 0; a < 32; ++a) {
        const float tij = T[(i0 + a) * 65 + j];
        u[a] = fmaf(tij, bv, u[a]);
        w[a] = fmaf(tij, bk, w[a]);
      }
    }
#pragma unroll
    for (int a = 0; a < 32; ++a) {
      out[ChunkWs::U + (i0 + a) * kD + e] = u[a];
      out[ChunkWs::W + (i0 + a) * kD + e] = w[a];
    }
  }
  const float cl = c[kC - 1];
  for (int i = tid; i < kC * kD; i += kThreads) {
    const int r = i / kD, e = i % kD;
    out[ChunkWs::Qe + i] = q[r * kP + e] * expf(c[r]);
    out[ChunkWs::Kd + i] = k[r * kP + e] * expf(cl - c[r]);
  }
  for (int i = tid; i < kC * kC; i += kThreads) out[ChunkWs::P + i] = QK[(i / kC) * 65 + (i % kC)];
  if (tid == 0) out[ChunkWs::GL] = expf(cl);
}

struct ScanParams {
  const float* ws;
  float* state;   // [B, H, D(k), D(v)]
  bf16* out;      // [B, L, H, D]
  int L, H, NC;
};

__global__ void __launch_bounds__(kThreads, 1) delta_chunk_scan_kernel(ScanParams p) {
  extern __shared__ __align__(16) float sm[];
  float* W = sm;                  // [64][132]
  float* Qe = W + kC * kPW;       // [64][132]
  float* Kd = Qe + kC * kPW;      // [64][128]
  float* P = Kd + kC * kD;        // [64][64]
  float* U = P + kC * kC;         // [64][16]
  float* Vn = U + kC * kVS;       // [64][16]
  float* S = Vn + kC * kVS;       // [128][16]
  __shared__ float gl_s;
  const int nvs = kD / kVS;
  const int vs = blockIdx.x % nvs;
  const int h = (blockIdx.x / nvs) % p.H;
  const int b = blockIdx.x / (nvs * p.H);
  const int tid = threadIdx.x;
  float* Sg = p.state + ((size_t)(b * p.H + h) * kD) * kD + vs * kVS;
  for (int i = tid; i < kD * kVS; i += kThreads) S[i] = Sg[(i / kVS) * kD + (i % kVS)];
  for (int ch = 0; ch < p.NC; ++ch) {
    const float* rec = p.ws + ((size_t)(b * p.H + h) * p.NC + ch) * ChunkWs::SIZE;
    __syncthreads();
    for (int i = tid; i < kC * kD / 4; i += kThreads) {
      const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
      *reinterpret_cast<float4*>(W + r * kPW + c4) = *reinterpret_cast<const float4*>(rec + ChunkWs::W + r * kD + c4);
      *reinterpret_cast<float4*>(Qe + r * kPW + c4) = *reinterpret_cast<const float4*>(rec + ChunkWs::Qe + r * kD + c4);
      *reinterpret_cast<float4*>(Kd + r * kD + c4) = *reinterpret_cast<const float4*>(rec + ChunkWs::Kd + r * kD + c4);
    }
    for (int i = tid; i < kC * kC / 4; i += kThreads)
      reinterpret_cast<float4*>(P)[i] = reinterpret_cast<const float4*>(rec + ChunkWs::P)[i];
    for (int i = tid; i < kC * kVS; i += kThreads) U[i] = rec[ChunkWs::U + (i / kVS) * kD + vs * kVS + (i % kVS)];
    if (tid == 0) gl_s = rec[ChunkWs::GL];
    __syncthreads();
    // Vn = U - W S (thread: column e, rows i0..i0+3)
    const int e = tid % kVS, i0 = (tid / kVS) * 4;
    {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kk = 0; kk < kD; ++kk) {
        const float sv = S[kk * kVS + e];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc[a] = fmaf(W[(i0 + a) * kPW + kk], sv, acc[a]);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) Vn[(i0 + a) * kVS + e] = U[(i0 + a) * kVS + e] - acc[a];
    }
    __syncthreads();
    // O = Qe S + P Vn
    {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kk = 0; kk < kD; ++kk) {
        const float sv = S[kk * kVS + e];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc[a] = fmaf(Qe[(i0 + a) * kPW + kk], sv, acc[a]);
      }
      for (int j = 0; j < kC; ++j) {
        const float vn = Vn[j * kVS + e];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc[a] = fmaf(P[(i0 + a) * kC + j], vn, acc[a]);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int t = ch * kC + i0 + a;
        if (t < p.L) p.out[(((int64_t)b * p.L + t) * p.H + h) * kD + vs * kVS + e] = f2bf(acc[a]);
      }
    }
    // S <- gl S + Kd^T Vn (thread: column e, key rows k0..k0+7)
    {
      const int k0 = (tid / kVS) * 8;
      float acc[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) acc[a] = 0.f;
      for (int j = 0; j < kC; ++j) {
        const float vn = Vn[j * kVS + e];
#pragma unroll
        for (int a = 0; a < 8; ++a) acc[a] = fmaf(Kd[j * kD + k0 + a], vn, acc[a]);
      }
      const float gl = gl_s;
      __syncthreads();  // every thread is done reading S for this chunk
#pragma unroll
      for (int a = 0; a < 8; ++a) S[(k0 + a) * kVS + e] = gl * S[(k0 + a) * kVS + e] + acc[a];
    }
  }
  __syncthreads();
  for (int i = tid; i < kD * kVS; i += kThreads) Sg[(i / kVS) * kD + (i % kVS)] = S[i];
}

constexpr size_t kPrepSmem = (size_t)(3 * kC * kP + 2 * kC * 65) * sizeof(float);
constexpr size_t kScanSmem = (size_t)(2 * kC * kPW + kC * kD + kC * kC + 2 * kC * kVS + kD * kVS) * sizeof(float);

}  // namespace

size_t q35_delta_chunk_workspace_bytes(int64_t batch, int64_t heads, int64_t max_len) {
  const int64_t nc = (max_len + kC - 1) / kC;
  return (size_t)batch * heads * nc * ChunkWs::SIZE * sizeof(float);
}

int q35_delta_chunked_launch(const void* qkv, const void* packed, const void* a_log, const void* dt_bias, float* state,
                             void* out, int64_t batch, int64_t seq_len, int64_t heads, int64_t packed_stride,
                             float* ws, cudaStream_t s) {
  if (batch * seq_len == 0) return Q35_OK;
  const int nc = (int)((seq_len + kC - 1) / kC);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(delta_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrepSmem);
    cudaFuncSetAttribute(delta_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem);
    attr = true;
  }
  PrepParams pp{(const bf16*)qkv, (const bf16*)packed, (const bf16*)a_log, (const bf16*)dt_bias, ws, (int)seq_len,
                (int)heads, nc, (int)packed_stride};
  delta_chunk_prep_kernel<<<(unsigned)(batch * heads * nc), kThreads, kPrepSmem, s>>>(pp);
  int rc = q35_check_launch("delta_chunk_prep");
  if (rc) return rc;
  ScanParams sp{ws, state, (bf16*)out, (int)seq_len, (int)heads, nc};
  delta_chunk_scan_kernel<<<(unsigned)(batch * heads * (kD / kVS)), kThreads, kScanSmem, s>>>(sp);
  return q35_check_launch("delta_chunk_scan");
}

extern "C" size_t q35_delta_chunked_workspace_size(int64_t batch, int64_t heads, int64_t seq_len) {
  return q35_delta_chunk_workspace_bytes(batch, heads, seq_len);
}

extern "C" int q35_delta_chunked(const void* qkv, const void* packed, const void* a_log, const void* dt_bias,
                                 float* state, void* out, int64_t batch, int64_t seq_len, int64_t heads, int64_t dim,
                                 int64_t packed_stride, void* workspace, size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(qkv && packed && a_log && dt_bias && state && out && workspace, "delta_chunked: null pointer");
  Q35_REQUIRE(dim == kD, "delta_chunked: head dim must be 128");
  Q35_REQUIRE(batch >= 0 && seq_len >= 0 && heads >= 1 && packed_stride >= 4 * heads * dim + 2 * heads,
              "delta_chunked: bad shape");
  Q35_REQUIRE(Q35_ALIGNED(qkv, 16) && Q35_ALIGNED(workspace, 16), "delta_chunked: 16-byte alignment");
  Q35_REQUIRE(workspace_bytes >= q35_delta_chunk_workspace_bytes(batch, heads, seq_len),
              "delta_chunked: workspace too small");
  return q35_delta_chunked_launch(qkv, packed, a_log, dt_bias, state, out, batch, seq_len, heads, packed_stride,
                                  static_cast<float*>(workspace), (cudaStream_t)stream);
}
