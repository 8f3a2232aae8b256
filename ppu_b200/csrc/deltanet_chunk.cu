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
// Phase B (one CTA per (batch, head, 16 value columns), chunks in order, products on the tensor
// cores in 3xTF32):  Vn = U - W S;  O = Qe S + P Vn;  S <- gl S + Kd^T Vn;  out = bf16(O).
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

  // ---- load the chunk (bf16 -> fp32), zero padding past L: every load issued before any use
  constexpr int kLoads = kC * 3 * (kD / 8) / kThreads;  // 12 16-byte loads per thread
  const float a_log = bf2f(p.a_log[h]), dt_bias = bf2f(p.dt_bias[h]);
  const int a_off = 4 * H * kD, b_off = a_off + H;
  __shared__ float araw[kC], braw[kC];
  {
    uint4 raw[kLoads];
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int i = tid + u * kThreads;
      const int r = i / (3 * kD / 8), rem = i % (3 * kD / 8);
      const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
      const int t = t0 + r;
      raw[u] = (t < L) ? *reinterpret_cast<const uint4*>(p.qkv + ((int64_t)b * L + t) * qkv_stride + which * H * kD +
                                                         h * kD + col)
                       : make_uint4(0, 0, 0, 0);
    }
    if (tid < 2 * kC) {  // the token's a (tid < 64) or b (64 <= tid < 128) projection
      const int r = tid % kC, t = t0 + r;
      float v = 0.f;
      if (t < L) v = bf2f(p.packed[((int64_t)b * L + t) * p.packed_stride + (tid < kC ? a_off : b_off) + h]);
      (tid < kC ? araw : braw)[r] = v;
    }
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int i = tid + u * kThreads;
      const int r = i / (3 * kD / 8), rem = i % (3 * kD / 8);
      const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
      float f[8];
      unpack_bf16x8(raw[u], f);
      float* dst = (which == 0 ? q : which == 1 ? k : v) + r * kP + col;
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = f[j];
    }
  }
  __syncthreads();
  // ---- per-token factors (one warp per token)
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
        const float a = araw[r] + dt_bias;
        const float sp = a > 20.0f ? a : log1pf(expf(a));
        g = -expf(a_log) * sp;
        bt = 1.0f / (1.0f + expf(-braw[r]));
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
  // ---- T = (I - A)^-1 (A strictly lower): T_ij = sum_{j <= m < i} A_im T_mj with T_jj = 1.
  // Blocked in 16 x 16 blocks: (a) the four diagonal blocks by forward substitution in parallel;
  // (b) block rows I = 1..3 in order: R_J = sum_{J <= K < I} A_IK T_KJ, then T_IJ = T_II R_J.
  {
    constexpr int B = 16;
    const int blk = tid / 64, lt = tid % 64;
    for (int r = 1; r < B; ++r) {  // (a) row r of every diagonal block
      float nv = 0.f;
      const int i = blk * B + r;
      if (lt < r) {
        const int jj = blk * B + lt;
        float acc = T[i * 65 + jj];
        for (int m = lt + 1; m < r; ++m) acc = fmaf(T[i * 65 + blk * B + m], T[(blk * B + m) * 65 + jj], acc);
        nv = acc;
      }
      __syncthreads();
      if (lt < r) T[i * 65 + blk * B + lt] = nv;
      __syncthreads();
    }
    float* R = QK + kC * 65;  // [48][16] scratch after QK
    for (int I = 1; I < kC / B; ++I) {
      // (b1) R_J for J < I: element (J, r, cc), r = row in the block, cc = column in the block
      for (int e = tid; e < I * B * B; e += kThreads) {
        const int J = e / (B * B), r = (e / B) % B, cc = e % B;
        const int row = I * B + r, col = J * B + cc;
        float acc = T[row * 65 + col];  // K = J term with T_JJ's unit diagonal
        for (int m = J * B + cc + 1; m < I * B; ++m) acc = fmaf(T[row * 65 + m], T[m * 65 + col], acc);
        R[(J * B + r) * B + cc] = acc;
      }
      __syncthreads();
      // (b2) T_IJ = T_II R_J (T_II unit lower triangular, strictly lower part in place)
      for (int e = tid; e < I * B * B; e += kThreads) {
        const int J = e / (B * B), r = (e / B) % B, cc = e % B;
        float acc = R[(J * B + r) * B + cc];
        for (int m = 0; m < r; ++m) acc = fmaf(T[(I * B + r) * 65 + I * B + m], R[(J * B + m) * B + cc], acc);
        T[(I * B + r) * 65 + J * B + cc] = acc;
      }
      __syncthreads();
    }
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

// ---- 3xTF32 tensor-core products (m16n8k8): x = hi + lo with hi, lo TF32; hi*hi + hi*lo + lo*hi
// keeps ~FP32 accuracy (the dropped lo*lo term is below FP32 rounding of the sum).
Q35_DEV uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
Q35_DEV void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_bits(x);
  lo = tf32_bits(x - __uint_as_float(hi));
}
Q35_DEV void mma_tf32(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d += A[16 x 8] * B[8 x 8] for one k-step; a = {A[g][c], A[g+8][c], A[g][c+4], A[g+8][c+4]},
// b = {B[c][g], B[c+4][g]} (g = lane / 4, c = lane % 4).
Q35_DEV void mma3(float d[4], const float a[4], const float b[2]) {
  uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], ah[i], al[i]);
  split_tf32(b[0], bh[0], bl[0]);
  split_tf32(b[1], bh[1], bl[1]);
  mma_tf32(d, al[0], al[1], al[2], al[3], bh[0], bh[1]);
  mma_tf32(d, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
  mma_tf32(d, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
}

Q35_DEV void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

constexpr int kPS = 24;   // row stride (floats) of S / Vn tiles: B-fragment loads hit distinct banks
constexpr int kPP = 68;   // row stride of P
constexpr int kPK2 = 132; // row stride of Kd (read transposed as the A operand of Kd^T Vn)

// Phase B on the tensor cores: the CTA's 8 warps split every product into 16 x 8 output tiles.
//   Vn (64 x 16) = U - W S        warp w: rows 16 (w & 3), cols 8 (w >> 2), K = 128
//   O  (64 x 16) = Qe S + P Vn    same tiles, K = 128 + 64
//   S' (128 x 16) = gl S + Kd^T Vn  warp w: rows 16 w, both column tiles, K = 64
__global__ void __launch_bounds__(kThreads, 1) delta_chunk_scan_kernel(ScanParams p) {
  extern __shared__ __align__(16) float sm[];
  float* W = sm;                   // [64][132]
  float* Qe = W + kC * kPW;        // [64][132]
  float* Kd = Qe + kC * kPW;       // [64][132]
  float* P = Kd + kC * kPK2;       // [64][68]
  float* U = P + kC * kPP;         // [64][16]
  float* Vn = U + kC * kVS;        // [64][24]
  float* S = Vn + kC * kPS;        // [128][24]
  __shared__ float gl_s;
  const int nvs = kD / kVS;
  const int vs = blockIdx.x % nvs;
  const int h = (blockIdx.x / nvs) % p.H;
  const int b = blockIdx.x / (nvs * p.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  float* Sg = p.state + ((size_t)(b * p.H + h) * kD) * kD + vs * kVS;
  for (int i = tid; i < kD * kVS; i += kThreads) S[(i / kVS) * kPS + (i % kVS)] = Sg[(i / kVS) * kD + (i % kVS)];
  const int mt = warp & 3, nt = warp >> 2;  // Vn / O tile of this warp
  for (int ch = 0; ch < p.NC; ++ch) {
    const float* rec = p.ws + ((size_t)(b * p.H + h) * p.NC + ch) * ChunkWs::SIZE;
    __syncthreads();
    // the chunk record: all copies in flight at once (cp.async), one wait
    for (int i = tid; i < kC * kD / 4; i += kThreads) {
      const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
      cp_async16(W + r * kPW + c4, rec + ChunkWs::W + r * kD + c4);
      cp_async16(Qe + r * kPW + c4, rec + ChunkWs::Qe + r * kD + c4);
      cp_async16(Kd + r * kPK2 + c4, rec + ChunkWs::Kd + r * kD + c4);
    }
    for (int i = tid; i < kC * kC / 4; i += kThreads) {
      const int r = i / (kC / 4), c4 = (i % (kC / 4)) * 4;
      cp_async16(P + r * kPP + c4, rec + ChunkWs::P + r * kC + c4);
    }
    for (int i = tid; i < kC * kVS / 4; i += kThreads) {
      const int r = i / (kVS / 4), c4 = (i % (kVS / 4)) * 4;
      cp_async16(U + r * kVS + c4, rec + ChunkWs::U + r * kD + vs * kVS + c4);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    if (tid == 0) gl_s = rec[ChunkWs::GL];
    __syncthreads();
    const int r0 = mt * 16 + g, n0 = nt * 8;
    // ---- Vn = U - W S
    {
      float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // two chains: even / odd k-steps
#pragma unroll 4
      for (int k0 = 0; k0 < kD; k0 += 16) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int k = k0 + 8 * hh;
          const float a[4] = {W[r0 * kPW + k + c], W[(r0 + 8) * kPW + k + c], W[r0 * kPW + k + c + 4],
                              W[(r0 + 8) * kPW + k + c + 4]};
          const float bb[2] = {S[(k + c) * kPS + n0 + g], S[(k + c + 4) * kPS + n0 + g]};
          mma3(hh ? e : d, a, bb);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] += e[i];
      const int col = n0 + 2 * c;
      Vn[r0 * kPS + col] = U[r0 * kVS + col] - d[0];
      Vn[r0 * kPS + col + 1] = U[r0 * kVS + col + 1] - d[1];
      Vn[(r0 + 8) * kPS + col] = U[(r0 + 8) * kVS + col] - d[2];
      Vn[(r0 + 8) * kPS + col + 1] = U[(r0 + 8) * kVS + col + 1] - d[3];
    }
    __syncthreads();
    // ---- O = Qe S + P Vn (rows r0, r0 + 8; columns n0 + 2c, +1)
    {
      float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // Qe S and P Vn in separate chains
#pragma unroll 4
      for (int k0 = 0; k0 < kC; k0 += 8) {
        {
          const float a[4] = {Qe[r0 * kPW + k0 + c], Qe[(r0 + 8) * kPW + k0 + c], Qe[r0 * kPW + k0 + c + 4],
                              Qe[(r0 + 8) * kPW + k0 + c + 4]};
          const float bb[2] = {S[(k0 + c) * kPS + n0 + g], S[(k0 + c + 4) * kPS + n0 + g]};
          mma3(d, a, bb);
        }
        {
          const int k = kC + k0;
          const float a[4] = {Qe[r0 * kPW + k + c], Qe[(r0 + 8) * kPW + k + c], Qe[r0 * kPW + k + c + 4],
                              Qe[(r0 + 8) * kPW + k + c + 4]};
          const float bb[2] = {S[(k + c) * kPS + n0 + g], S[(k + c + 4) * kPS + n0 + g]};
          mma3(d, a, bb);
        }
        const float a[4] = {P[r0 * kPP + k0 + c], P[(r0 + 8) * kPP + k0 + c], P[r0 * kPP + k0 + c + 4],
                            P[(r0 + 8) * kPP + k0 + c + 4]};
        const float bb[2] = {Vn[(k0 + c) * kPS + n0 + g], Vn[(k0 + c + 4) * kPS + n0 + g]};
        mma3(e, a, bb);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] += e[i];
      const int col = vs * kVS + n0 + 2 * c;
      const int t0 = ch * kC + r0, t1 = t0 + 8;
      if (t0 < p.L) {
        bf16* o = p.out + (((int64_t)b * p.L + t0) * p.H + h) * kD + col;
        o[0] = f2bf(d[0]);
        o[1] = f2bf(d[1]);
      }
      if (t1 < p.L) {
        bf16* o = p.out + (((int64_t)b * p.L + t1) * p.H + h) * kD + col;
        o[0] = f2bf(d[2]);
        o[1] = f2bf(d[3]);
      }
    }
    // ---- S' = gl S + Kd^T Vn (rows 16 warp + g (+8); columns 8 n + 2c (+1), n = 0, 1)
    {
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      const int m0 = warp * 16 + g;
#pragma unroll 4
      for (int k0 = 0; k0 < kC; k0 += 8) {
        const float a[4] = {Kd[(k0 + c) * kPK2 + m0], Kd[(k0 + c) * kPK2 + m0 + 8], Kd[(k0 + c + 4) * kPK2 + m0],
                            Kd[(k0 + c + 4) * kPK2 + m0 + 8]};
        const float b0[2] = {Vn[(k0 + c) * kPS + g], Vn[(k0 + c + 4) * kPS + g]};
        const float b1[2] = {Vn[(k0 + c) * kPS + 8 + g], Vn[(k0 + c + 4) * kPS + 8 + g]};
        mma3(d0, a, b0);
        mma3(d1, a, b1);
      }
      const float gl = gl_s;
      __syncthreads();  // every warp is done reading S for this chunk
      const int col = 2 * c;
      S[m0 * kPS + col] = gl * S[m0 * kPS + col] + d0[0];
      S[m0 * kPS + col + 1] = gl * S[m0 * kPS + col + 1] + d0[1];
      S[(m0 + 8) * kPS + col] = gl * S[(m0 + 8) * kPS + col] + d0[2];
      S[(m0 + 8) * kPS + col + 1] = gl * S[(m0 + 8) * kPS + col + 1] + d0[3];
      S[m0 * kPS + 8 + col] = gl * S[m0 * kPS + 8 + col] + d1[0];
      S[m0 * kPS + 8 + col + 1] = gl * S[m0 * kPS + 8 + col + 1] + d1[1];
      S[(m0 + 8) * kPS + 8 + col] = gl * S[(m0 + 8) * kPS + 8 + col] + d1[2];
      S[(m0 + 8) * kPS + 8 + col + 1] = gl * S[(m0 + 8) * kPS + 8 + col + 1] + d1[3];
    }
  }
  __syncthreads();
  for (int i = tid; i < kD * kVS; i += kThreads) Sg[(i / kVS) * kD + (i % kVS)] = S[(i / kVS) * kPS + (i % kVS)];
}

constexpr size_t kPrepSmem = (size_t)(3 * kC * kP + 2 * kC * 65 + 48 * 16) * sizeof(float);
constexpr size_t kScanSmem =
    (size_t)(2 * kC * kPW + kC * kPK2 + kC * kPP + kC * kVS + kC * kPS + kD * kPS) * sizeof(float);

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
