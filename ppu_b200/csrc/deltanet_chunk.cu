// Chunked (WY / UT-transform) Gated DeltaNet prefill, FP32 (reference semantics: the gated delta
// rule of qwen35_fused/kernels.py:768-851; chunked form of HF torch_chunk_gated_delta_rule,
// chunk 64, modeling_qwen3_5.py).
//
// Phase A (one CTA per (batch, head, 64-token chunk), all chunks in parallel, products on the
// tensor cores: bf16 for KK / QK, TF32-split left factor for U / W):
//   q_hat = q * rsqrt(|q|^2 + 1e-6) / sqrt(D), k_hat = k * rsqrt(|k|^2 + 1e-6),
//   g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b), c = cumsum(g) in the chunk;
//   A_ij = -beta_i (k_i . k_j) exp(c_i - c_j) (i > j); T = (I - A)^-1 by blocked substitution;
//   U = T diag(beta) V;  W = T diag(beta exp(c)) K;  P_ij = (q_i . k_j) exp(c_i - c_j) (i >= j);
//   Qe = q_hat exp(c);   Kd = k_hat exp(c_last - c);  gl = exp(c_last).
// Phase B, the recurrence (one CTA per (batch, head, 16 value columns), chunks in order, products
// on mma.sync in 3xTF32): keep S_c (the state entering chunk c);  Vn = U - W S;
// S <- gl S + Kd^T Vn.
// Phase C, the output (one CTA per (batch, head, chunk, 64 value columns), all chunks at once, on
// tcgen05 with a TMEM accumulator, 3xTF32): out = bf16(Qe S_c + P Vn).
// Padded tokens (beyond L) have beta = 0 and g = 0, as the reference's zero padding.
#include "common.cuh"
#include "tcgen05.cuh"

using namespace q35;

__device__ int q35_delta_chunk_error_word = 0;

namespace {

constexpr int kC = 64;      // chunk length
constexpr int kD = 128;     // key / value head dim
constexpr int kVS = 16;     // value columns per phase-B CTA
constexpr int kThreads = 256;
constexpr int kPW = 132;    // padded row stride of phase-B W tiles (16-byte aligned rows)
constexpr int kPK2 = 136;   // row stride of Kd (read transposed as the A operand of Kd^T Vn: distinct banks)

struct ChunkWs {  // per (b, h, chunk) record in the workspace, FP32
  // prep: W [64][kPW] and Kd [64][kPK2] (the recurrence's shared-memory row strides, so that each
  // arrives in one bulk copy), U [128 / kVS][64][kVS] (one recurrence CTA's value columns
  // contiguous), Qe [64][128], P [64][64], gl; recurrence: ST = S_c^T [128 value][128 key] (the
  // state entering the chunk, transposed) and VT = Vn^T [128 value][64 token]
  static constexpr size_t W = 0, U = W + kC * kPW, Qe = U + kC * kD, Kd = Qe + kC * kD, P = Kd + kC * kPK2,
                          GL = P + kC * kC, ST = GL + 4, VT = ST + kD * kD, SIZE = VT + kD * kC;
};
static_assert(ChunkWs::U % 4 == 0 && ChunkWs::Kd % 4 == 0 && ChunkWs::P % 4 == 0, "16-byte aligned records");
static_assert(ChunkWs::ST % 4 == 0 && ChunkWs::VT % 4 == 0 && ChunkWs::SIZE % 4 == 0, "16-byte aligned fields");

struct PrepParams {
  const bf16* qkv;       // [B, L, 3*H*D] conv output (when conv_w is null)
  const bf16* packed;    // [B, L, stride] ([qkv | z | a | b])
  const bf16* a_log;
  const bf16* dt_bias;
  const bf16* conv_w;    // [3*H*D, 4] or null: the causal conv (4 taps, zero history) runs in the prep
  bf16* conv_state;      // [B, 3*H*D, 4] receives the last 4 raw inputs (conv_w set, L >= 4)
  float* ws;             // [B, H, NC] x ChunkWs::SIZE
  int L, H, NC, packed_stride;
};
constexpr int kHalo = 3;  // raw rows before the chunk that the 4-tap conv reads

// ---- tensor-core helpers (mma.sync). Fragments of m16n8k8 TF32 (g = lane / 4, c = lane % 4):
// a = {A[g][c], A[g+8][c], A[g][c+4], A[g+8][c+4]}, b = {B[c][g], B[c+4][g]},
// d = {D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1]}. m16n8k16 bf16: a holds pairs
// {A[g][2c..2c+1], A[g+8][2c..], A[g][2c+8..], A[g+8][2c+8..]}, b = {B[2c..2c+1][g], B[2c+8..][g]}.
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
Q35_DEV void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
Q35_DEV uint32_t lds32(const bf16* p) { return *reinterpret_cast<const uint32_t*>(p); }
// a bf16 value as a TF32 operand: its FP32 bit pattern has the low 16 bits zero, so it is exact
Q35_DEV uint32_t bf16_as_tf32(bf16 x) { return (uint32_t)__bfloat16_as_ushort(x) << 16; }

constexpr int kPB = 136;  // row stride (bf16) of the raw q / k / v tiles: fragment loads hit distinct banks
constexpr int kTS = 68;   // row stride (floats) of T: A-fragment loads hit distinct banks

// Phase A on the tensor cores. q, k, v stay raw bf16 in shared memory (the normalisations are
// per-row scales): KK = k k^T and QK = q k^T are exact bf16 products with FP32 accumulation,
// scaled by the row factors afterwards; U = (T diag(beta)) V and W = (T diag(beta e^c ks)) k take
// the FP32 left factor split into TF32 high + low parts against the exactly representable bf16
// right factor (two MMAs per step, FP32-level accuracy). ~73 KB of shared memory: two CTAs per SM.
__global__ void __launch_bounds__(kThreads, 2) delta_chunk_prep_kernel(PrepParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // q, k, v tiles [kHalo + 64][136] (bf16) with row 0 of the chunk at kHalo: the halo rows hold the
  // conv's raw inputs before the chunk when the conv runs here
  bf16* qb = reinterpret_cast<bf16*>(smem_raw) + kHalo * kPB;
  bf16* kb = qb + (kHalo + kC) * kPB;
  bf16* vb = kb + (kHalo + kC) * kPB;
  float* T = reinterpret_cast<float*>(vb + kC * kPB);    // [64][68]  A, then T = (I - A)^-1
  float* R = T + kC * kTS;                               // [48][16]  solve scratch
  __shared__ float c[kC], beta[kC], qs[kC], ks[kC], araw[kC], braw[kC], su[kC], sw[kC], ec[kC], ed[kC];
  const int ch = blockIdx.x % p.NC;
  const int h = (blockIdx.x / p.NC) % p.H;
  const int b = blockIdx.x / (p.NC * p.H);
  const int H = p.H, L = p.L;
  const int t0 = ch * kC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, cq = lane & 3;
  const int qkv_stride = 3 * H * kD;

  // ---- load the chunk (raw bf16), zero padding past L: every load issued before any use
  constexpr int kLoads = kC * 3 * (kD / 8) / kThreads;  // 12 16-byte loads per thread
  const float a_log = bf2f(p.a_log[h]), dt_bias = bf2f(p.dt_bias[h]);
  const int a_off = 4 * H * kD, b_off = a_off + H;
  if (tid < 2 * kC) {  // the token's a (tid < 64) or b (64 <= tid < 128) projection
    const int r = tid % kC, t = t0 + r;
    float v = 0.f;
    if (t < L) v = bf2f(p.packed[((int64_t)b * L + t) * p.packed_stride + (tid < kC ? a_off : b_off) + h]);
    (tid < kC ? araw : braw)[r] = v;
  }
  if (p.conv_w != nullptr) {
    // raw projection rows t0 - 3 .. t0 + 63 (zero before 0 and from L on) into tile rows -3 .. 63:
    // every load issued before any store
    constexpr int kChunks = (kHalo + kC) * 3 * (kD / 8);
    constexpr int kCLoads = (kChunks + kThreads - 1) / kThreads;  // 13 16-byte loads per thread
    uint4 raw[kCLoads];
#pragma unroll
    for (int u = 0; u < kCLoads; ++u) {
      const int i = tid + u * kThreads;
      const int rr = i / (3 * kD / 8), rem = i % (3 * kD / 8);
      const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
      const int t = t0 - kHalo + rr;
      raw[u] = (i < kChunks && t >= 0 && t < L)
                   ? *reinterpret_cast<const uint4*>(p.packed + ((int64_t)b * L + t) * p.packed_stride + which * H * kD +
                                                     h * kD + col)
                   : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kCLoads; ++u) {
      const int i = tid + u * kThreads;
      if (i >= kChunks) break;
      const int rr = i / (3 * kD / 8), rem = i % (3 * kD / 8);
      const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
      *reinterpret_cast<uint4*>((which == 0 ? qb : which == 1 ? kb : vb) + (rr - kHalo) * kPB + col) = raw[u];
    }
    __syncthreads();
    // conv state: the chunk holding token L - 1 stores the head's last 4 raw inputs per channel
    // (causal_conv1d_fused's state update; rows L - 4 - t0 .. L - 1 - t0 lie in [-3, 63])
    if (ch == p.NC - 1) {
      for (int i = tid; i < 3 * kD * 4; i += kThreads) {
        const int c = i / 4, j = i % 4, which = c / kD, cc = c % kD;
        const bf16* tile = which == 0 ? qb : which == 1 ? kb : vb;
        p.conv_state[((int64_t)b * 3 * H * kD + which * H * kD + h * kD + cc) * 4 + j] =
            tile[(L - 4 + j - t0) * kPB + cc];
      }
    }
    __syncthreads();  // the state copy has read the raw rows the conv overwrites
    // causal conv + SiLU down each column with a 4-tap register window, in place (output row r
    // replaces raw row r once read); same tap order and rounding as the separate conv, zero past L.
    // Work unit: (two adjacent columns, quarter of the chunk's rows), three per thread run
    // interleaved, the two columns on paired FP32 FMAs (each half one IEEE fma, as the scalar
    // form); each unit reads its three rows of history before the barrier, so the in-place writes
    // cannot race.
    {
      constexpr int kQ = 4, kRows = kC / kQ, kPairs = 3 * kD / 2, kTasks = kPairs * kQ / kThreads;
      static_assert(kPairs * kQ == kTasks * kThreads, "whole units per thread");
      float2 wk[kTasks][4], hist[kTasks][4];
      int off[kTasks], rlim[kTasks];
      auto ld_pair = [&](int o) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(qb + o);
        return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
      };
#pragma unroll
      for (int k = 0; k < kTasks; ++k) {
        const int task = tid + k * kThreads, pidx = task % kPairs, qtr = task / kPairs;
        const int which = pidx / (kD / 2), cc = (pidx % (kD / 2)) * 2;
        off[k] = which * (int)((kHalo + kC) * kPB) + qtr * kRows * kPB + cc;  // from qb (tiles are contiguous)
        rlim[k] = L - t0 - qtr * kRows;
        const int chn = which * H * kD + h * kD + cc;
#pragma unroll
        for (int tap = 0; tap < 4; ++tap)
          wk[k][tap] = make_float2(bf2f(p.conv_w[(int64_t)chn * 4 + tap]), bf2f(p.conv_w[(int64_t)(chn + 1) * 4 + tap]));
#pragma unroll
        for (int j = 0; j < kHalo; ++j) hist[k][j] = ld_pair(off[k] + (j - kHalo) * kPB);
      }
      __syncthreads();  // all history rows read
#pragma unroll 2
      for (int r = 0; r < kRows; ++r) {
#pragma unroll
        for (int k = 0; k < kTasks; ++k) {
          const int o = off[k] + r * kPB;
          hist[k][3] = ld_pair(o);
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int tap = 0; tap < 4; ++tap) acc = __ffma2_rn(hist[k][tap], wk[k][tap], acc);
          const float2 y = __bfloat1622float2(__floats2bfloat162_rn(acc.x, acc.y));  // rbf of both
          const __nv_bfloat162 v = (r < rlim[k]) ? __floats2bfloat162_rn(silu_f(y.x), silu_f(y.y))
                                                 : __floats2bfloat162_rn(0.f, 0.f);
          *reinterpret_cast<__nv_bfloat162*>(qb + o) = v;
          hist[k][0] = hist[k][1];
          hist[k][1] = hist[k][2];
          hist[k][2] = hist[k][3];
        }
      }
    }
  } else {
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
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int i = tid + u * kThreads;
      const int r = i / (3 * kD / 8), rem = i % (3 * kD / 8);
      const int which = rem / (kD / 8), col = (rem % (kD / 8)) * 8;
      bf16* dst = (which == 0 ? qb : which == 1 ? kb : vb) + r * kPB + col;
      *reinterpret_cast<uint4*>(dst) = raw[u];
    }
  }
  __syncthreads();
  // ---- per-token factors. Squared norms: warp w sums tokens 8w .. 8w + 8 (interleaved, each in
  // the order of one warp per token: lane-strided partial sums, then the butterfly); the gates:
  // thread r < 64 for token r
  {
    float sq[8], sk[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = warp * 8 + j;
      float a = 0.f, bb = 0.f;
#pragma unroll
      for (int e = lane; e < kD; e += 32) {
        const float qv = bf2f(qb[r * kPB + e]), kv = bf2f(kb[r * kPB + e]);
        a += qv * qv;
        bb += kv * kv;
      }
      sq[j] = a;
      sk[j] = bb;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sq[j] = warp_sum(sq[j]);
      sk[j] = warp_sum(sk[j]);
    }
    if (lane < 8) {
      float mq = sq[0], mk = sk[0];
#pragma unroll
      for (int j = 1; j < 8; ++j)
        if (lane == j) {
          mq = sq[j];
          mk = sk[j];
        }
      qs[warp * 8 + lane] = rsqrt_ieee(mq + 1e-6f);
      ks[warp * 8 + lane] = rsqrt_ieee(mk + 1e-6f);
    }
    if (tid < kC) {
      const int t = t0 + tid;
      float gg = 0.f, bt = 0.f;
      if (t < L) {
        const float a = araw[tid] + dt_bias;
        const float sp = a > 20.0f ? a : log1pf(expf(a));
        gg = -expf(a_log) * sp;
        bt = 1.0f / (1.0f + expf(-braw[tid]));
      }
      c[tid] = gg;
      beta[tid] = bt;
    }
  }
  __syncthreads();
  if (tid == 0) {  // cumulative log decay, in token order (values in registers: one dependent add each)
    float v[kC];
#pragma unroll
    for (int r = 0; r < kC; ++r) v[r] = c[r];
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kC; ++r) {
      acc += v[r];
      c[r] = acc;
    }
  }
  __syncthreads();
  // ---- Qe = q_hat e^c, Kd = k_hat e^(c_last - c) with q_hat = (q qs) / sqrt(D) (kernels.py:826-827
  // association), k_hat = k ks; column scales of the U / W left factors
  float* out = p.ws + ((size_t)(b * H + h) * p.NC + ch) * ChunkWs::SIZE;
  const float cl = c[kC - 1];
  const float qscale = 1.0f / sqrtf((float)kD);
  if (tid < kC) {  // the row exponentials once per token
    ec[tid] = expf(c[tid]);
    ed[tid] = expf(cl - c[tid]);
  }
  __syncthreads();
  for (int i = tid; i < kC * kD; i += kThreads) {
    const int r = i / kD, e = i % kD;
    out[ChunkWs::Qe + i] = ((bf2f(qb[r * kPB + e]) * qs[r]) * qscale) * ec[r];
    out[ChunkWs::Kd + r * kPK2 + e] = (bf2f(kb[r * kPB + e]) * ks[r]) * ed[r];
  }
  if (tid < kC) {
    su[tid] = beta[tid];
    sw[tid] = (beta[tid] * ec[tid]) * ks[tid];
  }
  if (tid == 0) out[ChunkWs::GL] = expf(cl);
  // ---- KK = k k^T and QK = q k^T (64 x 64, K = 128) on bf16 mma.sync: warp w computes rows
  // 16 (w & 3) .. + 16 against key columns 32 (w >> 2) .. + 32 (four 8-column tiles)
  {
    const int mt = warp & 3, nb = (warp >> 2) * 4;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) kk[n][i] = qk[n][i] = 0.f;
#pragma unroll 2
    for (int k0 = 0; k0 < kD; k0 += 16) {
      const bf16* ka = kb + (16 * mt + g) * kPB + k0 + 2 * cq;
      const bf16* qa = qb + (16 * mt + g) * kPB + k0 + 2 * cq;
      const uint32_t ak[4] = {lds32(ka), lds32(ka + 8 * kPB), lds32(ka + 8), lds32(ka + 8 * kPB + 8)};
      const uint32_t aq[4] = {lds32(qa), lds32(qa + 8 * kPB), lds32(qa + 8), lds32(qa + 8 * kPB + 8)};
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const bf16* kbp = kb + (8 * (nb + n) + g) * kPB + k0 + 2 * cq;
        const uint32_t b0 = lds32(kbp), b1 = lds32(kbp + 8);
        mma_bf16(kk[n], ak, b0, b1);
        mma_bf16(qk[n], aq, b0, b1);
      }
    }
    // A_ij = -beta_i (k_hat_i . k_hat_j) e^(c_i - c_j) (j < i) into T; P_ij = (q_hat_i . k_hat_j)
    // e^(c_i - c_j) (j <= i) to the workspace
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = 16 * mt + g + 8 * half, j = 8 * (nb + n) + 2 * cq;
        float pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = j + e;
          const float dec = expf(c[i] - c[jj]);
          const float kkh = (kk[n][2 * half + e] * ks[i]) * ks[jj];
          T[i * kTS + jj] = (jj < i) ? -(beta[i] * kkh) * dec : 0.f;
          pv[e] = (jj <= i) ? (((qk[n][2 * half + e] * qs[i]) * qscale) * ks[jj]) * dec : 0.f;
        }
        *reinterpret_cast<float2*>(out + ChunkWs::P + i * kC + j) = make_float2(pv[0], pv[1]);
      }
  }
  __syncthreads();
  // ---- T = (I - A)^-1 (A strictly lower), in 16 x 16 blocks. The blocks below the diagonal
  // band are overwritten by T as it is formed, so their A values are first copied into q's tile
  // (q is no longer read: Qe and QK are done).
  // (a) Diagonal blocks T_II by forward substitution, one half-warp per block, lane = column:
  //     T_rj = A_rj + sum_{j < m < r} A_rm T_mj, m ascending, the column kept in registers.
  // (b) Off-diagonal blocks T_IJ = T_II (A_IJ T_JJ + sum_{J < K < I} A_IK T_KJ), by diagonals:
  //     I - J = 1 (three blocks at once), 2 (two), 3 (one); each diagonal is two 16 x 16 x 16k
  //     products (X = sum_K A_IK T_KJ into the scratch R, then T_IJ = T_II X), one output element
  //     per thread with the reduction unrolled.
  {
    constexpr int B = 16;
    float* Ac = reinterpret_cast<float*>(smem_raw);  // [64][kTS]: A rows 16 .. 63, columns < the row's block
    for (int e = tid; e < 6 * B * B; e += kThreads) {
      const int blk = e / (B * B), r = (e / B) % B, cc = e % B;
      const int I = blk < 1 ? 1 : blk < 3 ? 2 : 3, J = blk - (I * (I - 1)) / 2;  // (1,0) (2,0) (2,1) (3,0) (3,1) (3,2)
      Ac[(I * B + r) * kTS + J * B + cc] = T[(I * B + r) * kTS + J * B + cc];
    }
    if (warp < 2) {
      const int blk = warp * 2 + (lane >> 4), lt = lane & 15;
      float* Tb = T + blk * B * kTS + blk * B;  // the block's top-left corner
      float col[B];
#pragma unroll
      for (int r = 0; r < B; ++r) col[r] = 0.f;
#pragma unroll
      for (int r = 1; r < B; ++r) {
        float acc = Tb[r * kTS + lt];
#pragma unroll
        for (int m = 1; m < r; ++m)
          if (m > lt) acc = fmaf(Tb[r * kTS + m], col[m], acc);
        col[r] = acc;
      }
#pragma unroll
      for (int r = 1; r < B; ++r)
        if (r > lt) Tb[r * kTS + lt] = col[r];
    }
    __syncthreads();  // the diagonal blocks and the copy of A are complete
#pragma unroll 1
    for (int dg = 1; dg < kC / B; ++dg) {
      const int nblk = kC / B - dg;  // blocks (I, J = I - dg), I = dg .. 3
      // X_IJ = A_IJ T_JJ + sum_{J < K < I} A_IK T_KJ = sum_{J <= K < I} A_IK T_KJ (T_JJ unit diagonal)
      for (int e = tid; e < nblk * B * B; e += kThreads) {
        const int q = e / (B * B), r = (e / B) % B, cc = e % B;
        const int I = dg + q, J = q;
        const float* arow = Ac + (I * B + r) * kTS;
        float acc = 0.f;
        for (int K = J; K < I; ++K) {
#pragma unroll
          for (int m = 0; m < B; ++m) {
            const float tv = (K == J) ? (m == cc ? 1.f : (m > cc ? T[(K * B + m) * kTS + J * B + cc] : 0.f))
                                      : T[(K * B + m) * kTS + J * B + cc];
            acc = fmaf(arow[K * B + m], tv, acc);
          }
        }
        R[(q * B + r) * B + cc] = acc;
      }
      __syncthreads();
      // T_IJ = T_II X (T_II unit lower triangular)
      for (int e = tid; e < nblk * B * B; e += kThreads) {
        const int q = e / (B * B), r = (e / B) % B, cc = e % B;
        const int I = dg + q, J = q;
        const float* trow = T + (I * B + r) * kTS + I * B;
        float acc = R[(q * B + r) * B + cc];
#pragma unroll
        for (int m = 0; m < B; ++m)
          if (m < r) acc = fmaf(trow[m], R[(q * B + m) * B + cc], acc);
        T[(I * B + r) * kTS + J * B + cc] = acc;
      }
      __syncthreads();
    }
  }
  if (tid < kC) T[tid * kTS + tid] = 1.0f;
  __syncthreads();
  // ---- U = (T diag(beta)) V and W = (T diag(beta e^c ks)) k (64 x 128 each, K = 64 tokens):
  // warp w computes rows 16 (w & 3) .. + 16 and value / key columns 64 (w >> 2) .. + 64
  {
    const int mt = warp & 3, nb = (warp >> 2) * 8;
    float u[8][4], wv[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) u[n][i] = wv[n][i] = 0.f;
    const float* t_lo = T + (16 * mt + g) * kTS;
    const float* t_hi = t_lo + 8 * kTS;
#pragma unroll 2
    for (int j0 = 0; j0 < kC; j0 += 8) {
      const int ja = j0 + cq, jb = ja + 4;
      const float ta[4] = {t_lo[ja], t_hi[ja], t_lo[jb], t_hi[jb]};
      const float sua[2] = {su[ja], su[jb]}, swa[2] = {sw[ja], sw[jb]};
      uint32_t uh[4], ul[4], wh[4], wl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        split_tf32(ta[i] * sua[i >> 1], uh[i], ul[i]);
        split_tf32(ta[i] * swa[i >> 1], wh[i], wl[i]);
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int col = 8 * (nb + n) + g;
        const uint32_t bv0 = bf16_as_tf32(vb[ja * kPB + col]), bv1 = bf16_as_tf32(vb[jb * kPB + col]);
        const uint32_t bk0 = bf16_as_tf32(kb[ja * kPB + col]), bk1 = bf16_as_tf32(kb[jb * kPB + col]);
        mma_tf32(u[n], ul[0], ul[1], ul[2], ul[3], bv0, bv1);
        mma_tf32(u[n], uh[0], uh[1], uh[2], uh[3], bv0, bv1);
        mma_tf32(wv[n], wl[0], wl[1], wl[2], wl[3], bk0, bk1);
        mma_tf32(wv[n], wh[0], wh[1], wh[2], wh[3], bk0, bk1);
      }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = 16 * mt + g + 8 * half, e = 8 * (nb + n) + 2 * cq;
        *reinterpret_cast<float2*>(out + ChunkWs::U + ((e / kVS) * kC + i) * kVS + e % kVS) =
            make_float2(u[n][2 * half], u[n][2 * half + 1]);
        *reinterpret_cast<float2*>(out + ChunkWs::W + i * kPW + e) = make_float2(wv[n][2 * half], wv[n][2 * half + 1]);
      }
  }
}

struct ScanParams {
  float* ws;      // the chunk records (S_c^T and Vn^T are written here)
  float* state;   // [B, H, D(k), D(v)]
  int L, H, NC;
};

// ---- 3xTF32 products in the scan (m16n8k8): x = hi + lo with hi, lo TF32; hi*hi + hi*lo + lo*hi
// keeps ~FP32 accuracy (the dropped lo*lo term is below FP32 rounding of the sum).
constexpr int kPS = 24;   // row stride (words) of the pre-split S / Vn tiles: B-fragment loads hit distinct banks

// A fragment (16 x 8, row-major at `base` with row stride ld), split into TF32 high / low parts.
Q35_DEV void load_a_split(const float* base, int ld, int g, int c, uint32_t hi[4], uint32_t lo[4]) {
  const float a[4] = {base[g * ld + c], base[(g + 8) * ld + c], base[g * ld + c + 4], base[(g + 8) * ld + c + 4]};
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], hi[i], lo[i]);
}
// Transposed A fragment: A[m][t] = base[t * ld + m].
Q35_DEV void load_at_split(const float* base, int ld, int g, int c, uint32_t hi[4], uint32_t lo[4]) {
  const float a[4] = {base[c * ld + g], base[c * ld + g + 8], base[(c + 4) * ld + g], base[(c + 4) * ld + g + 8]};
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], hi[i], lo[i]);
}
// d += A * B[k0 .. k0 + 8][n0 .. n0 + 8] in 3xTF32, B given as pre-split [k][kPS] high / low tiles,
// with the three terms in three accumulators: the scan's dependent MMA chains
// are its latency (a chunk step measured ~4x its MMA issue time), so every product keeps
// independent chains (main hi*hi, corrections lo*hi and hi*lo) that are summed at the end.
struct Acc3 {
  float m[4], c1[4], c2[4];
};
Q35_DEV void acc3_zero(Acc3& a) {
#pragma unroll
  for (int i = 0; i < 4; ++i) a.m[i] = a.c1[i] = a.c2[i] = 0.f;
}
Q35_DEV float acc3_value(const Acc3& a, int i) { return a.m[i] + (a.c1[i] + a.c2[i]); }
Q35_DEV void mma3a(Acc3& d, const uint32_t ah[4], const uint32_t al[4], const uint32_t* Bh, const uint32_t* Bl,
                   int k0, int n0, int g, int c) {
  const int i0 = (k0 + c) * kPS + n0 + g, i1 = i0 + 4 * kPS;
  const uint32_t bh0 = Bh[i0], bh1 = Bh[i1], bl0 = Bl[i0], bl1 = Bl[i1];
  mma_tf32(d.c1, al[0], al[1], al[2], al[3], bh0, bh1);
  mma_tf32(d.c2, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
  mma_tf32(d.m, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
}

// Phase B, the recurrence. Warp w owns the FP32 state tile S[16 w .. 16 w + 16][0 .. 16] in
// registers across chunks; S and Vn also live in shared memory pre-split into TF32 high / low
// parts (the B operands), so each value is split once per chunk rather than once per reader.
//   chunk c: S_c^T to the record (for phase C); phase 1: X = W S (64 x 16, K = 128), warp w rows
//   16 (w & 3) .. + 16 of value columns 8 (w >> 2) .. + 8; Vn = U - X, published pre-split and as
//   Vn^T to the record; phase 2: every warp S <- gl S + Kd^T Vn on its tile.
// The chunk records {W, U, Kd} are double-buffered: chunk n + 2's rows are requested as bulk
// copies on the buffer's mbarrier once chunk n is done with it, a whole chunk step ahead of their
// use (a record load from L2 or HBM is longer than a chunk's products). The output products
// (Qe S_c + P Vn) are phase C's.
constexpr long long kScanWaitBudget = 2000000000LL;
constexpr uint32_t kScanW = kC * kPW * sizeof(float), kScanK = kC * kPK2 * sizeof(float),
                   kScanU = kC * kVS * sizeof(float), kScanRecBytes = kScanW + kScanK + kScanU;
__global__ void __launch_bounds__(kThreads, 1) delta_chunk_scan_kernel(ScanParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) float sm[];
  float* Wb = sm;                  // 2 x [64][132]
  float* Kb = Wb + 2 * kC * kPW;   // 2 x [64][136]
  float* Ub = Kb + 2 * kC * kPK2;  // 2 x [64][16]
  uint32_t* Vh = reinterpret_cast<uint32_t*>(Ub + 2 * kC * kVS);  // [64][24]
  uint32_t* Vl = Vh + kC * kPS;    // [64][24]
  uint32_t* Sh = Vl + kC * kPS;    // [128][24]
  uint32_t* Sl = Sh + kD * kPS;    // [128][24]
  const int nvs = kD / kVS;
  const int vs = blockIdx.x % nvs;
  const int h = (blockIdx.x / nvs) % p.H;
  const int b = blockIdx.x / (nvs * p.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  float* Sg = p.state + ((size_t)(b * p.H + h) * kD) * kD + vs * kVS;
  auto frag_row = [&](int i) { return warp * 16 + g + (i >= 2 ? 8 : 0); };
  auto frag_col = [&](int nt, int i) { return nt * 8 + 2 * c + (i & 1); };
  float s[2][4];  // this warp's state tile: [n-tile][mma fragment]
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[nt][i] = Sg[frag_row(i) * kD + frag_col(nt, i)];
  auto publish_s = [&]() {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int o = frag_row(i) * kPS + frag_col(nt, i);
        split_tf32(s[nt][i], Sh[o], Sl[o]);
      }
  };
  publish_s();
  auto rec_of = [&](int ch) { return p.ws + ((size_t)(b * p.H + h) * p.NC + ch) * ChunkWs::SIZE; };
  __shared__ __align__(8) uint64_t rec_bar[2];
  __shared__ int wait_failed;
  // W, Kd and this CTA's U columns of chunk ch into buffer ch % 2: three bulk copies (the prep
  // writes them in these shared-memory layouts), issued by thread 0 after arming the barrier
  auto issue = [&](int ch) {
    if (tid != 0) return;
    const float* rec = rec_of(ch);
    const int buf = ch & 1;
    const uint32_t bar = tc::smem_u32(&rec_bar[buf]);
    tc::mbar_expect_tx(bar, kScanRecBytes);
    tc::bulk_g2s(tc::smem_u32(Wb + buf * kC * kPW), rec + ChunkWs::W, kScanW, bar);
    tc::bulk_g2s(tc::smem_u32(Kb + buf * kC * kPK2), rec + ChunkWs::Kd, kScanK, bar);
    tc::bulk_g2s(tc::smem_u32(Ub + buf * kC * kVS), rec + ChunkWs::U + vs * kC * kVS, kScanU, bar);
  };
  if (tid == 0) {
    tc::mbar_init(tc::smem_u32(&rec_bar[0]), 1);
    tc::mbar_init(tc::smem_u32(&rec_bar[1]), 1);
    wait_failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (p.NC > 0) issue(0);
  if (p.NC > 1) issue(1);
  const int mt = warp & 3, nt1 = warp >> 2;  // phase-1 tile: token rows 16 mt, value columns 8 nt1
  for (int ch = 0; ch < p.NC; ++ch) {
    const float* W = Wb + (ch & 1) * kC * kPW;
    const float* Kd = Kb + (ch & 1) * kC * kPK2;
    const float* U = Ub + (ch & 1) * kC * kVS;
    float* rec = const_cast<float*>(rec_of(ch));
    const float gl = rec[ChunkWs::GL];  // issued now, used in phase 2
    // S_c^T (value column, key row) for phase C, from the registers before this chunk's update
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) rec[ChunkWs::ST + (size_t)(vs * kVS + frag_col(nt, i)) * kD + frag_row(i)] = s[nt][i];
    // this chunk's records: thread 0 waits with a budget and shares the outcome, then every
    // thread observes the completed phase itself (instant), which orders its reads after the copies
    const uint32_t bar = tc::smem_u32(&rec_bar[ch & 1]), parity = (uint32_t)(ch >> 1) & 1u;
    if (tid == 0 && !tc::mbar_wait_bounded(bar, parity, kScanWaitBudget)) {
      wait_failed = 1;
      atomicCAS(&q35_delta_chunk_error_word, 0, 2);
    }
    __syncthreads();  // the published S is visible; the wait's outcome is known
    if (wait_failed) {  // uniform: the recurrence stops and the error word is set
      if (tid == 0 && ch + 1 < p.NC)  // the other buffer's copies, with a budget, before exiting
        tc::mbar_wait_bounded(tc::smem_u32(&rec_bar[(ch + 1) & 1]), (uint32_t)((ch + 1) >> 1) & 1u, kScanWaitBudget);
      return;
    }
    tc::mbar_wait_bounded(bar, parity, kScanWaitBudget);
    // ---- phase 1: X = W S for token rows 16 mt .. + 16, value columns 8 nt1 .. + 8 (six chains:
    // even / odd k-step x three terms)
    float x[4];
    {
      Acc3 xa[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) acc3_zero(xa[q]);
      const float* A = W + mt * 16 * kPW;
#pragma unroll 4
      for (int k = 0; k < kD; k += 8) {
        uint32_t ah[4], al[4];
        load_a_split(A + k, kPW, g, c, ah, al);
        mma3a(xa[(k >> 3) & 1], ah, al, Sh, Sl, k, 8 * nt1, g, c);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = acc3_value(xa[0], i) + acc3_value(xa[1], i);
    }
    // Vn = U - W S, published pre-split for phase 2 and as Vn^T for phase C
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = mt * 16 + g + (i >= 2 ? 8 : 0), col = nt1 * 8 + 2 * c + (i & 1);
      const float vn = U[r * kVS + col] - x[i];
      split_tf32(vn, Vh[r * kPS + col], Vl[r * kPS + col]);
      rec[ChunkWs::VT + (size_t)(vs * kVS + col) * kC + r] = vn;
    }
    __syncthreads();  // Vn visible
    // ---- phase 2: S <- gl S + Kd^T Vn on this warp's tile (rows 16 warp .. + 16)
    {
      float d[2][4];
      {
        Acc3 da[2][2];  // [k-step parity][n-tile]
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) acc3_zero(da[q][nt]);
#pragma unroll
        for (int k0 = 0; k0 < kC; k0 += 8) {
          uint32_t ah[4], al[4];
          load_at_split(Kd + k0 * kPK2 + warp * 16, kPK2, g, c, ah, al);
          mma3a(da[(k0 >> 3) & 1][0], ah, al, Vh, Vl, k0, 0, g, c);
          mma3a(da[(k0 >> 3) & 1][1], ah, al, Vh, Vl, k0, 8, g, c);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) d[nt][i] = acc3_value(da[0][nt], i) + acc3_value(da[1][nt], i);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[nt][i] = gl * s[nt][i] + d[nt][i];
    }
    __syncthreads();  // readers of Sh / Sl, Vn and this chunk's record buffer are done
    publish_s();
    if (ch + 2 < p.NC) issue(ch + 2);
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) Sg[frag_row(i) * kD + frag_col(nt, i)] = s[nt][i];
}

// ---------------------------------------------------------------------------------------------
// Phase C: out[t, h, v] = bf16((Qe S_c + P Vn)[t, v]) for the chunk's 64 tokens and 64 of the 128
// value columns, on tcgen05 (kind::tf32, M = 64, N = 64, K = 128 + 64) with the FP32 accumulator
// in TMEM. 3xTF32: the A = [Qe | P] and B = [S_c ; Vn] operands are staged as TF32 high / low
// parts (K-major, 128-byte swizzle) and the three products hi.hi, lo.hi and hi.lo accumulate in
// one TMEM tile, so the result keeps FP32-level accuracy (the dropped lo.lo term is ~2^-22).
// K runs in three parts of 64 through one 64 KB staging area (three CTAs per SM): each part's loads
// are in flight while the previous part's MMAs run.
constexpr int kOutThreads = 256;            // staging; warps 0-3 also read one TMEM lane quarter each
constexpr int kOutParts = 3;                // K in three parts through one staging area
constexpr int kOutBatch = 4;                // 16-byte loads per operand in flight per thread
constexpr int kOutK = kD + kC;              // 192
constexpr int kOutKH = kOutK / kOutParts;   // 64: K per part
constexpr int kOutSlabs = kOutKH / 32;      // 2 slabs of 32 tf32 (128 bytes) per part
constexpr int kOutN = 64;                   // value columns per CTA
constexpr uint32_t kOutSlabBytes = 64 * 128;  // 64 rows of 128 bytes (A: tokens, B: value columns)
constexpr uint32_t kOutTile = kOutSlabs * kOutSlabBytes;  // 16 KB per operand part
constexpr size_t kOutSmem = 4 * (size_t)kOutTile + 1024 + 64;
constexpr long long kOutWaitBudget = 2000000000LL;

struct OutParams {
  const float* ws;
  bf16* out;  // [B, L, H, D]
  int L, H, NC;
};

__global__ void __launch_bounds__(kOutThreads, 3) delta_chunk_out_kernel(OutParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char out_smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)out_smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* A_hi = sm;
  unsigned char* A_lo = sm + kOutTile;
  unsigned char* B_hi = sm + 2 * kOutTile;
  unsigned char* B_lo = sm + 3 * kOutTile;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 4 * kOutTile);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int half = blockIdx.x & 1;
  const int ch = (blockIdx.x >> 1) % p.NC;
  const int h = (blockIdx.x / (2 * p.NC)) % p.H;
  const int b = blockIdx.x / (2 * p.NC * p.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* rec = p.ws + ((size_t)(b * p.H + h) * p.NC + ch) * ChunkWs::SIZE;

  if (warp == 0) tc::tmem_alloc(tmem_slot, 64);
  if (tid == 0) {
    tc::mbar_init(tc::smem_u32(bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // ---- stage A = [Qe | P] (64 token rows) and B = [S_c^T | Vn^T] (64 value rows of this half),
  // 16 bytes (4 values along K) per step, split into TF32 high / low parts
  auto stage = [&](unsigned char* hi, unsigned char* lo, int row, int k4, float4 v) {
    uint32_t h4[4], l4[4];
    tc::split_tf32(v.x, h4[0], l4[0]);
    tc::split_tf32(v.y, h4[1], l4[1]);
    tc::split_tf32(v.z, h4[2], l4[2]);
    tc::split_tf32(v.w, h4[3], l4[3]);
    const uint32_t off = (uint32_t)(k4 / 32) * kOutSlabBytes + tc::sw128_offset(row, (k4 % 32) / 4);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l4[0], l4[1], l4[2], l4[3]);
  };
  // one batch of kOutBatch 16-byte loads per operand per thread covers a part of K
  constexpr int kItems = 64 * (kOutKH / 4);  // 16-byte items per operand per part
  static_assert(kItems == kOutThreads * kOutBatch, "one batch per part");
  float4 a[kOutBatch], bv[kOutBatch];
  auto load_half = [&](int kh) {
#pragma unroll
    for (int u = 0; u < kOutBatch; ++u) {
      const int i = u * kOutThreads + tid;
      const int r = i / (kOutKH / 4), k4 = kh * kOutKH + (i % (kOutKH / 4)) * 4;
      const int v = half * kOutN + r;  // B row: value column
      a[u] = k4 < kD ? __ldcg(reinterpret_cast<const float4*>(rec + ChunkWs::Qe + r * kD + k4))
                     : __ldcg(reinterpret_cast<const float4*>(rec + ChunkWs::P + r * kC + (k4 - kD)));
      bv[u] = k4 < kD ? __ldcg(reinterpret_cast<const float4*>(rec + ChunkWs::ST + (size_t)v * kD + k4))
                      : __ldcg(reinterpret_cast<const float4*>(rec + ChunkWs::VT + (size_t)v * kC + (k4 - kD)));
    }
  };
  auto stage_half = [&]() {
#pragma unroll
    for (int u = 0; u < kOutBatch; ++u) {
      const int i = u * kOutThreads + tid;
      const int r = i / (kOutKH / 4), k4 = (i % (kOutKH / 4)) * 4;  // K offset within the part
      stage(A_hi, A_lo, r, k4, a[u]);
      stage(B_hi, B_lo, r, k4, bv[u]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy stores -> MMA reads
  };
  const uint32_t idesc = tc::idesc_f32acc(2, 64, kOutN);
  auto mma_half = [&](uint32_t tmem_acc, bool first) {
    const uint32_t ah = tc::smem_u32(A_hi), al = tc::smem_u32(A_lo), bh = tc::smem_u32(B_hi), bl = tc::smem_u32(B_lo);
    const uint32_t as[3] = {ah, al, ah}, bs[3] = {bh, bh, bl};  // hi.hi, lo.hi, hi.lo
    uint32_t acc = first ? 0u : 1u;
#pragma unroll
    for (int t = 0; t < 3; ++t)
#pragma unroll
      for (int sl = 0; sl < kOutSlabs; ++sl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t o = sl * kOutSlabBytes + kk * 32;
          tc::mma_tf32(tmem_acc, tc::desc_sw128(as[t] + o), tc::desc_sw128(bs[t] + o), idesc, acc);
          acc = 1;
        }
    tc::commit(tc::smem_u32(bar));
  };
  load_half(0);
  stage_half();
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) mma_half(tmem, true);
  bool ok = true;
#pragma unroll 1
  for (int part = 1; part < kOutParts; ++part) {
    load_half(part);  // in flight while the previous part's MMAs read the staging area
    // every thread waits for those MMAs before overwriting their operands
    ok = tc::mbar_wait_bounded(tc::smem_u32(bar), (uint32_t)(part - 1) & 1u, kOutWaitBudget) && ok;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    stage_half();
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (tid == 0) mma_half(tmem, false);
  }
  __syncwarp();
  if (warp < 4) {  // TMEM lane quarters
    ok = tc::mbar_wait_bounded(tc::smem_u32(bar), (uint32_t)(kOutParts - 1) & 1u, kOutWaitBudget) && ok;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // M = 64: token row 16 q + i sits in TMEM lane 32 q + i (i < 16) of warp q's lane quarter
    uint32_t v0[32], v1[32];
    const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
    tc::tmem_ld32(tq, v0);
    tc::tmem_ld32(tq + 32, v1);
    if (!ok) {
      if (lane == 0) atomicCAS(&q35_delta_chunk_error_word, 0, 1);
    } else if (lane < 16) {
      const int t = ch * kC + warp * 16 + lane;
      if (t < p.L) {
        bf16* o = p.out + (((int64_t)b * p.L + t) * p.H + h) * kD + half * kOutN;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __align__(16) bf16 w8[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) w8[j] = f2bf(__uint_as_float(v0[8 * q + j]));
          reinterpret_cast<uint4*>(o)[q] = *reinterpret_cast<const uint4*>(w8);
#pragma unroll
          for (int j = 0; j < 8; ++j) w8[j] = f2bf(__uint_as_float(v1[8 * q + j]));
          reinterpret_cast<uint4*>(o + 32)[q] = *reinterpret_cast<const uint4*>(w8);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
}

constexpr size_t kPrepSmem =
    (size_t)3 * (kHalo + kC) * kPB * sizeof(bf16) + (size_t)(kC * kTS + 48 * 16) * sizeof(float);
static_assert((3 * (kHalo + kC) * kPB * sizeof(bf16)) % 16 == 0, "T starts 16-byte aligned");
static_assert((kHalo * kPB * sizeof(bf16)) % 16 == 0, "tile rows stay 16-byte aligned");
static_assert((size_t)kC * kTS * sizeof(float) <= (size_t)(kHalo + kC) * kPB * sizeof(bf16),
              "the solve's copy of A fits in q's tile");
constexpr size_t kScanSmem =
    (size_t)(2 * kC * kPW + 2 * kC * kPK2 + 2 * kC * kVS + 2 * kC * kPS + 2 * kD * kPS) * sizeof(float);
static_assert(kScanSmem <= 227 * 1024, "scan shared memory");

}  // namespace

size_t q35_delta_chunk_workspace_bytes(int64_t batch, int64_t heads, int64_t max_len) {
  const int64_t nc = (max_len + kC - 1) / kC;
  return (size_t)batch * heads * nc * ChunkWs::SIZE * sizeof(float);
}

// conv_weight / conv_state non-null: `qkv` is ignored and the causal conv (4 taps, zero history,
// seq_len >= 4) runs inside the prep kernel on the raw [q k v] columns of `packed`, writing the
// conv state as causal_conv1d_fused does.
int q35_delta_chunked_launch(const void* qkv, const void* packed, const void* a_log, const void* dt_bias, float* state,
                             void* out, int64_t batch, int64_t seq_len, int64_t heads, int64_t packed_stride,
                             float* ws, cudaStream_t s, const void* conv_weight, void* conv_state, bool pdl) {
  if (batch * seq_len == 0) return Q35_OK;
  Q35_REQUIRE(conv_weight == nullptr || (conv_state != nullptr && seq_len >= 4),
              "delta_chunked: the fused conv needs a state and at least 4 tokens");
  const int nc = (int)((seq_len + kC - 1) / kC);
  static Q35PerDevice<bool> attr;
  attr.get([] {
    cudaFuncSetAttribute(delta_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrepSmem);
    cudaFuncSetAttribute(delta_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem);
    cudaFuncSetAttribute(delta_chunk_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kOutSmem);
    return true;
  });
  PrepParams pp{(const bf16*)qkv,         (const bf16*)packed,    (const bf16*)a_log, (const bf16*)dt_bias,
                (const bf16*)conv_weight, (bf16*)conv_state,      ws,                  (int)seq_len,
                (int)heads,               nc,                     (int)packed_stride};
  cudaError_t e =
      q35_launch(delta_chunk_prep_kernel, dim3((unsigned)(batch * heads * nc)), dim3(kThreads), kPrepSmem, s, pdl, pp);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "delta_chunk_prep launch: %s", cudaGetErrorString(e));
  ScanParams sp{ws, state, (int)seq_len, (int)heads, nc};
  e = q35_launch(delta_chunk_scan_kernel, dim3((unsigned)(batch * heads * (kD / kVS))), dim3(kThreads), kScanSmem, s,
                 pdl, sp);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "delta_chunk_scan launch: %s", cudaGetErrorString(e));
  OutParams op{ws, (bf16*)out, (int)seq_len, (int)heads, nc};
  e = q35_launch(delta_chunk_out_kernel, dim3((unsigned)(batch * heads * nc * 2)), dim3(kOutThreads), kOutSmem, s,
                 pdl, op);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "delta_chunk_out launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_delta_chunk_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_delta_chunk_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_delta_chunk_error_word, &zero, sizeof(int));
  return v;
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
                                  static_cast<float*>(workspace), (cudaStream_t)stream, nullptr, nullptr, false);
}

extern "C" int q35_delta_chunked_conv(const void* packed, const void* conv_weight, void* conv_state, const void* a_log,
                                      const void* dt_bias, float* state, void* out, int64_t batch, int64_t seq_len,
                                      int64_t heads, int64_t dim, int64_t packed_stride, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(packed && conv_weight && conv_state && a_log && dt_bias && state && out && workspace,
              "delta_chunked_conv: null pointer");
  Q35_REQUIRE(dim == kD, "delta_chunked_conv: head dim must be 128");
  Q35_REQUIRE(batch >= 0 && seq_len >= 4 && heads >= 1 && packed_stride >= 4 * heads * dim + 2 * heads,
              "delta_chunked_conv: bad shape (seq_len >= 4)");
  Q35_REQUIRE(Q35_ALIGNED(packed, 16) && packed_stride % 8 == 0 && Q35_ALIGNED(workspace, 16),
              "delta_chunked_conv: 16-byte alignment");
  Q35_REQUIRE(workspace_bytes >= q35_delta_chunk_workspace_bytes(batch, heads, seq_len),
              "delta_chunked_conv: workspace too small");
  return q35_delta_chunked_launch(nullptr, packed, a_log, dt_bias, state, out, batch, seq_len, heads, packed_stride,
                                  static_cast<float*>(workspace), (cudaStream_t)stream, conv_weight, conv_state,
                                  false);
}
