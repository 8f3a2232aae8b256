// Vision tower of Qwen3.5 (ViT encoder + 2x2 patch merger) for the multimodal request path.
//
// Reference: the fused vision operators of qwen35_fused/kernels.py (vision_qkv_rope :336-416,
// layer_norm :1188-1222, residual_add_layer_norm :1225-1287, position_embed_add :1290-1336) and
// the patched vision forward of integration.py:509-736 (run_blocks, then the merger); the eager
// math is Transformers' Qwen3_5VisionModel.
//
// Kernels (all HBM/latency-bound except the projections, which run on the tcgen05 GEMM with a
// bias / GELU epilogue, and the attention):
// * patchify: fp32 pixels [C, H, W] -> normalised bf16 patches in the Qwen2-VL processor order;
// * rope table: 2-D rotary cos/sin [tokens, 64] (row frequencies, column frequencies, twice);
// * position embed + norm1: bilinear position embedding added to the patch embedding and the
//   first block's LayerNorm, one warp per token;
// * layer_norm / residual_add_layer_norm: one warp per row, the row held in registers;
// * qkv rope: packed [tokens, 3 * heads * 64] -> q, k, v [heads, tokens, 64] with RoPE on q, k;
// * attention: bidirectional FlashAttention-style over one image (mma.sync m16n8k16 bf16,
//   FP32 online softmax), 64 queries per CTA.
// The C-ABI runner q35_vit_encode chains them over the blocks (8 launches per block).
#include <cfloat>
#include <vector>

#include "common.cuh"

int q35_gemm_tc_bias_launch(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n,
                            int64_t k, int epi, cudaStream_t s);

using namespace q35;

namespace {

constexpr int kVD = 64;  // vision head dim (width 1024 / 16 heads)

// ============================================================================ patchify
// out[p, f]: patch p = ((bh * gw/M + bw) * M + mh) * M + mw (merge-block order), feature
// f = ((c * T + tp) * P + py) * P + px; pixel row bh*M*P + mh*P + py, column bw*M*P + mw*P + px.
// A single image fills every temporal slot (the processor repeats the frame).
__global__ void __launch_bounds__(256) patchify_kernel(const float* __restrict__ px, bf16* __restrict__ out, int C,
                                                       int H, int W, int P, int T, int M, int n_patches,
                                                       float mean, float inv_std) {
  const int F = C * T * P * P;
  const int64_t i8 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-wide group of px
  if (i8 * 8 >= (int64_t)n_patches * F) return;
  const int64_t flat = i8 * 8;
  const int p = (int)(flat / F), f = (int)(flat - (int64_t)p * F);
  const int px0 = f % P, py = (f / P) % P, c = f / (T * P * P);
  const int gw = W / P, bw_n = gw / M;
  const int mw = p % M, mh = (p / M) % M, bw = (p / (M * M)) % bw_n, bh = p / (M * M * bw_n);
  const int y = (bh * M + mh) * P + py, x = (bw * M + mw) * P + px0;
  const int64_t img = blockIdx.y;  // images of a batch: [n, C, H, W] -> [n * patches, F]
  const float* src = px + img * C * H * W + ((int64_t)c * H + y) * W + x;
  __align__(16) bf16 o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = f2bf((src[j] - mean) * inv_std);
  *reinterpret_cast<uint4*>(out + img * n_patches * F + flat) = *reinterpret_cast<const uint4*>(o);
}

// Grid position of merge-ordered token p: row = bh * M + mh, column = bw * M + mw.
Q35_DEV void token_rc(int p, int gw, int M, int& row, int& col) {
  const int bw_n = gw / M;
  const int mw = p % M, mh = (p / M) % M, bw = (p / (M * M)) % bw_n, bh = p / (M * M * bw_n);
  row = bh * M + mh;
  col = bw * M + mw;
}

// ============================================================================ rope table
// HF Qwen3_5VisionModel.rot_pos_emb: freqs = pos * inv_freq (FP32) for the row (first half of the
// 32) and the column (second half); emb = cat(freqs, freqs); cos/sin in FP32.
__global__ void rope_table_kernel(float* __restrict__ cos_t, float* __restrict__ sin_t,
                                  const float* __restrict__ inv_freq, int n_tokens, int gw, int M) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tokens * kVD) return;
  const int p = i / kVD, d = i % kVD;
  int row, col;
  token_rc(p, gw, M, row, col);
  const int j = d & 31;
  const float ang = __fmul_rn((float)(j < 16 ? row : col), inv_freq[j & 15]);
  float s, c;
  sincosf(ang, &s, &c);
  cos_t[i] = c;
  sin_t[i] = s;
}

// torch.linspace(0, side - 1, steps) in FP32: the first half counts up from 0, the second half
// down from the end (ATen's symmetric form).
Q35_DEV float linspace_at(int idx, int steps, int side) {
  if (steps <= 1) return 0.f;
  const float end = (float)(side - 1);
  const float step = __fdiv_rn(end, (float)(steps - 1));
  return idx < steps / 2 ? __fmul_rn(step, (float)idx) : __fsub_rn(end, __fmul_rn(step, (float)(steps - 1 - idx)));
}

// ============================================================================ layer norms
// One warp per row of width 256 * CPL: lane l owns the 16-byte chunks l + 32 j. Mean, then the
// centred variance, over the FP32 values (kernels.py:1188-1222); out = c * rsqrt(var + eps) * w + b.
template <int CPL>
Q35_DEV void ln_row(float (&x)[CPL][8], const bf16* __restrict__ w, const bf16* __restrict__ b, bf16* __restrict__ out,
                    int width, float eps, int lane) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) s += x[j][e];
  const float mean = warp_sum(s) / (float)width;
  float v = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x[j][e] -= mean;
      v += x[j][e] * x[j][e];
    }
  const float r = rsqrt_ieee(warp_sum(v) / (float)width + eps);
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c8 = lane + 32 * j;
    float wf[8], bf[8];
    unpack_bf16x8(reinterpret_cast<const uint4*>(w)[c8], wf);
    unpack_bf16x8(reinterpret_cast<const uint4*>(b)[c8], bf);
    __align__(16) bf16 o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = f2bf(x[j][e] * r * wf[e] + bf[e]);
    reinterpret_cast<uint4*>(out)[c8] = *reinterpret_cast<const uint4*>(o);
  }
}

// RES = false: out = LN(x). RES = true: resid_out = bf16(x + u); out = LN(resid_out). resid_out may
// be x (every element is read before its own lane writes it).
template <int CPL, bool RES>
__global__ void __launch_bounds__(256) layer_norm_kernel(const bf16* x, const bf16* __restrict__ u,
                                                         const bf16* __restrict__ w, const bf16* __restrict__ b,
                                                         bf16* resid_out, bf16* __restrict__ out,
                                                         int rows, int width, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = (int64_t)row * width;
  float f[CPL][8];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c8 = lane + 32 * j;
    unpack_bf16x8(reinterpret_cast<const uint4*>(x + base)[c8], f[j]);
    if (RES) {
      float g[8];
      unpack_bf16x8(reinterpret_cast<const uint4*>(u + base)[c8], g);
      __align__(16) bf16 o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = f2bf(f[j][e] + g[e]);
        f[j][e] = bf2f(o[e]);
      }
      reinterpret_cast<uint4*>(resid_out + base)[c8] = *reinterpret_cast<const uint4*>(o);
    }
  }
  ln_row<CPL>(f, w, b, out + base, width, eps, lane);
}

// Any width (a multiple of 8 up to 16384): one CTA per row, the row staged in shared memory.
template <bool RES>
__global__ void __launch_bounds__(256) layer_norm_any_kernel(const bf16* x, const bf16* __restrict__ u,
                                                             const bf16* __restrict__ w, const bf16* __restrict__ b,
                                                             bf16* resid_out, bf16* __restrict__ out,
                                                             int width, float eps) {
  extern __shared__ float xs[];
  __shared__ float red[8];
  const int64_t base = (int64_t)blockIdx.x * width;
  float s = 0.f;
  for (int c = threadIdx.x; c < width; c += 256) {
    float v = bf2f(x[base + c]);
    if (RES) {
      const bf16 a = f2bf(v + bf2f(u[base + c]));
      resid_out[base + c] = a;
      v = bf2f(a);
    }
    xs[c] = v;
    s += v;
  }
  const float mean = block_sum<8>(s, red) / (float)width;
  float var = 0.f;
  for (int c = threadIdx.x; c < width; c += 256) {
    const float d = xs[c] - mean;
    var += d * d;
  }
  const float r = rsqrt_ieee(block_sum<8>(var, red) / (float)width + eps);
  for (int c = threadIdx.x; c < width; c += 256)
    out[base + c] = f2bf((xs[c] - mean) * r * bf2f(w[c]) + bf2f(b[c]));
}

// ============================================================================ position embedding
// kernels.py:1290-1336: out = bf16(hidden + bf16(sum_k w_k * table[idx_k])) with FP32 accumulation
// over the neighbours; the 4 bilinear neighbours and weights of HF fast_pos_embed_interpolate
// (torch.linspace grid over side x side, floor / clipped ceil, FP32 weights) are formed in the
// kernel from the token's grid position. NORM also writes LayerNorm(out) (the first block's norm1).
template <int CPL, bool NORM>
__global__ void __launch_bounds__(256) pos_embed_kernel(const bf16* __restrict__ hidden, const bf16* __restrict__ table,
                                                        const bf16* __restrict__ w, const bf16* __restrict__ b,
                                                        bf16* __restrict__ resid_out, bf16* __restrict__ norm_out,
                                                        int rows, int width, int gh, int gw, int M, int side,
                                                        float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  int r, c;
  token_rc(row % (gh * gw), gw, M, r, c);  // rows of a batch of images: the token within its image
  const float hv = linspace_at(r, gh, side), wv = linspace_at(c, gw, side);
  const int hf = (int)hv, wf = (int)wv;
  const int hc = min(hf + 1, side - 1), wc = min(wf + 1, side - 1);
  const float dh = __fsub_rn(hv, (float)hf), dw = __fsub_rn(wv, (float)wf);
  const int idx[4] = {hf * side + wf, hf * side + wc, hc * side + wf, hc * side + wc};
  const float wt[4] = {__fmul_rn(1.f - dh, 1.f - dw), __fmul_rn(1.f - dh, dw), __fmul_rn(dh, 1.f - dw),
                       __fmul_rn(dh, dw)};
  const int64_t base = (int64_t)row * width;
  float f[CPL][8];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c8 = lane + 32 * j;
    float pos[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float t[8];
      unpack_bf16x8(reinterpret_cast<const uint4*>(table + (int64_t)idx[k] * width)[c8], t);
#pragma unroll
      for (int e = 0; e < 8; ++e) pos[e] = fmaf(t[e], wt[k], pos[e]);
    }
    float h8[8];
    unpack_bf16x8(reinterpret_cast<const uint4*>(hidden + base)[c8], h8);
    __align__(16) bf16 o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o[e] = f2bf(h8[e] + rbf(pos[e]));
      f[j][e] = bf2f(o[e]);
    }
    reinterpret_cast<uint4*>(resid_out + base)[c8] = *reinterpret_cast<const uint4*>(o);
  }
  if (NORM) ln_row<CPL>(f, w, b, norm_out + base, width, eps, lane);
}

// Explicit-neighbour form of the same operator (the reference's API: indices / weights given).
__global__ void __launch_bounds__(256) pos_embed_given_kernel(const bf16* __restrict__ hidden,
                                                              const bf16* __restrict__ table,
                                                              const int64_t* __restrict__ idx,
                                                              const float* __restrict__ wt, bf16* __restrict__ out,
                                                              int width, int neighbors) {
  const int64_t row = blockIdx.x;
  for (int c = threadIdx.x; c < width; c += 256) {
    float pos = 0.f;
    for (int k = 0; k < neighbors; ++k)
      pos = fmaf(bf2f(table[idx[row * neighbors + k] * width + c]), wt[row * neighbors + k], pos);
    out[row * width + c] = f2bf(bf2f(hidden[row * width + c]) + rbf(pos));
  }
}

// ============================================================================ qkv + rope
// kernels.py:336-416: one warp per (token, head); lane l owns dims l and l + 32 of q and k, which
// are each other's rotate_half partners, so no exchange is needed. q*cos + partner*sign*sin in
// FP32 without fused multiply-adds (the reference launches it with enable_fp_fusion=False).
__global__ void __launch_bounds__(256) qkv_rope_kernel(const bf16* __restrict__ packed, const float* __restrict__ cos_t,
                                                       const float* __restrict__ sin_t, bf16* __restrict__ q_out,
                                                       bf16* __restrict__ k_out, bf16* __restrict__ v_out, int tokens,
                                                       int heads, int per_image) {
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (gw >= tokens * heads) return;
  const int t = gw / heads, h = gw - t * heads;
  const int img = t / per_image, tt = t - img * per_image;  // tables are per image; q/k/v [n, heads, L, 64]
  const int64_t stride = 3 * (int64_t)heads * kVD;
  const bf16* row = packed + (int64_t)t * stride;
  const int d0 = lane, d1 = lane + 32;
  const float c0 = cos_t[(int64_t)tt * kVD + d0], c1 = cos_t[(int64_t)tt * kVD + d1];
  const float s0 = sin_t[(int64_t)tt * kVD + d0], s1 = sin_t[(int64_t)tt * kVD + d1];
  const int64_t o = (((int64_t)img * heads + h) * per_image + tt) * kVD;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const bf16* src = row + (int64_t)which * heads * kVD + h * kVD;
    const float x0 = bf2f(src[d0]), x1 = bf2f(src[d1]);
    bf16* dst = (which == 0 ? q_out : k_out) + o;
    dst[d0] = f2bf(__fadd_rn(__fmul_rn(x0, c0), __fmul_rn(-x1, s0)));
    dst[d1] = f2bf(__fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1)));
  }
  const bf16* vsrc = row + 2 * (int64_t)heads * kVD + h * kVD;
  v_out[o + d0] = vsrc[d0];
  v_out[o + d1] = vsrc[d1];
}

// ============================================================================ attention
// Bidirectional attention over one image: q, k, v [heads, L, 64] bf16 -> out [L, heads * 64].
// CTA = 64 query rows of one head (4 warps x 16 rows); keys stream through shared memory in
// double-buffered 64-row tiles (cp.async, zero-filled past L, rows padded to 144 bytes so the
// ldmatrix row addresses fall in distinct banks). S = Q K^T and O += P V on mma.sync m16n8k16
// (bf16 in, FP32 accumulate); online softmax in FP32 (exp2 of log2e-scaled scores); P enters the
// second product rounded to bf16, as the eager path's bf16 attention weights do.
constexpr int kVaRows = 64, kVaKeys = 64, kVaStride = kVD + 8, kVaThreads = 128;

struct VisionAttnParams {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  bf16* out;
  int L, heads;
  float scale_log2;  // softmax scale * log2(e)
};

Q35_DEV void cp16_zfill(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}

__global__ void __launch_bounds__(kVaThreads) vision_attn_kernel(VisionAttnParams p) {
  __shared__ __align__(16) bf16 ks[2][kVaKeys * kVaStride];
  __shared__ __align__(16) bf16 vs[2][kVaKeys * kVaStride];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int h = blockIdx.y, img = blockIdx.z;  // images of a batch attend within themselves
  const int L = p.L;
  const int r0 = blockIdx.x * kVaRows + warp * 16 + g, r1 = r0 + 8;
  const int64_t hoff = ((int64_t)img * p.heads + h) * L * kVD;
  const bf16* qh = p.q + hoff;
  const bf16* kh = p.k + hoff;
  const bf16* vh = p.v + hoff;

  auto load_tile = [&](int tile, int buf) {
    for (int i = threadIdx.x; i < kVaKeys * 8; i += kVaThreads) {
      const int r = i >> 3, c = i & 7;
      const int key = tile * kVaKeys + r;
      const int bytes = key < L ? 16 : 0;
      const int64_t src = (int64_t)(key < L ? key : 0) * kVD + c * 8;
      cp16_zfill(&ks[buf][r * kVaStride + c * 8], kh + src, bytes);
      cp16_zfill(&vs[buf][r * kVaStride + c * 8], vh + src, bytes);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  const int ntiles = (L + kVaKeys - 1) / kVaKeys;
  load_tile(0, 0);

  // Q fragments (A operand, 16 rows x 64 dims = 4 k-steps), rows past L read as zero
  uint32_t qf[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int c = 16 * kk + 2 * tq;
    qf[kk][0] = r0 < L ? *reinterpret_cast<const uint32_t*>(qh + (int64_t)r0 * kVD + c) : 0u;
    qf[kk][1] = r1 < L ? *reinterpret_cast<const uint32_t*>(qh + (int64_t)r1 * kVD + c) : 0u;
    qf[kk][2] = r0 < L ? *reinterpret_cast<const uint32_t*>(qh + (int64_t)r0 * kVD + c + 8) : 0u;
    qf[kk][3] = r1 < L ? *reinterpret_cast<const uint32_t*>(qh + (int64_t)r1 * kVD + c + 8) : 0u;
  }

  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) {
      load_tile(tile + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint32_t kbase = (uint32_t)__cvta_generic_to_shared(&ks[buf][0]);
    const uint32_t vbase = (uint32_t)__cvta_generic_to_shared(&vs[buf][0]);

    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; kk += 2) {
        // keys 8nb..8nb+7; matrices: dims 16kk, 16kk+8, 16(kk+1), 16(kk+1)+8
        const int key = 8 * nb + (lane & 7);
        const int col = 16 * kk + 8 * ((lane >> 3) & 1) + 16 * (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + (uint32_t)((key * kVaStride + col) * 2), b0, b1, b2, b3);
        mma_bf16(s[nb], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16(s[nb], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
      }
    }
    // scale, mask keys past L, online softmax (rows g and g + 8 of the warp's 16)
    float mx0 = -FLT_MAX, mx1 = -FLT_MAX;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int key = tile * kVaKeys + 8 * nb + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = key + (e & 1) < L;
        s[nb][e] = ok ? s[nb][e] * p.scale_log2 : -FLT_MAX;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
    }
#pragma unroll
    for (int sh = 1; sh <= 2; sh <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] *= a0;
      o[n][1] *= a0;
      o[n][2] *= a1;
      o[n][3] *= a1;
    }
    uint32_t pf[8][2];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const float p0 = exp2f(s[nb][0] - mn0), p1 = exp2f(s[nb][1] - mn0);
      const float p2 = exp2f(s[nb][2] - mn1), p3 = exp2f(s[nb][3] - mn1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pf[nb][0] = pack_bf2(p0, p1);
      pf[nb][1] = pack_bf2(p2, p3);
    }
    // O += P V: k-step kk covers keys 16kk..16kk+15 = S blocks 2kk, 2kk+1
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a_0 = pf[2 * kk][0], a_1 = pf[2 * kk][1], a_2 = pf[2 * kk + 1][0], a_3 = pf[2 * kk + 1][1];
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        const int key = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int col = 8 * n + 8 * (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + (uint32_t)((key * kVaStride + col) * 2), b0, b1, b2, b3);
        mma_bf16(o[n], a_0, a_1, a_2, a_3, b0, b1);
        mma_bf16(o[n + 1], a_0, a_1, a_2, a_3, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with `buf` before the next iteration refills it
  }
#pragma unroll
  for (int sh = 1; sh <= 2; sh <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
    l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
  }
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  const int64_t ow = (int64_t)p.heads * kVD;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int c = h * kVD + 8 * n + 2 * tq;
    const int64_t orow = (int64_t)img * L;
    if (r0 < L) *reinterpret_cast<uint32_t*>(p.out + (orow + r0) * ow + c) = pack_bf2(o[n][0] * i0, o[n][1] * i0);
    if (r1 < L) *reinterpret_cast<uint32_t*>(p.out + (orow + r1) * ow + c) = pack_bf2(o[n][2] * i1, o[n][3] * i1);
  }
}

// ============================================================================ launch helpers
int ln_launch(const void* x, const void* u, const void* w, const void* b, void* resid_out, void* out, int64_t rows,
              int64_t width, float eps, cudaStream_t s) {
  if (rows == 0) return Q35_OK;
  const bool res = u != nullptr;
  const bool vec = width % 256 == 0 && width <= 2048 && Q35_ALIGNED(x, 16) && Q35_ALIGNED(out, 16) &&
                   Q35_ALIGNED(w, 16) && Q35_ALIGNED(b, 16) && (!res || (Q35_ALIGNED(u, 16) && Q35_ALIGNED(resid_out, 16)));
  const dim3 grid((unsigned)((rows + 7) / 8));
  const bf16 *X = (const bf16*)x, *U = (const bf16*)u, *Wt = (const bf16*)w, *B = (const bf16*)b;
  bf16 *R = (bf16*)resid_out, *O = (bf16*)out;
  if (vec) {
    const int cpl = (int)(width / 256);
#define Q35_LN_CASE(C)                                                                              \
  case C:                                                                                         \
    if (res)                                                                                      \
      layer_norm_kernel<C, true><<<grid, 256, 0, s>>>(X, U, Wt, B, R, O, (int)rows, (int)width, eps); \
    else                                                                                          \
      layer_norm_kernel<C, false><<<grid, 256, 0, s>>>(X, U, Wt, B, R, O, (int)rows, (int)width, eps); \
    return q35_check_launch("layer_norm");
    switch (cpl) {
      Q35_LN_CASE(1)
      Q35_LN_CASE(2)
      Q35_LN_CASE(4)
      Q35_LN_CASE(8)
      default: break;
    }
#undef Q35_LN_CASE
  }
  Q35_REQUIRE(width <= 16384, "layer_norm: width %lld too large", (long long)width);
  const size_t smem = (size_t)width * sizeof(float);
  if (res)
    layer_norm_any_kernel<true><<<(unsigned)rows, 256, smem, s>>>(X, U, Wt, B, R, O, (int)width, eps);
  else
    layer_norm_any_kernel<false><<<(unsigned)rows, 256, smem, s>>>(X, U, Wt, B, R, O, (int)width, eps);
  return q35_check_launch("layer_norm");
}

int pos_embed_norm_launch(const void* hidden, const void* table, const void* w, const void* b, void* resid_out,
                          void* norm_out, int64_t rows, int64_t width, int gh, int gw, int M, int side, float eps,
                          cudaStream_t s) {
  Q35_REQUIRE(width % 256 == 0 && width <= 2048, "vision position embedding: width %lld unsupported",
              (long long)width);
  const dim3 grid((unsigned)((rows + 7) / 8));
  const bool norm = norm_out != nullptr;
  const bf16 *H = (const bf16*)hidden, *T = (const bf16*)table, *Wt = (const bf16*)w, *B = (const bf16*)b;
  bf16 *R = (bf16*)resid_out, *N = (bf16*)norm_out;
  switch (width / 256) {
#define Q35_PE_CASE(C)                                                                                          \
  case C:                                                                                                      \
    if (norm)                                                                                                  \
      pos_embed_kernel<C, true><<<grid, 256, 0, s>>>(H, T, Wt, B, R, N, (int)rows, (int)width, gh, gw, M, side, eps); \
    else                                                                                                       \
      pos_embed_kernel<C, false><<<grid, 256, 0, s>>>(H, T, Wt, B, R, N, (int)rows, (int)width, gh, gw, M, side, eps); \
    return q35_check_launch("vision_position_embed");
    Q35_PE_CASE(1)
    Q35_PE_CASE(2)
    Q35_PE_CASE(4)
    Q35_PE_CASE(8)
#undef Q35_PE_CASE
    default:
      return q35_fail(Q35_ENOTSUP, "vision position embedding: width %lld unsupported", (long long)width);
  }
}

int attn_launch(const void* q, const void* k, const void* v, void* out, int64_t L, int64_t heads, float scale,
                cudaStream_t s, int64_t images = 1) {
  if (L == 0 || images == 0) return Q35_OK;
  VisionAttnParams p{(const bf16*)q, (const bf16*)k, (const bf16*)v, (bf16*)out, (int)L, (int)heads,
                     scale * 1.4426950408889634f};
  vision_attn_kernel<<<dim3((unsigned)((L + kVaRows - 1) / kVaRows), (unsigned)heads, (unsigned)images), kVaThreads, 0,
                       s>>>(p);
  return q35_check_launch("vision_attention");
}

struct VCarve {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~(size_t)255;
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
};

struct VitBuffers {
  bf16 *patches, *resid, *norm, *packed, *q, *k, *v, *attn, *upd, *mlp, *m1;
  float *cos_t, *sin_t;
};

VitBuffers vit_carve(const q35_vit_desc& d, void* base, size_t* total) {
  VCarve c{static_cast<char*>(base)};
  VitBuffers b;
  const int64_t N = d.max_patches, W = d.width;
  const int64_t F = (int64_t)d.in_channels * d.temporal_patch * d.patch * d.patch;
  b.patches = c.take<bf16>(N * F);
  b.resid = c.take<bf16>(N * W);
  b.norm = c.take<bf16>(N * W);
  b.packed = c.take<bf16>(N * 3 * W);
  b.q = c.take<bf16>(N * W);
  b.k = c.take<bf16>(N * W);
  b.v = c.take<bf16>(N * W);
  b.attn = c.take<bf16>(N * W);
  b.upd = c.take<bf16>(N * W);
  b.mlp = c.take<bf16>(N * d.intermediate);
  b.m1 = c.take<bf16>(N * W);  // merged rows [N / M^2, M^2 W]
  b.cos_t = c.take<float>(N * kVD);
  b.sin_t = c.take<float>(N * kVD);
  *total = c.off + 256;
  return b;
}

}  // namespace

// ================================================================================ C ABI
extern "C" int q35_layer_norm(const void* x, const void* weight, const void* bias, void* out, int64_t rows,
                              int64_t width, float eps, void* stream) {
  Q35_REQUIRE(x && weight && bias && out && rows >= 0 && width > 0, "layer_norm: bad argument");
  return ln_launch(x, nullptr, weight, bias, nullptr, out, rows, width, eps, (cudaStream_t)stream);
}

extern "C" int q35_residual_add_layer_norm(const void* residual, const void* update, const void* weight,
                                           const void* bias, void* residual_out, void* norm_out, int64_t rows,
                                           int64_t width, float eps, void* stream) {
  Q35_REQUIRE(residual && update && weight && bias && residual_out && norm_out && rows >= 0 && width > 0,
              "residual_add_layer_norm: bad argument");
  return ln_launch(residual, update, weight, bias, residual_out, norm_out, rows, width, eps, (cudaStream_t)stream);
}

extern "C" int q35_position_embed_add(const void* hidden, const void* table, const int64_t* indices,
                                      const float* weights, void* out, int64_t rows, int64_t width,
                                      int64_t neighbors, void* stream) {
  Q35_REQUIRE(hidden && table && indices && weights && out && rows >= 0 && width > 0 && neighbors >= 1,
              "position_embed_add: bad argument");
  if (rows == 0) return Q35_OK;
  pos_embed_given_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)hidden, (const bf16*)table, indices, weights, (bf16*)out, (int)width, (int)neighbors);
  return q35_check_launch("position_embed_add");
}

extern "C" int q35_vision_qkv_rope(const void* packed, const float* cos, const float* sin, void* q_out,
                                   void* k_out, void* v_out, int64_t tokens, int64_t heads, int64_t dim,
                                   void* stream) {
  Q35_REQUIRE(packed && cos && sin && q_out && k_out && v_out && tokens >= 0 && heads >= 1,
              "vision_qkv_rope: bad argument");
  Q35_REQUIRE(dim == kVD, "vision_qkv_rope: head dim %lld unsupported (64)", (long long)dim);
  if (tokens == 0) return Q35_OK;
  qkv_rope_kernel<<<(unsigned)((tokens * heads + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)packed, cos, sin, (bf16*)q_out, (bf16*)k_out, (bf16*)v_out, (int)tokens, (int)heads, (int)tokens);
  return q35_check_launch("vision_qkv_rope");
}

extern "C" int q35_vision_attention(const void* q, const void* k, const void* v, void* out, int64_t tokens,
                                    int64_t heads, int64_t dim, float scale, void* stream) {
  Q35_REQUIRE(q && k && v && out && tokens >= 0 && heads >= 1, "vision_attention: bad argument");
  Q35_REQUIRE(dim == kVD, "vision_attention: head dim %lld unsupported (64)", (long long)dim);
  Q35_REQUIRE(Q35_ALIGNED(q, 16) && Q35_ALIGNED(k, 16) && Q35_ALIGNED(v, 16) && Q35_ALIGNED(out, 4),
              "vision_attention: alignment");
  return attn_launch(q, k, v, out, tokens, heads, scale, (cudaStream_t)stream);
}

extern "C" int q35_vision_rope_table(const float* inv_freq, float* cos_out, float* sin_out, int64_t grid_h,
                                     int64_t grid_w, int64_t merge, void* stream) {
  Q35_REQUIRE(inv_freq && cos_out && sin_out && grid_h > 0 && grid_w > 0 && merge >= 1 && grid_h % merge == 0 &&
                  grid_w % merge == 0,
              "vision_rope_table: bad argument");
  const int n = (int)(grid_h * grid_w * kVD);
  rope_table_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(cos_out, sin_out, inv_freq,
                                                                        (int)(grid_h * grid_w), (int)grid_w,
                                                                        (int)merge);
  return q35_check_launch("vision_rope_table");
}

extern "C" int q35_vision_patchify(const float* pixels, void* out, int64_t channels, int64_t height, int64_t width,
                                   int64_t patch, int64_t temporal_patch, int64_t merge, float mean, float std,
                                   void* stream) {
  Q35_REQUIRE(pixels && out && channels >= 1 && patch >= 8 && patch % 8 == 0 && temporal_patch >= 1 && merge >= 1,
              "vision_patchify: bad argument");
  Q35_REQUIRE(height % (patch * merge) == 0 && width % (patch * merge) == 0,
              "vision_patchify: image %lldx%lld is not a multiple of patch x merge", (long long)height,
              (long long)width);
  Q35_REQUIRE(Q35_ALIGNED(out, 16) && std != 0.f, "vision_patchify: 16-byte aligned output, nonzero std");
  const int64_t n_patches = (height / patch) * (width / patch);
  const int64_t groups = n_patches * channels * temporal_patch * patch * patch / 8;
  patchify_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      pixels, (bf16*)out, (int)channels, (int)height, (int)width, (int)patch, (int)temporal_patch, (int)merge,
      (int)n_patches, mean, 1.0f / std);
  return q35_check_launch("vision_patchify");
}

// ------------------------------------------------------------------------------ ViT runner
struct q35_vit {
  q35_vit_desc d;
  std::vector<q35_vit_block_desc> blocks;
  VitBuffers buf;
};

extern "C" size_t q35_vit_workspace_size(const q35_vit_desc* desc) {
  if (!desc) return 0;
  size_t total = 0;
  vit_carve(*desc, nullptr, &total);
  return total;
}

extern "C" int q35_vit_create(const q35_vit_desc* desc, q35_vit** out) {
  Q35_REQUIRE(desc && out && desc->blocks && desc->depth > 0, "vit_create: bad descriptor");
  const q35_vit_desc& d = *desc;
  Q35_REQUIRE(d.width == d.heads * kVD, "vit_create: head dim must be 64 (width %d, heads %d)", d.width, d.heads);
  Q35_REQUIRE(d.width % 256 == 0 && d.width <= 2048 && d.intermediate % 64 == 0 && d.out_width % 8 == 0,
              "vit_create: width must be a multiple of 256 (<= 2048), intermediate of 64, out width of 8");
  Q35_REQUIRE(d.merge >= 1 && d.patch % 8 == 0 && d.temporal_patch >= 1 && d.in_channels >= 1 && d.pos_side >= 1,
              "vit_create: bad patch geometry");
  Q35_REQUIRE((d.in_channels * d.temporal_patch * d.patch * d.patch) % 64 == 0,
              "vit_create: patch features must be a multiple of 64");
  Q35_REQUIRE(d.patch_w && d.patch_b && d.pos_table && d.rope_inv_freq && d.merger_norm_w && d.merger_norm_b &&
                  d.merger_fc1_w && d.merger_fc1_b && d.merger_fc2_w && d.merger_fc2_b,
              "vit_create: missing weight");
  Q35_REQUIRE(d.max_patches > 0 && d.workspace && d.workspace_bytes >= q35_vit_workspace_size(desc),
              "vit_create: workspace too small");
  for (int i = 0; i < d.depth; ++i) {
    const q35_vit_block_desc& B = d.blocks[i];
    Q35_REQUIRE(B.norm1_w && B.norm1_b && B.norm2_w && B.norm2_b && B.qkv_w && B.qkv_b && B.proj_w && B.proj_b &&
                    B.fc1_w && B.fc1_b && B.fc2_w && B.fc2_b,
                "vit block %d: missing weight", i);
  }
  q35_vit* v = new q35_vit();
  v->d = d;
  v->blocks.assign(d.blocks, d.blocks + d.depth);
  v->d.blocks = v->blocks.data();
  size_t total = 0;
  v->buf = vit_carve(d, d.workspace, &total);
  *out = v;
  return Q35_OK;
}

extern "C" void q35_vit_destroy(q35_vit* v) { delete v; }

#define Q35_VTRY(x)       \
  do {                    \
    int _rc = (x);        \
    if (_rc) return _rc;  \
  } while (0)

// Processor output (fp32 patches) to the bf16 GEMM operand, 8 values per thread.
__global__ void patch_cast_kernel(const float* __restrict__ in, bf16* __restrict__ out, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const float4 a = reinterpret_cast<const float4*>(in)[2 * i], b = reinterpret_cast<const float4*>(in)[2 * i + 1];
  __align__(16) bf16 o[8] = {f2bf(a.x), f2bf(a.y), f2bf(a.z), f2bf(a.w), f2bf(b.x), f2bf(b.y), f2bf(b.z), f2bf(b.w)};
  reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<const uint4*>(o);
}

static int vit_blocks(q35_vit* vit, int64_t gh, int64_t gw, int64_t images, void* out, cudaStream_t s);

extern "C" int q35_vit_encode_patches(q35_vit* vit, const float* patches, int64_t grid_h, int64_t grid_w, void* out,
                                      void* stream) {
  Q35_REQUIRE(vit && patches && out, "vit_encode_patches: null argument");
  const q35_vit_desc& d = vit->d;
  Q35_REQUIRE(grid_h > 0 && grid_w > 0 && grid_h % d.merge == 0 && grid_w % d.merge == 0,
              "vit_encode_patches: grid %lldx%lld is not a multiple of the merge size", (long long)grid_h,
              (long long)grid_w);
  Q35_REQUIRE(grid_h * grid_w <= d.max_patches, "vit_encode_patches: %lld patches exceed max_patches %d",
              (long long)(grid_h * grid_w), d.max_patches);
  Q35_REQUIRE(Q35_ALIGNED(patches, 16), "vit_encode_patches: 16-byte aligned patches");
  const int64_t F = (int64_t)d.in_channels * d.temporal_patch * d.patch * d.patch;
  const int64_t n8 = grid_h * grid_w * F / 8;
  patch_cast_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(patches, vit->buf.patches, n8);
  Q35_VTRY(q35_check_launch("vit patch cast"));
  return vit_blocks(vit, grid_h, grid_w, 1, out, (cudaStream_t)stream);
}

extern "C" int q35_vit_encode_batch(q35_vit* vit, const float* pixels, int64_t images, int64_t height, int64_t width,
                                    void* out, void* stream) {
  Q35_REQUIRE(vit && pixels && out && images >= 1, "vit_encode: null argument or no image");
  const q35_vit_desc& d = vit->d;
  const VitBuffers& B = vit->buf;
  const int64_t P = d.patch, M = d.merge;
  Q35_REQUIRE(height % (P * M) == 0 && width % (P * M) == 0, "vit_encode: image size must be a multiple of %lld",
              (long long)(P * M));
  const int64_t gh = height / P, gw = width / P;
  Q35_REQUIRE(images * gh * gw <= d.max_patches, "vit_encode: %lld patches exceed max_patches %d",
              (long long)(images * gh * gw), d.max_patches);
  const int64_t groups = gh * gw * d.in_channels * d.temporal_patch * P * P / 8;
  patchify_kernel<<<dim3((unsigned)((groups + 255) / 256), (unsigned)images), 256, 0, (cudaStream_t)stream>>>(
      pixels, B.patches, d.in_channels, (int)height, (int)width, (int)P, d.temporal_patch, (int)M, (int)(gh * gw),
      d.pixel_mean, 1.0f / d.pixel_std);
  Q35_VTRY(q35_check_launch("vit patchify"));
  return vit_blocks(vit, gh, gw, images, out, (cudaStream_t)stream);
}

extern "C" int q35_vit_encode(q35_vit* vit, const float* pixels, int64_t height, int64_t width, void* out,
                              void* stream) {
  return q35_vit_encode_batch(vit, pixels, 1, height, width, out, stream);
}

// Patch embedding (from vit->buf.patches), position embedding, the blocks and the merger.
static int vit_blocks(q35_vit* vit, int64_t gh, int64_t gw, int64_t images, void* out, cudaStream_t s) {
  const q35_vit_desc& d = vit->d;
  const VitBuffers& B = vit->buf;
  void* stream = s;
  const int64_t P = d.patch, M = d.merge;
  const int64_t NI = gh * gw, N = images * NI, W = d.width;  // patches per image, in the batch
  const int64_t F = (int64_t)d.in_channels * d.temporal_patch * P * P;
  Q35_VTRY(q35_gemm_tc_bias_launch(B.patches, d.patch_w, d.patch_b, B.upd, N, W, F, Q35_EPI_BIAS, s));
  Q35_VTRY(q35_vision_rope_table(d.rope_inv_freq, B.cos_t, B.sin_t, gh, gw, M, stream));
  Q35_VTRY(pos_embed_norm_launch(B.upd, d.pos_table, d.blocks[0].norm1_w, d.blocks[0].norm1_b, B.resid, B.norm, N, W,
                                 (int)gh, (int)gw, (int)M, d.pos_side, d.eps, s));
  const float scale = 1.0f / sqrtf((float)kVD);
  for (int i = 0; i < d.depth; ++i) {
    const q35_vit_block_desc& L = vit->blocks[i];
    Q35_VTRY(q35_gemm_tc_bias_launch(B.norm, L.qkv_w, L.qkv_b, B.packed, N, 3 * W, W, Q35_EPI_BIAS, s));
    qkv_rope_kernel<<<(unsigned)((N * d.heads + 7) / 8), 256, 0, s>>>(B.packed, B.cos_t, B.sin_t, B.q, B.k, B.v, (int)N,
                                                                      d.heads, (int)NI);
    Q35_VTRY(q35_check_launch("vit qkv rope"));
    Q35_VTRY(attn_launch(B.q, B.k, B.v, B.attn, NI, d.heads, scale, s, images));
    Q35_VTRY(q35_gemm_tc_bias_launch(B.attn, L.proj_w, L.proj_b, B.upd, N, W, W, Q35_EPI_BIAS, s));
    Q35_VTRY(ln_launch(B.resid, B.upd, L.norm2_w, L.norm2_b, B.resid, B.norm, N, W, d.eps, s));
    Q35_VTRY(q35_gemm_tc_bias_launch(B.norm, L.fc1_w, L.fc1_b, B.mlp, N, d.intermediate, W,
                                     Q35_EPI_BIAS_GELU_TANH, s));
    Q35_VTRY(q35_gemm_tc_bias_launch(B.mlp, L.fc2_w, L.fc2_b, B.upd, N, W, d.intermediate, Q35_EPI_BIAS, s));
    // next block's norm1, or after the last block the merger's LayerNorm of (residual + update)
    const bool last = i + 1 == d.depth;
    const void* nw = last ? d.merger_norm_w : vit->blocks[i + 1].norm1_w;
    const void* nb = last ? d.merger_norm_b : vit->blocks[i + 1].norm1_b;
    Q35_VTRY(ln_launch(B.resid, B.upd, nw, nb, B.resid, B.norm, N, W, d.eps, s));
  }
  // merger: the LayerNorm'd tokens, M^2 consecutive rows as one [M^2 W] row -> fc1 + GELU -> fc2
  const int64_t NM = N / (M * M), WM = W * M * M;
  Q35_VTRY(q35_gemm_tc_bias_launch(B.norm, d.merger_fc1_w, d.merger_fc1_b, B.m1, NM, WM, WM, Q35_EPI_BIAS_GELU, s));
  return q35_gemm_tc_bias_launch(B.m1, d.merger_fc2_w, d.merger_fc2_b, out, NM, d.out_width, WM, Q35_EPI_BIAS, s);
}

extern "C" void* q35_vit_hidden(const q35_vit* vit) { return vit ? vit->buf.resid : nullptr; }
