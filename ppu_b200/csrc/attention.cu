// Gated GQA attention for Qwen3.5 (reference: kernels.py:419-573 qgkv_norm_rope, 940-1090
// gqa_decode_attention, 285-333 attention_gate_mul; integration.py:282-380).
//
// * qgkv_norm_rope: one CTA per (batch, token); thread d owns dimension d of every head, so the
//   per-head RMSNorm reductions and the RoPE partner exchange stay in shared memory.
// * decode attention: split-KV over the cache rows with all G = Hq/Hkv query heads of one KV
//   head in the same CTA (K/V are read once per group, not once per query head); FP32 online
//   softmax per warp, merged per CTA, then the last CTA of each (batch, KV head) combines the
//   splits (atomic ticket; no second launch) and applies the sigmoid output gate. The fused
//   variant also performs the Q/K norm + RoPE and the cache write of the current token, so a
//   whole decode attention layer (minus the projections) is one kernel.
// * prefill attention: causal, FP32 CUDA-core tiles (64 queries x 64 keys per step).
#include <cfloat>

#include "common.cuh"

using namespace q35;

namespace {

constexpr int kD = 256;  // head_dim of every Qwen3.5 attention layer

// ============================================================================ qgkv_norm_rope
template <bool TABLE>
__global__ void __launch_bounds__(kD) qgkv_rope_kernel(
    const bf16* __restrict__ packed, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const bf16* __restrict__ cos_t, const bf16* __restrict__ sin_t, const float* __restrict__ inv_freq,
    int64_t pos_base, bf16* __restrict__ q_out, bf16* __restrict__ k_out, bf16* __restrict__ v_out,
    const int64_t* __restrict__ cache_start, int L, int Hq, int Hkv, int rot, int kv_len, float eps,
    const int64_t* __restrict__ pos3 = nullptr, int sec_h = 0, int sec_w = 0, bf16* __restrict__ vt_out = nullptr,
    int vt_stride = 0) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  __shared__ float normed[kD];
  __shared__ float red[kD / 32];
  const int bt = blockIdx.x;  // b * L + t
  const int b = bt / L, t = bt - b * L;
  const int d = threadIdx.x;
  const int stride = 2 * Hq * kD + 2 * Hkv * kD;
  const bf16* row = packed + (int64_t)bt * stride;
  const int64_t start = cache_start ? *cache_start : 0;
  float c = 1.f, s = 0.f;
  if (d < rot) {
    if (TABLE) {
      c = bf2f(cos_t[(int64_t)bt * rot + d]);
      s = bf2f(sin_t[(int64_t)bt * rot + d]);
    } else {
      int64_t pos = pos_base + start + t;
      if (pos3) {  // interleaved M-RoPE: frequency j takes the height / width axis at j % 3 == 1 / 2
        const int j = d % (rot / 2);
        const int axis = (j % 3 == 1 && j < 3 * sec_h) ? 1 : (j % 3 == 2 && j < 3 * sec_w) ? 2 : 0;
        pos = pos3[((int64_t)axis * (gridDim.x / L) + b) * L + t];  // [3, batch, L]
      }
      rope_cs(d, rot / 2, (float)pos, inv_freq, c, s);
    }
  }
  for (int h = 0; h < Hq + Hkv; ++h) {
    const bool is_q = h < Hq;
    const int off = is_q ? h * 2 * kD : 2 * Hq * kD + (h - Hq) * kD;
    const float x = bf2f(row[off + d]);
    const float var = block_sum<kD / 32>(x * x, red) / (float)kD;
    const float w = bf2f(is_q ? qw[d] : kw[d]);
    normed[d] = rbf(x * rsqrt_ieee(var + eps) * (1.0f + w));
    __syncthreads();
    const float y = rope_apply(normed, d, rot, c, s);
    if (is_q) {
      q_out[(((int64_t)b * Hq + h) * L + t) * kD + d] = f2bf(y);
    } else if (start + t >= 0 && start + t < kv_len) {  // device-side start: never write past the cache
      const int kh = h - Hq;
      const int64_t o = (((int64_t)b * Hkv + kh) * kv_len + start + t) * kD + d;
      k_out[o] = f2bf(y);
      const bf16 vv = row[2 * Hq * kD + Hkv * kD + kh * kD + d];
      v_out[o] = vv;
      // V^T [b][kv head][dim][key] for the tcgen05 prefill attention (its K-major B operand)
      if (vt_out != nullptr && start + t < vt_stride) vt_out[(((int64_t)b * Hkv + kh) * kD + d) * vt_stride + start + t] = vv;
    }
    __syncthreads();
  }
}

// Prefill form of the decoder (positions, not tables; rotary_dim 64, Qwen3.5's): one warp per
// (token, head), lane l holding dims l + 32 i (i < 8), so the norm's sum is formed exactly as
// block_sum forms it in qgkv_rope_kernel (a butterfly over each 32-dim group, the 8 group sums in
// order) and the RoPE partner of dim d (d +- 32) sits in the same lane: no barrier, and the
// outputs are bit-identical to the one-CTA-per-token kernel.
__global__ void __launch_bounds__(256) qgkv_rope_warp_kernel(
    const bf16* __restrict__ packed, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const float* __restrict__ inv_freq, bf16* __restrict__ q_out, bf16* __restrict__ k_out, bf16* __restrict__ v_out,
    const int64_t* __restrict__ cache_start, int batch, int L, int Hq, int Hkv, int rot, int kv_len, float eps,
    const int64_t* __restrict__ pos3, int sec_h, int sec_w, bf16* __restrict__ vt_out, int vt_stride) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  constexpr int NG = kD / 32;  // dims per lane
  const int lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int heads = Hq + Hkv;
  if (pair >= (int64_t)batch * L * heads) return;
  const int h = (int)(pair % heads);
  const int bt = (int)(pair / heads), b = bt / L, t = bt - b * L;
  const bool is_q = h < Hq;
  const int stride = 2 * Hq * kD + 2 * Hkv * kD;
  const bf16* row = packed + (int64_t)bt * stride;
  const int off = is_q ? h * 2 * kD : 2 * Hq * kD + (h - Hq) * kD;
  const int64_t start = cache_start ? *cache_start : 0;
  float x[NG], wv[NG];
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    x[i] = bf2f(row[off + lane + 32 * i]);
    wv[i] = bf2f(is_q ? qw[lane + 32 * i] : kw[lane + 32 * i]);
  }
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < NG; ++i) var += warp_sum(x[i] * x[i]);
  var /= (float)kD;
  float nrm[NG];
#pragma unroll
  for (int i = 0; i < NG; ++i) nrm[i] = rbf(x[i] * rsqrt_ieee(var + eps) * (1.0f + wv[i]));
  constexpr int half = 32;  // rot / 2
  float y[NG];
#pragma unroll
  for (int i = 0; i < NG; ++i) y[i] = nrm[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // dims lane (partner lane + 32, negated) and lane + 32 (partner lane)
    const int d = lane + 32 * i;
    int64_t pos = start + t;
    if (pos3) {  // interleaved M-RoPE: frequency j takes the height / width axis at j % 3 == 1 / 2
      const int j = d % half;
      const int axis = (j % 3 == 1 && j < 3 * sec_h) ? 1 : (j % 3 == 2 && j < 3 * sec_w) ? 2 : 0;
      pos = pos3[((int64_t)axis * batch + b) * L + t];  // [3, batch, L]
    }
    float c, sn;
    rope_cs(d, half, (float)pos, inv_freq, c, sn);
    const float partner = i == 0 ? -nrm[1] : nrm[0];
    y[i] = rbf(rbf(nrm[i] * c) + rbf(partner * sn));
  }
  if (is_q) {
    bf16* o = q_out + (((int64_t)b * Hq + h) * L + t) * kD + lane;
#pragma unroll
    for (int i = 0; i < NG; ++i) o[32 * i] = f2bf(y[i]);
  } else if (start + t >= 0 && start + t < kv_len) {  // device-side start: never write past the cache
    const int kh = h - Hq;
    const int64_t o = (((int64_t)b * Hkv + kh) * kv_len + start + t) * kD + lane;
#pragma unroll
    for (int i = 0; i < NG; ++i) {
      k_out[o + 32 * i] = f2bf(y[i]);
      const bf16 vv = row[2 * Hq * kD + Hkv * kD + kh * kD + lane + 32 * i];
      v_out[o + 32 * i] = vv;
      if (vt_out != nullptr && start + t < vt_stride)
        vt_out[(((int64_t)b * Hkv + kh) * kD + lane + 32 * i) * vt_stride + start + t] = vv;
    }
  }
}

// ============================================================================ prefill attention, tensor cores
// FlashAttention-style causal GQA prefill on mma.sync m16n8k16 (bf16 in, FP32 accumulate).
// CTA = (16 query rows, group g of G query heads): warp w handles query head g * G + w, so each K/V tile in
// shared memory serves the G heads of the group. Keys stream in tiles of 32 (cp.async, double
// buffered, rows padded by 16 bytes so ldmatrix hits distinct banks). S = Q K^T from ldmatrix
// fragments (bf16 products are exact, FP32 accumulation), scaled, causally masked, online softmax
// in FP32; P.V uses P split into a bf16 high part and a bf16 remainder (two MMAs), which keeps the
// probabilities to ~16 bits so the result tracks an FP32 softmax.
constexpr int kFaRows = 16, kFaKeys = 32, kFaStride = kD + 8;

Q35_DEV void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

template <int G>
__global__ void __launch_bounds__(2 * G * 32) prefill_attn_mma_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                                     const bf16* __restrict__ V, bf16* __restrict__ O,
                                                                     int Hq, int Hkv, int L, int kv_len, int q_offset,
                                                                     float scale, int kv_div) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char fa_smem[];
  bf16* Qs = reinterpret_cast<bf16*>(fa_smem);        // [G][16][stride]
  bf16* KVs = Qs + G * kFaRows * kFaStride;            // per key group: K [2][32][stride], V [2][32][stride]
  constexpr int NG = G * 32;                           // threads of one key group
  constexpr int NT = 2 * NG;
  const int q0 = blockIdx.x * kFaRows, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kg = warp / G, wq = warp % G;  // key group (even / odd key tiles), query head in the group
  const int gt = threadIdx.x - kg * NG;    // thread index within the key group
  const int h = g * G + wq;
  bf16* Ks = KVs + kg * 4 * kFaKeys * kFaStride;
  bf16* Vs = Ks + 2 * kFaKeys * kFaStride;
  // blockIdx.y counts groups of G query heads; kv_div of them share one KV head
  const bf16* Kg = K + ((int64_t)b * Hkv + g / kv_div) * kv_len * kD;
  const bf16* Vg = V + ((int64_t)b * Hkv + g / kv_div) * kv_len * kD;
  // queries of the G heads (rows past L read as zero)
  for (int i = threadIdx.x; i < G * kFaRows * (kD / 8); i += NT) {
    const int hh = i / (kFaRows * (kD / 8)), r = (i / (kD / 8)) % kFaRows, c = (i % (kD / 8)) * 8;
    bf16* dst = Qs + (hh * kFaRows + r) * kFaStride + c;
    if (q0 + r < L)
      cp16(dst, Q + (((int64_t)b * Hq + g * G + hh) * L + q0 + r) * kD + c);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
  const int kend = min(kv_len, q0 + kFaRows - 1 + q_offset + 1);  // keys any row of the block may see
  const int ntiles = (kend + kFaKeys - 1) / kFaKeys;
  auto load_tile = [&](int t, int buf) {  // by this key group's threads
    const int k0 = t * kFaKeys;
    for (int i = gt; i < kFaKeys * (kD / 8); i += NG) {
      const int r = i / (kD / 8), c = (i % (kD / 8)) * 8;
      bf16* kd = Ks + (buf * kFaKeys + r) * kFaStride + c;
      bf16* vd = Vs + (buf * kFaKeys + r) * kFaStride + c;
      if (k0 + r < kv_len) {
        cp16(kd, Kg + (int64_t)(k0 + r) * kD + c);
        cp16(vd, Vg + (int64_t)(k0 + r) * kD + c);
      } else {
        *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + kg), "r"(NG) : "memory"); };
  if (kg < ntiles) load_tile(kg, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // the query tile (loaded by both groups) and the first key tiles are in place

  const int gq = lane >> 2, c4 = lane & 3;  // fragment row group / column pair
  float o[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;  // rows gq and gq + 8
  const int qi0 = q0 + gq + q_offset, qi1 = qi0 + 8;
  const uint32_t qbase = (uint32_t)__cvta_generic_to_shared(Qs + (wq * kFaRows + (lane & 15)) * kFaStride) +
                         (lane >> 4) * 16;
  int it = 0;
  for (int t = kg; t < ntiles; t += 2, ++it) {
    const int buf = it & 1;
    if (t + 2 < ntiles) load_tile(t + 2, buf ^ 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    group_sync();
    // ---- S = Q K^T for 16 rows x 32 keys
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    const uint32_t kbase = (uint32_t)__cvta_generic_to_shared(Ks + (buf * kFaKeys) * kFaStride);
#pragma unroll 4
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(qbase + ks * 32, a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 2; ++np) {  // key n-tiles 2np, 2np + 1
        uint32_t b0, b1, b2, b3;
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(kbase + key * kFaStride * 2 + ks * 32 + ((lane >> 3) & 1) * 16, b0, b1, b2, b3);
        mma_bf16(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- scale, causal mask, online softmax (rows gq and gq + 8; keys n*8 + 2*c4 + {0,1})
    const int k0 = t * kFaKeys;
    float mx0 = -FLT_MAX, mx1 = -FLT_MAX;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kj = k0 + n * 8 + 2 * c4 + e;
        const bool ok = kj < kv_len;
        s[n][e] = (ok && kj <= qi0) ? s[n][e] * scale : -FLT_MAX;
        s[n][2 + e] = (ok && kj <= qi1) ? s[n][2 + e] * scale : -FLT_MAX;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = (m0 == -FLT_MAX) ? 0.f : expf(m0 - mn0), al1 = (m1 == -FLT_MAX) ? 0.f : expf(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = (s[n][e] == -FLT_MAX) ? 0.f : expf(s[n][e] - mn0);
        s[n][2 + e] = (s[n][2 + e] == -FLT_MAX) ? 0.f : expf(s[n][2 + e] - mn1);
        rs0 += s[n][e];
        rs1 += s[n][2 + e];
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, off);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, off);
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    // ---- O += P V: P (16 x 32) as two k-steps of 16 keys, high and low bf16 parts
    const uint32_t vbase = (uint32_t)__cvta_generic_to_shared(Vs + (buf * kFaKeys) * kFaStride);
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const float* pa = s[2 * kk];
      const float* pb = s[2 * kk + 1];
      const uint32_t h0 = pack_bf2(pa[0], pa[1]), h1 = pack_bf2(pa[2], pa[3]);
      const uint32_t h2 = pack_bf2(pb[0], pb[1]), h3 = pack_bf2(pb[2], pb[3]);
      auto resid = [](float x, uint32_t packed, int half) {
        const float r = __uint_as_float(half ? (packed & 0xffff0000u) : (packed << 16));
        return x - r;
      };
      const uint32_t l0p = pack_bf2(resid(pa[0], h0, 0), resid(pa[1], h0, 1));
      const uint32_t l1p = pack_bf2(resid(pa[2], h1, 0), resid(pa[3], h1, 1));
      const uint32_t l2p = pack_bf2(resid(pb[0], h2, 0), resid(pb[1], h2, 1));
      const uint32_t l3p = pack_bf2(resid(pb[2], h3, 0), resid(pb[3], h3, 1));
      // B fragments of V (keys kk*16 .. +15 x dims): transposed 8x8 loads, two dim n-tiles per x4
      const int vrow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
      for (int np = 0; np < 16; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + vrow * kFaStride * 2 + (np * 16 + (lane >> 4) * 8) * 2, b0, b1, b2, b3);
        mma_bf16(o[2 * np], h0, h1, h2, h3, b0, b1);
        mma_bf16(o[2 * np], l0p, l1p, l2p, l3p, b0, b1);
        mma_bf16(o[2 * np + 1], h0, h1, h2, h3, b2, b3);
        mma_bf16(o[2 * np + 1], l0p, l1p, l2p, l3p, b2, b3);
      }
    }
    group_sync();  // this buffer is refilled two tiles later
  }
  // ---- merge the two key groups' partial softmax states (group 1 parks them in the freed key /
  // value tiles), then normalise and store (rows gq, gq + 8; dims n*8 + 2*c4 + {0,1})
  __syncthreads();
  constexpr int kPart = 4 + 32 * 4 + 1;  // m0 m1 l0 l1, o, pad (odd stride: no bank conflicts)
  float* pp = reinterpret_cast<float*>(KVs) + (wq * 32 + lane) * kPart;
  if (kg == 1) {
    pp[0] = m0;
    pp[1] = m1;
    pp[2] = l0;
    pp[3] = l1;
#pragma unroll
    for (int n = 0; n < 32; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) pp[4 + 4 * n + e] = o[n][e];
  }
  __syncthreads();
  if (kg == 1) return;
  {
    const float mb0 = pp[0], mb1 = pp[1], lb0 = pp[2], lb1 = pp[3];
    const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
    const float fa0 = (m0 == -FLT_MAX) ? 0.f : expf(m0 - mn0), fb0 = (mb0 == -FLT_MAX) ? 0.f : expf(mb0 - mn0);
    const float fa1 = (m1 == -FLT_MAX) ? 0.f : expf(m1 - mn1), fb1 = (mb1 == -FLT_MAX) ? 0.f : expf(mb1 - mn1);
    l0 = l0 * fa0 + lb0 * fb0;
    l1 = l1 * fa1 + lb1 * fb1;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      o[n][0] = o[n][0] * fa0 + pp[4 + 4 * n] * fb0;
      o[n][1] = o[n][1] * fa0 + pp[5 + 4 * n] * fb0;
      o[n][2] = o[n][2] * fa1 + pp[6 + 4 * n] * fb1;
      o[n][3] = o[n][3] * fa1 + pp[7 + 4 * n] * fb1;
    }
  }
  const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f, inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  const int r0 = q0 + gq, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < 32; ++n) {
    const int d = n * 8 + 2 * c4;
    if (r0 < L)
      *reinterpret_cast<uint32_t*>(O + (((int64_t)b * L + r0) * Hq + h) * kD + d) =
          pack_bf2(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < L)
      *reinterpret_cast<uint32_t*>(O + (((int64_t)b * L + r1) * Hq + h) * kD + d) =
          pack_bf2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

template <int G>
int launch_prefill_mma(const void* q, const void* k, const void* v, void* out, int64_t batch, int64_t q_heads,
                       int64_t kv_heads, int64_t seq_len, int64_t kv_len, int64_t q_offset, float scale,
                       cudaStream_t stream, bool pdl) {
  const int kv_div = (int)(q_heads / kv_heads / G);  // query-head groups of G per KV head
  // query tile + two key groups x two buffers x (K, V) tiles; the merge reuses the key tiles
  const size_t smem = (size_t)(G * kFaRows + 8 * kFaKeys) * kFaStride * sizeof(bf16);
  static_assert((size_t)4 * 32 * (4 + 32 * 4 + 1) * sizeof(float) <= (size_t)8 * kFaKeys * kFaStride * sizeof(bf16),
                "the merge partials fit in the key / value tiles");
  cudaFuncSetAttribute(prefill_attn_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const dim3 grid((unsigned)((seq_len + kFaRows - 1) / kFaRows), (unsigned)(kv_heads * kv_div), (unsigned)batch);
  const cudaError_t e = q35_launch(prefill_attn_mma_kernel<G>, grid, dim3(2 * G * 32), smem, stream, pdl,
                                   (const bf16*)q, (const bf16*)k, (const bf16*)v, (bf16*)out, (int)q_heads,
                                   (int)kv_heads, (int)seq_len, (int)kv_len, (int)q_offset, scale, kv_div);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "prefill_attention launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

}  // namespace

// ------------------------------------------------------------------------------------ C ABI
extern "C" int q35_qgkv_norm_rope(const void* packed, const void* q_weight, const void* k_weight,
                                  const void* cos, const void* sin, void* q_out, void* k_out, void* v_out,
                                  const int64_t* cache_start, int64_t batch, int64_t seq_len,
                                  int64_t q_heads, int64_t kv_heads, int64_t dim, int64_t rotary_dim,
                                  int64_t kv_len, float eps, void* stream) {
  Q35_REQUIRE(packed && q_weight && k_weight && cos && sin && q_out && k_out && v_out,
              "qgkv_norm_rope: null pointer");
  Q35_REQUIRE(dim == kD, "qgkv_norm_rope: head dim %lld unsupported (256)", (long long)dim);
  Q35_REQUIRE(rotary_dim > 0 && rotary_dim <= dim && rotary_dim % 2 == 0, "qgkv_norm_rope: bad rotary_dim");
  Q35_REQUIRE(batch >= 0 && seq_len >= 0 && q_heads > 0 && kv_heads > 0 && kv_len >= seq_len,
              "qgkv_norm_rope: bad shape");
  if (batch * seq_len == 0) return Q35_OK;
  qgkv_rope_kernel<true><<<(unsigned)(batch * seq_len), kD, 0, (cudaStream_t)stream>>>(
      (const bf16*)packed, (const bf16*)q_weight, (const bf16*)k_weight, (const bf16*)cos, (const bf16*)sin,
      nullptr, 0, (bf16*)q_out, (bf16*)k_out, (bf16*)v_out, cache_start, (int)seq_len, (int)q_heads,
      (int)kv_heads, (int)rotary_dim, (int)kv_len, eps);
  return q35_check_launch("qgkv_norm_rope");
}

// Prefill variant used by the decoder: RoPE from positions cache_start + t (text tokens).
// With pos3 (int64 [3, batch, seq_len]), the positions are 3-axis M-RoPE positions interleaved
// by (sec_h, sec_w) frequency pairs (Transformers apply_interleaved_mrope). With vt_out, V is also
// written transposed: vt_out [batch, kv_heads, 256, vt_stride].
namespace {
// the warp kernel is built for rotary_dim 64 (RoPE partners 32 dims apart, in one lane)
bool rot_ok_for_warp_kernel(int64_t rot) { return rot == 64; }
}  // namespace

int q35_qgkv_rope_positions_launch(const void* packed, const void* q_weight, const void* k_weight,
                                   const float* inv_freq, void* q_out, void* k_out, void* v_out,
                                   const int64_t* cache_start, int64_t batch, int64_t seq_len, int64_t q_heads,
                                   int64_t kv_heads, int64_t rotary_dim, int64_t kv_len, float eps,
                                   cudaStream_t stream, const int64_t* pos3, int sec_h, int sec_w, bool pdl,
                                   void* vt_out, int64_t vt_stride) {
  if (rot_ok_for_warp_kernel(rotary_dim)) {
    const int64_t pairs = batch * seq_len * (q_heads + kv_heads);
    const cudaError_t e = q35_launch(
        qgkv_rope_warp_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0, stream, pdl, (const bf16*)packed,
        (const bf16*)q_weight, (const bf16*)k_weight, inv_freq, (bf16*)q_out, (bf16*)k_out, (bf16*)v_out, cache_start,
        (int)batch, (int)seq_len, (int)q_heads, (int)kv_heads, (int)rotary_dim, (int)kv_len, eps, pos3, sec_h, sec_w,
        (bf16*)vt_out, (int)vt_stride);
    if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "qgkv_rope_positions launch: %s", cudaGetErrorString(e));
    return Q35_OK;
  }
  const cudaError_t e = q35_launch(
      qgkv_rope_kernel<false>, dim3((unsigned)(batch * seq_len)), dim3(kD), 0, stream, pdl, (const bf16*)packed,
      (const bf16*)q_weight, (const bf16*)k_weight, (const bf16*)nullptr, (const bf16*)nullptr, inv_freq, (int64_t)0,
      (bf16*)q_out, (bf16*)k_out, (bf16*)v_out, cache_start, (int)seq_len, (int)q_heads, (int)kv_heads,
      (int)rotary_dim, (int)kv_len, eps, pos3, sec_h, sec_w, (bf16*)vt_out, (int)vt_stride);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "qgkv_rope_positions launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

int q35_prefill_attention_launch(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                 int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len, int64_t q_offset,
                                 int64_t head_dim, float scale, cudaStream_t stream, bool pdl);

extern "C" int q35_prefill_attention(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                     int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len,
                                     int64_t q_offset, int64_t head_dim, float scale, void* stream) {
  return q35_prefill_attention_launch(q, k, v, out, batch, q_heads, kv_heads, seq_len, kv_len, q_offset, head_dim,
                                      scale, (cudaStream_t)stream, false);
}

// The causal prefill attention of the decoder (optionally chained with programmatic dependent
// launch): the argument checks and kernel choice of q35_prefill_attention.
int q35_prefill_attention_launch(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                 int64_t q_heads, int64_t kv_heads, int64_t seq_len, int64_t kv_len, int64_t q_offset,
                                 int64_t head_dim, float scale, cudaStream_t stream, bool pdl) {
  Q35_REQUIRE(q && k && v && out, "prefill_attention: null pointer");
  Q35_REQUIRE(head_dim == kD, "prefill_attention: head dim must be 256");
  Q35_REQUIRE(batch >= 0 && seq_len >= 0 && kv_heads >= 1 && q_heads % kv_heads == 0 && q_offset >= 0 &&
                  kv_len >= q_offset + seq_len,
              "prefill_attention: bad shape");
  if (batch * seq_len == 0) return Q35_OK;
  // tensor-core kernel for every group size: a group of G query heads per KV head runs as
  // G / G' CTA groups of G' = 4, 2 or 1 heads (the largest that divides G), sharing the KV head
  const int64_t group = q_heads / kv_heads;
  if (group % 4 == 0)
    return launch_prefill_mma<4>(q, k, v, out, batch, q_heads, kv_heads, seq_len, kv_len, q_offset, scale, stream,
                                 pdl);
  if (group % 2 == 0)
    return launch_prefill_mma<2>(q, k, v, out, batch, q_heads, kv_heads, seq_len, kv_len, q_offset, scale, stream,
                                 pdl);
  return launch_prefill_mma<1>(q, k, v, out, batch, q_heads, kv_heads, seq_len, kv_len, q_offset, scale, stream,
                               pdl);
}
