// Prefill projections C = A [M,K] . W [N,K]^T (reference: F.linear on the packed weights,
// integration.py:183, 245, 298; down/out/o proj :185, 272, 359) and the A8W8 int8 GEMM
// (explore_runtime_quantization.py:161-181).
//
// Tiles of 128 x 128 with a 64-byte K slab per stage (32 bf16 or 64 int8), 3-stage cp.async
// pipeline, ldmatrix fragments and warp-level MMA (bf16 -> fp32, or s8 -> exact s32).
// Epilogue through shared memory so that SwiGLU pairs and residual adds are row-coalesced:
//  STORE    out[m, n] = bf16(y)
//  RESIDUAL resid[m, n] = bf16(resid + bf16(y))
//  SWIGLU   tile columns interleave 16 gate / 16 up rows of W (rows n and n + N) -> 64 outputs
//  RAW_I32  acc[m, n] = exact int32 sum (int8 only)
// For int8 the dequantised value is y = (float(acc) * s_x[m]) * s_w[n].
#include "common.cuh"

using namespace q35;

namespace {

constexpr int BM = 128, BN = 128, BKB = 64;  // tile M, tile N (W rows), K bytes per stage
constexpr int kStages = 3;
constexpr int kPitch = BKB + 16;             // padded smem row pitch in bytes (80): ldmatrix conflict-free
constexpr int kGemmThreads = 256;
constexpr int EPI_RAW_I32 = 3;

struct GemmParams {
  const void* a;        // [M, K] bf16 or int8
  const void* w;        // [Nw, K]
  void* out;            // bf16 [M, Nout] or int32 (RAW)
  bf16* resid;          // RESIDUAL target [M, Nout]
  const float* sx;      // int8: per-row activation scale [M]
  const float* sw;      // int8: per-row weight scale [Nw]
  int M, N, K;          // N = output columns (SwiGLU: W has 2N rows)
};

Q35_DEV void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes) : "memory");
}
Q35_DEV void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
Q35_DEV void wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

Q35_DEV void ldmatrix_x4(unsigned r[4], const void* p) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

template <bool INT8>
Q35_DEV void mma(float c[4], const unsigned a[4], const unsigned b[2]);

template <>
Q35_DEV void mma<false>(float c[4], const unsigned a[4], const unsigned b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
Q35_DEV void mma<true>(float c[4], const unsigned a[4], const unsigned b[2]) {
  int* ci = reinterpret_cast<int*>(c);
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(ci[0]), "+r"(ci[1]), "+r"(ci[2]), "+r"(ci[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// W row feeding tile column j of output tile n0 (SwiGLU interleaves 16 gate / 16 up rows).
template <int EPI>
Q35_DEV int w_row_of(int n_tile0, int j, int N) {
  if (EPI == Q35_EPI_SWIGLU) {
    const int grp = j >> 5, within = j & 31;
    const int out_col = n_tile0 / 2 + grp * 16 + (within & 15);
    return within < 16 ? out_col : N + out_col;
  }
  return n_tile0 + j;
}

template <bool INT8, int EPI>
__global__ void __launch_bounds__(kGemmThreads) gemm_kernel(GemmParams p) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* As = smem;                           // [stages][BM][kPitch]
  unsigned char* Bs = smem + kStages * BM * kPitch;   // [stages][BN][kPitch]
  const int ES = INT8 ? 1 : 2;
  const int m0 = blockIdx.y * BM;
  const int n_tile0 = blockIdx.x * BN;                // position in the (interleaved) W-row space
  const int Nw = (EPI == Q35_EPI_SWIGLU) ? 2 * p.N : p.N;
  const int kbytes = p.K * ES;
  const int n_k = kbytes / BKB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps, warp tile 64 x 32
  const char* A = static_cast<const char*>(p.a);
  const char* W = static_cast<const char*>(p.w);

  auto load_stage = [&](int stage, int kt) {
    const int kb0 = kt * BKB;
    // A: 128 rows x 64 B = 512 x 16 B; W: same
    for (int i = threadIdx.x; i < BM * 4; i += kGemmThreads) {
      const int r = i >> 2, c = (i & 3) * 16;
      const int gm = m0 + r;
      const bool ok = gm < p.M;
      cp_async16_zfill(As + (stage * BM + r) * kPitch + c, A + (int64_t)(ok ? gm : 0) * kbytes + kb0 + c, ok);
    }
    for (int i = threadIdx.x; i < BN * 4; i += kGemmThreads) {
      const int r = i >> 2, c = (i & 3) * 16;
      const int j = n_tile0 + r;
      int wr = w_row_of<EPI>(n_tile0, r, p.N);
      bool ok = (EPI == Q35_EPI_SWIGLU) ? ((n_tile0 / 2 + (r >> 5) * 16 + (r & 15)) < p.N) : (j < Nw);
      cp_async16_zfill(Bs + (stage * BN + r) * kPitch + c, W + (int64_t)(ok ? wr : 0) * kbytes + kb0 + c, ok);
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < n_k) load_stage(s, s);
    commit();
  }
  for (int kt = 0; kt < n_k; ++kt) {
    wait_group<kStages - 2>();
    __syncthreads();
    const int nk = kt + kStages - 1;
    if (nk < n_k) load_stage(nk % kStages, nk);
    commit();
    const int st = kt % kStages;
    const unsigned char* a_st = As + st * BM * kPitch;
    const unsigned char* b_st = Bs + st * BN * kPitch;
#pragma unroll
    for (int ks = 0; ks < BKB; ks += 32) {  // 32 bytes of K per MMA (k16 bf16 / k32 int8)
      unsigned af[4][4], bfr[4][2];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int r = wm * 64 + mi * 16 + (lane & 15);
        const int c = ks + (lane >> 4) * 16;
        ldmatrix_x4(af[mi], a_st + r * kPitch + c);
      }
#pragma unroll
      for (int nj = 0; nj < 2; ++nj) {
        // x4 over two n8 tiles: matrices (n 0-7, k lo), (n 0-7, k hi), (n 8-15, k lo), (n 8-15, k hi)
        const int r = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks + ((lane >> 3) & 1) * 16;
        unsigned t[4];
        ldmatrix_x4(t, b_st + r * kPitch + c);
        bfr[nj * 2][0] = t[0];
        bfr[nj * 2][1] = t[1];
        bfr[nj * 2 + 1][0] = t[2];
        bfr[nj * 2 + 1][1] = t[3];
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) mma<INT8>(acc[mi][ni], af[mi], bfr[ni]);
    }
  }
  wait_group<0>();
  __syncthreads();

  // ---- epilogue through shared memory: tile [BM][BN] of bf16 (or int32/float for RAW)
  if (EPI == EPI_RAW_I32) {
    int* out = static_cast<int*>(p.out);
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = m0 + wm * 64 + mi * 16 + (lane >> 2) + (e >> 1) * 8;
          const int c = n_tile0 + wn * 32 + ni * 8 + (lane & 3) * 2 + (e & 1);
          if (r < p.M && c < p.N) out[(int64_t)r * p.N + c] = reinterpret_cast<int*>(acc[mi][ni])[e];
        }
    return;
  }
  bf16* tile = reinterpret_cast<bf16*>(smem);  // [BM][BN + 8]
  constexpr int TP = BN + 8;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = wm * 64 + mi * 16 + (lane >> 2) + (e >> 1) * 8;
        const int c = wn * 32 + ni * 8 + (lane & 3) * 2 + (e & 1);
        float y;
        if (INT8) {
          const int gm = m0 + r;
          const int wr = w_row_of<EPI>(n_tile0, c, p.N);
          const bool ok = gm < p.M && wr < Nw;
          const int a = reinterpret_cast<int*>(acc[mi][ni])[e];
          y = ok ? ((float)a * p.sx[gm]) * p.sw[wr] : 0.f;
        } else {
          y = acc[mi][ni][e];
        }
        tile[r * TP + c] = f2bf(y);
      }
  __syncthreads();
  if (EPI == Q35_EPI_SWIGLU) {
    const int ncols = BN / 2;  // 64 outputs per tile
    const int o0 = n_tile0 / 2;
    for (int i = threadIdx.x; i < BM * ncols; i += kGemmThreads) {
      const int r = i / ncols, oc = i % ncols;
      const int grp = oc >> 4, within = oc & 15;
      const int gm = m0 + r, gn = o0 + oc;
      if (gm >= p.M || gn >= p.N) continue;
      const float g = bf2f(tile[r * TP + grp * 32 + within]);
      const float u = bf2f(tile[r * TP + grp * 32 + 16 + within]);
      static_cast<bf16*>(p.out)[(int64_t)gm * p.N + gn] = f2bf(rbf(silu_f(g)) * u);
    }
  } else {
    for (int i = threadIdx.x; i < BM * BN; i += kGemmThreads) {
      const int r = i / BN, c = i % BN;
      const int gm = m0 + r, gn = n_tile0 + c;
      if (gm >= p.M || gn >= p.N) continue;
      const float y = bf2f(tile[r * TP + c]);
      if (EPI == Q35_EPI_RESIDUAL) {
        bf16* dst = p.resid + (int64_t)gm * p.N + gn;
        *dst = f2bf(bf2f(*dst) + y);
      } else {
        static_cast<bf16*>(p.out)[(int64_t)gm * p.N + gn] = f2bf(y);
      }
    }
  }
}

// Per-row symmetric int8 quantisation. TOK = false: the weight-side formula
// (explore_runtime_quantization.py:143-155); TOK = true: per-token activations with vllm
// scaled_int8_quant semantics (:167-172). See quant_i8 / quant_i8_tok.
template <bool TOK>
Q35_DEV int quant_code(float x, float s, float inv) {
  return TOK ? quant_i8_tok(x, inv) : quant_i8(x, s);
}

template <bool TOK>
__global__ void __launch_bounds__(256) quant_rows_kernel(const bf16* __restrict__ x, int8_t* __restrict__ q,
                                                         float* __restrict__ scale, int width) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * width;
  float amax = 0.f;
  for (int c = threadIdx.x; c < width; c += 256) amax = fmaxf(amax, fabsf(bf2f(xr[c])));
  amax = block_max<8>(amax, red);
  const float s = TOK ? tok_scale(amax) : (amax > 0.f ? amax / 127.0f : 1.0f);
  const float inv = tok_inv(amax);
  for (int c = threadIdx.x; c < width; c += 256) q[row * width + c] = (int8_t)quant_code<TOK>(bf2f(xr[c]), s, inv);
  if (threadIdx.x == 0) scale[row] = s;
}

// Width % 8 == 0, 16-byte aligned input and 8-byte aligned output: 16-byte loads, 8-byte int8
// stores; the second pass re-reads the row (4-12 KB, still in L1) instead of holding it.
template <bool TOK>
__global__ void __launch_bounds__(256) quant_rows_v8_kernel(const bf16* __restrict__ x, int8_t* __restrict__ q,
                                                            float* __restrict__ scale, int width) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * width);
  const int n8 = width / 8;
  float amax = 0.f;
  for (int c = threadIdx.x; c < n8; c += 256) {
    float f[8];
    unpack_bf16x8(xr[c], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  amax = block_max<8>(amax, red);
  const float s = TOK ? tok_scale(amax) : (amax > 0.f ? amax / 127.0f : 1.0f);
  const float inv = tok_inv(amax);
  for (int c = threadIdx.x; c < n8; c += 256) {
    float f[8];
    unpack_bf16x8(xr[c], f);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo |= (uint32_t)(quant_code<TOK>(f[j], s, inv) & 0xff) << (8 * j);
      hi |= (uint32_t)(quant_code<TOK>(f[4 + j], s, inv) & 0xff) << (8 * j);
    }
    reinterpret_cast<uint2*>(q + row * width)[c] = make_uint2(lo, hi);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

size_t gemm_smem() { return (size_t)kStages * (BM + BN) * kPitch; }

template <bool INT8, int EPI>
int launch_gemm(const GemmParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = gemm_smem();
  cudaFuncSetAttribute(gemm_kernel<INT8, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int nw_cols = (EPI == Q35_EPI_SWIGLU) ? 2 * p.N : p.N;
  dim3 grid((unsigned)((nw_cols + BN - 1) / BN), (unsigned)((p.M + BM - 1) / BM));
  const cudaError_t e = q35_launch(gemm_kernel<INT8, EPI>, grid, dim3(kGemmThreads), smem, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemm launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

template <bool INT8>
int dispatch_gemm(const GemmParams& p, int epi, cudaStream_t s, bool pdl) {
  switch (epi) {
    case Q35_EPI_STORE: return launch_gemm<INT8, Q35_EPI_STORE>(p, s, pdl);
    case Q35_EPI_RESIDUAL: return launch_gemm<INT8, Q35_EPI_RESIDUAL>(p, s, pdl);
    case Q35_EPI_SWIGLU: return launch_gemm<INT8, Q35_EPI_SWIGLU>(p, s, pdl);
    case EPI_RAW_I32:
      if (INT8) return launch_gemm<true, EPI_RAW_I32>(p, s, pdl);
  }
  return q35_fail(Q35_EINVAL, "gemm: bad epilogue %d", epi);
}

}  // namespace

int q35_gemm_launch(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k, int epi, bool int8,
                    const float* sx, const float* sw, cudaStream_t s, bool pdl) {
  Q35_REQUIRE(a && w && out, "gemm: null pointer");
  Q35_REQUIRE(m >= 0 && n > 0 && k > 0 && (k * (int8 ? 1 : 2)) % BKB == 0,
              "gemm: bad shape m=%lld n=%lld k=%lld (k bytes must be a multiple of 64)", (long long)m, (long long)n,
              (long long)k);
  Q35_REQUIRE(Q35_ALIGNED(a, 16) && Q35_ALIGNED(w, 16), "gemm: 16-byte alignment");
  Q35_REQUIRE(!int8 || epi == EPI_RAW_I32 || (sx && sw), "gemm: int8 needs scales");
  Q35_REQUIRE(epi != Q35_EPI_SWIGLU || n % 16 == 0, "gemm: SwiGLU width must be a multiple of 16");
  if (m == 0) return Q35_OK;
  GemmParams p;
  p.a = a;
  p.w = w;
  p.out = out;
  p.resid = static_cast<bf16*>(out);
  p.sx = sx;
  p.sw = sw;
  p.M = (int)m;
  p.N = (int)n;
  p.K = (int)k;
  return int8 ? dispatch_gemm<true>(p, epi, s, pdl) : dispatch_gemm<false>(p, epi, s, pdl);
}

template <bool TOK>
int quantize_launch(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width, cudaStream_t s, bool pdl) {
  if (rows == 0) return Q35_OK;
  const bool v8 = width % 8 == 0 && Q35_ALIGNED(x, 16) && Q35_ALIGNED(q, 8);
  const cudaError_t e = q35_launch(v8 ? quant_rows_v8_kernel<TOK> : quant_rows_kernel<TOK>, dim3((unsigned)rows),
                                   dim3(256), 0, s, pdl, (const bf16*)x, q, scale, (int)width);
  if (e != cudaSuccess)
    return q35_fail(Q35_ECUDA, "%s launch: %s", TOK ? "quantize_tokens" : "quantize_rows", cudaGetErrorString(e));
  return Q35_OK;
}

int q35_quantize_rows_launch(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width, cudaStream_t s) {
  return quantize_launch<false>(x, q, scale, rows, width, s, false);
}

int q35_quantize_tokens_launch(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                               cudaStream_t s, bool pdl) {
  return quantize_launch<true>(x, q, scale, rows, width, s, pdl);
}

extern "C" int q35_gemm_bf16(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k,
                             int32_t epilogue, void* stream) {
  Q35_REQUIRE(epilogue >= Q35_EPI_STORE && epilogue <= Q35_EPI_SWIGLU, "gemm_bf16: bad epilogue");
  return q35_gemm_launch(a, w, out, m, n, k, epilogue, false, nullptr, nullptr, (cudaStream_t)stream, false);
}

extern "C" int q35_quantize_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                                 void* stream) {
  Q35_REQUIRE(x && q && scale && rows >= 0 && width > 0, "quantize_rows: bad argument");
  return q35_quantize_rows_launch(x, q, scale, rows, width, (cudaStream_t)stream);
}

extern "C" int q35_quantize_tokens(const void* x, int8_t* q, float* scale, int64_t rows, int64_t width,
                                   void* stream) {
  Q35_REQUIRE(x && q && scale && rows >= 0 && width > 0, "quantize_tokens: bad argument");
  return q35_quantize_tokens_launch(x, q, scale, rows, width, (cudaStream_t)stream, false);
}

extern "C" size_t q35_a8w8_linear_workspace_size(int64_t m, int64_t k) {
  return (((size_t)m * k + 255) & ~(size_t)255) + (size_t)m * sizeof(float);
}

extern "C" int q35_a8w8_linear(const void* x, const int8_t* qw, const float* w_scale, void* out, int64_t m,
                               int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  Q35_REQUIRE(x && qw && w_scale && out && workspace, "a8w8_linear: null pointer");
  Q35_REQUIRE(k % 64 == 0 && n > 0 && m >= 0, "a8w8_linear: in/out features must be multiples of 64 / positive");
  Q35_REQUIRE(workspace_bytes >= q35_a8w8_linear_workspace_size(m, k), "a8w8_linear: workspace too small");
  int8_t* qx = static_cast<int8_t*>(workspace);
  float* sx = reinterpret_cast<float*>(static_cast<char*>(workspace) + (((size_t)m * k + 255) & ~(size_t)255));
  int rc = q35_quantize_tokens_launch(x, qx, sx, m, k, (cudaStream_t)stream, false);
  if (rc) return rc;
  return q35_gemm_launch(qx, qw, out, m, n, k, Q35_EPI_STORE, true, sx, w_scale, (cudaStream_t)stream, false);
}

extern "C" int q35_int8_gemm_i32(const int8_t* qx, const int8_t* qw, int32_t* acc, int64_t m, int64_t n, int64_t k,
                                 void* stream) {
  return q35_gemm_launch(qx, qw, acc, m, n, k, EPI_RAW_I32, true, nullptr, nullptr, (cudaStream_t)stream, false);
}
