// Row norms and elementwise activations (reference: qwen35_fused/kernels.py:24-333).
//
// One CTA per row for the 2048-wide norms (the reduction stays on chip, 16-byte chunks at width
// 2048); one warp per row for the 128-wide gated norm (8-byte chunks) and for the 256-1024-wide
// norms (16-byte chunks); 16-byte vector loops for the elementwise ops. Scalar kernels cover
// widths that are not multiples of 8 and unaligned tensors.
#include "common.cuh"

using namespace q35;

namespace {

constexpr int kRowThreads = 256;

// rows x width RMSNorm(1+w), optional residual add first (kernels.py:24-112).
template <bool ADD>
__global__ void __launch_bounds__(kRowThreads) rms_rows_kernel(const bf16* __restrict__ x,
                                                               const bf16* __restrict__ upd,
                                                               const bf16* __restrict__ w,
                                                               bf16* __restrict__ resid_out,
                                                               bf16* __restrict__ out, int width,
                                                               float eps) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * width;
  const bf16* ur = ADD ? upd + row * width : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x; c < width; c += kRowThreads) {
    float v = bf2f(xr[c]);
    if (ADD) {
      v = rbf(v + bf2f(ur[c]));
      resid_out[row * width + c] = f2bf(v);
    }
    ss += v * v;
  }
  const float var = block_sum<kRowThreads / 32>(ss, red) / (float)width;
  const float r = rsqrt_ieee(var + eps);
  for (int c = threadIdx.x; c < width; c += kRowThreads) {
    float v = bf2f(xr[c]);
    if (ADD) v = rbf(v + bf2f(ur[c]));
    out[row * width + c] = f2bf(v * r * (1.0f + bf2f(w[c])));
  }
}

// Width 2048: one 16-byte chunk per thread, x read once and kept in registers; the per-thread
// partial sums run over 8 consecutive elements, as in the decode GEMVs' RMSNorm prologue, so the
// prefill and decode norms of a row are bit-identical.
template <bool ADD>
__global__ void __launch_bounds__(kRowThreads) rms_rows2048_kernel(const bf16* __restrict__ x,
                                                                   const bf16* __restrict__ upd,
                                                                   const bf16* __restrict__ w,
                                                                   bf16* __restrict__ resid_out,
                                                                   bf16* __restrict__ out, float eps) {
  constexpr int kW = 2048;
  // the norm weights are constants: loaded before the wait, not after the block reduction
  const uint4 wraw = *reinterpret_cast<const uint4*>(w + 8 * threadIdx.x);
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  __shared__ float red[kRowThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kW + 8 * threadIdx.x;
  float f[8];
  unpack_bf16x8(*reinterpret_cast<const uint4*>(x + base), f);
  if (ADD) {
    float u[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(upd + base), u);
    __align__(16) bf16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      f[j] = rbf(f[j] + u[j]);
      o[j] = f2bf(f[j]);
    }
    *reinterpret_cast<uint4*>(resid_out + base) = *reinterpret_cast<const uint4*>(o);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  const float r = rsqrt_ieee(block_sum<kRowThreads / 32>(ss, red) / (float)kW + eps);
  float wv[8];
  unpack_bf16x8(wraw, wv);
  __align__(16) bf16 o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = f2bf(f[j] * r * (1.0f + wv[j]));
  *reinterpret_cast<uint4*>(out + base) = *reinterpret_cast<const uint4*>(o);
}

// Width 128 (the DeltaNet head): one warp per row, four consecutive values per lane in 8-byte
// loads and stores, x read once.
__global__ void gated_rms128_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate,
                                    const bf16* __restrict__ w, bf16* __restrict__ out, int64_t rows, float eps,
                                    int gate_group, int64_t gate_stride) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  constexpr int kW = 128;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  auto unpack4 = [](uint2 v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xFFFF0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xFFFF0000u);
  };
  float xf[4], gf[4], wf[4];
  unpack4(*reinterpret_cast<const uint2*>(x + row * kW + 4 * lane), xf);
  unpack4(*reinterpret_cast<const uint2*>(gate + (row / gate_group) * gate_stride + (row % gate_group) * kW + 4 * lane),
          gf);
  unpack4(*reinterpret_cast<const uint2*>(w + 4 * lane), wf);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss += xf[j] * xf[j];
  const float r = rsqrt_ieee(warp_sum(ss) / (float)kW + eps);
  __align__(8) bf16 o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float nrm = rbf(xf[j] * r);
    const float wt = rbf(nrm * wf[j]);
    o[j] = f2bf(wt * silu_f(gf[j]));
  }
  *reinterpret_cast<uint2*>(out + row * kW + 4 * lane) = *reinterpret_cast<const uint2*>(o);
}

// One warp per row: bf16(bf16(bf16(norm(x)) * w) * silu(gate)) (kernels.py:115-155).
// Gate row r starts at gate + (r / gate_group) * gate_stride + (r % gate_group) * width, so the z
// block of a packed projection ([L, rows] with `gate_group` heads per token) is read in place.
__global__ void gated_rms_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate,
                                 const bf16* __restrict__ w, bf16* __restrict__ out, int64_t rows,
                                 int width, float eps, int gate_group, int64_t gate_stride) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* xr = x + row * width;
  const bf16* gr = gate + (row / gate_group) * gate_stride + (row % gate_group) * width;
  float ss = 0.f;
  for (int c = lane; c < width; c += 32) {
    float v = bf2f(xr[c]);
    ss += v * v;
  }
  const float r = rsqrt_ieee(warp_sum(ss) / (float)width + eps);
  for (int c = lane; c < width; c += 32) {
    const float nrm = rbf(bf2f(xr[c]) * r);
    const float wt = rbf(nrm * bf2f(w[c]));
    out[row * width + c] = f2bf(wt * silu_f(bf2f(gr[c])));
  }
}

// ---- 16-byte vector forms (8 bf16 per thread per step); the scalar kernels above and below
// remain for widths that are not multiples of 8 or unaligned tensors.
Q35_DEV uint4 pack_bf16x8(const float (&f)[8]) {
  return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}

// RMSNorm(1+w) of rows of width 256 * CPL, one warp per row, CPL 16-byte chunks per lane.
template <bool ADD, int CPL>
__global__ void __launch_bounds__(256) rms_rows_warp_kernel(const bf16* __restrict__ x, const bf16* __restrict__ upd,
                                                            const bf16* __restrict__ w, bf16* __restrict__ resid_out,
                                                            bf16* __restrict__ out, int64_t rows, float eps) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  constexpr int W = 256 * CPL;
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * 8) {
    float f[CPL][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int64_t off = row * W + 8 * (lane + 32 * c);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(x + off), f[c]);
      if (ADD) {
        float u[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(upd + off), u);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[c][j] = rbf(f[c][j] + u[j]);
        *reinterpret_cast<uint4*>(resid_out + off) = pack_bf16x8(f[c]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[c][j] * f[c][j];
    }
    const float r = rsqrt_ieee(warp_sum(ss) / (float)W + eps);
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float wv[8], o[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(w + 8 * (lane + 32 * c)), wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = f[c][j] * r * (1.0f + wv[j]);
      *reinterpret_cast<uint4*>(out + row * W + 8 * (lane + 32 * c)) = pack_bf16x8(o);
    }
  }
}

// Gated RMSNorm of rows of width 256 * CPL, one warp per row (same rounding points as
// gated_rms_kernel).
template <int CPL>
__global__ void __launch_bounds__(256) gated_rms_warp_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate,
                                                             const bf16* __restrict__ w, bf16* __restrict__ out,
                                                             int64_t rows, float eps, int gate_group,
                                                             int64_t gate_stride) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  constexpr int W = 256 * CPL;
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * 8) {
    const bf16* gr = gate + (row / gate_group) * gate_stride + (row % gate_group) * W;
    float f[CPL][8], g[CPL][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(x + row * W + 8 * (lane + 32 * c)), f[c]);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(gr + 8 * (lane + 32 * c)), g[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[c][j] * f[c][j];
    }
    const float r = rsqrt_ieee(warp_sum(ss) / (float)W + eps);
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float wv[8], o[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(w + 8 * (lane + 32 * c)), wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float nrm = rbf(f[c][j] * r);
        const float wt = rbf(nrm * wv[j]);
        o[j] = wt * silu_f(g[c][j]);
      }
      *reinterpret_cast<uint4*>(out + row * W + 8 * (lane + 32 * c)) = pack_bf16x8(o);
    }
  }
}

// silu(gate) * up over [rows, 2 * width] -> [rows, width], width % 8 == 0; one CTA per row in a
// row-stride loop, 16-byte chunks.
__global__ void __launch_bounds__(256) silu_mul_v8_kernel(const bf16* __restrict__ packed, bf16* __restrict__ out,
                                                          int64_t rows, int width) {
  const int n8 = width / 8;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const bf16* pr = packed + r * 2 * width;
    for (int c = threadIdx.x; c < n8; c += blockDim.x) {
      float gf[8], uf[8], o[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(pr + 8 * c), gf);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(pr + width + 8 * c), uf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rbf(silu_f(gf[j])) * uf[j];
      *reinterpret_cast<uint4*>(out + r * width + 8 * c) = pack_bf16x8(o);
    }
  }
}

// x * sigmoid(gate) over n8 16-byte chunks.
__global__ void __launch_bounds__(256) sigmoid_mul_v8_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate,
                                                             bf16* __restrict__ out, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float xf[8], gf[8], o[8];
    unpack_bf16x8(reinterpret_cast<const uint4*>(x)[i], xf);
    unpack_bf16x8(reinterpret_cast<const uint4*>(gate)[i], gf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = xf[j] * rbf(sigmoid_f(gf[j]));
    reinterpret_cast<uint4*>(out)[i] = pack_bf16x8(o);
  }
}

// Attention output gate (the gate block of each head inside the packed QGKV row), 16-byte chunks;
// head_dim % 8 == 0 so a chunk never straddles two heads.
__global__ void __launch_bounds__(256) attn_gate_v8_kernel(const bf16* __restrict__ x, const bf16* __restrict__ packed,
                                                           bf16* __restrict__ out, int64_t rows, int hidden,
                                                           int64_t stride, int head_dim) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  const int n8 = hidden / 8;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    for (int c = threadIdx.x; c < n8; c += blockDim.x) {
      const int col = 8 * c, h = col / head_dim, d = col - h * head_dim;
      float xf[8], gf[8], o[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(x + r * hidden + col), xf);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(packed + r * stride + (int64_t)h * 2 * head_dim + head_dim + d), gf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = xf[j] * rbf(sigmoid_f(gf[j]));
      *reinterpret_cast<uint4*>(out + r * hidden + col) = pack_bf16x8(o);
    }
  }
}

__global__ void silu_mul_kernel(const bf16* __restrict__ packed, bf16* __restrict__ out,
                                int64_t rows, int64_t width) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    const float g = bf2f(packed[r * 2 * width + c]);
    const float u = bf2f(packed[r * 2 * width + width + c]);
    out[i] = f2bf(rbf(silu_f(g)) * u);
  }
}

__global__ void sigmoid_mul_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate,
                                   bf16* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f2bf(bf2f(x[i]) * rbf(sigmoid_f(bf2f(gate[i]))));
}

__global__ void attn_gate_kernel(const bf16* __restrict__ x, const bf16* __restrict__ packed,
                                 bf16* __restrict__ out, int64_t rows, int64_t hidden,
                                 int64_t stride, int64_t head_dim) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  const int64_t total = rows * hidden;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / hidden, c = i - r * hidden;
    const int64_t h = c / head_dim, d = c - h * head_dim;
    const float g = bf2f(packed[r * stride + h * 2 * head_dim + head_dim + d]);
    out[i] = f2bf(bf2f(x[i]) * rbf(sigmoid_f(g)));
  }
}

__global__ void embedding_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int64_t n, int64_t vocab, int64_t width) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  int64_t id = ids[row];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);  // clamp: never read outside the table
  const uint4* src = reinterpret_cast<const uint4*>(table + id * width);
  uint4* dst = reinterpret_cast<uint4*>(out + row * width);
  for (int64_t c = threadIdx.x; c < width / 8; c += blockDim.x) dst[c] = src[c];
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 8 * kNumSMs) g = 8 * kNumSMs;
  return (int)(g < 1 ? 1 : g);
}

// Widths the warp-per-row norms cover: 256, 512 or 1024 (1, 2 or 4 chunks per lane).
bool warp_rows_ok(int64_t width) { return width == 256 || width == 512 || width == 1024; }

unsigned warp_rows_grid(int64_t rows) {
  const int64_t g = (rows + 7) / 8;  // eight rows (warps) per CTA
  return (unsigned)(g < 8 * kNumSMs ? g : 8 * kNumSMs);
}

template <bool ADD>
void launch_rms_warp(const bf16* x, const bf16* upd, const bf16* w, bf16* resid_out, bf16* out, int64_t rows,
                     int64_t width, float eps, cudaStream_t s) {
  const unsigned grid = warp_rows_grid(rows);
  if (width == 256)
    rms_rows_warp_kernel<ADD, 1><<<grid, 256, 0, s>>>(x, upd, w, resid_out, out, rows, eps);
  else if (width == 512)
    rms_rows_warp_kernel<ADD, 2><<<grid, 256, 0, s>>>(x, upd, w, resid_out, out, rows, eps);
  else
    rms_rows_warp_kernel<ADD, 4><<<grid, 256, 0, s>>>(x, upd, w, resid_out, out, rows, eps);
}

void launch_gated_warp(const bf16* x, const bf16* gate, const bf16* w, bf16* out, int64_t rows, int64_t width,
                       float eps, int gate_group, int64_t gate_stride, cudaStream_t s) {
  const unsigned grid = warp_rows_grid(rows);
  if (width == 256)
    gated_rms_warp_kernel<1><<<grid, 256, 0, s>>>(x, gate, w, out, rows, eps, gate_group, gate_stride);
  else if (width == 512)
    gated_rms_warp_kernel<2><<<grid, 256, 0, s>>>(x, gate, w, out, rows, eps, gate_group, gate_stride);
  else
    gated_rms_warp_kernel<4><<<grid, 256, 0, s>>>(x, gate, w, out, rows, eps, gate_group, gate_stride);
}

}  // namespace

int q35_rms_norm_launch(const void* x, const void* weight, void* out, int64_t rows, int64_t width, float eps,
                        cudaStream_t stream, bool pdl);

extern "C" int q35_rms_norm(const void* x, const void* weight, void* out, int64_t rows,
                            int64_t width, float eps, void* stream) {
  return q35_rms_norm_launch(x, weight, out, rows, width, eps, (cudaStream_t)stream, false);
}

// q35_rms_norm, optionally chained with programmatic dependent launch (the width-2048 kernel).
int q35_rms_norm_launch(const void* x, const void* weight, void* out, int64_t rows, int64_t width, float eps,
                        cudaStream_t stream, bool pdl) {
  Q35_REQUIRE(x && weight && out, "rms_norm: null pointer");
  Q35_REQUIRE(rows >= 0 && width > 0 && width <= 65536, "rms_norm: bad shape rows=%lld width=%lld",
              (long long)rows, (long long)width);
  if (rows == 0) return Q35_OK;
  if (width == 2048 && Q35_ALIGNED(x, 16) && Q35_ALIGNED(weight, 16) && Q35_ALIGNED(out, 16)) {
    const cudaError_t e = q35_launch(rms_rows2048_kernel<false>, dim3((unsigned)rows), dim3(kRowThreads), 0, stream,
                                     pdl, (const bf16*)x, (const bf16*)nullptr, (const bf16*)weight, (bf16*)nullptr,
                                     (bf16*)out, eps);
    if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "rms_norm launch: %s", cudaGetErrorString(e));
    return Q35_OK;
  } else if (warp_rows_ok(width) && Q35_ALIGNED(x, 16) && Q35_ALIGNED(weight, 16) && Q35_ALIGNED(out, 16))
    launch_rms_warp<false>((const bf16*)x, nullptr, (const bf16*)weight, nullptr, (bf16*)out, rows, width, eps,
                           (cudaStream_t)stream);
  else
    rms_rows_kernel<false><<<(unsigned)rows, kRowThreads, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, nullptr, (const bf16*)weight, nullptr, (bf16*)out, (int)width, eps);
  return q35_check_launch("rms_norm");
}

extern "C" int q35_residual_add_rms_norm(const void* residual, const void* update,
                                         const void* weight, void* residual_out, void* norm_out,
                                         int64_t rows, int64_t width, float eps, void* stream) {
  Q35_REQUIRE(residual && update && weight && residual_out && norm_out,
              "residual_add_rms_norm: null pointer");
  Q35_REQUIRE(rows >= 0 && width > 0 && width <= 65536, "residual_add_rms_norm: bad shape");
  if (rows == 0) return Q35_OK;
  if (width == 2048 && Q35_ALIGNED(residual, 16) && Q35_ALIGNED(update, 16) && Q35_ALIGNED(weight, 16) &&
      Q35_ALIGNED(residual_out, 16) && Q35_ALIGNED(norm_out, 16))
    rms_rows2048_kernel<true><<<(unsigned)rows, kRowThreads, 0, (cudaStream_t)stream>>>(
        (const bf16*)residual, (const bf16*)update, (const bf16*)weight, (bf16*)residual_out, (bf16*)norm_out,
        eps);
  else if (warp_rows_ok(width) && Q35_ALIGNED(residual, 16) && Q35_ALIGNED(update, 16) && Q35_ALIGNED(weight, 16) &&
           Q35_ALIGNED(residual_out, 16) && Q35_ALIGNED(norm_out, 16))
    launch_rms_warp<true>((const bf16*)residual, (const bf16*)update, (const bf16*)weight, (bf16*)residual_out,
                          (bf16*)norm_out, rows, width, eps, (cudaStream_t)stream);
  else
    rms_rows_kernel<true><<<(unsigned)rows, kRowThreads, 0, (cudaStream_t)stream>>>(
        (const bf16*)residual, (const bf16*)update, (const bf16*)weight, (bf16*)residual_out,
        (bf16*)norm_out, (int)width, eps);
  return q35_check_launch("residual_add_rms_norm");
}

int q35_gated_rms_strided_launch(const void* x, const void* gate, int gate_group, int64_t gate_stride,
                                 const void* weight, void* out, int64_t rows, int64_t width, float eps,
                                 cudaStream_t stream, bool pdl = false);

extern "C" int q35_gated_rms_norm(const void* x, const void* gate, const void* weight, void* out,
                                  int64_t rows, int64_t width, float eps, void* stream) {
  Q35_REQUIRE(x && gate && weight && out, "gated_rms_norm: null pointer");
  Q35_REQUIRE(rows >= 0 && width > 0, "gated_rms_norm: bad shape");
  return q35_gated_rms_strided_launch(x, gate, 1, width, weight, out, rows, width, eps, (cudaStream_t)stream);
}

int q35_gated_rms_strided_launch(const void* x, const void* gate, int gate_group, int64_t gate_stride,
                                 const void* weight, void* out, int64_t rows, int64_t width, float eps,
                                 cudaStream_t stream, bool pdl) {
  if (rows == 0) return Q35_OK;
  const int rows_per_block = 8;
  const unsigned blocks = (unsigned)((rows + rows_per_block - 1) / rows_per_block);
  if (width == 128 && gate_stride % 4 == 0 && Q35_ALIGNED(x, 8) && Q35_ALIGNED(gate, 8) && Q35_ALIGNED(weight, 8) &&
      Q35_ALIGNED(out, 8)) {
    const cudaError_t e = q35_launch(gated_rms128_kernel, dim3(blocks), dim3(32 * rows_per_block), 0, stream, pdl,
                                     (const bf16*)x, (const bf16*)gate, (const bf16*)weight, (bf16*)out, rows, eps,
                                     gate_group, gate_stride);
    if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gated_rms launch: %s", cudaGetErrorString(e));
    return Q35_OK;
  } else if (warp_rows_ok(width) && gate_stride % 8 == 0 && Q35_ALIGNED(x, 16) && Q35_ALIGNED(gate, 16) &&
           Q35_ALIGNED(weight, 16) && Q35_ALIGNED(out, 16))
    launch_gated_warp((const bf16*)x, (const bf16*)gate, (const bf16*)weight, (bf16*)out, rows, width, eps,
                      gate_group, gate_stride, stream);
  else
    gated_rms_kernel<<<blocks, 32 * rows_per_block, 0, stream>>>((const bf16*)x, (const bf16*)gate,
                                                                 (const bf16*)weight, (bf16*)out, rows,
                                                                 (int)width, eps, gate_group, gate_stride);
  return q35_check_launch("gated_rms_strided");
}

__global__ void set_counters_kernel(int64_t* a, int64_t* b, int64_t value) {
  pdl_wait();  // programmatic dependent launch: inputs only after the previous kernel
  pdl_launch_dependents();
  if (a) *a = value;
  if (b) *b = value;
}

int q35_set_counters_launch(int64_t* a, int64_t* b, int64_t value, cudaStream_t stream, bool pdl) {
  const cudaError_t e = q35_launch(set_counters_kernel, dim3(1), dim3(1), 0, stream, pdl, a, b, value);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "set_counters launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_silu_and_mul(const void* packed, void* out, int64_t rows, int64_t width,
                                void* stream) {
  Q35_REQUIRE(packed && out && rows >= 0 && width > 0, "silu_and_mul: bad argument");
  if (rows == 0) return Q35_OK;
  if (width % 8 == 0 && width <= (1 << 30) && Q35_ALIGNED(packed, 16) && Q35_ALIGNED(out, 16))
    silu_mul_v8_kernel<<<(unsigned)(rows < 8 * kNumSMs ? rows : 8 * kNumSMs), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)packed, (bf16*)out, rows, (int)width);
  else
    silu_mul_kernel<<<grid_for(rows * width, 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)packed, (bf16*)out, rows, width);
  return q35_check_launch("silu_and_mul");
}

extern "C" int q35_sigmoid_mul(const void* x, const void* gate, void* out, int64_t n,
                               void* stream) {
  Q35_REQUIRE(x && gate && out && n >= 0, "sigmoid_mul: bad argument");
  if (n == 0) return Q35_OK;
  if (n % 8 == 0 && Q35_ALIGNED(x, 16) && Q35_ALIGNED(gate, 16) && Q35_ALIGNED(out, 16))
    sigmoid_mul_v8_kernel<<<grid_for(n / 8, 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)gate, (bf16*)out, n / 8);
  else
    sigmoid_mul_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)gate, (bf16*)out, n);
  return q35_check_launch("sigmoid_mul");
}

int q35_attention_gate_launch(const void* x, const void* packed, void* out, int64_t rows, int64_t hidden,
                              int64_t packed_stride, int64_t head_dim, cudaStream_t stream, bool pdl);

extern "C" int q35_attention_gate_mul(const void* x, const void* packed, void* out, int64_t rows,
                                      int64_t hidden, int64_t packed_stride, int64_t head_dim,
                                      void* stream) {
  return q35_attention_gate_launch(x, packed, out, rows, hidden, packed_stride, head_dim, (cudaStream_t)stream,
                                   false);
}

// q35_attention_gate_mul, optionally chained with programmatic dependent launch (16-byte kernel).
int q35_attention_gate_launch(const void* x, const void* packed, void* out, int64_t rows, int64_t hidden,
                              int64_t packed_stride, int64_t head_dim, cudaStream_t stream, bool pdl) {
  Q35_REQUIRE(x && packed && out, "attention_gate_mul: null pointer");
  Q35_REQUIRE(rows >= 0 && head_dim > 0 && hidden % head_dim == 0 && packed_stride >= 2 * hidden,
              "attention_gate_mul: bad shape");
  if (rows == 0) return Q35_OK;
  if (hidden % 8 == 0 && head_dim % 8 == 0 && packed_stride % 8 == 0 && hidden <= (1 << 30) &&
      Q35_ALIGNED(x, 16) && Q35_ALIGNED(packed, 16) && Q35_ALIGNED(out, 16)) {
    const cudaError_t e = q35_launch(attn_gate_v8_kernel, dim3((unsigned)(rows < 8 * kNumSMs ? rows : 8 * kNumSMs)),
                                     dim3(256), 0, stream, pdl, (const bf16*)x, (const bf16*)packed, (bf16*)out, rows,
                                     (int)hidden, packed_stride, (int)head_dim);
    if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "attention_gate launch: %s", cudaGetErrorString(e));
    return Q35_OK;
  } else
    attn_gate_kernel<<<grid_for(rows * hidden, 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)packed, (bf16*)out, rows, hidden, packed_stride, head_dim);
  return q35_check_launch("attention_gate_mul");
}

int q35_embedding_launch(const int64_t* ids, const void* table, void* out, int64_t n, int64_t vocab, int64_t width,
                         cudaStream_t stream, bool pdl) {
  Q35_REQUIRE(ids && table && out && n >= 0 && vocab > 0 && width % 8 == 0,
              "embedding: bad argument");
  Q35_REQUIRE(Q35_ALIGNED(table, 16) && Q35_ALIGNED(out, 16), "embedding: 16-byte alignment");
  if (n == 0) return Q35_OK;
  const cudaError_t e = q35_launch(embedding_kernel, dim3((unsigned)n), dim3(128), 0, stream, pdl, ids,
                                   (const bf16*)table, (bf16*)out, n, vocab, width);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "embedding launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" int q35_embedding(const int64_t* ids, const void* table, void* out, int64_t n,
                             int64_t vocab, int64_t width, void* stream) {
  return q35_embedding_launch(ids, table, out, n, vocab, width, (cudaStream_t)stream, false);
}
