// Shared device helpers for the Qwen3.5 sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "qwen35_b200.h"

#define Q35_DEV __device__ __forceinline__

typedef __nv_bfloat16 bf16;

namespace q35 {

constexpr int kNumSMs = 148;

Q35_DEV float bf2f(bf16 x) { return __bfloat162float(x); }
Q35_DEV bf16 f2bf(float x) { return __float2bfloat16_rn(x); }
Q35_DEV float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// SiLU / sigmoid exactly as the reference kernels write them (kernels.py:135, 166, 272).
Q35_DEV float silu_f(float x) { return x / (1.0f + expf(-x)); }
Q35_DEV float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
// GELU of the vision tower: the tanh form ("gelu_pytorch_tanh", the ViT MLP) and the erf form
// (nn.GELU(), the patch merger), as torch writes them: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715
// x^3))) and 0.5 x (1 + erf(x / sqrt(2))).
Q35_DEV float gelu_tanh_f(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}
Q35_DEV float gelu_erf_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }
// IEEE square root and division (no approximate rsqrt), closest to torch.rsqrt on the CPU.
Q35_DEV float rsqrt_ieee(float x) { return 1.0f / sqrtf(x); }

Q35_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
Q35_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Warp reduction of NV per-lane partial sums at once (transpose butterfly: each level halves the
// values a lane keeps, exchanging the other half with its partner), NV a power of two <= 32:
// NV - 1 + 5 - log2(NV) shuffles instead of 5 NV. Afterwards the returned value of lane l is the
// warp total of value index butterfly_index<NV>(l); lanes that differ only in bits below the
// levels used agree, and butterfly_writer<NV>(l) picks one of them. Each level adds the same lane
// pairs as warp_sum (offsets 16, 8, 4, 2, 1), so every total is bit-identical to warp_sum's.
template <int NV>
Q35_DEV float butterfly_sum(float (&v)[NV], int lane) {
  int n = NV;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const int half = n / 2;
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[i + half];
          const float keep = upper ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}
template <int NV>
Q35_DEV int butterfly_index(int lane) {
  int idx = 0;
#pragma unroll
  for (int nn = NV, bit = 4; nn > 1; nn /= 2, --bit) idx = idx * 2 + ((lane >> bit) & 1);
  return idx;
}
template <int NV>
Q35_DEV bool butterfly_writer(int lane) {
  int levels = 0;
#pragma unroll
  for (int nn = NV; nn > 1; nn /= 2) ++levels;
  return (lane & ((1 << (5 - levels)) - 1)) == 0;
}

// Block-wide sum; every thread gets the result. `red` needs NWARPS floats.
template <int NWARPS>
Q35_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NWARPS; ++i) t += red[i];
  return t;
}
template <int NWARPS>
Q35_DEV float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int i = 1; i < NWARPS; ++i) t = fmaxf(t, red[i]);
  return t;
}

// 16-byte read-only streaming load: weights are touched once per step, keep them out of L1.
Q35_DEV uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

Q35_DEV void unpack_bf16x8(const uint4& u, float f[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

Q35_DEV float dot_bf16x8(const uint4& a, const uint4& b, float acc) {
  float fa[8], fb[8];
  unpack_bf16x8(a, fa);
  unpack_bf16x8(b, fb);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = fmaf(fa[i], fb[i], acc);
  return acc;
}

Q35_DEV int dot_i8x16(const uint4& a, const uint4& b, int acc) {
  acc = __dp4a((int)a.x, (int)b.x, acc);
  acc = __dp4a((int)a.y, (int)b.y, acc);
  acc = __dp4a((int)a.z, (int)b.z, acc);
  acc = __dp4a((int)a.w, (int)b.w, acc);
  return acc;
}

// Weight side (explore_runtime_quantization.py:143-155, a torch formula): per output row
// s = amax / 127 (1 for an all-zero row), code = clamp(rne(x / s), -127, 127).
Q35_DEV int quant_i8(float x, float s) {
  int q = __float2int_rn(__fdiv_rn(x, s));
  return max(-127, min(127, q));
}

// Activation side: dynamic per-token symmetric quantisation with the semantics of vllm's
// scaled_int8_quant(x, scale=None, azp=None, symmetric=True), which the reference calls at
// explore_runtime_quantization.py:167-172. The stored scale is amax / 127 (0 for an all-zero
// row); each code is x times the reciprocal 127 / amax (0 for an all-zero row), rounded to
// nearest even and saturated to [-128, 127]. Multiplying by the reciprocal is not the same as
// dividing by the scale: at exact half-way products (x = amax / 2, or amax with mantissa 127)
// the two round differently, so the two sides keep their own formulas.
Q35_DEV float tok_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
Q35_DEV float tok_inv(float amax) { return amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f; }
Q35_DEV int quant_i8_tok(float x, float inv) {
  const int q = __float2int_rn(__fmul_rn(x, inv));
  return max(-128, min(127, q));
}

// Programmatic dependent launch: wait for the producer grid's writes / let the consumer start.
Q35_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
Q35_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// RoPE factors for dimension d at position pos: cos/sin rounded to BF16 as the HF rotary
// embedding returns them (cat(freqs, freqs); FP32 angle = pos * inv_freq).
Q35_DEV void rope_cs(int d, int half, float pos, const float* inv_freq, float& c, float& s) {
  const float ang = pos * inv_freq[d % half];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  c = rbf(cs);
  s = rbf(sn);
}

// Partial RoPE of a normed head held in shared memory, with the BF16 rounding of each partial
// product of the eager path (kernels.py:455-472).
Q35_DEV float rope_apply(const float* normed, int d, int rot, float c, float s) {
  if (d >= rot) return normed[d];
  const int half = rot / 2;
  const float partner = d < half ? -normed[d + half] : normed[d - half];
  return rbf(rbf(normed[d] * c) + rbf(partner * s));
}

// Order-preserving 32-bit key of a float (larger float -> larger key); -0 folds onto +0.
Q35_DEV uint32_t float_order_key(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- warp-level tensor-core helpers (mma.sync m16n8k16 bf16, ldmatrix)
Q35_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
Q35_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
Q35_DEV void mma_bf16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
Q35_DEV uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
}  // namespace q35

// Per-step device counters the decoder's last kernel advances (cache rows, RoPE position, token log).
struct q35_step_counters {
  int64_t* cache_len;
  int64_t* rope_pos;
  int64_t* token_log;
  int64_t* log_pos;
  int log_len;
};

// Host-side error reporting shared by every entry point.
int q35_fail(int code, const char* fmt, ...);
int q35_check_launch(const char* what);

#define Q35_REQUIRE(cond, ...)                         \
  do {                                                 \
    if (!(cond)) return q35_fail(Q35_EINVAL, __VA_ARGS__); \
  } while (0)

#define Q35_ALIGNED(p, n) ((((uintptr_t)(p)) % (n)) == 0)

// Launch with optional programmatic dependent launch (PDL): the kernel may start while the
// previous kernel on the stream drains; it must call pdl_wait() before touching that kernel's
// outputs. Without the attribute pdl_wait()/pdl_launch_dependents() are no-ops.
template <typename... KArgs, typename... Args>
static inline cudaError_t q35_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host-side set-up that belongs to one device's context: kernel attributes (dynamic shared
// memory, carve-out, non-portable cluster sizes) and occupancy answers are per device, so a
// process that drives several GPUs must set and cache them per device ordinal. `get` runs `init`
// once per device (the first caller on that device, under a mutex; `init` runs with that device
// current) and afterwards returns the cached value with one acquire load.
constexpr int kQ35MaxDevices = 64;

template <class T>
class Q35PerDevice {
 public:
  template <class F>
  T get(F&& init) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kQ35MaxDevices) {
      cudaGetLastError();
      return init();  // no cacheable ordinal: set up on every call
    }
    if (ready_[dev].load(std::memory_order_acquire)) return val_[dev];
    std::lock_guard<std::mutex> lock(mu_);
    if (!ready_[dev].load(std::memory_order_relaxed)) {
      val_[dev] = init();
      ready_[dev].store(true, std::memory_order_release);
    }
    return val_[dev];
  }

 private:
  std::mutex mu_;
  T val_[kQ35MaxDevices] = {};
  std::atomic<bool> ready_[kQ35MaxDevices] = {};
};
