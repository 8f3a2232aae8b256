// Decode GEMV with the weights staged through shared memory by bulk asynchronous copies.
//
// Included inside gemv.cu's anonymous namespace (uses GemvParams, build_input, epilogue).
//
// Each CTA owns a contiguous range of output units, i.e. a contiguous byte range of the weight
// (two ranges for SwiGLU: gate rows and the matching up rows). Thread 0 streams it through a ring
// of kStages 24 KB shared-memory stages with cp.async.bulk (TMA bulk copy, no tensor map, no
// multicast), completing on one mbarrier per stage. The first stages are issued before the PDL
// wait — weights do not depend on the previous kernel — so they are in flight while the producer
// kernel drains. A stage holds RS = 24 KB / row_bytes rows cut into 1 KB parts; the 24 parts go
// 3 per warp: a lane dots 32 contiguous weight bytes with the matching slice of the input vector
// (shared memory), a warp reduces, and per-row partials are summed in a fixed order by one thread
// per unit, which applies the epilogue. In-flight bytes live in shared memory, not registers, so
// a CTA of the next kernel fits beside a running one (~90 KB each).

constexpr int kBulkStages = 3;
constexpr int kBulkStageBytes = 24 * 1024;
constexpr int kBulkPart = 1024;                       // bytes per work item
constexpr int kBulkItems = kBulkStageBytes / kBulkPart;  // 24 items per stage, 3 per warp
constexpr long long kBulkWaitBudget = 4000000000LL;   // ~2 s: a wait that exceeds it reports and exits

__device__ int q35_gemv_error_word = 0;

Q35_DEV uint32_t bulk_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

Q35_DEV bool bulk_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kBulkWaitBudget) return false;
  }
}

Q35_DEV void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int K, bool INT8, int RPU>
struct BulkShape {
  static constexpr int ES = INT8 ? 1 : 2;
  static constexpr int RB = K * ES;                   // row bytes
  static constexpr int RS = kBulkStageBytes / RB;     // rows per stage
  static constexpr int SU = RS / RPU;                 // units per stage
  static constexpr int PPR = RB / kBulkPart;          // parts per row
  static_assert(RB % kBulkPart == 0 && kBulkStageBytes % RB == 0, "row size must tile the stage");
  static_assert(RS % RPU == 0 && SU >= 1, "stage must hold whole units");
};

template <int K, int PRO, int EPI, bool INT8>
__global__ void __launch_bounds__(kThreads) gemv_bulk_kernel(GemvParams p) {
  constexpr int RPU = (EPI == Q35_EPI_SWIGLU) ? 2 : 1;
  using Sh = BulkShape<K, INT8, RPU>;
  constexpr int RB = Sh::RB, SU = Sh::SU, PPR = Sh::PPR;
  extern __shared__ __align__(16) unsigned char smem_raw[];  // bulk copies need 16-byte alignment
  unsigned char* stages = smem_raw;                                     // [kBulkStages][24 KB]
  __shared__ __align__(16) bf16 xs[K];
  __shared__ __align__(16) int8_t xq[INT8 ? K : 16];
  __shared__ float red[kWarps];
  __shared__ float sx_s;
  __shared__ float partf[kBulkItems];
  __shared__ int parti[kBulkItems];
  __shared__ __align__(8) uint64_t full[kBulkStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = p.n_out;
  const int u0 = (int)(((long long)n_out * blockIdx.x) / gridDim.x);
  const int u1 = (int)(((long long)n_out * (blockIdx.x + 1)) / gridDim.x);
  const int n_st = (u1 - u0 + SU - 1) / SU;
  const char* W = static_cast<const char*>(p.weight);

  auto issue = [&](int i) {  // thread 0: stage i -> slot i % kBulkStages
    const int ua = u0 + i * SU;
    const int nu = min(SU, u1 - ua);
    const uint32_t bar = bulk_smem_u32(&full[i % kBulkStages]);
    const uint32_t dst = bulk_smem_u32(stages + (i % kBulkStages) * kBulkStageBytes);
    const uint32_t bytes = (uint32_t)(nu * RB);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes * RPU) : "memory");
    bulk_copy(dst, W + (int64_t)ua * RB, bytes, bar);
    if (RPU == 2) bulk_copy(dst + SU * RB, W + ((int64_t)n_out + ua) * RB, bytes, bar);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bulk_smem_u32(&full[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < kBulkStages && i < n_st; ++i) issue(i);
  }
  if (PRO != Q35_PRO_PLAIN)
    for (int i = threadIdx.x; i < K / 64; i += kThreads) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.norm_w + 64 * i));
  pdl_wait();
  pdl_launch_dependents();
  build_input<PRO, INT8>(p, K, xs, xq, &sx_s, red);  // ends with __syncthreads (barrier init visible)
  const float sx = INT8 ? sx_s : 1.0f;

  bool ok = true;
  for (int i = 0; i < n_st; ++i) {
    const int slot = i % kBulkStages;
    if (!bulk_wait(bulk_smem_u32(&full[slot]), (i / kBulkStages) & 1)) {
      if (threadIdx.x == 0) atomicCAS(&q35_gemv_error_word, 0, 1);
      ok = false;
    }
    if (!__syncthreads_and(ok)) break;
    const unsigned char* st = stages + slot * kBulkStageBytes;
    const int ua = u0 + i * SU;
    const int nu = min(SU, u1 - ua);
#pragma unroll
    for (int j = 0; j < kBulkItems / kWarps; ++j) {
      const int item = warp + j * kWarps;
      const int row = item / PPR, part = item % PPR;  // row within the stage
      const int urow = (RPU == 2) ? (row % SU) : row;  // unit of this row
      float accf = 0.f;
      int acci = 0;
      if (urow < nu) {
        const uint4* wv = reinterpret_cast<const uint4*>(st + row * RB + part * kBulkPart + lane * 32);
        const uint4 w0 = wv[0], w1 = wv[1];
        if (INT8) {
          const uint4* xv = reinterpret_cast<const uint4*>(xq + part * kBulkPart + lane * 32);
          acci = dot_i8x16(w1, xv[1], dot_i8x16(w0, xv[0], 0));
        } else {
          const uint4* xv = reinterpret_cast<const uint4*>(xs + (part * kBulkPart + lane * 32) / 2);
          accf = dot_bf16x8(w1, xv[1], dot_bf16x8(w0, xv[0], 0.f));
        }
      }
      if (INT8) {
        acci = warp_sum_i(acci);
        if (lane == 0) parti[item] = acci;
      } else {
        accf = warp_sum(accf);
        if (lane == 0) partf[item] = accf;
      }
    }
    __syncthreads();  // parts complete; stage slot free
    if (threadIdx.x == 0 && i + kBulkStages < n_st) issue(i + kBulkStages);
    if (threadIdx.x < nu) {
      const int u = threadIdx.x;
      float y[2];
#pragma unroll
      for (int r = 0; r < RPU; ++r) {
        const int row = u + r * SU;
        if (INT8) {
          int t = 0;
#pragma unroll
          for (int q = 0; q < PPR; ++q) t += parti[row * PPR + q];
          y[r] = ((float)t * sx) * p.w_scale[(int64_t)(ua + u) + (int64_t)r * n_out];
        } else {
          float t = 0.f;
#pragma unroll
          for (int q = 0; q < PPR; ++q) t += partf[row * PPR + q];
          y[r] = t;
        }
      }
      epilogue<EPI, INT8>(p, ua + u, y[0], RPU > 1 ? y[1] : 0.f);
    }
  }
}

template <int K, int PRO, int EPI, bool INT8>
int launch_bulk(const GemvParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)kBulkStages * kBulkStageBytes;
  static Q35PerDevice<bool> attr;
  attr.get([smem] {
    cudaFuncSetAttribute(gemv_bulk_kernel<K, PRO, EPI, INT8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return true;
  });
  int grid = kNumSMs;
  if (p.n_out < grid) grid = p.n_out;
  cudaError_t e = q35_launch(gemv_bulk_kernel<K, PRO, EPI, INT8>, dim3(grid), dim3(kThreads), smem, s, pdl, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemv_bulk launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}
