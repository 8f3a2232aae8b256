// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// C[M, N] = A[M, K] . W[N, K]^T with BF16 inputs / FP32 accumulation (kind::f16), or int8 inputs /
// exact int32 accumulation (kind::i8, A8W8). Persistent: one CTA per SM walks the 128 x TBN output
// tiles (TBN = 256, or 128 when that fills the machine in fewer waves) in M-fastest order, so the
// CTAs running at once share each weight tile. Warp roles:
//   warp 0 lane 0  TMA producer: A box 128 x 128 B and W box TBN x 128 B per stage (128-byte
//                  swizzle, K-major) into a 4-stage ring guarded by full / empty mbarriers
//                  (6 stages, or L2 prefetches of the weight boxes ahead of their loads, measured
//                  no faster / 30-50 % slower);
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16 bf16 / 32 int8 each) per stage into one of
//                  two 128 x TBN FP32/S32 TMEM accumulators; tcgen05.commit frees the stage and,
//                  after a tile's last stage, hands the accumulator to the epilogue;
//   warps 2-9      epilogue, two warps per TMEM lane quarter taking alternate 32-column chunks:
//                  tcgen05.ld from the warp's 32 TMEM lanes, dequantise (int8), store / add to the
//                  residual / apply SwiGLU, then release the accumulator, while the MMA warp
//                  already fills the other one.
// A second kernel runs the same pipeline on SM pairs (tcgen05 cta_group::2, 256 x 256 tiles); see
// gemm_tc2_kernel. The launcher picks the kernel and tile width per shape.
// SwiGLU tiles load W rows [o0, o0+TBN/2) (gate) and [N+o0, N+o0+TBN/2) (up) as the two halves of
// the B tile, so gate and up of an output sit TBN/2 TMEM columns apart.
// No cluster multicast anywhere (loads are per CTA). Every mbarrier wait is bounded by a clock
// budget; a wait that gives up records an error code in q35_tc_error and raises a CTA-wide abort
// flag that ends every role's loop.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

using namespace q35;

__device__ int q35_tc_error_word = 0;

namespace {

constexpr int BM = 128, BKB = 128;  // tile rows, K bytes per stage (tile cols: 256, or 128 for narrow N)
constexpr int kABytes = BM * BKB;   // 16 KB
constexpr int kThreads = 320;       // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;        // two per TMEM lane quarter, alternate 32-column chunks
constexpr long long kWaitBudget = 4000000000LL;  // ~2 s at 2 GHz
constexpr int stages_for(int) { return 4; }

struct TcParams {
  void* out;          // bf16 [M, N] or int32 (RAW)
  bf16* resid;        // RESIDUAL: [M, N] updated in place
  const bf16* bias;   // BIAS*: [N]
  const float* sx;    // int8: [M]
  const float* sw;    // int8: [Nw]
  int M, N, K;        // K in elements
};

Q35_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

Q35_DEV void report(int code);

// Bounded wait for the phase of `parity` to complete. Gives up (false) when another role raised
// the CTA's abort flag, or after the clock budget, raising the flag and recording `code`.
Q35_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
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
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBudget) {
      *abort_flag = 1;
      report(code);
      return false;
    }
  }
}

Q35_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

Q35_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

Q35_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

Q35_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major operand tile with 128-byte swizzle: 8-row core groups 1024 bytes apart (SBO), version 1.
Q35_DEV uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);          // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset
  d |= (uint64_t)1 << 46;                         // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
  return d;
}

template <bool INT8>
Q35_DEV void mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  if (INT8)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

Q35_DEV void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

Q35_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

Q35_DEV void report(int code) { atomicCAS(&q35_tc_error_word, 0, code); }

// ---------------------------------------------------------------- CTA-pair (cta_group::2) helpers
Q35_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
Q35_DEV uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
Q35_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory that completes bytes on an mbarrier of either CTA of the pair.
Q35_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}
template <bool INT8>
Q35_DEV void mma_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  if (INT8)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive (once the pair's MMAs issued so far complete) on the mbarrier at `bar` in both CTAs.
Q35_DEV void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)0x3)
      : "memory");
}
Q35_DEV void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
Q35_DEV void mbar_expect_tx_only(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Epilogue of one accumulator tile for one thread's output row: the warp takes the 32-column
// chunks h, h + 2, ... of its TMEM lane quarter. The residual reads of chunk c + 2 are issued
// before chunk c's TMEM load, so the chunks' memory round trips overlap instead of following one
// another (with one read round trip per chunk, 8 chunks in a row made the tile's tail several us).
template <bool INT8, int EPI, int TBN>
Q35_DEV void epilogue_row(const TcParams& p, uint32_t trow, int row, int col0, int h) {
  constexpr int kCols = (EPI == Q35_EPI_SWIGLU) ? TBN / 2 : TBN;
  const bool row_ok = row < p.M;
  bf16* base = (EPI == Q35_EPI_RESIDUAL ? p.resid : static_cast<bf16*>(p.out)) + (int64_t)(row_ok ? row : 0) * p.N;
  const float sx = (INT8 && row_ok) ? p.sx[row] : 0.f;
  uint4 res[4], res_n[4];
  auto fetch = [&](int c, uint4 (&r)[4]) {
    const int gc = col0 + c;
    if (EPI == Q35_EPI_RESIDUAL && row_ok && gc + 32 <= p.N) {
#pragma unroll
      for (int i = 0; i < 4; ++i) r[i] = *reinterpret_cast<const uint4*>(base + gc + 8 * i);
    }
  };
  if (32 * h < kCols) fetch(32 * h, res);
  for (int c = 32 * h; c < kCols; c += 64) {
    if (c + 64 < kCols) fetch(c + 64, res_n);
    const int gc = col0 + c;
    uint32_t v[32], u[32];
    tmem_ld32(trow + c, v);
    if (EPI == Q35_EPI_SWIGLU) tmem_ld32(trow + TBN / 2 + c, u);
    if (row_ok && gc < p.N) {
      float y[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        y[j] = INT8 ? ((gc + j < p.N) ? ((float)(int)v[j] * sx) * __ldg(p.sw + gc + j) : 0.f) : __uint_as_float(v[j]);
      if (EPI == Q35_EPI_SWIGLU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float up =
              INT8 ? ((gc + j < p.N) ? ((float)(int)u[j] * sx) * __ldg(p.sw + p.N + gc + j) : 0.f) : __uint_as_float(u[j]);
          y[j] = rbf(silu_f(rbf(y[j]))) * rbf(up);
        }
      }
      if (EPI >= Q35_EPI_BIAS) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float b = (gc + j < p.N) ? bf2f(p.bias[gc + j]) : 0.f;
          y[j] = y[j] + b;
          if (EPI == Q35_EPI_BIAS_GELU_TANH) y[j] = gelu_tanh_f(rbf(y[j]));
          if (EPI == Q35_EPI_BIAS_GELU) y[j] = gelu_erf_f(rbf(y[j]));
        }
      }
      bf16* dst = base + gc;
      if (gc + 32 <= p.N) {
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          __align__(16) bf16 o[8];
          if (EPI == Q35_EPI_RESIDUAL) {
            float rf[8];
            unpack_bf16x8(res[qq], rf);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = f2bf(rf[j] + rbf(y[8 * qq + j]));
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = f2bf(y[8 * qq + j]);
          }
          *reinterpret_cast<uint4*>(dst + 8 * qq) = *reinterpret_cast<const uint4*>(o);
        }
      } else {
        for (int j = 0; j < 32 && gc + j < p.N; ++j) {
          if (EPI == Q35_EPI_RESIDUAL)
            dst[j] = f2bf(bf2f(dst[j]) + rbf(y[j]));
          else
            dst[j] = f2bf(y[j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) res[i] = res_n[i];
  }
}

template <bool INT8, int EPI, int TBN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, TcParams p) {
  constexpr int S = stages_for(TBN);
  constexpr int kBB = TBN * BKB;  // B bytes per stage
  constexpr int kCols = (EPI == Q35_EPI_SWIGLU) ? TBN / 2 : TBN;  // output columns per tile
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sA = smem;
  unsigned char* sB = smem + S * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * kBB);  // full[S], empty[S], tfull[2], tempty[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kstep = BKB / (INT8 ? 1 : 2);  // K elements per stage
  const int n_k = p.K / kstep;
  const int num_m = (p.M + BM - 1) / BM;
  const int ntiles = num_m * ((p.N + kCols - 1) / kCols);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  const uint32_t tfull0 = smem_u32(bars + 2 * S), tempty0 = smem_u32(bars + 2 * S + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, kEpiWarps);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * TBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: the set-up above overlapped the previous kernel's tail; A,
  // the residual and the outputs are touched only after it has completed
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile % num_m) * BM, c0 = (tile / num_m) * kCols;
        for (int kt = 0; kt < n_k; ++kt, ++it) {
          const int s = it % S, r = it / S;
          if (r > 0 && !mbar_wait(empty0 + 8 * s, (r - 1) & 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full0 + 8 * s, kABytes + kBB);
          const int kx = kt * kstep;
          tma_load_2d(smem_u32(sA + s * kABytes), &tmA, kx, m0, full0 + 8 * s);
          if (EPI == Q35_EPI_SWIGLU) {
            tma_load_2d(smem_u32(sB + s * kBB), &tmB, kx, c0, full0 + 8 * s);
            tma_load_2d(smem_u32(sB + s * kBB + kBB / 2), &tmB, kx, p.N + c0, full0 + 8 * s);
          } else {
            tma_load_2d(smem_u32(sB + s * kBB), &tmB, kx, c0, full0 + 8 * s);
          }
        }
      }
      // drain: every copy this thread issued has landed before the CTA can exit
      // (only matters after an abort: otherwise the MMA warp consumed them all)
      static __shared__ int no_abort;  // a flag nobody raises: these waits end on landing or budget
      no_abort = 0;
      for (int j = it - S > 0 ? it - S : 0; j < it; ++j)
        mbar_wait(full0 + 8 * (j % S), (uint32_t)((j / S) & 1), &no_abort, 5);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      // instruction descriptor: D fp32 (1) / s32 (2); A, B bf16 (1) / signed int8 (1); K-major;
      // N = TBN (>> 3 at bit 17), M = 128 (>> 4 at bit 24)
      const uint32_t idesc = ((INT8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TBN >> 3) << 17) |
                             ((uint32_t)(BM >> 4) << 24);
      int it = 0, tc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++tc) {
        const int acc = tc & 1, use = tc >> 1;
        if (use > 0 && !mbar_wait(tempty0 + 8 * acc, (use - 1) & 1, abort_flag, 4)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(acc * TBN);
        for (int kt = 0; kt < n_k; ++kt, ++it) {
          const int s = it % S, r = it / S;
          if (!mbar_wait(full0 + 8 * s, r & 1, abort_flag, 2)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sB + s * kBB);
#pragma unroll
          for (int k = 0; k < BKB / 32; ++k)  // 32 bytes of K per MMA
            mma<INT8>(d, smem_desc(a0 + 32 * k), smem_desc(b0 + 32 * k), idesc, (kt > 0 || k > 0) ? 1u : 0u);
          mma_commit(empty0 + 8 * s);
        }
        if (ok) mma_commit(tfull0 + 8 * acc);
      }
    }
  } else {
    // ---------------- epilogue: warp w owns TMEM lanes / tile rows [32 (w % 4), 32 (w % 4) + 32)
    const int q = warp & 3, h = (warp - 2) >> 2;
    int tc = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tc) {
      const int acc = tc & 1, use = tc >> 1;
      if (!mbar_wait(tfull0 + 8 * acc, use & 1, abort_flag, 3)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (tile % num_m) * BM, col0 = (tile / num_m) * kCols;
      const uint32_t trow = tmem + (uint32_t)(acc * TBN) + ((uint32_t)(q * 32) << 16);
      epilogue_row<INT8, EPI, TBN>(p, trow, m0 + q * 32 + lane, col0, h);
      // the accumulator is drained (tcgen05.ld waited): hand it back to the MMA warp
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TBN) : "memory");
}

// ---------------------------------------------------------------- CTA-pair kernel
// The same persistent pipeline on pairs of SMs (thread-block clusters of 2, tcgen05 cta_group::2):
// a pair computes a 256 x TBN tile as ONE MMA of M = 256. CTA r of the pair loads its own A rows
// [128 r, 128 r + 128) and B rows [r TBN/2, (r + 1) TBN/2) and holds output rows 128 r .. in its
// TMEM; the MMA reads both CTAs' shared memory. Each SM therefore streams half the B bytes per
// FLOP of the single-CTA kernel. Protocol (rank 0 = leader):
//   full[s]   leader only: the leader's producer arrives with the pair's total bytes; both CTAs'
//             loads complete their bytes on it (cta_group::2 TMA, mbarrier mapped to rank 0);
//   empty[s]  each CTA: the leader's tcgen05.commit arrives on both (multicast commit);
//   tfull[a]  each CTA: multicast commit after a tile's last MMA;
//   tempty[a] leader only: the 8 epilogue warps of each CTA arrive (remote arrive from rank 1).
constexpr int stages_pair(int bn) { return bn == 256 ? 6 : 8; }
constexpr size_t smem_bytes_pair(int bn) {
  return 1024 + (size_t)stages_pair(bn) * (kABytes + (size_t)(bn / 2) * BKB) + 256;
}

template <bool INT8, int EPI, int TBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, TcParams p) {
  constexpr int S = stages_pair(TBN);
  constexpr int kBB = (TBN / 2) * BKB;  // this CTA's B bytes per stage
  constexpr int kCols = (EPI == Q35_EPI_SWIGLU) ? TBN / 2 : TBN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sA = smem;
  unsigned char* sB = smem + S * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * kBB);  // full[S], empty[S], tfull[2], tempty[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int kstep = BKB / (INT8 ? 1 : 2);
  const int n_k = p.K / kstep;
  const int num_m = (p.M + 2 * BM - 1) / (2 * BM);
  const int ntiles = num_m * ((p.N + kCols - 1) / kCols);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  const uint32_t tfull0 = smem_u32(bars + 2 * S), tempty0 = smem_u32(bars + 2 * S + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * TBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA signal
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // as in gemm_tc_kernel: inputs and outputs only after the previous kernel completed
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < ntiles && ok; tile += npairs) {
        const int m0 = (tile % num_m) * 2 * BM + (int)rank * BM, c0 = (tile / num_m) * kCols;
        for (int kt = 0; kt < n_k; ++kt, ++it) {
          const int s = it % S, r = it / S;
          if (r > 0 && !mbar_wait(empty0 + 8 * s, (r - 1) & 1, abort_flag, 11)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx_only(full0 + 8 * s, 2 * (kABytes + kBB));
          const uint32_t fbar = map_to_rank(full0 + 8 * s, 0);
          const int kx = kt * kstep;
          tma_load_2d_pair(smem_u32(sA + s * kABytes), &tmA, kx, m0, fbar);
          const int brow = (EPI == Q35_EPI_SWIGLU) ? (rank == 0 ? c0 : p.N + c0) : c0 + (int)rank * (TBN / 2);
          tma_load_2d_pair(smem_u32(sB + s * kBB), &tmB, kx, brow, fbar);
        }
      }
      (void)ok;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader): M = 256 across the pair, N = TBN
      const uint32_t idesc = ((INT8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TBN >> 3) << 17) |
                             ((uint32_t)((2 * BM) >> 4) << 24);
      int it = 0, tc = 0;
      bool ok = true;
      for (int tile = pair; tile < ntiles && ok; tile += npairs, ++tc) {
        const int acc = tc & 1, use = tc >> 1;
        if (use > 0 && !mbar_wait(tempty0 + 8 * acc, (use - 1) & 1, abort_flag, 14)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(acc * TBN);
        for (int kt = 0; kt < n_k; ++kt, ++it) {
          const int s = it % S, r = it / S;
          if (!mbar_wait(full0 + 8 * s, r & 1, abort_flag, 12)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sB + s * kBB);
#pragma unroll
          for (int k = 0; k < BKB / 32; ++k)
            mma_pair<INT8>(d, smem_desc(a0 + 32 * k), smem_desc(b0 + 32 * k), idesc, (kt > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair(empty0 + 8 * s);
        }
        if (ok) mma_commit_pair(tfull0 + 8 * acc);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): warp w owns TMEM lanes [32 (w % 4), +32) of this CTA
    const int q = warp & 3, h = (warp - 2) >> 2;
    const uint32_t tempty_leader = map_to_rank(tempty0, 0);
    int tc = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++tc) {
      const int acc = tc & 1, use = tc >> 1;
      if (!mbar_wait(tfull0 + 8 * acc, use & 1, abort_flag, 13)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (tile % num_m) * 2 * BM + (int)rank * BM, col0 = (tile / num_m) * kCols;
      const uint32_t trow = tmem + (uint32_t)(acc * TBN) + ((uint32_t)(q * 32) << 16);
      epilogue_row<INT8, EPI, TBN>(p, trow, m0 + q * 32 + lane, col0, h);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + 8 * acc);
    }
  }
  // Every load, MMA and cross-CTA arrival of the pair is done before either CTA frees TMEM or exits:
  // the producers' last loads were consumed by the leader's MMAs, whose completion both epilogues
  // waited for (or the CTA aborted, whose waits are bounded).
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TBN) : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// 2-D K-major map: rows x k elements, box = (128 bytes of K) x box_rows, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t k, uint32_t box_rows, bool int8) {
  auto fn = encode_fn();
  if (!fn) return false;
  const uint64_t esz = int8 ? 1 : 2;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {k * esz};
  cuuint32_t box[2] = {(cuuint32_t)(BKB / esz), box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr size_t smem_bytes(int bn) { return 1024 + (size_t)stages_for(bn) * (kABytes + (size_t)bn * BKB) + 256; }

template <bool INT8, int EPI, int TBN>
int launch_tc_bn(const void* a, const void* w, const TcParams& p, cudaStream_t s, bool pdl) {
  CUtensorMap ma, mb;
  const uint64_t wrows = (EPI == Q35_EPI_SWIGLU) ? 2 * (uint64_t)p.N : (uint64_t)p.N;
  if (!make_map(&ma, a, p.M, p.K, BM, INT8) ||
      !make_map(&mb, w, wrows, p.K, EPI == Q35_EPI_SWIGLU ? TBN / 2 : TBN, INT8))
    return q35_fail(Q35_ECUDA, "gemm_tc: tensor map encoding failed");
  cudaFuncSetAttribute(gemm_tc_kernel<INT8, EPI, TBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem_bytes(TBN));
  const int cols_per_tile = (EPI == Q35_EPI_SWIGLU) ? TBN / 2 : TBN;
  const int64_t tiles = (int64_t)((p.N + cols_per_tile - 1) / cols_per_tile) * ((p.M + BM - 1) / BM);
  const unsigned grid = (unsigned)(tiles < kNumSMs ? tiles : kNumSMs);
  const cudaError_t e = q35_launch(gemm_tc_kernel<INT8, EPI, TBN>, dim3(grid), dim3(kThreads), smem_bytes(TBN), s, pdl,
                                   ma, mb, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemm_tc launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

int g_tc_pairs = 1;  // process-wide: CTA-pair kernel (1) or single-CTA kernel (0)

template <bool INT8, int EPI>
int max_active_pairs() {
  static Q35PerDevice<int> max_pairs;  // pairs resident at once (clusters of 2 need both SMs in one GPC)
  return max_pairs.get([] {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(kNumSMs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes_pair(256);
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaFuncSetAttribute(gemm_tc2_kernel<INT8, EPI, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem_bytes_pair(256));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<INT8, EPI, 256>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = kNumSMs / 2;
    }
    return n < kNumSMs / 2 ? n : kNumSMs / 2;
  });
}

// Pair tiles are 256 x 256 (an N = 128 MMA runs at about half the rate of N = 256 on either kernel).
template <bool INT8, int EPI>
int launch_tc2(const void* a, const void* w, const TcParams& p, cudaStream_t s, bool pdl) {
  constexpr int TBN = 256;
  const int npairs = max_active_pairs<INT8, EPI>();
  const int cols = (EPI == Q35_EPI_SWIGLU) ? TBN / 2 : TBN;
  const int64_t tiles = (int64_t)((p.N + cols - 1) / cols) * ((p.M + 2 * BM - 1) / (2 * BM));
  CUtensorMap ma, mb;
  const uint64_t wrows = (EPI == Q35_EPI_SWIGLU) ? 2 * (uint64_t)p.N : (uint64_t)p.N;
  if (!make_map(&ma, a, p.M, p.K, BM, INT8) || !make_map(&mb, w, wrows, p.K, TBN / 2, INT8))
    return q35_fail(Q35_ECUDA, "gemm_tc: tensor map encoding failed");
  const int64_t pairs = tiles < npairs ? tiles : npairs;
  cudaFuncSetAttribute(gemm_tc2_kernel<INT8, EPI, TBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem_bytes_pair(TBN));
  const cudaError_t e = q35_launch(gemm_tc2_kernel<INT8, EPI, TBN>, dim3((unsigned)(2 * pairs)), dim3(kThreads),
                                   smem_bytes_pair(TBN), s, pdl, ma, mb, p);
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "gemm_tc2 launch: %s", cudaGetErrorString(e));
  return Q35_OK;
}

// Kernel and tile choice (measured at M = 1024 on B200): when single-CTA 128-column tiles fill
// the machine in one wave while 256-column tiles would leave most SMs idle (N = 2048: 128 vs 64
// tiles), the single-CTA 128-column kernel (down 41 us, out_proj 19.5 us; pairs: 44.5 / 23.3).
// Otherwise 256-column tiles, on SM pairs by default (in_proj 35 us, QKV + gate 34, gate/up 47.5;
// single CTAs: 37.7 / 35.7 / 51.4). Splitting K over more pairs to fill the idle SMs (partial
// sums through global memory, fixed-order combine) measured slower for every shape and was removed.
template <bool INT8, int EPI>
int launch_tc(const void* a, const void* w, const TcParams& p, cudaStream_t s, bool pdl) {
  const int64_t mt = (p.M + BM - 1) / BM;
  const int cols128 = (EPI == Q35_EPI_SWIGLU) ? 64 : 128;
  const int64_t t128 = (int64_t)((p.N + cols128 - 1) / cols128) * mt;
  if (t128 <= kNumSMs && mt * 2 <= t128) return launch_tc_bn<INT8, EPI, 128>(a, w, p, s, pdl);
  if (g_tc_pairs) return launch_tc2<INT8, EPI>(a, w, p, s, pdl);
  return launch_tc_bn<INT8, EPI, 256>(a, w, p, s, pdl);
}

}  // namespace

// Used by the decoder prefill and q35_gemm_tc: tensor-core projection with fused epilogue.
int q35_gemm_tc_launch(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k, int epi, bool int8,
                       const float* sx, const float* sw, cudaStream_t s, const void* bias = nullptr, bool pdl = false) {
  Q35_REQUIRE(a && w && out, "gemm_tc: null pointer");
  Q35_REQUIRE(m >= 1 && n >= 1 && k >= 1 && (k * (int8 ? 1 : 2)) % BKB == 0,
              "gemm_tc: k=%lld must fill 128-byte K slabs", (long long)k);
  Q35_REQUIRE(Q35_ALIGNED(a, 16) && Q35_ALIGNED(w, 16) && Q35_ALIGNED(out, 16), "gemm_tc: 16-byte alignment");
  Q35_REQUIRE(n % 8 == 0, "gemm_tc: n must be a multiple of 8");
  Q35_REQUIRE(!int8 || (sx && sw), "gemm_tc: int8 needs scales");
  Q35_REQUIRE(epi == Q35_EPI_STORE || epi == Q35_EPI_RESIDUAL || epi == Q35_EPI_SWIGLU ||
                  (!int8 && epi >= Q35_EPI_BIAS && epi <= Q35_EPI_BIAS_GELU && bias),
              "gemm_tc: bad epilogue %d", epi);
  Q35_REQUIRE(!bias || Q35_ALIGNED(bias, 16), "gemm_tc: bias must be 16-byte aligned");
  TcParams p = {};
  p.bias = static_cast<const bf16*>(bias);
  p.out = out;
  p.resid = static_cast<bf16*>(out);
  p.sx = sx;
  p.sw = sw;
  p.M = (int)m;
  p.N = (int)n;
  p.K = (int)k;
  if (int8) {
    switch (epi) {
      case Q35_EPI_STORE: return launch_tc<true, Q35_EPI_STORE>(a, w, p, s, pdl);
      case Q35_EPI_RESIDUAL: return launch_tc<true, Q35_EPI_RESIDUAL>(a, w, p, s, pdl);
      default: return launch_tc<true, Q35_EPI_SWIGLU>(a, w, p, s, pdl);
    }
  }
  switch (epi) {
    case Q35_EPI_STORE: return launch_tc<false, Q35_EPI_STORE>(a, w, p, s, pdl);
    case Q35_EPI_RESIDUAL: return launch_tc<false, Q35_EPI_RESIDUAL>(a, w, p, s, pdl);
    case Q35_EPI_BIAS: return launch_tc<false, Q35_EPI_BIAS>(a, w, p, s, pdl);
    case Q35_EPI_BIAS_GELU_TANH: return launch_tc<false, Q35_EPI_BIAS_GELU_TANH>(a, w, p, s, pdl);
    case Q35_EPI_BIAS_GELU: return launch_tc<false, Q35_EPI_BIAS_GELU>(a, w, p, s, pdl);
    default: return launch_tc<false, Q35_EPI_SWIGLU>(a, w, p, s, pdl);
  }
}

int q35_gemm_tc_bias_launch(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n,
                            int64_t k, int epi, cudaStream_t s) {
  Q35_REQUIRE(bias, "gemm_tc_bias: null bias");
  Q35_REQUIRE(epi >= Q35_EPI_BIAS && epi <= Q35_EPI_BIAS_GELU, "gemm_tc_bias: bad epilogue %d", epi);
  return q35_gemm_tc_launch(a, w, out, m, n, k, epi, false, nullptr, nullptr, s, bias);
}

extern "C" int q35_gemm_tc_bias(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n,
                                int64_t k, int32_t epilogue, void* stream) {
  return q35_gemm_tc_bias_launch(a, w, bias, out, m, n, k, epilogue, (cudaStream_t)stream);
}

extern "C" int q35_gemm_tc(const void* a, const void* w, void* out, int64_t m, int64_t n, int64_t k,
                           int32_t epilogue, void* stream) {
  return q35_gemm_tc_launch(a, w, out, m, n, k, epilogue, false, nullptr, nullptr, (cudaStream_t)stream);
}

extern "C" int q35_gemm_tc_a8w8(const int8_t* qa, const float* sx, const int8_t* qw, const float* sw, void* out,
                                int64_t m, int64_t n, int64_t k, int32_t epilogue, void* stream) {
  return q35_gemm_tc_launch(qa, qw, out, m, n, k, epilogue, true, sx, sw, (cudaStream_t)stream);
}

extern "C" int q35_set_gemm_tc_pairs(int on) {
  Q35_REQUIRE(on == 0 || on == 1, "gemm_tc: pairs must be 0 or 1");
  g_tc_pairs = on;
  return Q35_OK;
}

extern "C" int q35_tc_error(void) {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q35_tc_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q35_tc_error_word, &zero, sizeof(int));
  return v;
}
