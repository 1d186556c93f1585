// gemm_tc.cuh - C[M,N] = A[M,K] * W[N,K]^T on sm_100a tensor cores.
//
// A (activations) and W (weights, row = output feature, the reference's
// row-major Matrix layout core/cortex.nim:24-27) are both K-major.  One CTA
// computes one 128 x BN tile:
//   warp 0 / lane 0 : TMA producer, STAGES-deep shared-memory ring of
//                     128-byte-wide K slices (SWIZZLE_128B), one mbarrier pair
//                     per stage;
//   warp 1          : allocates BN TMEM columns; lane 0 issues
//                     tcgen05.mma (M=128, N=BN, fp32 accumulate in TMEM) and
//                     releases each stage with tcgen05.commit;
//   all 4 warps     : epilogue, each warp reading its 32 TMEM lanes (= 32 rows)
//                     with tcgen05.ld and handing 16-column runs to `Epi`.
// TIn = __nv_bfloat16 -> kind::f16 (bf16 x bf16), TIn = float -> kind::tf32.
// Rows >= M and columns >= N are zero-filled by TMA and never stored; K tails
// are zero-filled and contribute nothing.  Every wait is bounded (common.cuh).
#pragma once

#include <cuda.h>
#include "common.cuh"

namespace snai {

template <typename TIn> struct TcKind;
template <> struct TcKind<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;  // BF16
  static constexpr int kBK = 64;       // elements per 128-byte K slice
  static constexpr int kUK = 16;       // K per tcgen05.mma (32 bytes)
};
template <> struct TcKind<float> {
  static constexpr uint32_t kFmt = 2;  // TF32
  static constexpr int kBK = 32;
  static constexpr int kUK = 8;
};

constexpr int kTcBM = 128;

template <int BN, int STAGES>
struct TcSmem {
  static constexpr int kABytes = kTcBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
};

// Shared-memory matrix descriptor of a K-major tile stored as rows of 128
// bytes with the 128-byte swizzle (8-row atoms 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused here)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // SWIZZLE_128B
  return d;
}

template <typename TIn, int BN>
__device__ __forceinline__ constexpr uint32_t tc_idesc() {
  return (1u << 4)                                      // D: fp32
         | (TcKind<TIn>::kFmt << 7) | (TcKind<TIn>::kFmt << 10)  // A, B formats
         | ((uint32_t)(BN >> 3) << 17)                  // N
         | ((uint32_t)(kTcBM >> 4) << 24);              // M
}

template <typename TIn>
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate);

template <>
__device__ __forceinline__ void tc_mma<__nv_bfloat16>(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                      uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <>
__device__ __forceinline__ void tc_mma<float>(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <typename TIn, int BN, int STAGES, int MIN_BLOCKS, class Epi>
__global__ void __launch_bounds__(128, MIN_BLOCKS)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, Epi epi, int *err) {
  using Sm = TcSmem<BN, STAGES>;
  constexpr int BK = TcKind<TIn>::kBK;
  constexpr int KSTEPS = BK / TcKind<TIn>::kUK;
  constexpr uint32_t IDESC = tc_idesc<TIn, BN>();

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Sm::kBarOffset);
  uint64_t *empty = full + STAGES;
  uint64_t *accb = empty + STAGES;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(accb + 1);
  int *cta_fail = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTcBM, n0 = blockIdx.y * BN;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    *cta_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int issued = 0;
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, kErrWaitEmpty)) {
        atomicExch(cta_fail, 1);
        break;
      }
      if (*(volatile int *)cta_fail) break;
      mbar_arrive_expect_tx(&full[s], Sm::kStageBytes);
      uint8_t *st = smem + s * Sm::kStageBytes;
      tma_load_2d(st, &tmA, &full[s], kb * BK, m0);
      tma_load_2d(st + Sm::kABytes, &tmB, &full[s], kb * BK, n0);
      ++issued;
    }
    // Do not leave while a copy into this CTA's shared memory is in flight.
    for (int kb = issued - 1; kb >= 0 && kb >= issued - STAGES; --kb) {
      const int s = kb % STAGES;
      if (!mbar_wait_bounded(&full[s], (uint32_t)(kb / STAGES) & 1u, err, kErrWaitDrain)) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!mbar_wait_bounded(&full[s], ph, err, kErrWaitFull)) {
        atomicExch(cta_fail, 1);
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(smem + s * Sm::kStageBytes);
      const uint32_t b0 = a0 + Sm::kABytes;
      const uint64_t adesc = sw128_desc(a0), bdesc = sw128_desc(b0);
#pragma unroll
      for (int k = 0; k < KSTEPS; ++k) {
        // +32 bytes per K step inside the swizzle atom (start address is in 16-byte units)
        tc_mma<TIn>(tmem, adesc + 2u * k, bdesc + 2u * k, IDESC, (kb | k) != 0 ? 1u : 0u);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(accb);
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> Epi ----
  const bool acc_ok = mbar_wait_bounded(accb, 0, err, kErrWaitAccum);
  tc_fence_after();
  if (acc_ok && !*(volatile int *)cta_fail) {
    const int row = m0 + warp * 32 + lane;
    const uint32_t tbase = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      if (n0 + c >= N) break;  // warp-uniform
      float v[16];
      tmem_ld16(tbase + (uint32_t)c, v);
      if (row < M) {
        const int cnt = min(16, N - (n0 + c));
        epi.store(row, n0 + c, v, cnt);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, BN);
}

}  // namespace snai
