// gemm_tc.cuh - C[M,N] = A[M,K] * W[N,K]^T on sm_100a tensor cores.
//
// A (activations) and W (weights, row = output feature, the reference's
// row-major Matrix layout core/cortex.nim:24-27) are both K-major and staged
// by TMA as 128-byte-wide K slices with the 128-byte swizzle; tcgen05.mma
// (M = 128, N = BN, fp32 accumulate in TMEM) consumes them and the epilogue
// reads TMEM back with tcgen05.ld.
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

}  // namespace snai

namespace snai {

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int BN, int STAGES>
struct TcpSmem {
  static constexpr int kABytes = kTcBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
};

// Persistent, warp-specialised C = A * W^T.  One CTA per SM walks the tiles
// t = blockIdx.x, + gridDim.x, ... (M-fastest, so CTAs running together share
// weight tiles in L2).  Roles:
//   warp 0 lane 0   TMA producer over a STAGES-deep ring (all tiles, one
//                   running k-block counter);
//   warp 1          allocates 2*BN TMEM columns (two accumulators); lane 0
//                   issues the tcgen05.mma of tile i into accumulator i % 2;
//   warps 2..9      epilogue: two warps per 32-lane TMEM quarter, each taking
//                   half of the tile's columns; wait for accumulator i % 2,
//                   tcgen05.ld, hand 16-column runs to Epi, release the
//                   accumulator; this overlaps the MMAs of tile i + 1.
// All waits are bounded (common.cuh); a failed wait records an error and the
// CTA winds down.
template <typename TIn, int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(320, 1)
    gemm_tcp_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                    int K, Epi epi, int *err) {
  using Sm = TcpSmem<BN, STAGES>;
  constexpr int BK = TcKind<TIn>::kBK;
  constexpr int KSTEPS = BK / TcKind<TIn>::kUK;
  constexpr uint32_t IDESC = tc_idesc<TIn, BN>();
  constexpr uint32_t TCOLS = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Sm::kBarOffset);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(tempty + 2);
  int *cta_fail = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kTcBM - 1) / kTcBM;
  const int num_tiles = num_m * ((N + BN - 1) / BN);
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    *cta_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile % num_m) * kTcBM, n0 = (tile / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, kErrWaitEmpty) || *(volatile int *)cta_fail) {
            atomicExch(cta_fail, 1);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Sm::kStageBytes);
          uint8_t *st = smem + s * Sm::kStageBytes;
          tma_load_2d(st, &tmA, &full[s], kb * BK, m0);
          tma_load_2d(st + Sm::kABytes, &tmB, &full[s], kb * BK, n0);
        }
      }
      // do not leave while a copy into this CTA's shared memory is in flight
      for (int j = it - 1; j >= 0 && j >= it - STAGES; --j)
        if (!mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, err, kErrWaitDrain)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, tc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++tc) {
        const int acc = tc & 1;
        if (!mbar_wait_bounded(&tempty[acc], ((uint32_t)(tc >> 1) & 1u) ^ 1u, err, kErrWaitEmpty)) {
          atomicExch(cta_fail, 1);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, err, kErrWaitFull) || *(volatile int *)cta_fail) {
            atomicExch(cta_fail, 1);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * Sm::kStageBytes);
          const uint64_t adesc = sw128_desc(a0), bdesc = sw128_desc(a0 + Sm::kABytes);
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k)
            tc_mma<TIn>(d, adesc + 2u * k, bdesc + 2u * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter = warp % 4, column half by warp
    const int q = warp & 3;
    const int c_lo = ((warp - 2) >> 2) * (BN / 2);
    int tc = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
      const int acc = tc & 1;
      if (!mbar_wait_bounded(&tfull[acc], (uint32_t)(tc >> 1) & 1u, err, kErrWaitAccum) ||
          *(volatile int *)cta_fail) {
        atomicExch(cta_fail, 1);
        break;
      }
      tc_fence_after();
      const int m0 = (tile % num_m) * kTcBM, n0 = (tile / num_m) * BN;
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = c_lo; c < c_lo + BN / 2; c += 16) {
        if (n0 + c >= N) break;  // warp-uniform
        float v[16];
        tmem_ld16(tbase + (uint32_t)c, v);
        if (row < M) epi.store(row, n0 + c, v, min(16, N - (n0 + c)));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TCOLS);
}

}  // namespace snai
