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

// Epilogue warps per CTA: four per TMEM lane quarter, each taking a quarter
// of the tile's columns, so a warp drains its accumulator slice with one
// round of TMEM loads.
constexpr int kEpiWarps = 16;
constexpr int kGemmThreads = (2 + kEpiWarps) * 32;

constexpr int kStageFloats = 32 * 16;  // per-warp transpose buffer: 32 rows x 16 columns

// Drains COLS accumulator columns of one TMEM lane quarter (rows row0 ..
// row0 + 31), 32 columns per round of TMEM loads and one wait.  Each
// 16-column run then goes through the warp's shared-memory buffer (16-byte
// chunks XOR-swizzled by row pair, conflict-free both ways) so that each
// store instruction covers 8 rows x 64 contiguous bytes instead of 32 rows x
// 16 bytes; the epilogue functor takes 4-column groups (rows >= M and
// columns >= N are skipped).
// A lane's copy of another lane's trivially copyable value (32-bit words).
template <class T>
__device__ __forceinline__ T shfl_any(const T &v, int src) {
  if constexpr (sizeof(T) % 4 != 0 || sizeof(T) == 0) {
    return v;
  } else {
    T out;
    const uint32_t *pi = reinterpret_cast<const uint32_t *>(&v);
    uint32_t *po = reinterpret_cast<uint32_t *>(&out);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(T) / 4); ++i) po[i] = __shfl_sync(0xffffffffu, pi[i], src);
    return out;
  }
}

// TMA reduce-add of a staged 32-row x 16-column fp32 run into the tensor at
// (column x, row y); the staging buffer is in the map's 64-byte swizzle.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *tmap, const float *stg, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(stg)), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// TMA store of a staged 32-row x 16-column fp32 run to the tensor at (x, y).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *tmap, const float *stg, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(stg)), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int COLS, class Epi>
__device__ __forceinline__ void drain_accumulator(uint32_t tbase, int row0, int M, int n0, int N, const Epi &epi,
                                                  float *stg) {
  const int lane = threadIdx.x & 31;
  using Row = typename Epi::Row;
  const Row mine = row0 + lane < M ? epi.row(row0 + lane) : Row{};
  float4 *buf = reinterpret_cast<float4 *>(stg);
  constexpr int BLK = COLS < 32 ? COLS : 32;  // columns per TMEM load round
#pragma unroll
  for (int c0 = 0; c0 < COLS; c0 += BLK) {
  if (n0 + c0 >= N) break;  // warp-uniform
  uint32_t rb[BLK];
#pragma unroll
  for (int c = 0; c < BLK; c += 16) tmem_ld16_nowait(tbase + (uint32_t)(c0 + c), rb + c);
  tmem_wait_ld();
  uint32_t *r = rb - c0;  // r[c0 + j] == rb[j]
#pragma unroll
  for (int c = c0; c < c0 + BLK; c += 16) {
    if (n0 + c >= N) break;  // warp-uniform
    if constexpr (Epi::kTmaReduce) {
      // stage the run (the 64-byte swizzle: chunk ch of row l at ch ^ ((l >> 1) & 3)),
      // then one lane adds it into the tensor; rows >= M and columns >= N
      // fall outside the map and are dropped by the copy
      if (lane == 0) bulk_wait_read_all();  // the previous run has been read out of the buffer
      __syncwarp();
#pragma unroll
      for (int ch = 0; ch < 4; ++ch)
        buf[lane * 4 + (ch ^ ((lane >> 1) & 3))] =
            make_float4(__uint_as_float(r[c + 4 * ch]), __uint_as_float(r[c + 4 * ch + 1]),
                        __uint_as_float(r[c + 4 * ch + 2]), __uint_as_float(r[c + 4 * ch + 3]));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0 && row0 < M) tma_reduce_add_2d(&epi.tmap, stg, n0 + c, row0);
    } else {
    // runs the epilogue stores by TMA (same staging; the run's tensor and
    // column come from the epilogue)
    int tx = 0;
    const CUtensorMap *tm = nullptr;
    if constexpr (Epi::kTmaStore) tm = epi.tma_out(n0 + c, tx);
    if (tm != nullptr) {
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int ch = 0; ch < 4; ++ch)
        buf[lane * 4 + (ch ^ ((lane >> 1) & 3))] =
            make_float4(__uint_as_float(r[c + 4 * ch]), __uint_as_float(r[c + 4 * ch + 1]),
                        __uint_as_float(r[c + 4 * ch + 2]), __uint_as_float(r[c + 4 * ch + 3]));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0 && row0 < M) tma_store_2d(tm, stg, tx, row0);
    } else {
    // this run's reads (residual) go out first and overlap the transpose
    typename Epi::Pre pre[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = row0 + 8 * i + (lane >> 2), n = n0 + c + 4 * (lane & 3);
      if (m < M && n < N) pre[i] = epi.load4(m, n, min(4, N - n));
    }
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
      buf[lane * 4 + (ch ^ ((lane >> 1) & 3))] =
          make_float4(__uint_as_float(r[c + 4 * ch]), __uint_as_float(r[c + 4 * ch + 1]),
                      __uint_as_float(r[c + 4 * ch + 2]), __uint_as_float(r[c + 4 * ch + 3]));
    __syncwarp();
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = 8 * i + (lane >> 2), qq = lane & 3;
      v[i] = buf[rr * 4 + (qq ^ ((rr >> 1) & 3))];
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = 8 * i + (lane >> 2);
      const Row ri = shfl_any(mine, rr);
      const int m = row0 + rr, n = n0 + c + 4 * (lane & 3);
      if (m < M && n < N) epi.store4(m, n, v[i], min(4, N - n), pre[i], ri);
    }
    }
    }
  }
  }
  if constexpr (Epi::kTmaReduce || Epi::kTmaStore) {
    if (lane == 0) bulk_wait_all();  // the adds / stores are done before the accumulator is released
    __syncwarp();
  }
}

template <int BN, int STAGES>
struct TcpSmem {
  static constexpr int kABytes = kTcBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStgOffset = STAGES * kStageBytes;  // epilogue transpose buffers
  static constexpr int kBarOffset = kStgOffset + kEpiWarps * kStageFloats * 4;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
};

// Persistent, warp-specialised C = A * W^T.  One CTA per SM walks the tiles
// t = blockIdx.x, + gridDim.x, ... (M-fastest, so CTAs running together share
// weight tiles in L2).  Roles:
//   warp 0 lane 0   TMA producer over a STAGES-deep ring (all tiles, one
//                   running k-block counter);
//   warp 1          allocates 2*BN TMEM columns (two accumulators); lane 0
//                   issues the tcgen05.mma of tile i into accumulator i % 2;
//   warps 2..17     epilogue: four warps per 32-lane TMEM quarter, each taking
//                   a quarter of the tile's columns; wait for accumulator
//                   i % 2, tcgen05.ld, hand 16-column runs to Epi, release
//                   the accumulator; this overlaps the MMAs of tile i + 1.
// All waits are bounded (common.cuh); a failed wait records an error and the
// CTA winds down.
template <typename TIn, int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    snai_tileproj_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                    int K, const __grid_constant__ Epi epi, int *err) {
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
      mbar_init(&tempty[a], kEpiWarps);
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
  // launched as a programmatic dependent: the set-up above (barriers, TMEM,
  // descriptor prefetch) overlapped the previous kernel's tail; nothing it
  // wrote is read before this wait.  The next kernel may then start its own
  // set-up (a GEMM's shared memory keeps it off this kernel's SMs).
  grid_dep_wait();
  grid_dep_launch();

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
    // epilogue warps: TMEM lane quarter = warp % 4, column quarter by warp
    const int q = warp & 3;
    const int c_lo = ((warp - 2) >> 2) * (BN / 4);
    int tc = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
      const int acc = tc & 1;
      {
        const int pm = (tile % num_m) * kTcBM + q * 32 + lane, pn = (tile / num_m) * BN + c_lo;
        if (pm < M && pn < N) epi.prefetch(pm, pn, min(BN / 4, N - pn));
      }
      if (!mbar_wait_bounded(&tfull[acc], (uint32_t)(tc >> 1) & 1u, err, kErrWaitAccum) ||
          *(volatile int *)cta_fail) {
        atomicExch(cta_fail, 1);
        break;
      }
      tc_fence_after();
      const int m0 = (tile % num_m) * kTcBM, n0 = (tile / num_m) * BN;
      const uint32_t tbase = tmem + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
      if (n0 + c_lo < N)
        drain_accumulator<BN / 4>(tbase + (uint32_t)c_lo, m0 + q * 32, M, n0 + c_lo, N, epi,
                                  reinterpret_cast<float *>(smem + Sm::kStgOffset) + (warp - 2) * kStageFloats);
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

// ============================================================================
// CTA-pair GEMM (tcgen05 cta_group::2): a cluster of two CTAs on two SMs
// computes one 256 x 256 tile.  Each CTA stages its own 128 rows of A and
// its own 128 rows of W (half of the tile's N) with TMA loads that complete
// on the leader CTA's barrier; the leader issues M=256, N=256 MMAs that read
// both CTAs' shared memory and write a 128 x 256 fp32 accumulator into each
// CTA's TMEM.  Per SM this moves 32 KB per 64-deep k-block for 128x256x64
// MACs, two thirds of the 128 x 256 single-CTA tile's bytes: the projections
// are bound by L2 -> SM bandwidth, not by the tensor cores.  Each CTA loads
// only its own halves: no load is shared between the two CTAs.
// ============================================================================

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity, int *err, int code) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_acq_cluster(bar, parity)) return true;
    if ((it & 63u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}
// 2-D tiled load into this CTA's shared memory, completing on a barrier of
// either CTA of the pair (cluster address); one destination CTA.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on `bar` in both CTAs of the pair once the pair MMAs issued so far
// are done: one commit to this CTA's barrier, one to the peer's (by its
// cluster address).
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar) {
  const uint32_t local = smem_u32(bar);
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(local)
               : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mapa_shared(local, 1))
               : "memory");
}

template <typename TIn>
__device__ __forceinline__ void tc_mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate);
template <>
__device__ __forceinline__ void tc_mma_pair<__nv_bfloat16>(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
template <>
__device__ __forceinline__ void tc_mma_pair<float>(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// M = 256, N = 256 instruction descriptor
template <typename TIn>
__device__ __forceinline__ constexpr uint32_t tc_idesc_pair() {
  return (1u << 4) | (TcKind<TIn>::kFmt << 7) | (TcKind<TIn>::kFmt << 10) | ((uint32_t)(256 >> 3) << 17) |
         ((uint32_t)(256 >> 4) << 24);
}

template <int STAGES>
struct Tc2Smem {
  static constexpr int kABytes = kTcBM * 128;  // this CTA's 128 rows of A, one 128-byte K slice each
  static constexpr int kBBytes = 128 * 128;    // this CTA's 128 rows of W
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStgOffset = STAGES * kStageBytes;  // epilogue transpose buffers
  static constexpr int kBarOffset = kStgOffset + kEpiWarps * kStageFloats * 4;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
};

// Persistent CTA-pair GEMM.  Pair p = blockIdx.x / 2 walks the 256 x 256
// tiles p, p + pairs, ... (M-fastest).  Roles as in snai_tileproj_tc_kernel; the MMA
// warp of the leader (cluster rank 0) issues for both CTAs, its commits
// arrive on both CTAs' barriers, and both CTAs' epilogue warps release an
// accumulator on the leader's barrier (kEpiWarps per CTA).  Every wait is
// bounded.
template <typename TIn, int STAGES, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    snai_pairproj_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                    int K, const __grid_constant__ Epi epi, int *err) {
  using Sm = Tc2Smem<STAGES>;
  constexpr int BK = TcKind<TIn>::kBK;
  constexpr int KSTEPS = BK / TcKind<TIn>::kUK;
  constexpr uint32_t IDESC = tc_idesc_pair<TIn>();
  constexpr uint32_t TCOLS = 512;  // two 256-column accumulators

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Sm::kBarOffset);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(tempty + 2);
  int *cta_fail = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + 255) / 256;
  const int num_tiles = num_m * ((N + 255) / 256);
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    *cta_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, TCOLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // programmatic dependent launch, as in the single-CTA kernel
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
        const int m0 = (tile % num_m) * 256 + (int)rank * 128;
        const int n0 = (tile / num_m) * 256 + (int)rank * 128;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, kErrWaitEmpty) || *(volatile int *)cta_fail) {
            atomicExch(cta_fail, 1);
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Sm::kStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
          uint8_t *st = smem + s * Sm::kStageBytes;
          tma_load_2d_pair(st, &tmA, fb, kb * BK, m0);
          tma_load_2d_pair(st + Sm::kABytes, &tmB, fb, kb * BK, n0);
        }
      }
      // the leader's full barriers also count the peer's copies: do not leave
      // while one into either CTA is in flight
      if (leader)
        for (int j = it - 1; j >= 0 && j >= it - STAGES; --j)
          if (!mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, err, kErrWaitDrain)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int it = 0, tc = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs, ++tc) {
        const int acc = tc & 1;
        if (!mbar_wait_cluster_bounded(&tempty[acc], ((uint32_t)(tc >> 1) & 1u) ^ 1u, err, kErrWaitEmpty)) {
          atomicExch(cta_fail, 1);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * 256);
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
            tc_mma_pair<TIn>(d, adesc + 2u * k, bdesc + 2u * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          tc_commit_pair(&empty[s]);
        }
        tc_commit_pair(&tfull[acc]);
      }
    }
  } else {
    // epilogue warps: TMEM lane quarter = warp % 4, column quarter by warp
    const int q = warp & 3;
    const int c_lo = ((warp - 2) >> 2) * 64;
    const uint32_t te0 = mapa_shared(smem_u32(&tempty[0]), 0), te1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int tc = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++tc) {
      const int acc = tc & 1;
      {
        const int pm = (tile % num_m) * 256 + (int)rank * 128 + q * 32 + lane, pn = (tile / num_m) * 256 + c_lo;
        if (pm < M && pn < N) epi.prefetch(pm, pn, min(64, N - pn));
      }
      if (!mbar_wait_bounded(&tfull[acc], (uint32_t)(tc >> 1) & 1u, err, kErrWaitAccum) ||
          *(volatile int *)cta_fail) {
        atomicExch(cta_fail, 1);
        break;
      }
      tc_fence_after();
      const int m0 = (tile % num_m) * 256 + (int)rank * 128, n0 = (tile / num_m) * 256;
      const uint32_t tbase = tmem + (uint32_t)(acc * 256) + ((uint32_t)(q * 32) << 16);
      if (n0 + c_lo < N)
        drain_accumulator<64>(tbase + (uint32_t)c_lo, m0 + q * 32, M, n0 + c_lo, N, epi,
                              reinterpret_cast<float *>(smem + Sm::kStgOffset) + (warp - 2) * kStageFloats);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? te1 : te0);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer is done with this CTA's TMEM and barriers
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, TCOLS);
}

}  // namespace snai
