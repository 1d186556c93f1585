// forward.cu - the .snai forward step on sm_100a (core/cortex.nim:487-563).
//
// A pass runs a list of rows (slot, position, token) through the model in
// chunks.  Per chunk:
//   embed_norm     h = E[token] (ids outside [0,V) read row 0, :493);
//                  x = RMSNorm(h, rms_att[0]); hist[slot][pos] = token
//   per layer l:   QKV projection -> RoPE, q rows, k/v appended to the cache
//                  attention      -> att (per row and head, positions 0..pos)
//                  Wo projection  -> h += .
//                  rmsnorm        -> x = RMSNorm(h, rms_ffn[l])
//                  W_up projection-> u = SiLU(.)
//                  W_down proj.   -> h += .
//                  rmsnorm        -> x = RMSNorm(h, rms_att[l+1])
//   rows that need logits: x = RMSNorm(h, rms_final) -> W_out projection.
// Projections run as fp32 GEMV in FP32 mode and as tcgen05 GEMMs
// (gemm_tc.cuh) in TF32 or BF16 mode, for any number of rows.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <climits>
#include <atomic>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "engine.h"
#include "epilogue.cuh"
#include "gemm_tc.cuh"

namespace snai {

// ============================================================================
// element-wise / row kernels
// ============================================================================

__global__ void fill_f32_kernel(float *dst, size_t n, float v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) dst[i] = v;
}

__global__ void to_bf16_kernel(const float *__restrict__ src, __nv_bfloat16 *__restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// Every tensor of a segment table in one launch: blockIdx.y picks the
// segment, the grid's x dimension strides over it with 4-element steps
// (every segment's length is a multiple of 4: d is).
__global__ void to_bf16_segments_kernel(const Bf16Segments segs) {
  const Bf16Segments::Seg s = segs.seg[blockIdx.y];
  const size_t n4 = s.n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(reinterpret_cast<const float4 *>(s.src) + i);
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t *>(&lo);
    pk.y = *reinterpret_cast<uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(s.dst + 4 * i) = pk;
  }
}

constexpr int kNormThreads = 256;

// The block's sum of its threads' partial sums: warp sums, then the warps'
// in warp order (every thread gets it).
__device__ __forceinline__ float block_reduce_sum(float s, float *red) {
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  __syncthreads();
  return t;
}

// Block sum of squares of a D-vector (parallel tree; the reference sums
// sequentially, core/cortex.nim:119).
__device__ __forceinline__ float block_sumsq(const float *x, int D, float *red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) s = __fmaf_rn(x[i], x[i], s);
  return block_reduce_sum(s, red);
}

// 1 / sqrt(ss/D + 1e-5), in the reference's float operations (:121).
__device__ __forceinline__ float rms_inv(float ss, int D) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
}

// rms_inv of a D-row computed by one warp in exactly the operations and order
// of block_sumsq in a kNormThreads CTA (virtual warp w = threads 32w..32w+31),
// so a GEMV that normalises its own input rows reads the values the norm
// kernel would have written.
template <bool COHERENT = false>
__device__ __forceinline__ float warp_row_rms_inv(const float *__restrict__ hr, int D, int lane) {
  constexpr int NW = kNormThreads / 32;
  float p[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) p[w] = 0.f;
  // 4 * kNormThreads elements per round, all loads in flight before the
  // sums; a missing element adds 0 * 0, which leaves the sum as it is
  for (int base = 0; base < D; base += 4 * kNormThreads) {
    float v[NW][4];
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = base + 32 * w + lane + kNormThreads * j;
        v[w][j] = i < D ? (COHERENT ? __ldcg(hr + i) : __ldg(hr + i)) : 0.f;
      }
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int j = 0; j < 4; ++j) p[w] = __fmaf_rn(v[w][j], v[w][j], p[w]);
  }
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) t += warp_sum(p[w]);
  return rms_inv(t, D);
}

// The rows of a pass of at most kRowPackMax rows, passed by value to the
// pass's first kernel (the embedding kernel, or the QKV GEMV that does its
// work), which writes them to the device row arrays for the later kernels of
// the pass (so the pass needs no host-to-device copy), and to the split
// attention, which reads its row before its dependency wait.  n = 0: the rows
// are on the device already.
constexpr int kRowPackMax = 8;
struct RowPack {
  RowDesc r[kRowPackMax];
  int2 out[kRowPackMax];
  int n, n_out;
};

// h[m] = emb[token], x[m] = RMSNorm(h[m], w); the token into the history.
// Rows of D <= 16 * kNormThreads keep their values in registers between the
// copy and the norm (the same sums as block_sumsq over h).
template <typename TA>
__global__ void __launch_bounds__(kNormThreads) embed_norm_kernel(const RowDesc *rows, const RowPack pk,
                                                                  RowDesc *rows_w,
                                                                  int2 *__restrict__ outrows_w,
                                                                  const int *__restrict__ tokens_d,
                                                                  const float *__restrict__ emb,
                                                                  const float *__restrict__ w, float *__restrict__ h,
                                                                  TA *__restrict__ x, int *__restrict__ hist,
                                                                  int *__restrict__ seq_len, int V, int D, int ctx) {
  constexpr int RV = 16;
  __shared__ float red[kNormThreads / 32];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const RowDesc rd = pk.n ? pk.r[m] : rows[m];
  if (pk.n) {
    if (threadIdx.x == 0) rows_w[m] = rd;
    if (m == 0 && (int)threadIdx.x < pk.n_out) outrows_w[threadIdx.x] = pk.out[threadIdx.x];
  }
  const int raw = tokens_d ? tokens_d[rd.token] : rd.token;
  const int tid = (raw < 0 || raw >= V) ? 0 : raw;
  const float *e = emb + (size_t)tid * D;
  float *hr = h + (size_t)m * D;
  if (threadIdx.x == 0) {
    hist[(size_t)rd.slot * ctx + rd.pos] = raw;
    atomicMax(&seq_len[rd.slot], rd.pos + 1);
  }
  TA *xr = x + (size_t)m * D;
  if (D <= RV * kNormThreads) {
    float v[RV];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      v[j] = i < D ? e[i] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < D) {
        hr[i] = v[j];
        s = __fmaf_rn(v[j], v[j], s);
      }
    }
    const float inv = rms_inv(block_reduce_sum(s, red), D);
#pragma unroll
    for (int j = 0; j < RV; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < D) ActIO<TA>::store(xr + i, __fmul_rn(__fmul_rn(v[j], inv), w[i]));
    }
    return;
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) hr[i] = e[i];
  __syncthreads();
  const float inv = rms_inv(block_sumsq(hr, D, red), D);
  for (int i = threadIdx.x; i < D; i += blockDim.x) ActIO<TA>::store(xr + i, __fmul_rn(__fmul_rn(hr[i], inv), w[i]));
}

// x[i] = RMSNorm(h[src(i)], w); src(i) = i, or outrows[i].x when gathering.
template <typename TA>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float *__restrict__ h, const int2 *__restrict__ gather,
                                                               const float *__restrict__ w, TA *__restrict__ x, int D) {
  __shared__ float red[kNormThreads / 32];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const int src = gather ? gather[m].x : m;
  const float *hr = h + (size_t)src * D;
  const float inv = rms_inv(block_sumsq(hr, D, red), D);
  TA *xr = x + (size_t)m * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ActIO<TA>::store(xr + i, __fmul_rn(__fmul_rn(hr[i], inv), w[i]));
}

// ============================================================================
// attention over the KV cache (core/cortex.nim:512-538)
// ============================================================================
//
// One CTA per (row, head).  Scores s_t = (q . k_t) / sqrtf(hs) for t <= pos go
// to shared memory; max starts at -9999 as in the reference (:517); then
// e_t = exp(s_t - max), the sum, w_t = e_t / sum, and att = sum_t w_t v_t.
// Channels >= heads*hs of att are zero (:512-513).
//
// Fast path HS = 64: a warp reads two positions per load instruction (16
// lanes x 16 bytes per 256-byte key row), so every load is a contiguous
// 512-byte span of the head-major cache.

constexpr int kAttThreads = 128;

template <typename TA>
__device__ __forceinline__ void att_zero_tail(TA *out_row, int att_ch, int D) {
  for (int c = att_ch + threadIdx.x; c < D; c += blockDim.x) ActIO<TA>::store(out_row + c, 0.f);
}

// softmax over s[0..n) in place: s_t <- exp(s_t - max)/sum.  Returns nothing;
// uses red[32] scratch.
__device__ __forceinline__ void att_softmax(float *s, int n, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float mx = -9999.0f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) mx = fmaxf(mx, s[t]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < nw; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float e = expf(__fsub_rn(s[t], mx));
    s[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < nw; ++w) sum += red[w];
  for (int t = threadIdx.x; t < n; t += blockDim.x) s[t] = __fdiv_rn(s[t], sum);
  __syncthreads();
}

// RoPE of one 4-channel group (two pairs) with (cos, sin) of both pairs
// (core/cortex.nim:74-87).
__device__ __forceinline__ float4 rope4(float4 v, float4 c) {
  return make_float4(__fsub_rn(__fmul_rn(v.x, c.x), __fmul_rn(v.y, c.y)),
                     __fadd_rn(__fmul_rn(v.x, c.y), __fmul_rn(v.y, c.x)),
                     __fsub_rn(__fmul_rn(v.z, c.z), __fmul_rn(v.w, c.w)),
                     __fadd_rn(__fmul_rn(v.z, c.w), __fmul_rn(v.w, c.z)));
}

// ---- attention of passes with few rows, head size 64: a chunked formula ----
//
// The whole-row kernel below (a CTA per (row, head), the passes of many
// rows) computes the reference's order: all scores, max, exponentials, sum,
// weights, weighted values.  Passes with few rows (rows x heads below the SM
// count) need more CTAs per (row, head), so the split kernel, and the
// persistent one-row pass kernel, compute a chunked formula instead:
// the positions 0..n-1 of a (row, head) are cut into chunks of 64 (4 warps x
// 8 position pairs).  Warp w of a chunk loads the K and V rows of its 8 pairs
// at once (a warp reads two 256-byte rows per instruction, so every load is a
// contiguous 512-byte span of the head-major cache) and computes
//   m_w = max(-9999, s_t) (the reference's initialisation, core/cortex.nim:517),
//   l_w = sum exp(s_t - m_w),  o_w = sum exp(s_t - m_w) v_t   (t in pair order),
// s_t = (q . k_t) / sqrtf(hs).  A chunk's four warps combine in warp order:
//   M_c = max_w m_w,  L_c = sum_w exp(m_w - M_c) l_w,  O_c = sum_w exp(m_w - M_c) o_w,
// and the chunks in chunk order:
//   M = max(-9999, M_c),  att = (sum_c exp(M_c - M) O_c) / (sum_c exp(M_c - M) L_c).
// The split kernel and the pass kernel run exactly these operations, so a
// row's attention has the same bits in either; against the whole-row kernel
// they differ by rounding (a few fp32 ulps), so a row's bits depend on
// whether its pass has few rows.  (A chunked whole-row kernel was measured
// 8-10 % slower than the one below at the d=1024 benchmark's HBM roofline,
// so passes of many rows keep the reference's order.)  Channels >=
// heads*hs of att are zero (:512-513).
//
// kvs non-null (a decode pass, one row per slot): K and V of position pos
// come from the row's staging entry ([M, 2, att_ch], without RoPE, as q) and
// are appended to the cache here, where the slot's cache pages are read
// anyway; RoPE of q and k is applied here then.
constexpr int kAttChunk = 64;  // positions per chunk
constexpr int kAttPW = 68;     // floats per partial: max, sum, (pad), 64 weighted value sums from [4]
constexpr int kSplitCounters = 256;  // (row, head) arrival counters of the split kernel
constexpr int kSplitMax = 128;       // chunks (= CTAs) per (row, head) in the split kernel: ctx <= 8192

struct AttRow {
  float *kbase, *vbase;
  float4 qv, knew, vnew;
  int n, nc;  // positions, and positions below nc read from the cache
};

// The row's q (rotated in a decode pass), its cache pointers and the staged
// K/V of position pos.  `append` writes the staged row to the cache (one
// warp of one CTA per (row, head)).
// COHERENT: q and the staged K/V were written earlier in the same kernel by
// other CTAs (the persistent pass kernel): read them from L2.
template <bool COHERENT = false>
__device__ __forceinline__ AttRow att_row(const RowDesc &rd, const float *__restrict__ q, float *__restrict__ kv,
                                          int m, int head, int att_ch, size_t slot_stride, size_t layer_off,
                                          size_t part_stride, size_t head_stride, const float *__restrict__ kvs,
                                          const float2 *__restrict__ rope, bool append,
                                          const float4 *cs_pre = nullptr) {
  constexpr int HS = 64;
  const int lane = threadIdx.x & 31, half = lane >> 4, pi = lane & 15;
  AttRow r;
  r.n = rd.pos + 1;
  r.nc = kvs ? r.n - 1 : r.n;
  r.kbase = kv + (size_t)rd.slot * slot_stride + layer_off + (size_t)head * head_stride;
  r.vbase = r.kbase + part_stride;
  auto ld4 = [](const float *p) {
    return COHERENT ? __ldcg(reinterpret_cast<const float4 *>(p)) : *reinterpret_cast<const float4 *>(p);
  };
  r.qv = ld4(q + (size_t)m * att_ch + head * HS + pi * 4);
  r.knew = make_float4(0.f, 0.f, 0.f, 0.f);
  r.vnew = r.knew;
  if (kvs) {
    const float *kst = kvs + (size_t)m * 2 * att_ch + head * HS;
    const float4 cs = cs_pre ? *cs_pre : *reinterpret_cast<const float4 *>(rope + (size_t)rd.pos * (HS / 2) + pi * 2);
    r.qv = rope4(r.qv, cs);
    r.knew = rope4(ld4(kst + pi * 4), cs);
    r.vnew = ld4(kst + att_ch + pi * 4);
    if (append)  // lanes 0..15 the K row, lanes 16..31 the V row
      *reinterpret_cast<float4 *>((half ? r.vbase : r.kbase) + (size_t)rd.pos * HS + pi * 4) = half ? r.vnew : r.knew;
  }
  return r;
}

// Warp `warp` (0..3)'s K and V rows of the chunk starting at t0 that come
// from the cache (positions below nc; zero elsewhere).
constexpr int kAttU = 8;  // position pairs per warp of a chunk
__device__ __forceinline__ void att_chunk_load(const float *kbase, const float *vbase, int nc, int n, int t0, int warp,
                                               float4 (&kr)[kAttU], float4 (&vr)[kAttU]) {
  constexpr int HS = 64, U = kAttU;
  const int lane = threadIdx.x & 31, half = lane >> 4, pi = lane & 15;
  const int t1 = min(n, t0 + kAttChunk);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int t = t0 + 2 * (warp * U + u) + half;
    const bool cached = t < min(nc, t1);
    kr[u] = cached ? __ldcs(reinterpret_cast<const float4 *>(kbase + (size_t)t * HS + pi * 4))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    vr[u] = cached ? __ldcs(reinterpret_cast<const float4 *>(vbase + (size_t)t * HS + pi * 4))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Warp `warp` (0..3)'s (m_w, l_w, o_w) of the chunk starting at t0 into wp
// (kAttPW floats), from its cached rows (att_chunk_load) and the new position's.
__device__ __forceinline__ void att_chunk_compute(const AttRow &r, int t0, float sqrt_hs, float *wp, int warp,
                                                  float4 (&kr)[kAttU], float4 (&vr)[kAttU]) {
  constexpr int U = kAttU;
  const int lane = threadIdx.x & 31, half = lane >> 4, pi = lane & 15;
  const int t1 = min(r.n, t0 + kAttChunk);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int t = t0 + 2 * (warp * U + u) + half;
    if (!(t < min(r.nc, t1)) && t < t1) {
      kr[u] = r.knew;
      vr[u] = r.vnew;
    }
  }
  float sc[U];
  float mx = -9999.0f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    float d = r.qv.x * kr[u].x + r.qv.y * kr[u].y + r.qv.z * kr[u].z + r.qv.w * kr[u].w;
    d += __shfl_xor_sync(0xffffffffu, d, 8);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    sc[u] = __fdiv_rn(d, sqrt_hs);
    if (t0 + 2 * (warp * U + u) + half < t1) mx = fmaxf(mx, sc[u]);
  }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
  // each position's exponential once: lane u of a half computes it for its
  // half's position u, the half's lanes read it by shuffle
  float own = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (pi == u) own = expf(__fsub_rn(sc[u], mx));
  float ls = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const float e = __shfl_sync(0xffffffffu, own, (lane & 16) | u);
    if (t0 + 2 * (warp * U + u) + half < t1) {
      ls = __fadd_rn(ls, e);
      o.x = __fadd_rn(o.x, __fmul_rn(vr[u].x, e));
      o.y = __fadd_rn(o.y, __fmul_rn(vr[u].y, e));
      o.z = __fadd_rn(o.z, __fmul_rn(vr[u].z, e));
      o.w = __fadd_rn(o.w, __fmul_rn(vr[u].w, e));
    }
  }
  ls = __fadd_rn(ls, __shfl_xor_sync(0xffffffffu, ls, 16));
  o.x = __fadd_rn(o.x, __shfl_xor_sync(0xffffffffu, o.x, 16));
  o.y = __fadd_rn(o.y, __shfl_xor_sync(0xffffffffu, o.y, 16));
  o.z = __fadd_rn(o.z, __shfl_xor_sync(0xffffffffu, o.z, 16));
  o.w = __fadd_rn(o.w, __shfl_xor_sync(0xffffffffu, o.w, 16));
  if (lane < 16) *reinterpret_cast<float4 *>(wp + 4 + 4 * pi) = o;
  if (lane == 0) {
    wp[0] = mx;
    wp[1] = ls;
  }
}

// Warp `warp` (0..3)'s (m_w, l_w, o_w) of the chunk starting at t0 into wp (kAttPW floats).
__device__ __forceinline__ void att_warp_chunk(const AttRow &r, int t0, float sqrt_hs, float *wp, int warp) {
  float4 kr[kAttU], vr[kAttU];
  att_chunk_load(r.kbase, r.vbase, r.nc, r.n, t0, warp, kr, vr);
  att_chunk_compute(r, t0, sqrt_hs, wp, warp, kr, vr);
}

// Channel ch (< 64) of a chunk's partial from its four warps' (warp order).
__device__ __forceinline__ void att_chunk_combine(const float *wp4, int ch, float *dst) {
  float M = wp4[0];
#pragma unroll
  for (int w = 1; w < 4; ++w) M = fmaxf(M, wp4[w * kAttPW]);
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float s = expf(__fsub_rn(wp4[w * kAttPW], M));
    L = __fadd_rn(L, __fmul_rn(s, wp4[w * kAttPW + 1]));
    O = __fadd_rn(O, __fmul_rn(s, wp4[w * kAttPW + 4 + ch]));
  }
  dst[4 + ch] = O;
  if (ch == 0) {
    dst[0] = M;
    dst[1] = L;
  }
}

// Channel ch of att from C chunk partials (chunk order); LD reads a float.
template <class LD>
__device__ __forceinline__ float att_merge(const float *cp, int C, int ch, LD ld) {
  float M = -9999.0f;
  for (int c = 0; c < C; ++c) M = fmaxf(M, ld(cp + c * kAttPW));
  float L = 0.f, O = 0.f;
  for (int c = 0; c < C; ++c) {
    const float s = expf(__fsub_rn(ld(cp + c * kAttPW), M));
    L = __fadd_rn(L, __fmul_rn(s, ld(cp + c * kAttPW + 1)));
    O = __fadd_rn(O, __fmul_rn(s, ld(cp + c * kAttPW + 4 + ch)));
  }
  return __fdiv_rn(O, L);
}

// Whole-row kernel: one CTA per (row, head).  Scores s_t = (q . k_t) /
// sqrtf(hs) for t <= pos go to shared memory; max starts at -9999 as in the
// reference (:517); then e_t = exp(s_t - max), the sum, w_t = e_t / sum, and
// att = sum_t w_t v_t.  A warp reads two positions per load instruction (16
// lanes x 16 bytes per 256-byte key row), so every load is a contiguous
// 512-byte span of the head-major cache.
// kvs non-null: K and V of position pos come from the row's staging entry
// ([M, 2, att_ch], without RoPE, as q) and are appended to the cache here,
// where the slot's cache pages are being read anyway (one row per slot in
// the pass); RoPE of q and k is applied here then.
template <typename TA>
__global__ void __launch_bounds__(kAttThreads) attention_hs64_kernel(
    const RowDesc *__restrict__ rows, const float *__restrict__ q, float *__restrict__ kv, TA *__restrict__ out,
    int D, int att_ch, size_t slot_stride, size_t layer_off, size_t part_stride, size_t head_stride, float sqrt_hs,
    const float *__restrict__ kvs, const float2 *__restrict__ rope) {
  constexpr int HS = 64;
  extern __shared__ float smem_att[];
  float *red = smem_att;        // [32]
  float *acc = smem_att + 32;   // [4 warps][64]
  float *s = smem_att + 32 + 4 * HS;
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.y, head = blockIdx.x;
  const RowDesc rd = rows[m];
  const int n = rd.pos + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = lane >> 4, part = lane & 15;

  float *kbase = kv + (size_t)rd.slot * slot_stride + layer_off + (size_t)head * head_stride;
  float *vbase = kbase + part_stride;
  float4 qv = *reinterpret_cast<const float4 *>(q + (size_t)m * att_ch + head * HS + part * 4);
  // cache positions below nc; position pos from the staging entry when deferred
  const int nc = kvs ? n - 1 : n;
  const float *kst = kvs ? kvs + (size_t)m * 2 * att_ch + head * HS : nullptr;
  const float *vst = kvs ? kst + att_ch : nullptr;
  float4 knew = make_float4(0.f, 0.f, 0.f, 0.f), vnew = knew;
  if (kvs) {
    const float4 cs = *reinterpret_cast<const float4 *>(rope + (size_t)rd.pos * (HS / 2) + part * 2);
    qv = rope4(qv, cs);
    knew = rope4(*reinterpret_cast<const float4 *>(kst + part * 4), cs);
    vnew = *reinterpret_cast<const float4 *>(vst + part * 4);
    if (warp == 0)  // append: lanes 0..15 the K row, lanes 16..31 the V row
      *reinterpret_cast<float4 *>((half ? vbase : kbase) + (size_t)rd.pos * HS + part * 4) = half ? vnew : knew;
  }

  // ---- scores: warp w takes position pairs w, w+4, ...; 8 pairs per sweep ----
  constexpr int U = 8;
  for (int p0 = warp * U; 2 * p0 < n; p0 += 4 * U) {
    float4 kr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = 2 * (p0 + u) + half;
      kr[u] = t < nc   ? __ldcs(reinterpret_cast<const float4 *>(kbase + (size_t)t * HS + part * 4))
              : t < n ? knew
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float d = qv.x * kr[u].x + qv.y * kr[u].y + qv.z * kr[u].z + qv.w * kr[u].w;
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      const int t = 2 * (p0 + u) + half;
      if (part == 0 && t < n) s[t] = __fdiv_rn(d, sqrt_hs);
    }
  }
  __syncthreads();
  att_softmax(s, n, red);

  // ---- weighted sum of values ----
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int p0 = warp * U; 2 * p0 < n; p0 += 4 * U) {
    float4 vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = 2 * (p0 + u) + half;
      vr[u] = t < nc   ? __ldcs(reinterpret_cast<const float4 *>(vbase + (size_t)t * HS + part * 4))
              : t < n ? vnew
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = 2 * (p0 + u) + half;
      const float wt = t < n ? s[t] : 0.f;
      a.x = __fadd_rn(a.x, __fmul_rn(vr[u].x, wt));
      a.y = __fadd_rn(a.y, __fmul_rn(vr[u].y, wt));
      a.z = __fadd_rn(a.z, __fmul_rn(vr[u].z, wt));
      a.w = __fadd_rn(a.w, __fmul_rn(vr[u].w, wt));
    }
  }
  a.x += __shfl_xor_sync(0xffffffffu, a.x, 16);
  a.y += __shfl_xor_sync(0xffffffffu, a.y, 16);
  a.z += __shfl_xor_sync(0xffffffffu, a.z, 16);
  a.w += __shfl_xor_sync(0xffffffffu, a.w, 16);
  if (half == 0) *reinterpret_cast<float4 *>(acc + warp * HS + part * 4) = a;
  __syncthreads();
  TA *orow = out + (size_t)m * D;
  if (threadIdx.x < HS) {
    const float r = acc[threadIdx.x] + acc[HS + threadIdx.x] + acc[2 * HS + threadIdx.x] + acc[3 * HS + threadIdx.x];
    ActIO<TA>::store(orow + head * HS + threadIdx.x, r);
  }
  if (head == gridDim.x - 1) att_zero_tail(orow, att_ch, D);
}

// Split kernel for passes of few rows (rows x heads below the SM count, e.g.
// the one-row decode pass of the PHP host): CTA (head, row, c) computes chunk
// c (when the row has it) into part[row][head][c]; the last CTA of the
// (row, head) to arrive (an arrival counter, reset by it for the next launch;
// nobody waits on it) merges the chunks.  gridDim.z = ceil(ctx / 64), so a
// captured launch serves every later step.
template <typename TA>
__global__ void __launch_bounds__(kAttThreads) attention_split_hs64_kernel(
    const RowDesc *__restrict__ rows, const RowPack pk, const float *__restrict__ q, float *__restrict__ kv,
    TA *__restrict__ out, int D, int att_ch, size_t slot_stride, size_t layer_off, size_t part_stride,
    size_t head_stride, float sqrt_hs, const float *__restrict__ kvs, const float2 *__restrict__ rope,
    float *__restrict__ part, int *__restrict__ cnt) {
  constexpr int HS = 64;
  __shared__ __align__(16) float wp4[4 * kAttPW];
  __shared__ int is_last;
  const int head = blockIdx.x, m = blockIdx.y, c = blockIdx.z, S = gridDim.z, H = gridDim.x;
  const int warp = threadIdx.x >> 5, pi = threadIdx.x & 15;
  // A decode pass whose rows came by value: the row, this chunk's cached K
  // and V rows and the RoPE factors are read before the wait for the
  // previous kernel (QKV), which writes none of them: earlier passes wrote
  // the cache, and no kernel of this pass starts before the previous pass
  // has finished (the pass's first kernel, the embedding kernel or the QKV
  // GEMV that does its work, waits before it lets the next one start).
  const bool early = pk.n > 0 && kvs != nullptr;
  float4 kr[kAttU], vr[kAttU], cs = make_float4(0.f, 0.f, 0.f, 0.f);
  RowDesc rd = early ? pk.r[m] : RowDesc{};
  if (early) {
    const int n = rd.pos + 1;
    if (c * kAttChunk < n) {
      const float *kbase = kv + (size_t)rd.slot * slot_stride + layer_off + (size_t)head * head_stride;
      att_chunk_load(kbase, kbase + part_stride, n - 1, n, c * kAttChunk, warp, kr, vr);
      cs = *reinterpret_cast<const float4 *>(rope + (size_t)rd.pos * (HS / 2) + pi * 2);
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  if (!early) rd = rows[m];
  const int n = rd.pos + 1, C = (n + kAttChunk - 1) / kAttChunk;
  float *pp = part + (size_t)(m * H + head) * S * kAttPW;
  // the row's C chunks take part; the other CTAs of the (row, head) leave
  if (c >= C) return;
  TA *orow = out + (size_t)m * D;
  const AttRow r = att_row(rd, q, kv, m, head, att_ch, slot_stride, layer_off, part_stride, head_stride, kvs, rope,
                           warp == 0 && c == (n - 1) / kAttChunk, early ? &cs : nullptr);
  if (!early) att_chunk_load(r.kbase, r.vbase, r.nc, r.n, c * kAttChunk, warp, kr, vr);
  att_chunk_compute(r, c * kAttChunk, sqrt_hs, wp4 + warp * kAttPW, warp, kr, vr);
  __syncthreads();
  if (C == 1) {
    // one chunk: its partial (att_chunk_combine's operations) and the merge
    // of that one partial (att_merge's), in registers, straight to att
    if (threadIdx.x < HS) {
      const int ch = threadIdx.x;
      float Mc = wp4[0];
#pragma unroll
      for (int w = 1; w < 4; ++w) Mc = fmaxf(Mc, wp4[w * kAttPW]);
      float Lc = 0.f, Oc = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float s = expf(__fsub_rn(wp4[w * kAttPW], Mc));
        Lc = __fadd_rn(Lc, __fmul_rn(s, wp4[w * kAttPW + 1]));
        Oc = __fadd_rn(Oc, __fmul_rn(s, wp4[w * kAttPW + 4 + ch]));
      }
      const float Mm = fmaxf(-9999.0f, Mc);
      const float s = expf(__fsub_rn(Mc, Mm));
      const float L = __fadd_rn(0.f, __fmul_rn(s, Lc)), O = __fadd_rn(0.f, __fmul_rn(s, Oc));
      ActIO<TA>::store(orow + head * HS + ch, __fdiv_rn(O, L));
    }
    if (head == H - 1) att_zero_tail(orow, att_ch, D);
    return;
  }
  if (threadIdx.x < HS) att_chunk_combine(wp4, threadIdx.x, pp + c * kAttPW);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(&cnt[m * H + head], 1) == C - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x < HS)
    ActIO<TA>::store(orow + head * HS + threadIdx.x,
                     att_merge(pp, C, threadIdx.x, [](const float *p) { return __ldcg(p); }));
  if (threadIdx.x == 0) cnt[m * H + head] = 0;
  if (head == H - 1) att_zero_tail(orow, att_ch, D);
}

// Any even head size: threads take positions for the scores and channels for
// the weighted sum.
template <typename TA>
__global__ void __launch_bounds__(kAttThreads) attention_generic_kernel(
    const RowDesc *__restrict__ rows, const float *__restrict__ q, float *__restrict__ kv, TA *__restrict__ out,
    int D, int att_ch, int hs, size_t slot_stride, size_t layer_off, size_t part_stride, size_t head_stride,
    float sqrt_hs, const float *__restrict__ kvs, const float2 *__restrict__ rope) {
  extern __shared__ float smem_att[];
  float *red = smem_att;
  float *s = smem_att + 32;
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.y, head = blockIdx.x;
  const RowDesc rd = rows[m];
  const int n = rd.pos + 1;
  float *kbase = kv + (size_t)rd.slot * slot_stride + layer_off + (size_t)head * head_stride;
  float *vbase = kbase + part_stride;
  const float *qr = q + (size_t)m * att_ch + (size_t)head * hs;
  const float *kst = kvs ? kvs + (size_t)m * 2 * att_ch + (size_t)head * hs : nullptr;
  const float *vst = kvs ? kst + att_ch : nullptr;
  float *qrot = smem_att + 32 + n;  // [hs] q after RoPE (deferred mode)
  float *krot = qrot + hs;          // [hs] new k after RoPE
  if (kvs) {
    // RoPE of q and of the new k (the staging entries hold them unrotated)
    for (int p = threadIdx.x; p < hs / 2; p += blockDim.x) {
      const float2 cs = rope[(size_t)rd.pos * (hs / 2) + p];
      const float a = qr[2 * p], b = qr[2 * p + 1], ka = kst[2 * p], kb = kst[2 * p + 1];
      qrot[2 * p] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
      qrot[2 * p + 1] = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
      krot[2 * p] = __fsub_rn(__fmul_rn(ka, cs.x), __fmul_rn(kb, cs.y));
      krot[2 * p + 1] = __fadd_rn(__fmul_rn(ka, cs.y), __fmul_rn(kb, cs.x));
    }
    __syncthreads();
    for (int j = threadIdx.x; j < 2 * hs; j += blockDim.x)
      (j < hs ? kbase : vbase)[(size_t)rd.pos * hs + (j % hs)] = (j < hs ? krot : vst)[j % hs];
    qr = qrot;
  }
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float *kr = (kvs && t == n - 1) ? krot : kbase + (size_t)t * hs;
    float d = 0.f;
    for (int j = 0; j < hs; ++j) d = __fadd_rn(d, __fmul_rn(qr[j], kr[j]));
    s[t] = __fdiv_rn(d, sqrt_hs);
  }
  __syncthreads();
  att_softmax(s, n, red);
  TA *orow = out + (size_t)m * D;
  for (int j = threadIdx.x; j < hs; j += blockDim.x) {
    float a = 0.f;
    for (int t = 0; t < n; ++t)
      a = __fadd_rn(a, __fmul_rn((kvs && t == n - 1) ? vst[j] : vbase[(size_t)t * hs + j], s[t]));
    ActIO<TA>::store(orow + (size_t)head * hs + j, a);
  }
  if (head == gridDim.x - 1) att_zero_tail(orow, att_ch, D);
}

// ============================================================================
// fp32 GEMV for small row counts: C[M,N] = X[M,K] * W[N,K]^T
// ============================================================================
//
// A warp owns four consecutive weight rows (two RoPE pairs) over one slice of
// K; the S warps of a row quad split K between them and P quads share a CTA
// (S * P <= 8 warps).  A pass covers up to 512 columns of the slice: each
// lane loads its 4 x 16 weights of the pass into registers at once (8 KB of
// loads in flight per warp), so with one pass per slice (K <= 4096) a quad is
// read from HBM once whatever M is.  Activation rows come through L1 in
// groups of MB; the 4 * MB partial dot products of a group are summed over
// the warp by a transposing butterfly (a stage halves the values each lane
// keeps, so a group costs about 4 * MB shuffles instead of 20 * MB), the S
// slice sums are added in slice order through shared memory, and the lanes
// owning an even row emit (row, row + 1) pairs to the epilogue.
//
// With NORM the input rows are RMSNorm(X[src(m)], nw) (src(m) = m, or
// gather[m].x): each warp computes the rows' rms_inv itself, so a pass of at
// most a few rows needs no separate norm launch.

constexpr int kGemvMaxWarps = 8;
constexpr int kGemvPass = 512;  // K columns per warp pass: 4 float4 per lane per row

// Butterfly reduce-scatter over the warp: stage O (16, 8, ...) pairs lane
// with lane ^ O; while a lane holds C > 1 values it keeps the lower or upper
// half (by lane & O) and adds the partner's copy of that half.  Afterwards
// the lane holds in v[0] the warp sum of value lane / (32 / NV).
template <int C, int O, int NV>
__device__ __forceinline__ void gemv_reduce(float (&v)[NV], int lane) {
  if constexpr (O > 0) {
    if constexpr (C > 1) {
      constexpr int H = C / 2;
      const bool up = (lane & O) != 0;
#pragma unroll
      for (int j = 0; j < H; ++j) {
        const float send = up ? v[j] : v[j + H];
        const float keep = up ? v[j + H] : v[j];
        v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, O));
      }
      gemv_reduce<H, O / 2, NV>(v, lane);
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], O));
      gemv_reduce<1, O / 2, NV>(v, lane);
    }
  }
}

// The first QKV GEMV of a one-row pass whose row came by value also does the
// embedding kernel's work: X is the embedding table, the row's token picks
// the input row, and CTA 0 writes h, the history and the pass's row
// descriptors (after the wait for the previous kernel, which may read them).
struct GemvEmbed {
  const int *tokens_d;  // the row's token: tokens_d[r.token], or r.token when nullptr
  float *h;
  int *hist, *seq_len;
  int V, ctx;
  RowDesc *rows_w;
  int2 *outrows_w;
};

struct GemvNorm {
  const float *w;       // RMSNorm weights [K]; nullptr: X is the input as is
  const int2 *gather;   // input row m = X[gather[m].x], or X[m] when nullptr
  int emb = 0;          // 1: the embedding fold above (one row, staged-tile kernel)
  GemvEmbed ef{};
  RowPack pk{};
};

template <int MB, bool NORM, class Epi>
__global__ void __launch_bounds__(kGemvMaxWarps * 32, 2)
    snai_rowproj_f32_kernel(const float *__restrict__ W, int N, int K, const float *__restrict__ X, int M, int S, int slice,
                    Epi epi, GemvNorm nrm) {
  constexpr int NV = 4 * MB;   // values a lane reduces per group: [m][row]
  constexpr int G = 32 / NV;   // lanes holding each reduced value
  __shared__ float part[kGemvMaxWarps][NV];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = warp % S;
  const int n0 = (blockIdx.x * (blockDim.x >> 5) / S + warp / S) * 4;
  const bool live = n0 < N;
  const int ks = s * slice, ke = min(K, ks + slice);
  const int passes = ke > ks ? (ke - ks + kGemvPass - 1) / kGemvPass : 0;
  float4 w[4][4];
  auto load_w = [&](int kb) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = kb + lane * 4 + 128 * i;
        w[r][i] = (live && n0 + r < N && k < ke)
                      ? __ldcg(reinterpret_cast<const float4 *>(W + (size_t)(n0 + r) * K + k))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
  };
  auto dot_group = [&](int kb, int m0, float (&acc)[NV]) {
#pragma unroll
    for (int j = 0; j < MB; ++j) {
      if (m0 + j >= M) break;
      const float *xr;
      float inv = 1.f;
      if constexpr (NORM) {
        xr = X + (size_t)(nrm.gather ? nrm.gather[m0 + j].x : m0 + j) * K;
        inv = warp_row_rms_inv(xr, K, lane);
      } else {
        xr = X + (size_t)(m0 + j) * K;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = kb + lane * 4 + 128 * i;
        if (k < ke) {
          float4 xv = __ldg(reinterpret_cast<const float4 *>(xr + k));
          if constexpr (NORM) {
            const float4 nw = __ldg(reinterpret_cast<const float4 *>(nrm.w + k));
            xv.x = __fmul_rn(__fmul_rn(xv.x, inv), nw.x);
            xv.y = __fmul_rn(__fmul_rn(xv.y, inv), nw.y);
            xv.z = __fmul_rn(__fmul_rn(xv.z, inv), nw.z);
            xv.w = __fmul_rn(__fmul_rn(xv.w, inv), nw.w);
          }
#pragma unroll
          for (int r = 0; r < 4; ++r)
            acc[4 * j + r] = fmaf(w[r][i].x, xv.x, fmaf(w[r][i].y, xv.y, fmaf(w[r][i].z, xv.z,
                                                                               fmaf(w[r][i].w, xv.w, acc[4 * j + r]))));
        }
      }
    }
  };
  // nothing before the wait reads what an earlier kernel writes: the next
  // kernel may start at once (it waits for this one in turn), and with one
  // pass the weights are in flight before the wait for the previous results
  grid_dep_launch();
  if (passes == 1) load_w(ks);
  grid_dep_wait();
  for (int m0 = 0; m0 < M; m0 += MB) {
    float acc[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[j] = 0.f;
    if (passes == 1) {
      dot_group(ks, m0, acc);
    } else {
      for (int p = 0; p < passes; ++p) {
        load_w(ks + p * kGemvPass);
        dot_group(ks + p * kGemvPass, m0, acc);
      }
    }
    gemv_reduce<NV, 16, NV>(acc, lane);
    float tot = acc[0];
    if (S > 1) {
      if (lane % G == 0) part[warp][lane / G] = tot;
      __syncthreads();
      if (s == 0) {
        tot = part[warp][lane / G];
        for (int t = 1; t < S; ++t) tot = __fadd_rn(tot, part[warp + t][lane / G]);
      }
      __syncthreads();
    }
    if (s == 0) {
      const float t1 = __shfl_down_sync(0xffffffffu, tot, G);
      const int idx = lane / G, m = m0 + idx / 4, r = idx % 4;
      if (live && lane % G == 0 && (r & 1) == 0 && m < M && n0 + r < N) {
        float v[16] = {tot, t1};
        epi.store(m, n0 + r, v, n0 + r + 1 < N ? 2 : 1);
      }
    }
  }
}

// ============================================================================
// fp32 GEMV for one or two rows: the CTA's weight rows staged in shared memory
// ============================================================================
//
// A pass of one or two rows reads every weight once and does little
// arithmetic with it, so a chain of these GEMVs is bound by how early each
// one's weights are on their way.  Here a CTA owns R consecutive weight rows
// over all of K (one contiguous block of R * K * 4 <= 64 KB) and copies them
// into shared memory with bulk copies issued before it waits for the
// previous kernel.  The CTA holds few registers, so CTAs of the next GEMV of
// the chain find room beside it and start their own copies while this one
// computes.  The arithmetic is the register GEMV's: the same slices of K, the
// same lane FMA chains over four float4 per slice, the same warp butterfly,
// and the slice sums added in slice order, so a row gets the same bits from
// either kernel.
constexpr int kRowTileBytes = 64 * 1024;
constexpr int kRowTileThreads = 128;
constexpr int kRowTileMaxItems = 16;  // (row quad, K slice) pairs of a CTA
constexpr uint32_t kRowTileCopy = 16 * 1024;

template <int MB, bool NORM, class Epi>
__global__ void __launch_bounds__(kRowTileThreads)
    snai_rowtile_f32_kernel(const float *__restrict__ W, int N, int K, const float *__restrict__ X, int M, int S,
                            int slice, int R, Epi epi, GemvNorm nrm, int *err) {
  constexpr int NV = 4 * MB;  // values a lane reduces per item: [m][row]
  constexpr int G = 32 / NV;
  extern __shared__ __align__(128) uint8_t rowtile_smem[];
  __shared__ __align__(8) uint64_t full;
  __shared__ float part[kRowTileMaxItems][NV];
  const float *tile = reinterpret_cast<const float *>(rowtile_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * R;
  const int rows = min(R, N - row0);
  // the weights never change during a pass: they may be fetched before the
  // previous kernel has finished
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)rows * (uint32_t)K * 4u;
    mbar_init(&full, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&full, bytes);
    const char *src = reinterpret_cast<const char *>(W + (size_t)row0 * K);
    for (uint32_t o = 0; o < bytes; o += kRowTileCopy) {
      const uint32_t n = min(kRowTileCopy, bytes - o);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(rowtile_smem + o)),
          "l"(src + o), "r"(n), "r"(smem_u32(&full))
          : "memory");
    }
  }
  __syncthreads();
  // a pass's first kernel (the embedding fold) lets the next one start only
  // once the previous pass has finished, as the embedding kernel does
  const bool first = NORM && nrm.emb;
  if (!first) grid_dep_launch();
  grid_dep_wait();
  if (first) grid_dep_launch();
  const int nq = (rows + 3) / 4, items = nq * S;
  // input row of row j: the token's embedding row (embedding fold), or
  // gather[j].x, or j
  int src[MB];
#pragma unroll
  for (int j = 0; j < MB; ++j) src[j] = NORM && nrm.gather ? nrm.gather[j].x : j;
  if constexpr (NORM) {
    if (nrm.emb) {
      const RowDesc rd = nrm.pk.r[0];
      const int raw = nrm.ef.tokens_d ? nrm.ef.tokens_d[rd.token] : rd.token;
      src[0] = (raw < 0 || raw >= nrm.ef.V) ? 0 : raw;
      if (blockIdx.x == 0) {
        // the embedding kernel's writes: h, the history, the row descriptors
        const float *er = X + (size_t)src[0] * K;
        for (int k = threadIdx.x; k < K; k += blockDim.x) nrm.ef.h[k] = er[k];
        if (threadIdx.x == 0) {
          nrm.ef.hist[(size_t)rd.slot * nrm.ef.ctx + rd.pos] = raw;
          atomicMax(&nrm.ef.seq_len[rd.slot], rd.pos + 1);
          nrm.ef.rows_w[0] = rd;
        }
        if ((int)threadIdx.x < nrm.pk.n_out) nrm.ef.outrows_w[threadIdx.x] = nrm.pk.out[threadIdx.x];
      }
    }
  }
  // this lane's input values of item `it`'s K slice, as read (and the norm
  // weights there with NORM) ...
  auto load_x = [&](int it, float4(&xv)[MB][4], float4(&nw)[4]) {
    const int qi = it / S, s = it - qi * S;
    const int ks = s * slice, ke = min(K, ks + slice);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = ks + lane * 4 + 128 * i;
      nw[i] = NORM && k < ke ? __ldg(reinterpret_cast<const float4 *>(nrm.w + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < MB; ++j) {
      const float *xr = X + (size_t)src[j] * K;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = ks + lane * 4 + 128 * i;
        xv[j][i] = j < M && k < ke ? __ldg(reinterpret_cast<const float4 *>(xr + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  // ... then normalised (NORM): x * inv * w
  float inv[MB];
#pragma unroll
  for (int j = 0; j < MB; ++j) inv[j] = 1.f;
  auto norm_x = [&](int it, float4(&xv)[MB][4], const float4(&nw)[4]) {
    if constexpr (NORM) {
      const int qi = it / S, s = it - qi * S;
      const int ks = s * slice, ke = min(K, ks + slice);
#pragma unroll
      for (int j = 0; j < MB; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = ks + lane * 4 + 128 * i;
          if (j < M && k < ke) {
            float4 &v = xv[j][i];
            v.x = __fmul_rn(__fmul_rn(v.x, inv[j]), nw[i].x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv[j]), nw[i].y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv[j]), nw[i].z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv[j]), nw[i].w);
          }
        }
    }
  };
  float4 xv[MB][4], nw[4];
  // the first item's inputs are on their way while the rows' rms is taken
  if (warp < items) load_x(warp, xv, nw);
  if constexpr (NORM) {
#pragma unroll
    for (int j = 0; j < MB; ++j)
      if (j < M && warp < items) inv[j] = warp_row_rms_inv(X + (size_t)src[j] * K, K, lane);
  }
  if (warp < items) norm_x(warp, xv, nw);
  // every thread sees the copies land (or the whole CTA gives up together)
  const bool late = !mbar_wait_bounded(&full, 0u, err, kErrWaitFull);
  if (__syncthreads_or(late)) {
    // do not leave while copies into this CTA's shared memory may be in flight
    if (threadIdx.x == 0) mbar_wait_bounded(&full, 0u, err, kErrWaitDrain);
    return;
  }
  for (int it = warp; it < items; it += kRowTileThreads / 32) {
    if (it != warp) {
      load_x(it, xv, nw);
      norm_x(it, xv, nw);
    }
    const int qi = it / S, s = it - qi * S;
    const int ks = s * slice, ke = min(K, ks + slice);
    float acc[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[j] = 0.f;
#pragma unroll
    for (int j = 0; j < MB; ++j) {
      if (j >= M) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = ks + lane * 4 + 128 * i;
        if (k < ke) {
          const float4 x4 = xv[j][i];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float4 w = 4 * qi + r < rows ? *reinterpret_cast<const float4 *>(tile + (size_t)(4 * qi + r) * K + k)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
            acc[4 * j + r] =
                fmaf(w.x, x4.x, fmaf(w.y, x4.y, fmaf(w.z, x4.z, fmaf(w.w, x4.w, acc[4 * j + r]))));
          }
        }
      }
    }
    gemv_reduce<NV, 16, NV>(acc, lane);
    if (lane % G == 0) part[it][lane / G] = acc[0];
  }
  __syncthreads();
  // per quad and (row, weight row) pair: the slice sums in slice order
  for (int t = threadIdx.x; t < nq * NV; t += blockDim.x) {
    const int qi = t / NV, jv = t - qi * NV, m = jv / 4, r = jv % 4;
    const int n = row0 + 4 * qi + r;
    if ((r & 1) == 0 && m < M && n < N) {
      float v0 = part[qi * S][jv], v1 = part[qi * S][jv + 1];
      for (int s = 1; s < S; ++s) {
        v0 = __fadd_rn(v0, part[qi * S + s][jv]);
        v1 = __fadd_rn(v1, part[qi * S + s][jv + 1]);
      }
      float v[16] = {v0, v1};
      epi.store(m, n, v, n + 1 < N ? 2 : 1);
    }
  }
}

// ============================================================================
// fp32 GEMV for one or two rows over many weight rows: a shared-memory ring
// ============================================================================
//
// For a matrix of many rows (the logits, V x D) the staged-tile kernel runs
// in waves, and each wave's copies start only when a CTA of the wave before
// has finished.  Here one CTA per SM streams its contiguous share of row
// quads through shared memory: consumer warp w takes the CTA's quads w,
// w + 8, ... through its own D slots (a quad of rows over all of K, K <=
// 1024, per slot), and one producer thread refills each slot as soon as its
// warp has read it, issuing the first copies before the dependency wait.  A
// warp's slots are used strictly in turn, so a wait on a slot's phase never
// sees an older phase of the same parity.  A consumer warp computes a whole
// quad, both K slices in slice order, with the register GEMV's lane FMA
// chains and butterfly, so a row's bits are those of the other GEMVs.
constexpr int kRingConsumers = 8;
constexpr int kRingThreads = (kRingConsumers + 1) * 32;
constexpr int kRingSlotsMax = 16;
constexpr int kRingBytes = 128 * 1024;
constexpr int kRingMinQuadsPerSm = 16;  // below this the staged-tile kernel's one wave is as quick

template <int MB, bool NORM, class Epi>
__global__ void __launch_bounds__(kRingThreads, 1)
    snai_rowring_f32_kernel(const float *__restrict__ W, int N, int K, const float *__restrict__ X, int M, int S,
                            int slice, int D, Epi epi, GemvNorm nrm, int *err) {
  constexpr int NV = 4 * MB;
  constexpr int G = 32 / NV;
  constexpr int SMAX = 2;  // K <= 1024: at most two 512-column slices
  extern __shared__ __align__(128) uint8_t ring_smem[];
  __shared__ __align__(8) uint64_t full[kRingSlotsMax], empty[kRingSlotsMax];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quads = (N + 3) / 4;
  const int q0 = (int)((long long)quads * blockIdx.x / gridDim.x);
  const int q1 = (int)((long long)quads * (blockIdx.x + 1) / gridDim.x);
  const uint32_t slot_bytes = 16u * (uint32_t)K;
  const int NS = kRingConsumers * D;  // slot w * D + d: warp w's d-th
  // quad j of the CTA: warp j % 8, its (j / 8)-th, slot use (j / 8) / D
  auto slot_of = [&](int j) { return (j % kRingConsumers) * D + (j / kRingConsumers) % D; };
  auto use_of = [&](int j) { return (j / kRingConsumers) / D; };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  grid_dep_launch();
  if (warp == kRingConsumers) {
    // ---- producer: the CTA's quads in order, each once its slot is free ----
    // (the weights never change during a pass: the first copies go out before
    // the wait for the previous kernel)
    if (lane == 0) {
      int j = 0;
      for (int q = q0; q < q1; ++q, ++j) {
        const int sl = slot_of(j), u = use_of(j);
        if (u > 0 && (!mbar_wait_bounded(&empty[sl], (uint32_t)(u - 1) & 1u, err, kErrWaitEmpty) ||
                      *(volatile int *)&abort_flag)) {
          abort_flag = 1;
          break;
        }
        const uint32_t bytes = (uint32_t)min(4, N - 4 * q) * (uint32_t)K * 4u;
        mbar_arrive_expect_tx(&full[sl], bytes);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(ring_smem + (size_t)sl * slot_bytes)),
            "l"(W + (size_t)q * 4 * K), "r"(bytes), "r"(smem_u32(&full[sl]))
            : "memory");
      }
      // do not leave while a copy into this CTA's shared memory is in flight
      for (int i = j - 1; i >= 0 && i >= j - NS; --i)
        if (!mbar_wait_bounded(&full[slot_of(i)], (uint32_t)use_of(i) & 1u, err, kErrWaitDrain)) break;
    }
    return;
  }
  // ---- consumers ----
  grid_dep_wait();
  // the lane's inputs of both slices as read, then (NORM) the rows' rms while
  // they are on their way, then x * inv * w
  float4 xv[MB][SMAX][4], nw[SMAX][4];
#pragma unroll
  for (int s = 0; s < SMAX; ++s)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ks = s * slice, ke = min(K, ks + slice);
      const int k = ks + lane * 4 + 128 * i;
      const bool in = s < S && k < ke;
      nw[s][i] = NORM && in ? __ldg(reinterpret_cast<const float4 *>(nrm.w + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < MB; ++j) {
        const float *xr = X + (size_t)(NORM && nrm.gather ? nrm.gather[j].x : j) * K;
        xv[j][s][i] = j < M && in ? __ldg(reinterpret_cast<const float4 *>(xr + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  if constexpr (NORM) {
#pragma unroll
    for (int j = 0; j < MB; ++j) {
      if (j >= M) break;
      const float inv = warp_row_rms_inv(X + (size_t)(nrm.gather ? nrm.gather[j].x : j) * K, K, lane);
#pragma unroll
      for (int s = 0; s < SMAX; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ks = s * slice, ke = min(K, ks + slice);
          const int k = ks + lane * 4 + 128 * i;
          if (s < S && k < ke) {
            float4 &v = xv[j][s][i];
            v.x = __fmul_rn(__fmul_rn(v.x, inv), nw[s][i].x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), nw[s][i].y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), nw[s][i].z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), nw[s][i].w);
          }
        }
    }
  }
  for (int j = warp; q0 + j < q1; j += kRingConsumers) {
    const int sl = slot_of(j), n0 = (q0 + j) * 4;
    if (!mbar_wait_bounded(&full[sl], (uint32_t)use_of(j) & 1u, err, kErrWaitFull) ||
        *(volatile int *)&abort_flag) {
      abort_flag = 1;
      break;
    }
    const float *wq = reinterpret_cast<const float *>(ring_smem + (size_t)sl * slot_bytes);
    float tot = 0.f;
#pragma unroll
    for (int s = 0; s < SMAX; ++s) {
      if (s >= S) break;
      const int ks = s * slice, ke = min(K, ks + slice);
      float acc[NV];
#pragma unroll
      for (int v = 0; v < NV; ++v) acc[v] = 0.f;
#pragma unroll
      for (int jm = 0; jm < MB; ++jm) {
        if (jm >= M) break;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = ks + lane * 4 + 128 * i;
          if (k < ke) {
            const float4 x4 = xv[jm][s][i];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float4 w = n0 + r < N ? *reinterpret_cast<const float4 *>(wq + (size_t)r * K + k)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
              acc[4 * jm + r] =
                  fmaf(w.x, x4.x, fmaf(w.y, x4.y, fmaf(w.z, x4.z, fmaf(w.w, x4.w, acc[4 * jm + r]))));
            }
          }
        }
      }
      if (s == S - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);  // every lane has read the slot
      }
      gemv_reduce<NV, 16, NV>(acc, lane);
      tot = s == 0 ? acc[0] : __fadd_rn(tot, acc[0]);
    }
    const float t1 = __shfl_down_sync(0xffffffffu, tot, G);
    const int idx = lane / G, m = idx / 4, r = idx % 4;
    if (lane % G == 0 && (r & 1) == 0 && m < M && n0 + r < N) {
      float v[16] = {tot, t1};
      epi.store(m, n0 + r, v, n0 + r + 1 < N ? 2 : 1);
    }
  }
}

// ============================================================================
// the small-batch decode pass in one persistent kernel
// ============================================================================
//
// A decode pass of one or two rows (the PHP host's cortex_forward step) reads
// every weight once: 168 MB at d=1024, as fp32 matrices whose dot products
// are tiny.  As separate launches (embedding, per layer QKV / attention / Wo
// / W_up / W_down, logits) every kernel pays its own DRAM ramp and tail.
// Here one CTA per SM runs the whole pass:
//   * warp 0 streams this CTA's share of every weight matrix of the pass, in
//     pass order, into a shared-memory ring with bulk copies (slots of 16*d
//     bytes: a quad of rows of a d-wide matrix, or one row of W_down), never
//     waiting for activations, so the weight stream keeps running through
//     the stage boundaries;
//   * warps 1..8 compute each stage from the ring and the stage's input
//     vector in shared memory, then meet the other CTAs at a grid barrier
//     (a monotonic counter, bounded spin) before the next stage reads what
//     this one wrote.
// Stages per layer: QKV (input RMSNorm(h), or of the embedding row in layer
// 0), attention (64-position chunks of every (row, head) over the CTAs, the
// last chunk of a (row, head) merging), Wo (+h), W_up (input RMSNorm(h),
// SiLU), W_down (+h); then the logits (input RMSNorm(h)).  The arithmetic is
// the fp32 GEMV's and the attention kernels' operation for operation (a
// row's K in 512-column slices, lanes' FMA chains over four float4 per
// slice, the warp butterfly, the slice sums in slice order; norms by the
// GEMV's rms_inv; the canonical chunked attention), so the pass gives the
// bits of the kernel-per-stage path.  Cross-CTA data written inside the
// kernel (h, q, staged K/V, attention partials, att, u) is read from L2.
// Used for FP32 passes of 1 or 2 rows of distinct slots that all want
// logits, d = 512 or 1024, head size 64, vocab a multiple of 4, ctx <= 8192.
constexpr int kPassThreads = 9 * 32;
constexpr int kPassMaxRows = 2;
constexpr int kPassMaxSlots = 32;
constexpr size_t kPassRingBytes = 176 * 1024;

struct PassArgs {
  int M, D, F, V, L, H, S, ctx;
  const RowDesc *rows;
  const int *tokens_d;
  const float *emb, *w_out, *rms_final;
  const PassLayer *layers;
  float *kv;
  size_t slot_stride, layer_stride, part_stride, head_stride;
  const float2 *rope;
  float sqrt_hs;
  float *h, *q, *kvs, *att, *u, *logits;
  int *hist, *seq_len;
  float *part;
  int *cnt;
  unsigned *bar;  // [0] arrivals, [1] finished CTAs; zero between launches
  int *err;
};

struct PassSmem {
  uint64_t full[kPassMaxSlots], empty[kPassMaxSlots];
  float xs[kPassMaxRows * 4096];       // the stage's input rows
  __align__(16) float wp4[2][4 * kAttPW];  // attention: two 4-warp groups
  float inv[kPassMaxRows];
  int flag[2];
  int abort;
};

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every consumer thread of every CTA: returns once all CTAs have arrived at
// barrier number `no` (their writes before it visible), or false (error
// recorded) if that takes longer than kWaitTimeoutNs.
__device__ bool pass_grid_sync(const PassArgs &a, PassSmem &sm, unsigned no) {
  named_sync(1, 256);
  if (threadIdx.x == 32) {
    __threadfence();
    atomicAdd(&a.bar[0], 1u);
    const unsigned target = (no + 1) * gridDim.x;
    bool ok = true;
    if (ld_acquire_u32(&a.bar[0]) < target) {
      const unsigned long long t0 = global_timer_ns();
      for (uint32_t it = 1;; ++it) {
        if (ld_acquire_u32(&a.bar[0]) >= target) break;
        if ((it & 63u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) {
          record_error(a.err, kErrWaitAccum);
          ok = false;
          break;
        }
      }
    }
    sm.flag[0] = ok;
    if (!ok) sm.abort = 1;
  }
  named_sync(1, 256);
  return sm.flag[0] != 0;
}

// xs[m][k] = RMSNorm(src row m, w)[k] for the pass's rows; src row m is the
// embedding row of the row's token (layer 0) or h.
template <bool EMB>
__device__ void pass_norm(const PassArgs &a, PassSmem &sm, const float *w) {
  const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31, ct = threadIdx.x - 32;
  auto src = [&](int m) -> const float * {
    if constexpr (EMB) {
      const RowDesc rd = a.rows[m];
      const int raw = a.tokens_d ? a.tokens_d[rd.token] : rd.token;
      const int tid = (raw < 0 || raw >= a.V) ? 0 : raw;
      return a.emb + (size_t)tid * a.D;
    } else {
      return a.h + (size_t)m * a.D;
    }
  };
  if (cw < a.M) {
    const float inv = EMB ? warp_row_rms_inv<false>(src(cw), a.D, lane) : warp_row_rms_inv<true>(src(cw), a.D, lane);
    if (lane == 0) sm.inv[cw] = inv;
  }
  named_sync(1, 256);
  for (int m = 0; m < a.M; ++m) {
    const float *s = src(m);
    for (int k = 4 * ct; k < a.D; k += 4 * 256) {
      const float4 hv = EMB ? __ldg(reinterpret_cast<const float4 *>(s + k)) : __ldcg(reinterpret_cast<const float4 *>(s + k));
      const float4 wv = __ldg(reinterpret_cast<const float4 *>(w + k));
      const float inv = sm.inv[m];
      *reinterpret_cast<float4 *>(sm.xs + m * a.D + k) =
          make_float4(__fmul_rn(__fmul_rn(hv.x, inv), wv.x), __fmul_rn(__fmul_rn(hv.y, inv), wv.y),
                      __fmul_rn(__fmul_rn(hv.z, inv), wv.z), __fmul_rn(__fmul_rn(hv.w, inv), wv.w));
    }
  }
  named_sync(1, 256);
}

// xs[m][0..K) = src[m * K ..] (a vector written earlier in this kernel).
__device__ void pass_load(const PassArgs &a, PassSmem &sm, const float *src, int K) {
  const int ct = threadIdx.x - 32;
  for (int m = 0; m < a.M; ++m)
    for (int k = 4 * ct; k < K; k += 4 * 256)
      *reinterpret_cast<float4 *>(sm.xs + m * K + k) = __ldcg(reinterpret_cast<const float4 *>(src + (size_t)m * K + k));
  named_sync(1, 256);
}

// This CTA's quads of an R-row matrix: [q0, q1) of R / 4.
__device__ __forceinline__ void pass_quads(int R, int &q0, int &q1) {
  const long long Q = R / 4;
  q0 = (int)(Q * blockIdx.x / gridDim.x);
  q1 = (int)(Q * (blockIdx.x + 1) / gridDim.x);
}

// One weight stage of the consumers: the CTA's rows of W (R x K, K = D or
// F = 4D) from the ring, dot products with xs, Epi(m, n, v, cnt) on the
// results.  Consumer warp w takes the stage's slots w, w + 8, ...: it waits
// for its slot, computes every row of it (K in 512-column slices, each
// slice's lanes FMA-chained over four float4 and butterfly-summed, the
// slices added in order), releases the slot and stores the rows itself, so
// the warps never wait for each other inside a stage.  `it` counts ring
// slots in step with the producer.
template <class Epi>
__device__ bool pass_stage(const PassArgs &a, PassSmem &sm, const uint8_t *ring, int ns, int R, int K, int &it,
                           const Epi &epi) {
  const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
  const int slot_bytes = 16 * a.D;
  const int rows_per_slot = K == a.D ? 4 : 1;
  const int T = K / 512;  // 512-column slices of a row
  int q0, q1;
  pass_quads(R, q0, q1);
  const int nslots = (q1 - q0) * (4 / rows_per_slot);
  bool ok = true;
  for (int j = cw; ok && j < nslots; j += 8) {
    const int sl = (it + j) % ns;
    if (!mbar_wait_bounded(&sm.full[sl], (uint32_t)((it + j) / ns) & 1u, a.err, kErrWaitFull) || sm.abort) {
      ok = false;
      sm.abort = 1;
      break;
    }
    const float *wsl = reinterpret_cast<const float *>(ring + (size_t)sl * slot_bytes);
    float tot[4][kPassMaxRows];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (r >= rows_per_slot) break;
      for (int t = 0; t < T; ++t) {
        float acc[kPassMaxRows];
#pragma unroll
        for (int m = 0; m < kPassMaxRows; ++m) acc[m] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = t * 512 + lane * 4 + 128 * i;
          const float4 w = *reinterpret_cast<const float4 *>(wsl + r * K + k);
#pragma unroll
          for (int m = 0; m < kPassMaxRows; ++m) {
            const float4 xv = m < a.M ? *reinterpret_cast<const float4 *>(sm.xs + m * K + k)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            acc[m] = fmaf(w.x, xv.x, fmaf(w.y, xv.y, fmaf(w.z, xv.z, fmaf(w.w, xv.w, acc[m]))));
          }
        }
#pragma unroll
        for (int m = 0; m < kPassMaxRows; ++m) {
          const float s = warp_sum(acc[m]);
          tot[r][m] = t == 0 ? s : __fadd_rn(tot[r][m], s);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[sl]);  // every lane has read the slot
    if (rows_per_slot == 4) {
      if (lane < 2 * a.M) {  // row pairs of a d-wide matrix
        const int pr = lane / a.M, m = lane % a.M;
        float v[16] = {};
#pragma unroll
        for (int r = 0; r < 4; r += 2)
          if (pr == r / 2) {
#pragma unroll
            for (int mm = 0; mm < kPassMaxRows; ++mm)
              if (mm == m) {
                v[0] = tot[r][mm];
                v[1] = tot[r + 1][mm];
              }
          }
        epi.store(m, (q0 + j) * 4 + 2 * pr, v, 2);
      }
    } else if (lane < a.M) {  // one row of W_down
      float v[16] = {};
#pragma unroll
      for (int mm = 0; mm < kPassMaxRows; ++mm)
        if (mm == lane) v[0] = tot[0][mm];
      epi.store(lane, q0 * 4 + j, v, 1);
    }
  }
  it += nslots;
  named_sync(1, 256);
  return ok && !sm.abort;
}

// logits[rows[m].out][n] = C (core/cortex.nim:555-561)
struct PassLogits {
  float *logits;
  const RowDesc *rows;
  int V;
  __device__ __forceinline__ void store(int m, int n, const float *v, int cnt) const {
    float *p = logits + (size_t)rows[m].out * V + n;
    for (int i = 0; i < cnt; ++i) p[i] = v[i];
  }
};

// The attention stage: work items (row, head, chunk) over the CTAs, two at a
// time (warps 1-4 and 5-8); the last chunk of a (row, head) to finish merges
// into att.
__device__ bool pass_attention(const PassArgs &a, PassSmem &sm, int l) {
  const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
  const int grp = cw >> 2, wq = cw & 3, gt = wq * 32 + lane;  // group, warp and thread in group
  const size_t layer_off = (size_t)l * a.layer_stride;
  int C[kPassMaxRows] = {0, 0};
  int total = 0;
  for (int m = 0; m < a.M; ++m) {
    C[m] = (a.rows[m].pos + 1 + kAttChunk - 1) / kAttChunk;
    total += a.H * C[m];
  }
  const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
  const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
  for (int base = i0; base < i1; base += 2) {
    const int item = base + grp;
    if (item < i1) {
      int m = 0, rem = item;
      while (m + 1 < a.M && rem >= a.H * C[m]) rem -= a.H * C[m++];
      const int head = rem / C[m], c = rem % C[m];
      const RowDesc rd = a.rows[m];
      const int n = rd.pos + 1;
      const AttRow r = att_row<true>(rd, a.q, a.kv, m, head, a.D, a.slot_stride, layer_off, a.part_stride,
                                     a.head_stride, a.kvs, a.rope, wq == 0 && c == (n - 1) / kAttChunk);
      att_warp_chunk(r, c * kAttChunk, a.sqrt_hs, sm.wp4[grp] + wq * kAttPW, wq);
      named_sync(2 + grp, 128);
      float *pp = a.part + (size_t)(m * a.H + head) * a.S * kAttPW;
      if (gt < 64) att_chunk_combine(sm.wp4[grp], gt, pp + c * kAttPW);
      __threadfence();
      named_sync(2 + grp, 128);
      if (gt == 0) sm.flag[grp] = atomicAdd(&a.cnt[m * a.H + head], 1) == C[m] - 1;
      named_sync(2 + grp, 128);
      if (sm.flag[grp]) {
        __threadfence();
        if (gt < 64)
          a.att[(size_t)m * a.D + head * 64 + gt] = att_merge(pp, C[m], gt, [](const float *p) { return __ldcg(p); });
        if (gt == 0) a.cnt[m * a.H + head] = 0;
      }
      named_sync(2 + grp, 128);
    }
  }
  return true;
}

__global__ void __launch_bounds__(kPassThreads, 1) snai_pass_kernel(const __grid_constant__ PassArgs a) {
  extern __shared__ __align__(1024) uint8_t pass_smem[];
  PassSmem &sm = *reinterpret_cast<PassSmem *>(pass_smem);
  uint8_t *ring = pass_smem + ((sizeof(PassSmem) + 1023) & ~size_t(1023));
  const int slot_bytes = 16 * a.D;
  const int ns = min(kPassMaxSlots, (int)(kPassRingBytes / slot_bytes));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    // ---- producer: every weight slot of this CTA, in pass order ----
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      auto stream = [&](const float *W, int R, int K) {
        int q0, q1;
        pass_quads(R, q0, q1);
        const int nslots = (q1 - q0) * (K == a.D ? 1 : 4);
        const char *base = reinterpret_cast<const char *>(W + (size_t)q0 * 4 * K);
        for (int j = 0; ok && j < nslots; ++j, ++it) {
          const int sl = it % ns;
          if (!mbar_wait_bounded(&sm.empty[sl], ((uint32_t)(it / ns) & 1u) ^ 1u, a.err, kErrWaitEmpty) ||
              *(volatile int *)&sm.abort) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[sl], (uint32_t)slot_bytes);
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  smem_u32(ring + (size_t)sl * slot_bytes)),
              "l"(base + (size_t)j * slot_bytes), "r"(slot_bytes), "r"(smem_u32(&sm.full[sl]))
              : "memory");
        }
      };
      for (int l = 0; ok && l < a.L; ++l) {
        const PassLayer &ly = a.layers[l];
        stream(ly.wqkv, 3 * a.D, a.D);
        stream(ly.wo, a.D, a.D);
        stream(ly.wup, a.F, a.D);
        stream(ly.wdown, a.D, a.F);
      }
      if (ok) stream(a.w_out, a.V, a.D);
      // do not leave while a copy into this CTA's shared memory is in flight
      for (int j = it - 1; j >= 0 && j >= it - ns; --j)
        if (!mbar_wait_bounded(&sm.full[j % ns], (uint32_t)(j / ns) & 1u, a.err, kErrWaitDrain)) break;
    }
  } else {
    // ---- consumers ----
    const int ct = threadIdx.x - 32;
    int it = 0;
    unsigned bar = 0;
    bool ok = true;
    // the embedding row into h (a share per CTA), the token into the history
    if (blockIdx.x == 0 && ct < a.M) {
      const RowDesc rd = a.rows[ct];
      const int raw = a.tokens_d ? a.tokens_d[rd.token] : rd.token;
      a.hist[(size_t)rd.slot * a.ctx + rd.pos] = raw;
      atomicMax(&a.seq_len[rd.slot], rd.pos + 1);
    }
    {
      const int tot = a.M * a.D;
      const int e0 = (int)((long long)tot * blockIdx.x / gridDim.x), e1 = (int)((long long)tot * (blockIdx.x + 1) / gridDim.x);
      for (int e = e0 + ct; e < e1; e += 256) {
        const int m = e / a.D, k = e - m * a.D;
        const RowDesc rd = a.rows[m];
        const int raw = a.tokens_d ? a.tokens_d[rd.token] : rd.token;
        const int tid = (raw < 0 || raw >= a.V) ? 0 : raw;
        a.h[(size_t)m * a.D + k] = a.emb[(size_t)tid * a.D + k];
      }
    }
    for (int l = 0; ok && l < a.L; ++l) {
      const PassLayer &ly = a.layers[l];
      EpiQKV eq{a.rows, a.q, a.kv, a.rope, a.D, a.D, 64, a.slot_stride, (size_t)l * a.layer_stride,
                a.part_stride, a.head_stride, a.kvs};
      eq.tma = 0;
      if (l == 0)
        pass_norm<true>(a, sm, ly.rms_att);
      else
        pass_norm<false>(a, sm, ly.rms_att);
      ok = pass_stage(a, sm, ring, ns, 3 * a.D, a.D, it, eq) && pass_grid_sync(a, sm, bar++);
      if (!ok) break;
      pass_attention(a, sm, l);
      ok = pass_grid_sync(a, sm, bar++);
      if (!ok) break;
      pass_load(a, sm, a.att, a.D);
      EpiResidual er{};
      er.h = a.h;
      er.ld = a.D;
      ok = pass_stage(a, sm, ring, ns, a.D, a.D, it, er) && pass_grid_sync(a, sm, bar++);
      if (!ok) break;
      pass_norm<false>(a, sm, ly.rms_ffn);
      ok = pass_stage(a, sm, ring, ns, a.F, a.D, it, EpiSilu<float>{a.u, a.F}) && pass_grid_sync(a, sm, bar++);
      if (!ok) break;
      pass_load(a, sm, a.u, a.F);
      ok = pass_stage(a, sm, ring, ns, a.D, a.F, it, er) && pass_grid_sync(a, sm, bar++);
    }
    if (ok) {
      pass_norm<false>(a, sm, a.rms_final);
      ok = pass_stage(a, sm, ring, ns, a.V, a.D, it, PassLogits{a.logits, a.rows, a.V});
    }
    if (!ok) sm.abort = 1;
    // the last CTA to finish resets the counters for the next launch (every
    // CTA has passed every barrier by then)
    named_sync(1, 256);
    if (ct == 0 && ok) {
      __threadfence();
      if (atomicAdd(&a.bar[1], 1u) == gridDim.x - 1) {
        a.bar[0] = 0;
        a.bar[1] = 0;
      }
    }
  }
}

// ============================================================================
// host side
// ============================================================================

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  // a function-local static: initialised once, thread-safe
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// 2-D K-major operand [rows][K] with 128-byte-wide, box_rows-high boxes.
static bool make_tmap(CUtensorMap *map, const void *base, bool bf16, int K, int rows, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  const size_t es = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * es};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The residual epilogue of M rows: h and its tensor map for the drains'
// reduce-adds (16 x 32 fp32 boxes, 64-byte swizzle; valid for every engine
// shape: d is a multiple of 4 and h is 256-byte aligned).  Returns false
// (with the error set) if the map cannot be made.
static bool residual_epi(Engine &e, int M, EpiResidual *r) {
  *r = EpiResidual{};
  r->h = e.h;
  r->ld = e.d.D;
  auto enc = get_encode_fn();
  cuuint64_t dims[2] = {(cuuint64_t)e.d.D, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)e.d.D * 4};
  cuuint32_t box[2] = {16, 32};
  cuuint32_t estr[2] = {1, 1};
  if (!enc || enc(&r->tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.h, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed for the residual (M=%d D=%d)", M, e.d.D);
    return false;
  }
  return true;
}

// TMA stores for the QKV drains when K and V go to the staging buffer and
// every channel is an attention channel: q as [M][att_ch], the staging
// buffer as [M][2 att_ch], fp32, 16 x 32 boxes, 64-byte swizzle.  Leaves the
// plain stores on any failure.
static void qkv_tma_maps(Engine &e, int M, EpiQKV *q) {
  q->tma = 0;
  if (q->kvs == nullptr || e.d.att_ch != e.d.D || (e.d.att_ch & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(e.q) & 15) != 0 || (reinterpret_cast<uintptr_t>(e.kvs) & 15) != 0)
    return;
  auto enc = get_encode_fn();
  if (!enc) return;
  cuuint32_t box[2] = {16, 32};
  cuuint32_t estr[2] = {1, 1};
  cuuint64_t dq[2] = {(cuuint64_t)e.d.att_ch, (cuuint64_t)M};
  cuuint64_t sq[1] = {(cuuint64_t)e.d.att_ch * 4};
  cuuint64_t dk[2] = {(cuuint64_t)e.d.att_ch * 2, (cuuint64_t)M};
  cuuint64_t sk[1] = {(cuuint64_t)e.d.att_ch * 8};
  if (enc(&q->tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.q, dq, sq, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return;
  if (enc(&q->tkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.kvs, dk, sk, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return;
  q->tma = 1;
}

// TF32 / BF16 modes run every projection on the tensor cores, whatever the
// row count: a row's result must not depend on how many rows share its pass
// (a decode pass of 3 rows, the logits rows of a prompt chunk, a shard of
// the sequences), and the tensor-core kernels give a row the same bits for
// any M (same K order, one accumulator per output).
static bool tc_path(const Engine &e, int M) {
  return e.precision != kFP32 && M >= 1 && e.d.D % 16 == 0 && e.d.D >= 64;
}

static int sm_count(int dev) { return device_sm_count(dev); }

int device_sm_count(int dev) {
  static std::atomic<int> cached[64];
  const bool slot = dev >= 0 && dev < 64;
  if (slot) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148;
  }
  if (slot) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Launches kern on the engine's stream; with pdl as a programmatic dependent
// launch (the kernel begins with grid_dep_wait before it reads anything the
// previous kernel writes).
template <typename... KArgs, typename... Args>
static void launch_k(Engine &e, bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e.stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  e.launches++;
}

// Persistent tcgen05 GEMM (snai_tileproj_tc_kernel): 128 x BN tiles, one CTA per SM.
template <typename TIn, int BN, class Epi>
static int launch_tcp(Engine &e, int M, int N, int K, const void *A, const void *W, const Epi &epi, bool pdl) {
  constexpr int STAGES = BN == 256 ? 4 : 6;
  using Sm = TcpSmem<BN, STAGES>;
  auto kern = snai_tileproj_tc_kernel<TIn, BN, STAGES, Epi>;
  static DeviceOnce attr;  // per instantiation
  if (!attr.run(e.device, [&] { return set_dyn_smem(kern, (int)Sm::kBytes); })) {
    set_error("cudaFuncSetAttribute failed for the tensor-core projection");
    return -5;
  }
  CUtensorMap ta, tb;
  const bool bf = sizeof(TIn) == 2;
  if (!make_tmap(&ta, A, bf, K, M, kTcBM) || !make_tmap(&tb, W, bf, K, N, BN)) {
    set_error("cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
    return -5;
  }
  const int tiles = ((M + kTcBM - 1) / kTcBM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count(e.device));
  launch_k(e, pdl, kern, dim3(grid), dim3(kGemmThreads), Sm::kBytes, ta, tb, M, N, K, epi, e.err_d);
  return 0;
}

// CTA-pair tcgen05 GEMM (snai_pairproj_tc_kernel): 256 x 256 tiles on SM pairs.
template <typename TIn, class Epi>
static int launch_tc2(Engine &e, int M, int N, int K, const void *A, const void *W, const Epi &epi, bool pdl) {
  constexpr int STAGES = 6;
  using Sm = Tc2Smem<STAGES>;
  auto kern = snai_pairproj_tc_kernel<TIn, STAGES, Epi>;
  static DeviceOnce attr;  // per instantiation
  if (!attr.run(e.device, [&] { return set_dyn_smem(kern, (int)Sm::kBytes); })) {
    set_error("cudaFuncSetAttribute failed for the CTA-pair projection");
    return -5;
  }
  CUtensorMap ta, tb;
  const bool bf = sizeof(TIn) == 2;
  if (!make_tmap(&ta, A, bf, K, M, kTcBM) || !make_tmap(&tb, W, bf, K, N, 128)) {
    set_error("cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
    return -5;
  }
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int pairs = std::max(1, std::min(tiles, sm_count(e.device) / 2));
  launch_k(e, pdl, kern, dim3(2 * pairs), dim3(kGemmThreads), Sm::kBytes, ta, tb, M, N, K, epi, e.err_d);
  return 0;
}

// pdl: launch as a programmatic dependent of the previous kernel (its set-up
// overlaps that kernel's tail).  Not after a long kernel of small CTAs
// (attention): the GEMM's CTAs, parked on every SM with their shared memory
// until it ends, would take that kernel's room.
template <typename TIn, class Epi>
static int launch_tc(Engine &e, int M, int N, int K, const void *A, const void *W, const Epi &epi, bool pdl = true) {
  // Tile shape by a per-CTA cost model: a CTA streams (rows of A + rows of W)
  // per k-block for every tile it owns and multiplies them, so the cost is
  // (tiles per CTA) x max(128 + BN, MMA time), with the CTA pair's 256 x 256
  // tile at 128 + 128 rows and a 128 x 256 block per CTA.
  // Large M keeps the pair tiles; few rows (one GPU's share of the
  // sequences, small batches) take narrower single-CTA tiles on more SMs.
  // Every shape gives a row the same bits (same K order, one accumulator).
  const int sms = sm_count(e.device);
  auto waves = [](long long tiles, long long slots) { return (tiles + slots - 1) / slots; };
  // per k-block a CTA loads 128 + BN rows of 128 bytes and multiplies a
  // 128 x BN block, about 1.14 BN row-loads of time at the SM's L2 and
  // tensor rates; whichever is longer is the tile's cost (so a 512-row QKV
  // takes 128 x 128 tiles on 96 SMs rather than 48 CTA pairs)
  auto cost = [](long long rows, long long bn) { return std::max(rows, bn + bn / 8); };
  const long long mt = (M + kTcBM - 1) / kTcBM;
  long long best = (M >= 256 && N >= 256)
                       ? waves((long long)((M + 255) / 256) * ((N + 255) / 256), sms / 2) * cost(256, 256)
                       : LLONG_MAX;
  int pick = 0;  // 0 pair, else BN
  for (int bn : {256, 128, 64}) {
    const long long c = waves(mt * ((N + bn - 1) / bn), sms) * cost(128 + bn, bn);
    if (c < best) {
      best = c;
      pick = bn;
    }
  }
  if (pick == 0) return launch_tc2<TIn>(e, M, N, K, A, W, epi, pdl);
  if (pick == 256) return launch_tcp<TIn, 256>(e, M, N, K, A, W, epi, pdl);
  if (pick == 128) return launch_tcp<TIn, 128>(e, M, N, K, A, W, epi, pdl);
  return launch_tcp<TIn, 64>(e, M, N, K, A, W, epi, pdl);
}

// A product of the training step on the TF32 tensor cores: C[M, N] =
// A[M, K] * W[N, K]^T, both fp32 and K-major (rows 16-byte aligned), with the
// training epilogue.
int train_gemm_tc(Engine &e, int M, int N, int K, const float *A, const float *W, const EpiTrain &epi) {
  if (M <= 0 || N <= 0) return 0;
  return launch_tc<float>(e, M, N, K, A, W, epi);
}

template <class Epi>
static int launch_gemv(Engine &e, int M, int N, int K, const float *X, const float *W, const Epi &epi,
                       GemvNorm nrm) {
  // S warps split K into slices of whole 128-column steps (one 512-column
  // pass each up to K = 4096); P row quads per CTA while that still leaves
  // two CTAs per SM
  const int S = std::max(1, std::min(kGemvMaxWarps, (K + kGemvPass - 1) / kGemvPass));
  const int slice = ((K + S - 1) / S + 127) / 128 * 128;
  // one or two rows over many weight rows (K <= 1024): the ring kernel, one
  // CTA per SM
  const int sms = sm_count(e.device);
  if (!nrm.emb && M <= 2 && K <= 1024 && (K & 3) == 0 && (N + 3) / 4 >= kRingMinQuadsPerSm * sms) {
    const int D = std::max(1, std::min(kRingSlotsMax / kRingConsumers, kRingBytes / (kRingConsumers * 16 * K)));
    void (*kern)(const float *, int, int, const float *, int, int, int, int, Epi, GemvNorm, int *) =
        nrm.w ? snai_rowring_f32_kernel<1, true, Epi>
              : (M <= 1 ? snai_rowring_f32_kernel<1, false, Epi> : snai_rowring_f32_kernel<2, false, Epi>);
    static DeviceOnce attr;  // per Epi: the three instantiations at once
    const bool ready = attr.run(e.device, [] {
      const bool a = set_dyn_smem(snai_rowring_f32_kernel<1, true, Epi>, kRingBytes);
      const bool b = set_dyn_smem(snai_rowring_f32_kernel<1, false, Epi>, kRingBytes);
      return set_dyn_smem(snai_rowring_f32_kernel<2, false, Epi>, kRingBytes) && a && b;
    });
    if (ready) {
      launch_k(e, true, kern, dim3(sms), dim3(kRingThreads), (size_t)kRingConsumers * D * 16 * K, W, N, K, X, M, S,
               slice, D, epi, nrm, e.err_d);
      return 0;
    }
  }
  // one or two rows: the staged-tile kernel, R rows of W per CTA (the most
  // that fit its 64 KB, fewer while that leaves under two CTAs per SM)
  if (M <= 2 && (size_t)K * 16 <= kRowTileBytes && (K & 3) == 0) {
    int R = 16;
    while (R > 4 && (size_t)R * K * 4 > kRowTileBytes) R /= 2;
    while (R > 4 && (N + R - 1) / R < 2 * sm_count(e.device)) R /= 2;
    if ((R / 4) * S <= kRowTileMaxItems) {
      void (*kern)(const float *, int, int, const float *, int, int, int, int, Epi, GemvNorm, int *) =
          nrm.w ? snai_rowtile_f32_kernel<1, true, Epi>
                : (M <= 1 ? snai_rowtile_f32_kernel<1, false, Epi> : snai_rowtile_f32_kernel<2, false, Epi>);
      static DeviceOnce attr;  // per Epi: the three instantiations at once
      const bool ready = attr.run(e.device, [] {
        const bool a = set_dyn_smem(snai_rowtile_f32_kernel<1, true, Epi>, kRowTileBytes);
        const bool b = set_dyn_smem(snai_rowtile_f32_kernel<1, false, Epi>, kRowTileBytes);
        return set_dyn_smem(snai_rowtile_f32_kernel<2, false, Epi>, kRowTileBytes) && a && b;
      });
      if (ready) {
        launch_k(e, true, kern, dim3((N + R - 1) / R), dim3(kRowTileThreads), (size_t)R * K * 4, W, N, K, X, M, S,
                 slice, R, epi, nrm, e.err_d);
        return 0;
      }
    }
  }
  if (nrm.emb) {
    set_error("the embedding fold needs the staged-tile GEMV (M=%d K=%d)", M, K);
    return -5;
  }
  const int quads = (N + 3) / 4, target = 2 * sm_count(e.device);
  int P = 1;
  while (2 * P * S <= kGemvMaxWarps && quads / (2 * P) >= target) P *= 2;
  const dim3 grid((quads + P - 1) / P), block(32 * S * P);
  void (*kern)(const float *, int, int, const float *, int, int, int, Epi, GemvNorm);
  if (nrm.w)  // one row (kGemvNormRows)
    kern = snai_rowproj_f32_kernel<1, true, Epi>;
  else
    kern = M <= 1   ? snai_rowproj_f32_kernel<1, false, Epi>
           : M <= 2 ? snai_rowproj_f32_kernel<2, false, Epi>
           : M <= 4 ? snai_rowproj_f32_kernel<4, false, Epi>
                    : snai_rowproj_f32_kernel<8, false, Epi>;
  launch_k(e, true, kern, grid, block, 0, W, N, K, X, M, S, slice, epi, nrm);
  return 0;
}

// C[M,N] = A[M,K] * W[N,K]^T with the epilogue `epi`.  `a_bytes` / `out_bytes`:
// bytes per element of A and algorithmic output bytes (for the profiler).
// With nrm.w (GEMV path only) A is the residual stream h and the input rows
// are RMSNorm(h, nrm.w), normalised inside the GEMV.  after_long: the previous
// kernel is a long one (attention), so a tensor-core launch does not start
// early as its programmatic dependent.
template <class Epi>
static int project(Engine &e, int kind, int M, int N, int K, const void *A, const float *W32,
                   const __nv_bfloat16 *W16, const Epi &epi, double out_bytes, GemvNorm nrm = GemvNorm{},
                   bool after_long = false) {
  if (M <= 0) return 0;
  const bool tc = tc_path(e, M);
  const bool bf = tc && e.precision == kBF16;
  const double w_bytes = (double)N * K * (bf ? 2 : 4), a_bytes = (double)M * K * (bf ? 2 : 4);
  const int tok = prof_begin(e);
  int rc = 0;
  if (tc) {
    rc = bf ? launch_tc<__nv_bfloat16>(e, M, N, K, A, W16, epi, !after_long)
            : launch_tc<float>(e, M, N, K, A, W32, epi, !after_long);
  } else {
    rc = launch_gemv(e, M, N, K, static_cast<const float *>(A), W32, epi, nrm);
  }
  prof_end(e, tok, kind, w_bytes + a_bytes + out_bytes, 2.0 * M * N * K);
  return rc;
}

// Attention is a programmatic dependent only on the GEMV path: after a
// tensor-core projection, its grid of many small CTAs launched early measured
// 15 % slower (9.2 against 8.0 ms per d=1024 decode step of 4096 rows).
template <typename TA>
static void launch_attention(Engine &e, int M, int layer, TA *out, double kv_positions, bool defer,
                             const RowPack &pk) {
  const Dims &d = e.d;
  const int tok = prof_begin(e);
  const size_t layer_off = (size_t)layer * e.kv_layer_stride;
  dim3 grid(d.heads, M);
  const int max_n = d.ctx;
  static DeviceOnce attr;  // per instantiation
  attr.run(e.device, [] {
    const bool a = set_dyn_smem(attention_hs64_kernel<TA>, 200 * 1024);
    const bool b = set_dyn_smem(attention_split_hs64_kernel<TA>, 200 * 1024);
    return set_dyn_smem(attention_generic_kernel<TA>, 200 * 1024) && a && b;
  });
  // few rows: a CTA per 64-position chunk of every (row, head), whatever the
  // row's position (the chunk count follows ctx, so a captured launch fits
  // every later step); same bits as the whole-row kernel
  const int rh = M * d.heads, nsm = sm_count(e.device), chunks = (d.ctx + kAttChunk - 1) / kAttChunk;
  const bool split = d.hs == 64 && e.att_split && e.att_part && rh < nsm && rh <= kSplitCounters &&
                     chunks <= kSplitMax && (size_t)rh * chunks <= e.att_part_entries;
  if (split) {
    launch_k(e, !tc_path(e, M), attention_split_hs64_kernel<TA>, dim3(d.heads, M, chunks), dim3(kAttThreads), 0,
             e.rows_d, pk, e.q, e.kv, out, d.D, d.att_ch, e.kv_slot_stride, layer_off, e.kv_part_stride,
             e.kv_head_stride, e.sqrt_hs, defer ? e.kvs : nullptr, e.rope, e.att_part, e.att_cnt);
  } else if (d.hs == 64) {
    const size_t sm = (32 + 4 * 64 + (size_t)max_n) * sizeof(float);
    launch_k(e, !tc_path(e, M), attention_hs64_kernel<TA>, grid, dim3(kAttThreads), sm, e.rows_d, e.q, e.kv, out,
             d.D, d.att_ch, e.kv_slot_stride, layer_off, e.kv_part_stride, e.kv_head_stride, e.sqrt_hs,
             defer ? e.kvs : nullptr, e.rope);
  } else {
    const size_t sm = (32 + (size_t)max_n + 2 * (size_t)d.hs) * sizeof(float);
    launch_k(e, !tc_path(e, M), attention_generic_kernel<TA>, grid, dim3(kAttThreads), sm, e.rows_d, e.q, e.kv,
             out, d.D, d.att_ch, d.hs, e.kv_slot_stride, layer_off, e.kv_part_stride, e.kv_head_stride, e.sqrt_hs,
             defer ? e.kvs : nullptr, e.rope);
  }
  // K and V of positions 0..pos per row, q in, att out
  prof_end(e, tok, kProfAttention, kv_positions * 2.0 * d.att_ch * 4 + (double)M * d.att_ch * 4 + (double)M * d.D * sizeof(TA),
           kv_positions * 4.0 * d.att_ch);
}

template <typename TA>
static void launch_norm(Engine &e, int M, const int2 *gather, const float *w, TA *x) {
  const int tok = prof_begin(e);
  launch_k(e, true, rmsnorm_kernel<TA>, dim3(M), dim3(kNormThreads), 0, e.h, gather, w, x, e.d.D);
  prof_end(e, tok, kProfNorm, (double)M * e.d.D * (4 + sizeof(TA)), 0.0);
}

// Passes of at most this many rows on the GEMV path normalise inside the
// GEMVs that consume the norms.  Each warp recomputes a row's rms_inv (one
// more L2 round trip per row before its dot products), which pays for the
// norm launch it saves at one row (80.9 -> 72.2 us per d=1024 decode pass),
// breaks even at two and loses from three rows on.
constexpr int kGemvNormRows = 1;

static bool gemv_norm(const Engine &e, int M) { return !tc_path(e, M) && M <= kGemvNormRows; }

// The persistent pass kernel serves FP32 decode passes of 1-2 rows of
// distinct slots that all want logits (the shapes it is written for), when
// the stream is not being captured into a graph.
static bool pass_kernel_ok(Engine &e, int M, int n_out, bool defer) {
  const Dims &d = e.d;
  if (!(e.pass_kernel && e.precision == kFP32 && e.pass_layers && M >= 1 && M <= kPassMaxRows && n_out == M && defer &&
        d.hs == 64 && d.att_ch == d.D && (d.D == 512 || d.D == 1024) && d.V % 4 == 0 && d.ctx <= 8192 &&
        (size_t)M * d.heads * ((d.ctx + kAttChunk - 1) / kAttChunk) <= e.att_part_entries && M * d.heads <= kSplitCounters))
    return false;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(e.stream, &st) != cudaSuccess || st != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;
  }
  static DeviceOnce attr;
  static std::atomic<int> fits[64];
  const size_t smem = ((sizeof(PassSmem) + 1023) & ~size_t(1023)) + kPassRingBytes + 1024;
  attr.run(e.device, [&] { return set_dyn_smem(snai_pass_kernel, (int)smem); });
  if (e.device < 0 || e.device >= 64) return false;
  int f = fits[e.device].load();
  if (f == 0) {  // one CTA per SM must fit, or the cooperative launch is refused
    int nb = 0;
    f = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, snai_pass_kernel, kPassThreads, smem) == cudaSuccess &&
                nb >= 1
            ? 1
            : -1;
    cudaGetLastError();
    fits[e.device].store(f);
  }
  return f == 1;
}

static int launch_pass(Engine &e, int M, const int *tokens_d, double kv_positions) {
  const Dims &d = e.d;
  PassArgs a{};
  a.M = M;
  a.D = d.D;
  a.F = d.F;
  a.V = d.V;
  a.L = d.L;
  a.H = d.heads;
  a.S = (d.ctx + kAttChunk - 1) / kAttChunk;
  a.ctx = d.ctx;
  a.rows = e.rows_d;
  a.tokens_d = tokens_d;
  a.emb = e.emb;
  a.w_out = e.w_out;
  a.rms_final = e.rms_final;
  a.layers = e.pass_layers;
  a.kv = e.kv;
  a.slot_stride = e.kv_slot_stride;
  a.layer_stride = e.kv_layer_stride;
  a.part_stride = e.kv_part_stride;
  a.head_stride = e.kv_head_stride;
  a.rope = e.rope;
  a.sqrt_hs = e.sqrt_hs;
  a.h = e.h;
  a.q = e.q;
  a.kvs = e.kvs;
  a.att = static_cast<float *>(e.att);
  a.u = static_cast<float *>(e.u);
  a.logits = e.logits;
  a.hist = e.hist;
  a.seq_len = e.seq_len_d;
  a.part = e.att_part;
  a.cnt = e.att_cnt;
  a.bar = e.pass_bar;
  a.err = e.err_d;
  const size_t smem = ((sizeof(PassSmem) + 1023) & ~size_t(1023)) + kPassRingBytes + 1024;
  void *args[] = {&a};
  const int tok = prof_begin(e);
  const cudaError_t r = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(snai_pass_kernel),
                                                    dim3(sm_count(e.device)), dim3(kPassThreads), args, smem,
                                                    e.stream);
  e.launches++;
  const double wbytes = 4.0 * ((double)d.L * (4.0 * d.D * d.D + 2.0 * d.F * d.D) + (double)d.V * d.D);
  prof_end(e, tok, kProfPass,
           wbytes + kv_positions * 2.0 * d.att_ch * 4 * d.L + 4.0 * M * (d.V + d.D * (6.0 * d.L + 2)),
           2.0 * M * (d.L * (4.0 * d.D * d.D + 2.0 * d.F * d.D) + (double)d.V * d.D) + kv_positions * 4.0 * d.att_ch * d.L);
  if (r != cudaSuccess) {
    cudaGetLastError();
    set_error("pass kernel launch failed: %s", cudaGetErrorString(r));
    return -4;
  }
  return 0;
}

// Copies a chunk's rows (e.rows_stage, e.out_stage) to the device.
static int upload_rows(Engine &e, int M, int n_out) {
  if (cudaMemcpyAsync(e.rows_d, e.rows_stage.data(), sizeof(RowDesc) * M, cudaMemcpyHostToDevice, e.stream) !=
          cudaSuccess ||
      (n_out && cudaMemcpyAsync(e.outrows_d, e.out_stage.data(), sizeof(int2) * n_out, cudaMemcpyHostToDevice,
                                e.stream) != cudaSuccess)) {
    set_error("row upload failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -4;
  }
  return 0;
}

// pack: the chunk's rows by value (the embedding kernel writes them to the
// device), or nullptr when they are on the device already.
template <typename TA>
static int run_chunk_typed(Engine &e, int M, const int *tokens_d, int n_out, bool out_tc, double kv_positions,
                           bool defer, const RowPack *pack) {
  const Dims &d = e.d;
  if constexpr (sizeof(TA) == 4) {
    if (pass_kernel_ok(e, M, n_out, defer)) {
      if (pack) {
        const int rc = upload_rows(e, M, n_out);
        if (rc) return rc;
      }
      return launch_pass(e, M, tokens_d, kv_positions);
    }
  }
  RowPack pk{};
  if (pack) pk = *pack;
  const double ea = sizeof(TA);
  TA *x = static_cast<TA *>(e.x);
  TA *att = static_cast<TA *>(e.att);
  TA *u = static_cast<TA *>(e.u);
  // a one-row pass whose row came by value: the first QKV GEMV does the
  // embedding kernel's work (one launch fewer)
  const bool fold = gemv_norm(e, M) && pk.n == 1 && d.D % 4 == 0 && (size_t)d.D * 16 <= kRowTileBytes;
  if (!fold) {
    const int tok = prof_begin(e);
    launch_k(e, true, embed_norm_kernel<TA>, dim3(M), dim3(kNormThreads), 0, e.rows_d, pk, e.rows_d, e.outrows_d,
             tokens_d, e.emb, e.layers[0].rms_att, e.h, x, e.hist, e.seq_len_d, d.V, d.D, d.ctx);
    prof_end(e, tok, kProfEmbed, (double)M * d.D * (8 + ea), 0.0);
  }
  for (int l = 0; l < d.L; ++l) {
    const LayerWeights &w = e.layers[l];
    EpiQKV eq{e.rows_d, e.q, e.kv, e.rope, d.D, d.att_ch, d.hs, e.kv_slot_stride, (size_t)l * e.kv_layer_stride,
              e.kv_part_stride, e.kv_head_stride, defer ? e.kvs : nullptr};
    if (tc_path(e, M)) qkv_tma_maps(e, M, &eq);
    // layer 0 reads the embedding kernel's normalised rows; later layers
    // normalise h inside the QKV GEMV on a small pass
    const bool fuse = gemv_norm(e, M);
    const bool fq = fuse && l > 0;
    GemvNorm nq = fq ? GemvNorm{w.rms_att, nullptr} : GemvNorm{};
    const void *qa = fq ? static_cast<const void *>(e.h) : x;
    if (fold && l == 0) {
      nq = GemvNorm{w.rms_att, nullptr};
      nq.emb = 1;
      nq.ef = GemvEmbed{tokens_d, e.h, e.hist, e.seq_len_d, d.V, d.ctx, e.rows_d, e.outrows_d};
      nq.pk = pk;
      qa = e.emb;
    }
    int rc = project(e, kProfQKV, M, 3 * d.D, d.D, qa, w.wqkv, w.wqkv_h, eq, 3.0 * M * d.att_ch * 4, nq);
    if (rc) return rc;
    launch_attention<TA>(e, M, l, att, kv_positions, defer, pk);
    EpiResidual res;
    if (!residual_epi(e, M, &res)) return -5;
    rc = project(e, kProfWo, M, d.D, d.D, att, w.wo, w.wo_h, res, 8.0 * M * d.D, GemvNorm{}, true);
    if (rc) return rc;
    if (!fuse) launch_norm<TA>(e, M, nullptr, w.rms_ffn, x);
    rc = project(e, kProfUp, M, d.F, d.D, fuse ? static_cast<const void *>(e.h) : x, w.wup, w.wup_h,
                 EpiSilu<TA>{u, d.F}, ea * M * d.F, fuse ? GemvNorm{w.rms_ffn, nullptr} : GemvNorm{});
    if (rc) return rc;
    rc = project(e, kProfDown, M, d.D, d.F, u, w.wdown, w.wdown_h, res, 8.0 * M * d.D);
    if (rc) return rc;
    if (l + 1 < d.L && !fuse) launch_norm<TA>(e, M, nullptr, e.layers[l + 1].rms_att, x);
  }
  if (n_out > 0) {
    EpiLogits el{e.logits, e.outrows_d, (long long)d.V};
    const double ob = 4.0 * n_out * d.V;
    if (out_tc && e.precision == kBF16) {
      __nv_bfloat16 *xo = static_cast<__nv_bfloat16 *>(e.xo);
      launch_norm<__nv_bfloat16>(e, n_out, e.outrows_d, e.rms_final, xo);
      return project(e, kProfLogits, n_out, d.V, d.D, xo, e.w_out, e.w_out_h, el, ob);
    }
    if (gemv_norm(e, n_out))
      return project(e, kProfLogits, n_out, d.V, d.D, e.h, e.w_out, e.w_out_h, el, ob,
                     GemvNorm{e.rms_final, e.outrows_d});
    float *xo = static_cast<float *>(e.xo);
    launch_norm<float>(e, n_out, e.outrows_d, e.rms_final, xo);
    return project(e, kProfLogits, n_out, d.V, d.D, xo, e.w_out, e.w_out_h, el, ob);
  }
  return 0;
}

// ---- bounded-wait self-test ----
//
// One warp initialises an mbarrier that expects one arrival and waits on its
// first phase, which nothing completes.  The wait gives up after limit_ns,
// records kErrWaitSelfTest in the engine's error word (the same path every
// kernel's expired wait takes) and the kernel returns normally, so the
// context stays usable.  `out` receives 1 if the wait gave up, 0 if it
// (impossibly) completed.
__global__ void wait_selftest_kernel(int *__restrict__ err, int *__restrict__ out, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  const bool done = mbar_wait_bounded_ns(&bar, 0, err, kErrWaitSelfTest, limit_ns);
  if (threadIdx.x == 0) *out = done ? 0 : 1;
}

int wait_selftest(Engine &e, long long limit_ns) {
  wait_selftest_kernel<<<1, 32, 0, e.stream>>>(e.err_d, e.ids_d, (unsigned long long)limit_ns);
  e.launches++;
  const cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) {
    set_error("kernel launch failed: %s", cudaGetErrorString(le));
    return -4;
  }
  return 0;
}

// ---- decode step on the device (graph body) ----

// Per-step uniforms of the current step into the sampler's buffer.
__global__ void stage_step_kernel(const float *__restrict__ unif_all, float *__restrict__ unif,
                                  const int *__restrict__ step, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) unif[b] = unif_all[(size_t)(*step) * batch + b];
}

// Row descriptors of a decode step: slot, its current position, token index b
// (ids_d[b]), logits into the slot; the logits row map (row b, slot).
__global__ void decode_rows_kernel(const int *__restrict__ slots, const int *__restrict__ seq_len,
                                   RowDesc *__restrict__ rows, int2 *__restrict__ outrows, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) {
    const int s = slots[b];
    rows[b] = RowDesc{s, seq_len[s], b, s};
    outrows[b] = make_int2(b, s);
  }
}

// The step's ids out, then the counter advances (one thread does the
// increment after every thread of its block has read the counter).
__global__ void finish_step_kernel(const int *__restrict__ ids, int *__restrict__ ids_all, int *__restrict__ step,
                                   int batch) {
  const int st = *step;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) ids_all[(size_t)st * batch + b] = ids[b];
  __syncthreads();
  if (threadIdx.x == 0) *step = st + 1;
}

// One chunk of rows in the operand type of its path.
static int run_chunk(Engine &e, int M, const int *tokens_d, int n_out, bool out_tc, double kv_positions, bool defer,
                     const RowPack *pack = nullptr) {
  return (tc_path(e, M) && e.precision == kBF16)
             ? run_chunk_typed<__nv_bfloat16>(e, M, tokens_d, n_out, out_tc, kv_positions, defer, pack)
             : run_chunk_typed<float>(e, M, tokens_d, n_out, out_tc, kv_positions, defer, pack);
}

int decode_step_device(Engine &e, int batch, const SampleLaunch &sampler) {
  const int tpb = 256, nb = (batch + tpb - 1) / tpb;
  stage_step_kernel<<<nb, tpb, 0, e.stream>>>(e.unif_all, e.unif_d, e.step_d, batch);
  e.launches++;
  int rc = launch_sampler(sampler, e.stream);
  if (rc) return rc;
  e.launches++;
  decode_rows_kernel<<<nb, tpb, 0, e.stream>>>(e.slots_d, e.seq_len_d, e.rows_d, e.outrows_d, batch);
  e.launches++;
  const bool tc = tc_path(e, batch);
  rc = run_chunk(e, batch, e.ids_d, batch, tc, 0.0, true);
  if (rc) return rc;
  finish_step_kernel<<<1, 1024, 0, e.stream>>>(e.ids_d, e.ids_all, e.step_d, batch);
  e.launches++;
  const cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) {
    set_error("kernel launch failed: %s", cudaGetErrorString(le));
    return -4;
  }
  return 0;
}

int run_rows(Engine &e, const RowDesc *rows, int n, const int *tokens_d) {
  for (int c0 = 0; c0 < n; c0 += e.m_max) {
    const int M = std::min(e.m_max, n - c0);
    // rows of this chunk and the ones that need logits
    e.rows_stage.assign(rows + c0, rows + c0 + M);
    e.out_stage.clear();
    double kv_positions = 0;
    for (int i = 0; i < M; ++i) {
      kv_positions += e.rows_stage[i].pos + 1;
      if (e.rows_stage[i].out >= 0) e.out_stage.push_back(make_int2(i, e.rows_stage[i].out));
    }
    const int n_out = (int)e.out_stage.size();
    // every slot at most once in the chunk (a decode step): the new K and V
    // are staged and appended by the attention kernel
    bool defer = true;
    e.slot_seen.assign((size_t)e.max_seqs, 0);
    for (int i = 0; i < M && defer; ++i) {
      const int s = e.rows_stage[i].slot;
      defer = !e.slot_seen[s];
      e.slot_seen[s] = 1;
    }
    // a chunk of a few rows goes to the device by value, with the first kernel
    const bool by_value = M <= kRowPackMax;
    RowPack pack{};
    if (by_value) {
      for (int i = 0; i < M; ++i) pack.r[i] = e.rows_stage[i];
      for (int i = 0; i < n_out; ++i) pack.out[i] = e.out_stage[i];
      pack.n = M;
      pack.n_out = n_out;
    } else {
      const int rc = upload_rows(e, M, n_out);
      if (rc) return rc;
    }
    const bool out_tc = tc_path(e, n_out);
    const int rc = run_chunk(e, M, tokens_d, n_out, out_tc, kv_positions, defer, by_value ? &pack : nullptr);
    if (rc) return rc;
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      set_error("kernel launch failed: %s", cudaGetErrorString(le));
      return -4;
    }
  }
  return 0;
}

// ---- profiler ----
static cudaEvent_t prof_event(Engine &e) {
  if (!e.prof_free.empty()) {
    cudaEvent_t ev = e.prof_free.back();
    e.prof_free.pop_back();
    return ev;
  }
  cudaEvent_t ev = nullptr;
  cudaEventCreate(&ev);
  return ev;
}

int prof_begin(Engine &e) {
  if (!e.prof) return -1;
  cudaEvent_t a = prof_event(e);
  cudaEventRecord(a, e.stream);
  e.prof_pending.push_back(Engine::ProfPending{-1, a, nullptr, 0.0, 0.0});
  return (int)e.prof_pending.size() - 1;
}

void prof_end(Engine &e, int token, int kind, double bytes, double flops) {
  if (token < 0 || token >= (int)e.prof_pending.size()) return;
  cudaEvent_t b = prof_event(e);
  cudaEventRecord(b, e.stream);
  Engine::ProfPending &p = e.prof_pending[token];
  p.kind = kind;
  p.b = b;
  p.bytes = bytes;
  p.flops = flops;
}

void prof_collect(Engine &e) {
  if (e.prof_pending.empty()) return;
  cudaStreamSynchronize(e.stream);
  for (auto &p : e.prof_pending) {
    if (p.b && p.kind >= 0 && p.kind < kProfKinds) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
        e.prof_ms[p.kind] += ms;
        e.prof_count[p.kind] += 1;
        e.prof_bytes[p.kind] += p.bytes;
        e.prof_flops[p.kind] += p.flops;
      }
      e.prof_free.push_back(p.b);
    }
    e.prof_free.push_back(p.a);
  }
  e.prof_pending.clear();
}

int convert_bf16_segments(Engine &e, const Bf16Segments &segs) {
  if (segs.count <= 0) return 0;
  to_bf16_segments_kernel<<<dim3(2 * device_sm_count(e.device), segs.count), 256, 0, e.stream>>>(segs);
  e.launches++;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int convert_bf16(Engine &e, const float *src, __nv_bfloat16 *dst, size_t n) {
  to_bf16_kernel<<<1184, 256, 0, e.stream>>>(src, dst, n);
  e.launches++;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int fill_f32(Engine &e, float *dst, size_t n, float v) {
  fill_f32_kernel<<<592, 256, 0, e.stream>>>(dst, n, v);
  e.launches++;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace snai
