// sampler.cu - the reference's two logits -> token samplers on sm_100a.
//
// One CTA of 512 threads per row.  Both kernels reproduce the PHP code's
// double-precision arithmetic *bit for bit* for given logits and uniform u:
//
// Variant A (src/snai_inference.php:151-195).
//   t_v = fp32(L_v / T); penalised ids (the unique history, held as a bitmap
//   in shared memory): t = fp32(t / rep) if t > 0 else fp32(t * rep).
//   Greedy (T <= 0.01): first index of the maximum.  Otherwise
//   p_v = exp(t_v - max) in double (snai_exp.h), S = sequential sum of p_v
//   in vocab order, r = u*S, id = first v whose running sum >= r.
//   The sequential sum is replaced by a parallel one whose distance from the
//   sequential one is bounded (below); when r is far enough from the running
//   sums around the chosen id, the choice provably equals the sequential
//   one.  Otherwise (probability ~ V^2 2^-52) warp 0 redoes the row
//   sequentially.  Either way the id is the sequential algorithm's id.
//
// Variant B (src/tensor_ffi_adapter.php:168-204).
//   val_v = L_v - rep for ids in the input set, else L_v (double).  Stable
//   descending sort + top_k = the k smallest (-val, v).  The kernel
//   radix-selects a threshold on 32-bit keys of fp32 lower bounds of val,
//   gathers every element whose fp32 upper bound reaches the threshold (a
//   superset of the top k), sorts that set exactly by (val desc, v asc) and
//   runs the PHP softmax / top-p / draw sequentially over the k survivors.
#include <cfloat>
#include <cmath>
#include <climits>
#include <cstdio>

#include "common.cuh"
#include "engine.h"
#include "snai_exp.h"

namespace snai {

constexpr int kSampThreads = 512;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kMaxTopK = 1024;
constexpr int kCandCap = 4096;  // exact-sort capacity of variant B
constexpr int kMaxVocab = 1 << 19;
constexpr int kMaxSeg = kMaxVocab / 2048;

struct SampArgs {
  const float *logits;
  long long ld;
  const int *row_map;
  int V;
  const int *hist;
  long long hist_ld;
  int hist_cols;
  const int *hist_len;
  const float *uniforms;
  double T, Tinv, rep, top_p;
  int top_k;
  int nan_guard;
  int *out;
  int *err;
};

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------

// Marks the row's history ids (each once, ids outside [0,V) ignored) in a
// shared bitmap of V bits.  Ends with a barrier.
__device__ void build_bitmap(const SampArgs &a, int mrow, uint32_t *bits) {
  const int words = (a.V + 31) >> 5;
  for (int i = threadIdx.x; i < words; i += blockDim.x) bits[i] = 0u;
  __syncthreads();
  int n = a.hist_len ? a.hist_len[mrow] : a.hist_cols;
  n = min(max(n, 0), a.hist_cols);
  const int *hr = a.hist + (size_t)mrow * a.hist_ld;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = hr[i];
    if (t >= 0 && t < a.V) atomicOr(&bits[t >> 5], 1u << (t & 31));
  }
  __syncthreads();
}

__device__ __forceinline__ bool in_set(const uint32_t *bits, int v) { return (bits[v >> 5] >> (v & 31)) & 1u; }

// fp32(x / T) for the double T, exactly as fp32(double(x) / T):
// q = x * (1/T) is within 2 ulp of x/T; rounding q to fp32 gives the same
// float as rounding the correctly rounded quotient unless q lies within a few
// double ulps of a float rounding midpoint, or outside the normal float
// range, and then the real division is done.
__device__ __forceinline__ float div_to_f32(float x, double T, double Tinv) {
  const double q = __dmul_rn((double)x, Tinv);
  const unsigned long long b = (unsigned long long)__double_as_longlong(q);
  const int ex = (int)((b >> 52) & 0x7FF) - 1023;
  const long long low = (long long)(b & 0x1FFFFFFFull);
  const bool safe = (q == 0.0) || (ex >= -126 && ex <= 127 && llabs(low - 0x10000000ll) > 4);
  return safe ? __double2float_rn(q) : __double2float_rn(__ddiv_rn((double)x, T));
}

// Variant A's stored value for vocab entry v (src/snai_inference.php:153, 160-164).
__device__ __forceinline__ float tempered(const SampArgs &a, const uint32_t *bits, float x, int v) {
  float t = div_to_f32(x, a.T, a.Tinv);
  if (in_set(bits, v)) {
    const double d = (double)t;
    t = d > 0.0 ? __double2float_rn(__ddiv_rn(d, a.rep)) : __double2float_rn(__dmul_rn(d, a.rep));
  }
  return t;
}

// Exclusive block scan of doubles in thread order; `tot` = block total.
// Summation order is fixed (warp Kogge-Stone, then warp totals in order).
__device__ double block_excl_scan(double v, double *wsum, double &tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl = __dadd_rn(incl, n);
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  double base = 0.0, all = 0.0;
  for (int w = 0; w < kSampWarps; ++w) {
    if (w == warp) base = all;
    all = __dadd_rn(all, wsum[w]);
  }
  __syncthreads();
  tot = all;
  // exclusive prefix inside the warp = the previous lane's inclusive tree sum
  double ex = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) ex = 0.0;
  return __dadd_rn(base, ex);
}

// ---------------------------------------------------------------------------
// Variant A
// ---------------------------------------------------------------------------

struct SmemA {
  double seg[kMaxSeg];      // per-segment sums (segment = 2048 entries)
  double wsum[kSampWarps];
  float bmax[kSampWarps];
  int bidx[kSampWarps];
  double S, r;
  int seg_star;
  double seg_base;
  int cand;
  double cand_hi, cand_lo;  // running sums at cand and cand-1
  int certified;
};

// p_v for an index (t_v known) in the contract's arithmetic.
__device__ __forceinline__ double prob_a(float t, double maxv) { return snai_exp(__dsub_rn((double)t, maxv)); }

// The sequential algorithm of src/snai_inference.php:178-194, by warp 0.
__device__ int sequential_a(const SampArgs &a, const uint32_t *bits, const float *L, double maxv, double u) {
  const int lane = threadIdx.x & 31;
  double sum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const double p = v < a.V ? prob_a(tempered(a, bits, L[v], v), maxv) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) sum = __dadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
  }
  const double r = __dmul_rn(u, sum);
  double cum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const double p = v < a.V ? prob_a(tempered(a, bits, L[v], v), maxv) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) {
      cum = __dadd_rn(cum, __shfl_sync(0xffffffffu, p, j));
      if (cum >= r) return b + j;
    }
  }
  return 0;  // `$best_token = 0` when nothing qualifies (NaN sums)
}

__global__ void __launch_bounds__(kSampThreads) sample_a_kernel(SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemA &sm = *reinterpret_cast<SmemA *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemA));
  const int b = blockIdx.x;
  const int mrow = a.row_map ? a.row_map[b] : b;
  const float *L = a.logits + (size_t)mrow * a.ld;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int V = a.V;

  if (a.nan_guard) {
    const float l0 = L[0];
    if (l0 != l0) {
      if (threadIdx.x == 0) a.out[b] = -1;
      return;
    }
  }
  build_bitmap(a, mrow, bits);

  // ---- pass 1: tempered values, maximum and the first index attaining it ----
  float best = -INFINITY;
  int bi = INT_MAX;
  const bool vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  for (int v0 = threadIdx.x * 4; v0 < V; v0 += kSampThreads * 4) {
    float x[4];
    if (vec && v0 + 3 < V) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(L + v0));
      x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = v0 + j < V ? L[v0 + j] : NAN;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (v0 + j >= V) break;
      const float t = tempered(a, bits, x[j], v0 + j);
      if (t > best) { best = t; bi = v0 + j; }  // indices ascend per thread: ties keep the first
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  if (lane == 0) { sm.bmax[warp] = best; sm.bidx[warp] = bi; }
  __syncthreads();
  best = sm.bmax[0];
  bi = sm.bidx[0];
  for (int w = 1; w < kSampWarps; ++w)
    if (sm.bmax[w] > best || (sm.bmax[w] == best && sm.bidx[w] < bi)) { best = sm.bmax[w]; bi = sm.bidx[w]; }
  // PHP: max starts at -INF and only a strictly larger value moves it.
  const bool any = best > -INFINITY;
  const double maxv = any ? (double)best : -INFINITY;
  if (a.T <= 0.01) {
    if (threadIdx.x == 0) a.out[b] = any ? bi : 0;
    return;
  }
  const double u = (double)a.uniforms[b];

  // ---- pass 2: segment sums of p_v (segment = 2048 consecutive ids) ----
  const int nseg = (V + 2047) / 2048;
  for (int s = 0; s < nseg; ++s) {
    const int v0 = s * 2048 + threadIdx.x * 4;
    double c = 0.0;
    if (v0 < V) {
      float x[4];
      if (vec && v0 + 3 < V) {
        const float4 q = __ldg(reinterpret_cast<const float4 *>(L + v0));
        x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = v0 + j < V ? L[v0 + j] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v0 + j < V) c = __dadd_rn(c, prob_a(tempered(a, bits, x[j], v0 + j), maxv));
    }
    double tot;
    block_excl_scan(c, sm.wsum, tot);
    if (threadIdx.x == 0) sm.seg[s] = tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double S = 0.0;
    for (int s = 0; s < nseg; ++s) S = __dadd_rn(S, sm.seg[s]);
    const double r = __dmul_rn(u, S);
    int ss = -1;
    double base = 0.0, run = 0.0;
    for (int s = 0; s < nseg; ++s) {
      const double nxt = __dadd_rn(run, sm.seg[s]);
      if (nxt >= r) { ss = s; base = run; break; }
      run = nxt;
    }
    sm.S = S;
    sm.r = r;
    sm.seg_star = ss;
    sm.seg_base = base;
    sm.cand = INT_MAX;
    sm.certified = 0;
  }
  __syncthreads();
  const double S = sm.S, r = sm.r;
  const int ss = sm.seg_star;
  bool fallback = !(isfinite(S) && isfinite(r) && ss >= 0 && u >= 0.0 && u <= 1.0);

  if (!fallback) {
    // ---- pass 3: scan inside the crossing segment ----
    const int v0 = ss * 2048 + threadIdx.x * 4;
    double p[4] = {0.0, 0.0, 0.0, 0.0};
    double c = 0.0;
    if (v0 < V) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v0 + j < V) {
          p[j] = prob_a(tempered(a, bits, L[v0 + j], v0 + j), maxv);
          c = __dadd_rn(c, p[j]);
        }
    }
    double tot;
    const double ex = block_excl_scan(c, sm.wsum, tot);
    double prev = __dadd_rn(sm.seg_base, ex);
    for (int j = 0; j < 4; ++j) {
      if (v0 + j >= V) break;
      const double cur = __dadd_rn(prev, p[j]);
      if (cur >= r) {
        atomicMin(&sm.cand, v0 + j);
        break;
      }
      prev = cur;
    }
    __syncthreads();
    const int cand = sm.cand;
    if (cand >= v0 && cand < v0 + 4 && v0 < V) {
      // running sums P'(cand-1), P'(cand) as this thread formed them
      double pre = __dadd_rn(sm.seg_base, ex);
      for (int j = 0; j < cand - v0; ++j) pre = __dadd_rn(pre, p[j]);
      sm.cand_lo = pre;
      sm.cand_hi = __dadd_rn(pre, p[cand - v0]);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int ok = 0;
      if (cand != INT_MAX) {
        // Any summation tree of depth h over non-negative terms is within
        // h 2^-53 (1+o(1)) of the exact sum.  The sequential running sum at v
        // has depth v; ours has depth <= nseg + 56 (4 per chunk, 5 per warp
        // scan, 16 warps, nseg segments, twice).  Bounds below use 2^-52,
        // twice the first-order constant.
        const double slack = (double)(nseg + 64);
        const double Er = ((double)V + slack) * 0x1p-52 * r;
        const double hi = sm.cand_hi, lo = sm.cand_lo;
        const bool up = hi - ((double)cand + slack) * 0x1p-52 * hi >= r + Er;
        const bool dn = cand == 0 || lo + ((double)cand + slack) * 0x1p-52 * lo < r - Er;
        ok = up && dn;
      }
      sm.certified = ok;
    }
    __syncthreads();
    if (sm.certified) {
      if (threadIdx.x == 0) a.out[b] = cand;
      return;
    }
    fallback = true;
  }
  if (warp == 0) {
    const int id = sequential_a(a, bits, L, maxv, u);
    if (lane == 0) a.out[b] = id;
  }
}

// ---------------------------------------------------------------------------
// Variant B
// ---------------------------------------------------------------------------

struct SmemB {
  unsigned int hist[4096];
  unsigned int wtot[kSampWarps];
  unsigned long long ckey[kCandCap];  // exact order key of a candidate
  int cidx[kCandCap];
  int ncand;
  unsigned int prefix, pmask;
  int need;
  int bstar;
  unsigned int bcount;
  int ties_left;
  int order[kMaxTopK];
  double val[kMaxTopK];
  double p[kMaxTopK];
  double cum[kMaxTopK];
  int nf;
  int overflow;
};

// Monotone 32-bit key of a float (NaN lowest; -0 and +0 equal, as PHP
// compares them).
__device__ __forceinline__ unsigned int okey32(float f) {
  if (f != f) return 0u;
  if (f == 0.f) f = 0.f;
  const unsigned int u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Monotone 64-bit key of a double (NaN lowest).
__device__ __forceinline__ unsigned long long okey64(double d) {
  if (d != d) return 0ull;
  if (d == 0.0) d = 0.0;
  const unsigned long long u = (unsigned long long)__double_as_longlong(d);
  return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}
__device__ __forceinline__ double key_to_double(unsigned long long k) {
  const unsigned long long u = (k & 0x8000000000000000ull) ? (k & 0x7FFFFFFFFFFFFFFFull) : ~k;
  return __longlong_as_double((long long)u);
}

// val_v and the fp32 keys bracketing it.
struct ValB {
  double val;
  unsigned int klo, khi;
  bool pen;
};
__device__ __forceinline__ ValB val_b(const SampArgs &a, const uint32_t *bits, float x, int v) {
  ValB r;
  r.pen = in_set(bits, v);
  if (!r.pen) {
    r.val = (double)x;
    r.klo = r.khi = okey32(x);
  } else {
    r.val = __dsub_rn((double)x, a.rep);
    r.klo = okey32(__double2float_rd(r.val));
    r.khi = okey32(__double2float_ru(r.val));
  }
  return r;
}

__device__ __forceinline__ void hist_add(unsigned int *hist, unsigned int bin, bool active) {
  const unsigned int mask = __ballot_sync(0xffffffffu, active);
  if (!active) return;
  const unsigned int peers = __match_any_sync(mask, bin);
  if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned int)__popc(peers));
}

__device__ __forceinline__ void push_cand(SmemB &sm, double val, int v) {
  const int slot = atomicAdd(&sm.ncand, 1);
  if (slot < kCandCap) {
    sm.ckey[slot] = okey64(val);
    sm.cidx[slot] = v;
  } else {
    sm.overflow = 1;
  }
}

// candidate i precedes candidate j in PHP's arsort order
__device__ __forceinline__ bool precedes(unsigned long long ki, int vi, unsigned long long kj, int vj) {
  return ki > kj || (ki == kj && vi < vj);
}

__global__ void __launch_bounds__(kSampThreads) sample_b_kernel(SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB));
  const int b = blockIdx.x;
  const int mrow = a.row_map ? a.row_map[b] : b;
  const float *L = a.logits + (size_t)mrow * a.ld;
  const int V = a.V;
  const int k = min(a.top_k, V);
  build_bitmap(a, mrow, bits);

  const int iters = (V + kSampThreads - 1) / kSampThreads;  // warp-uniform trip count

  // ---- radix select on klo: 12 + 12 + 8 bits, most significant first ----
  if (threadIdx.x == 0) {
    sm.prefix = 0u;
    sm.pmask = 0u;
    sm.need = k;
    sm.ncand = 0;
    sm.overflow = 0;
  }
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
  bool exact = false;
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], wd = widths[pass];
    const unsigned int bmask = (1u << wd) - 1u;
    for (int i = threadIdx.x; i < 4096; i += kSampThreads) sm.hist[i] = 0u;
    __syncthreads();
    const unsigned int prefix = sm.prefix, pmask = sm.pmask;
    for (int it = 0; it < iters; ++it) {
      const int v = it * kSampThreads + threadIdx.x;
      bool act = false;
      unsigned int bin = 0;
      if (v < V) {
        const ValB x = val_b(a, bits, L[v], v);
        act = (x.klo & pmask) == prefix;
        bin = (x.klo >> sh) & bmask;
      }
      hist_add(sm.hist, bin, act);
    }
    __syncthreads();
    // largest bin whose suffix count reaches `need`: warp 0 scans from the top
    if (threadIdx.x < 32) {
      const int need = sm.need;
      const int nb = 1 << wd;
      const int per = nb / 32;  // bins per lane, lane 31 owns the top ones
      const int lo = threadIdx.x * per;
      unsigned int mine = 0;
      for (int i = 0; i < per; ++i) mine += sm.hist[lo + i];
      // inclusive suffix sum over lanes (lane l: bins >= lo)
      unsigned int suf = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int n = __shfl_down_sync(0xffffffffu, suf, o);
        if ((int)threadIdx.x + o < 32) suf += n;
      }
      const unsigned int above_lane = suf - mine;  // bins above this lane's range
      const bool here = above_lane < (unsigned)need && suf >= (unsigned)need;
      if (here) {
        unsigned int acc = above_lane;
        int bs = lo;
        for (int i = per - 1; i >= 0; --i) {
          const unsigned int c = sm.hist[lo + i];
          if (acc + c >= (unsigned)need) { bs = lo + i; break; }
          acc += c;
        }
        sm.bstar = bs;
        sm.bcount = sm.hist[bs];
        sm.need = need - (int)acc;
        sm.prefix = prefix | ((unsigned int)bs << sh);
        sm.pmask = pmask | (bmask << sh);
      }
    }
    __syncthreads();
    exact = (pass == 2);
    const unsigned int bcount = sm.bcount;
    __syncthreads();  // everyone has read bcount before the next pass clears hist
    if (bcount <= 1024u) break;
  }
  const unsigned int tau = sm.prefix;  // klo threshold (low unresolved bits 0)
  const bool tie_path = exact && sm.bcount > 1024u;
  __syncthreads();

  // ---- gather the superset {khi >= tau} ----
  // On the tie path the many non-penalised entries equal to tau are taken
  // only as the first `need` of them in vocab order (the later ones cannot
  // reach the top k: they tie in value and lose on index).
  for (int it = 0; it < iters; ++it) {
    const int v = it * kSampThreads + threadIdx.x;
    if (v < V) {
      const ValB x = val_b(a, bits, L[v], v);
      if (x.khi >= tau) {
        if (!(tie_path && !x.pen && x.klo == tau)) push_cand(sm, x.val, v);
      }
    }
  }
  if (tie_path) {
    if (threadIdx.x == 0) sm.ties_left = sm.need;
    __syncthreads();
    for (int it = 0; it < iters; ++it) {
      const int v = it * kSampThreads + threadIdx.x;
      bool f = false;
      double val = 0.0;
      if (v < V) {
        const ValB x = val_b(a, bits, L[v], v);
        f = !x.pen && x.klo == tau;
        val = x.val;
      }
      // rank of this flag among the block's flags in index order
      const unsigned int bal = __ballot_sync(0xffffffffu, f);
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      if (lane == 0) sm.wtot[warp] = __popc(bal);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < kSampWarps; ++w) {
        if (w < warp) before += sm.wtot[w];
        total += sm.wtot[w];
      }
      const int rank = before + __popc(bal & ((1u << lane) - 1u));
      const int left = sm.ties_left;
      if (f && rank < left) push_cand(sm, val, v);
      __syncthreads();
      if (threadIdx.x == 0) sm.ties_left = left - min(total, left);
      __syncthreads();
      if (sm.ties_left <= 0) break;
    }
  }
  __syncthreads();
  if (sm.overflow) {
    if (threadIdx.x == 0) {
      a.out[b] = -2;
      record_error(a.err, kErrSamplerArgs);
    }
    return;
  }
  const int nc = sm.ncand;

  // ---- exact order of the candidates: rank by counting ----
  for (int i = threadIdx.x; i < nc; i += kSampThreads) {
    const unsigned long long ki = sm.ckey[i];
    const int vi = sm.cidx[i];
    int rank = 0;
    for (int j = 0; j < nc; ++j) rank += precedes(sm.ckey[j], sm.cidx[j], ki, vi) ? 1 : 0;
    if (rank < k) {
      sm.order[rank] = vi;
      sm.val[rank] = key_to_double(ki);
    }
  }
  __syncthreads();

  // ---- src/tensor_ffi_adapter.php:180-204 over the k survivors ----
  if (a.T < 0.01) {
    if (threadIdx.x == 0) a.out[b] = sm.order[0];
    return;
  }
  for (int i = threadIdx.x; i < k; i += kSampThreads) sm.p[i] = snai_exp(__ddiv_rn(sm.val[i], a.T));
  __syncthreads();
  __shared__ double sum_sh;
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < k; ++i) s = __dadd_rn(s, sm.p[i]);
    sum_sh = s;
  }
  __syncthreads();
  const double sum = sum_sh;
  for (int i = threadIdx.x; i < k; i += kSampThreads) sm.p[i] = __ddiv_rn(sm.p[i], sum);
  __syncthreads();
  if (threadIdx.x == 0) {
    double cum = 0.0;
    int nf = 0;
    for (int i = 0; i < k; ++i) {
      cum = __dadd_rn(cum, sm.p[i]);
      sm.cum[i] = cum;  // $cum_check after i+1 terms is this same sum
      nf = i + 1;
      if (cum >= a.top_p) break;
    }
    const double r = __dmul_rn((double)a.uniforms[b], cum);
    int id = sm.order[0];
    for (int i = 0; i < nf; ++i)
      if (r <= sm.cum[i]) { id = sm.order[i]; break; }
    a.out[b] = id;
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

int check_sample_args(const SampleLaunch &s) {
  if (s.rows < 0) { set_error("sampler: rows < 0"); return -2; }
  if (s.V < 1 || s.V > kMaxVocab) { set_error("sampler: vocab %d outside [1, %d]", s.V, kMaxVocab); return -2; }
  if (s.ld < s.V) { set_error("sampler: row stride %lld < vocab %d", s.ld, s.V); return -2; }
  if (!s.logits || !s.out_ids || (s.rows > 0 && !s.uniforms && s.temperature > 0.01)) {
    set_error("sampler: null logits / uniforms / output");
    return -2;
  }
  if (s.hist_cols < 0 || (s.hist_cols > 0 && !s.hist) || s.hist_ld < s.hist_cols) {
    set_error("sampler: bad history arguments");
    return -2;
  }
  if (s.variant == 0) {
    if (s.temperature == 0.0 || s.temperature != s.temperature) {
      // PHP 8 raises DivisionByZeroError for `/ 0.0`
      set_error("sampler variant 0: temperature must be non-zero");
      return -2;
    }
  } else if (s.variant == 1) {
    if (s.top_k < 1 || s.top_k > kMaxTopK) { set_error("sampler variant 1: top_k %d outside [1, %d]", s.top_k, kMaxTopK); return -2; }
  } else {
    set_error("sampler: unknown variant %d", s.variant);
    return -2;
  }
  return 0;
}

int launch_sampler(const SampleLaunch &s, cudaStream_t stream) {
  int rc = check_sample_args(s);
  if (rc) return rc;
  if (s.rows == 0) return 0;
  SampArgs a;
  a.logits = s.logits;
  a.ld = s.ld;
  a.row_map = s.row_map;
  a.V = s.V;
  a.hist = s.hist;
  a.hist_ld = s.hist_ld;
  a.hist_cols = s.hist_cols;
  a.hist_len = s.hist_len;
  a.uniforms = s.uniforms;
  a.T = s.temperature;
  a.Tinv = 1.0 / s.temperature;
  a.rep = s.rep;
  a.top_p = s.top_p;
  a.top_k = s.top_k;
  a.nan_guard = s.nan_guard;
  a.out = s.out_ids;
  a.err = s.err;
  const size_t bitmap = (size_t)((s.V + 31) / 32) * 4;
  int dev = 0;
  cudaGetDevice(&dev);
  if (s.variant == 0) {
    const size_t sm = sizeof(SmemA) + bitmap;
    static unsigned long long set_mask = 0;
    if (!(set_mask & (1ull << dev))) {
      cudaFuncSetAttribute(sample_a_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      set_mask |= 1ull << dev;
    }
    sample_a_kernel<<<s.rows, kSampThreads, sm, stream>>>(a);
  } else {
    const size_t sm = sizeof(SmemB) + bitmap;
    static unsigned long long set_mask = 0;
    if (!(set_mask & (1ull << dev))) {
      cudaFuncSetAttribute(sample_b_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      set_mask |= 1ull << dev;
    }
    sample_b_kernel<<<s.rows, kSampThreads, sm, stream>>>(a);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("sampler launch failed: %s", cudaGetErrorString(e));
    return -4;
  }
  return 0;
}

}  // namespace snai
