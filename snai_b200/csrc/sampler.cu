// sampler.cu - the reference's two logits -> token samplers on sm_100a.
//
// One CTA of 512 threads per row; a row of up to 32768 logits is held in
// registers (thread t owns the 16-byte chunks t, t+512, ...), larger rows are
// re-read from L2 on every pass.  Both kernels reproduce the PHP code's
// double-precision decisions bit for bit for given logits and uniform u.
//
// Variant A (src/snai_inference.php:151-195).
//   t_v = fp32(L_v / T); penalised ids (the unique history, a bitmap in shared
//   memory): t = fp32(t / rep) if t > 0 else fp32(t * rep).  Greedy
//   (T <= 0.01): first index of the maximum.  Otherwise p_v = exp(t_v - max)
//   in double (snai_exp.h), S = sequential sum in vocab order, r = u*S, and
//   the id is the first v whose running sum reaches r.
//   The kernel replaces the sequential running sums by parallel ones with a
//   proven error bound and accepts the id only when r is farther from the
//   running sums around it than the bound ("certified"):
//     tier 1: p_v from fp32 expf (error bound per element: expf is within
//             2 ulp, the argument's rounding to float adds |x| 2^-24);
//     tier 2: p_v from the contract exponential itself (no exp error);
//     tier 3: warp 0 runs the sequential loop.
//   Each tier is exact whenever it answers, so the id is always the
//   sequential algorithm's id.
//
// Variant B (src/tensor_ffi_adapter.php:168-204).
//   val_v = L_v - rep for ids in the input set, else L_v (double).  The
//   stable descending sort + top_k keeps the k smallest (-val, v).  Fast
//   path: a histogram of fp32 lower bounds of val over distance bins below
//   the row maximum finds a threshold bin holding the k-th largest; every
//   element whose fp32 upper bound reaches that bin is gathered (a superset
//   of the top k), sorted exactly by (val desc, v asc), and the PHP softmax
//   / top-p / draw runs sequentially over the k survivors.  Rows the fast
//   path cannot settle (non-finite maxima, huge exact ties) go through a
//   general radix select.
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "engine.h"
#include "snai_exp.h"

namespace snai {

constexpr int kSampThreads = 512;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kMaxTopK = 1024;
constexpr int kCandCap = 4096;   // exact-sort capacity (general path)
constexpr int kFastCand = 2048;  // candidates the fast path accepts
constexpr int kMaxVocab = 1 << 19;
constexpr int kMaxSeg = kMaxVocab / 2048;
constexpr int kSegGroup = 32;    // segments reduced per shared-memory round

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

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
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

// A row of logits: 16-byte chunk i of thread t covers entries
// 4*(t + 512*i) .. +3.  NV4 > 0: the row (V <= 2048*NV4) sits in registers;
// NV4 == 0: every access reads global memory (L2 after the first pass).
template <int NV4>
struct Row {
  const float *L;
  int V;
  bool vec;
  float4 r[NV4 > 0 ? NV4 : 1];

  __device__ __forceinline__ int layers() const { return NV4 > 0 ? NV4 : (V + 2047) / 2048; }
  __device__ __forceinline__ float4 fetch(int i) const {
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
    if (vec && v0 + 3 < V) return __ldg(reinterpret_cast<const float4 *>(L + v0));
    float4 f;
    f.x = v0 < V ? L[v0] : 0.f;
    f.y = v0 + 1 < V ? L[v0 + 1] : 0.f;
    f.z = v0 + 2 < V ? L[v0 + 2] : 0.f;
    f.w = v0 + 3 < V ? L[v0 + 3] : 0.f;
    return f;
  }
  __device__ __forceinline__ void load() {
    if constexpr (NV4 > 0) {
#pragma unroll
      for (int i = 0; i < NV4; ++i) r[i] = fetch(i);
    }
  }
  // Chunk layer i; with registers the choice is a chain of predicated moves,
  // so a run-time i never sends the array to local memory.
  __device__ __forceinline__ float4 get(int i) const {
    if constexpr (NV4 > 0) {
      float4 o = r[0];
#pragma unroll
      for (int q = 1; q < NV4; ++q)
        if (q == i) o = r[q];
      return o;
    } else {
      return fetch(i);
    }
  }
};

__device__ __forceinline__ float f4_at(const float4 &f, int j) { return j == 0 ? f.x : j == 1 ? f.y : j == 2 ? f.z : f.w; }
__device__ __forceinline__ void f4_set(float4 &f, int j, float v) {
  if (j == 0) f.x = v;
  else if (j == 1) f.y = v;
  else if (j == 2) f.z = v;
  else f.w = v;
}

// ---------------------------------------------------------------------------
// Variant A
// ---------------------------------------------------------------------------

struct SmemA {
  double wp[kSegGroup][kSampWarps];  // per-warp partial sums of p
  double we[kSegGroup][kSampWarps];  // per-warp partial sums of the error bound
  double seg[kMaxSeg];
  double segerr[kMaxSeg];
  double wsum[kSampWarps];
  float bmax[kSampWarps];
  int bidx[kSampWarps];
  double S, r, seg_base, err_base, err_tot;
  int seg_star;
  int cand;
  double cand_hi, cand_lo, ecand_hi, ecand_lo;
  int certified;
};

// p_v and its error bound.  EXACT: the contract exponential, error 0.  Else
// fp32 expf (CUDA: at most 2 ulp) of the argument rounded to float (relative
// error |x| 2^-24 after exp), bounded as p~ (3e-7 + 7e-8 |x|); below -87 the
// float result underflows and the bound is e^-87.
template <bool EXACT>
__device__ __forceinline__ double prob(float t, double maxv, double &err) {
  const double xd = __dsub_rn((double)t, maxv);
  if constexpr (EXACT) {
    err = 0.0;
    return snai_exp(xd);
  } else {
    if (!(xd >= -87.0)) {
      err = 1.7e-38;
      return 0.0;
    }
    const float xf = __double2float_rn(xd);
    const float pf = expf(xf);
    err = (double)pf * (3e-7 + 7e-8 * (double)fabsf(xf));
    return (double)pf;
  }
}

// tier 1 / tier 2 of variant A: returns the id, or -1 if not certified.
// `tv(i)` gives this thread's chunk i of tempered values.
template <bool EXACT, class TV>
__device__ int certified_draw(SmemA &sm, int V, int nl, double maxv, double u, const TV &tv) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // ---- segment sums (segment i = chunk layer i = 2048 consecutive ids) ----
  for (int g0 = 0; g0 < nl; g0 += kSegGroup) {
    const int g1 = min(nl, g0 + kSegGroup);
    for (int i = g0; i < g1; ++i) {
      const float4 t = tv(i);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      double c = 0.0, ce = 0.0;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v0 + j < V) {
          double e;
          c = __dadd_rn(c, prob<EXACT>(f4_at(t, j), maxv, e));
          ce += e;
        }
      c = warp_sum_d(c);
      ce = warp_sum_d(ce);
      if (lane == 0) {
        sm.wp[i - g0][warp] = c;
        sm.we[i - g0][warp] = ce;
      }
    }
    __syncthreads();
    if (threadIdx.x < g1 - g0) {
      double s = 0.0, e = 0.0;
      for (int w = 0; w < kSampWarps; ++w) {
        s = __dadd_rn(s, sm.wp[threadIdx.x][w]);
        e += sm.we[threadIdx.x][w];
      }
      sm.seg[g0 + threadIdx.x] = s;
      sm.segerr[g0 + threadIdx.x] = e;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double S = 0.0, Et = 0.0;
    for (int s = 0; s < nl; ++s) {
      S = __dadd_rn(S, sm.seg[s]);
      Et += sm.segerr[s];
    }
    const double r = __dmul_rn(u, S);
    int ss = -1;
    double base = 0.0, run = 0.0, eb = 0.0;
    for (int s = 0; s < nl; ++s) {
      const double nxt = __dadd_rn(run, sm.seg[s]);
      if (nxt >= r) {
        ss = s;
        base = run;
        break;
      }
      run = nxt;
      eb += sm.segerr[s];
    }
    sm.S = S;
    sm.r = r;
    sm.err_tot = Et;
    sm.err_base = eb;
    sm.seg_star = ss;
    sm.seg_base = base;
    sm.cand = INT_MAX;
    sm.certified = 0;
  }
  __syncthreads();
  const double S = sm.S, r = sm.r;
  const int ss = sm.seg_star;
  if (!(isfinite(S) && isfinite(r) && ss >= 0 && u >= 0.0 && u <= 1.0)) return -1;

  // ---- running sums inside the crossing segment ----
  const int v0 = (threadIdx.x + kSampThreads * ss) * 4;
  const float4 t = tv(ss);
  double p[4] = {0.0, 0.0, 0.0, 0.0}, pe[4] = {0.0, 0.0, 0.0, 0.0};
  double c = 0.0, ce = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (v0 + j < V) {
      p[j] = prob<EXACT>(f4_at(t, j), maxv, pe[j]);
      c = __dadd_rn(c, p[j]);
      ce += pe[j];
    }
  double tot, etot;
  const double ex = block_excl_scan(c, sm.wsum, tot);
  const double eex = block_excl_scan(ce, sm.wsum, etot);
  double prev = __dadd_rn(sm.seg_base, ex);
  int mine = -1;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (mine < 0 && v0 + j < V) {
      const double cur = __dadd_rn(prev, p[j]);
      if (cur >= r) mine = j;
      prev = cur;
    }
  }
  if (mine >= 0) atomicMin(&sm.cand, v0 + mine);
  __syncthreads();
  const int cand = sm.cand;
  if (cand >= v0 && cand < v0 + 4 && v0 < V) {
    double pre = __dadd_rn(sm.seg_base, ex);
    double ep = sm.err_base + eex;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < cand - v0) {
        pre = __dadd_rn(pre, p[j]);
        ep += pe[j];
      }
    double phi = pre, ehi = ep;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j == cand - v0) {
        phi = __dadd_rn(pre, p[j]);
        ehi = ep + pe[j];
      }
    sm.cand_lo = pre;
    sm.cand_hi = phi;
    sm.ecand_lo = ep;
    sm.ecand_hi = ehi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 0;
    if (cand != INT_MAX) {
      // A summation tree of depth h over non-negative terms is within
      // h 2^-53 (1+o(1)) of the exact sum.  The sequential running sum at v has
      // depth v; ours at most nl + 50 (4 per chunk, 5 + 16 per reduction or
      // scan, nl segments).  The rounding bounds below use 2^-52 (twice the
      // first-order constant); the exp-error sums get a (1 + 1e-6) margin for
      // their own rounding.
      const double slack = (double)(nl + 64);
      const double Er = u * (sm.err_tot * (1.0 + 1e-6) + ((double)V + slack) * 0x1p-52 * S) + 0x1p-52 * r;
      const double hi = sm.cand_hi, lo = sm.cand_lo;
      const double Ehi = sm.ecand_hi * (1.0 + 1e-6) + ((double)cand + slack) * 0x1p-52 * hi;
      const double Elo = sm.ecand_lo * (1.0 + 1e-6) + ((double)cand + slack) * 0x1p-52 * lo;
      const bool up = hi - Ehi >= r + Er;
      const bool dn = cand == 0 || lo + Elo < r - Er;
      ok = up && dn;
    }
    sm.certified = ok;
  }
  __syncthreads();
  return sm.certified ? cand : -1;
}

// The sequential algorithm of src/snai_inference.php:178-194, by warp 0.
__device__ int sequential_a(const SampArgs &a, const uint32_t *bits, const float *L, double maxv, double u) {
  const int lane = threadIdx.x & 31;
  double sum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    double e;
    const double p = v < a.V ? prob<true>(tempered(a, bits, L[v], v), maxv, e) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) sum = __dadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
  }
  const double r = __dmul_rn(u, sum);
  double cum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    double e;
    const double p = v < a.V ? prob<true>(tempered(a, bits, L[v], v), maxv, e) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) {
      cum = __dadd_rn(cum, __shfl_sync(0xffffffffu, p, j));
      if (cum >= r) return b + j;
    }
  }
  return 0;  // `$best_token = 0` when nothing qualifies (NaN sums)
}

template <int NV4>
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
  Row<NV4> row;
  row.L = L;
  row.V = V;
  row.vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  row.load();
  build_bitmap(a, mrow, bits);
  const int nl = row.layers();

  // ---- pass 1: tempered values (kept in registers), maximum, first argmax ----
  auto temper = [&](int i) {
    float4 x = row.fetch(i);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) f4_set(x, j, v0 + j < V ? tempered(a, bits, f4_at(x, j), v0 + j) : -INFINITY);
    return x;
  };
  if constexpr (NV4 > 0) {
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        f4_set(row.r[i], j, v0 + j < V ? tempered(a, bits, f4_at(row.r[i], j), v0 + j) : -INFINITY);
    }
  }
  auto tv = [&](int i) {
    if constexpr (NV4 > 0)
      return row.get(i);
    else
      return temper(i);
  };
  float best = -INFINITY;
  int bi = INT_MAX;
#pragma unroll
  for (int i = 0; i < nl; ++i) {
    const float4 t = tv(i);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float tj = f4_at(t, j);
      if (tj > best) {  // ids ascend along a thread's chunks: ties keep the first
        best = tj;
        bi = v0 + j;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if (lane == 0) {
    sm.bmax[warp] = best;
    sm.bidx[warp] = bi;
  }
  __syncthreads();
  best = sm.bmax[0];
  bi = sm.bidx[0];
  for (int w = 1; w < kSampWarps; ++w)
    if (sm.bmax[w] > best || (sm.bmax[w] == best && sm.bidx[w] < bi)) {
      best = sm.bmax[w];
      bi = sm.bidx[w];
    }
  // PHP: max starts at -INF and only a strictly larger value moves it.
  const bool any = best > -INFINITY;
  const double maxv = any ? (double)best : -INFINITY;
  if (a.T <= 0.01) {
    if (threadIdx.x == 0) a.out[b] = any ? bi : 0;
    return;
  }
  const double u = (double)a.uniforms[b];
  if (any) {
    int id = certified_draw<false>(sm, V, nl, maxv, u, tv);
    if (id < 0) id = certified_draw<true>(sm, V, nl, maxv, u, tv);
    if (id >= 0) {
      if (threadIdx.x == 0) a.out[b] = id;
      return;
    }
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
  int overflow;
  float fmax[kSampWarps];
  float fsum[kSampWarps], fsq[kSampWarps];
  int fcnt[kSampWarps];
  float R;
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

// val_v and the fp32 values bracketing it (lo <= val <= hi; equal unless the
// entry is penalised).
struct ValB {
  double val;
  float lo, hi;
  bool pen;
};
__device__ __forceinline__ ValB val_b(const SampArgs &a, const uint32_t *bits, float x, int v) {
  ValB r;
  r.pen = in_set(bits, v);
  if (!r.pen) {
    r.val = (double)x;
    r.lo = r.hi = x;
  } else {
    r.val = __dsub_rn((double)x, a.rep);
    r.lo = __double2float_rd(r.val);
    r.hi = __double2float_ru(r.val);
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

// Warp-cooperative append (every lane calls it; `want` selects).
__device__ __forceinline__ void push_cand_warp(SmemB &sm, bool want, double val, int v, int cap) {
  const unsigned int m = __ballot_sync(0xffffffffu, want);
  if (!m) return;
  const int lane = threadIdx.x & 31;
  int base = 0;
  if (lane == 0) base = atomicAdd(&sm.ncand, __popc(m));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (want) {
    const int slot = base + __popc(m & ((1u << lane) - 1u));
    if (slot < cap) {
      sm.ckey[slot] = okey64(val);
      sm.cidx[slot] = v;
    }
  }
}

// candidate i precedes candidate j in PHP's arsort order
__device__ __forceinline__ bool precedes(unsigned long long ki, int vi, unsigned long long kj, int vj) {
  return ki > kj || (ki == kj && vi < vj);
}

// Sorts the nc gathered candidates and keeps the first k in sm.order / sm.val.
__device__ void rank_candidates(SmemB &sm, int nc, int k) {
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
}

// Fast selection (see the file comment).  Returns false when the row needs
// the general path.  All threads return the same value.
template <int NV4>
__device__ bool fast_select_b(const SampArgs &a, const uint32_t *bits, const Row<NV4> &row, SmemB &sm, int k) {
  const int V = a.V, nl = row.layers();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // pass 1: maximum of the lower bounds, and their spread
  float mx = -INFINITY, s1 = 0.f, s2 = 0.f;
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < nl; ++i) {
    const float4 x = row.get(i);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (v0 + j < V) {
        const ValB e = val_b(a, bits, f4_at(x, j), v0 + j);
        if (isfinite(e.lo)) {
          mx = fmaxf(mx, e.lo);
          s1 += e.lo;
          s2 = fmaf(e.lo, e.lo, s2);
          ++cnt;
        } else if (e.lo > 0.f) {
          cnt = -(1 << 24);  // +inf: leave the row to the general path
        }
      }
    }
  }
  mx = warp_max(mx);
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) {
    sm.fmax[warp] = mx;
    sm.fsum[warp] = s1;
    sm.fsq[warp] = s2;
    sm.fcnt[warp] = cnt;
  }
  __syncthreads();
  mx = -INFINITY;
  s1 = s2 = 0.f;
  cnt = 0;
  for (int w = 0; w < kSampWarps; ++w) {
    mx = fmaxf(mx, sm.fmax[w]);
    s1 += sm.fsum[w];
    s2 += sm.fsq[w];
    cnt += sm.fcnt[w];
  }
  __syncthreads();
  if (!isfinite(mx) || cnt < k) return false;
  const float mean = s1 / cnt;
  const float sd = sqrtf(fmaxf(s2 / cnt - mean * mean, 0.f));
  float R = 2.5f * sd;
  if (!(R > 0.f) || !isfinite(R)) return false;  // all equal: ties, general path

  // pass 2: histogram of the distance below the maximum, 255 bins over [0, R)
  int bstar = 255;
  for (int attempt = 0; attempt < 3 && bstar >= 255; ++attempt, R *= 8.f) {
    const float inv_w = 255.f / R;
    for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < nl; ++i) {
      const float4 x = row.get(i);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (v0 + j < V) {
          const float d = mx - val_b(a, bits, f4_at(x, j), v0 + j).lo;
          if (d >= 0.f && d < R) atomicAdd(&sm.hist[min((int)(d * inv_w), 254)], 1u);
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
      // inclusive prefix over bins 0..255, 8 per lane
      unsigned int c[8], run = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        run += sm.hist[lane * 8 + q];
        c[q] = run;
      }
      unsigned int incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const unsigned int before = incl - run;
      int bs = 255;
#pragma unroll
      for (int q = 7; q >= 0; --q)
        if (before + c[q] >= (unsigned)k) bs = lane * 8 + q;
      // smallest bin reaching k
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bs = min(bs, __shfl_xor_sync(0xffffffffu, bs, o));
      if (lane == 0) {
        sm.bstar = bs;
        sm.R = R;
      }
    }
    __syncthreads();
    bstar = sm.bstar;
    __syncthreads();
  }
  if (bstar >= 255) return false;
  R = sm.R;
  const float inv_w = 255.f / R;

  // pass 3: gather every entry whose upper bound falls in a bin <= bstar
  if (threadIdx.x == 0) sm.ncand = 0;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < nl; ++i) {
    const float4 x = row.get(i);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      bool want = false;
      double val = 0.0;
      if (v0 + j < V) {
        const ValB e = val_b(a, bits, f4_at(x, j), v0 + j);
        const float d = mx - e.hi;
        want = d < R && min((int)(d * inv_w), 254) <= bstar;
        val = e.val;
      }
      push_cand_warp(sm, want, val, v0 + j, kFastCand);
    }
  }
  __syncthreads();
  const int nc = sm.ncand;
  __syncthreads();
  if (nc > kFastCand || nc < k) return false;
  rank_candidates(sm, nc, k);
  return true;
}

// General selection: radix select on the 32-bit keys of the lower bounds
// (12 + 12 + 8 bits), superset gather by the upper bounds, exact sort.
// Handles ties of any size: when more than 1024 entries share the exact
// threshold value, only the first `need` of them in vocab order are kept
// (the later ones tie in value and lose on index).
__device__ bool general_select_b(const SampArgs &a, const uint32_t *bits, const float *L, SmemB &sm, int k) {
  const int V = a.V;
  const int iters = (V + kSampThreads - 1) / kSampThreads;  // warp-uniform trip count
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
        const unsigned int klo = okey32(val_b(a, bits, L[v], v).lo);
        act = (klo & pmask) == prefix;
        bin = (klo >> sh) & bmask;
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
          if (acc + c >= (unsigned)need) {
            bs = lo + i;
            break;
          }
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
  const unsigned int tau = sm.prefix;  // lower-bound key threshold (low unresolved bits 0)
  const bool tie_path = exact && sm.bcount > 1024u;
  __syncthreads();

  // gather the superset {key(hi) >= tau}
  for (int it = 0; it < iters; ++it) {
    const int v = it * kSampThreads + threadIdx.x;
    if (v < V) {
      const ValB x = val_b(a, bits, L[v], v);
      if (okey32(x.hi) >= tau) {
        if (!(tie_path && !x.pen && okey32(x.lo) == tau)) push_cand(sm, x.val, v);
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
        f = !x.pen && okey32(x.lo) == tau;
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
  if (sm.overflow) return false;
  rank_candidates(sm, sm.ncand, k);
  return true;
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads) sample_b_kernel(SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB));
  const int b = blockIdx.x;
  const int mrow = a.row_map ? a.row_map[b] : b;
  const float *L = a.logits + (size_t)mrow * a.ld;
  const int V = a.V;
  const int k = min(a.top_k, V);
  Row<NV4> row;
  row.L = L;
  row.V = V;
  row.vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  row.load();
  build_bitmap(a, mrow, bits);

  if (!fast_select_b<NV4>(a, bits, row, sm, k)) {
    if (!general_select_b(a, bits, L, sm, k)) {
      if (threadIdx.x == 0) {
        a.out[b] = -2;
        record_error(a.err, kErrSamplerArgs);
      }
      return;
    }
  }

  // ---- src/tensor_ffi_adapter.php:180-204 over the k survivors ----
  if (a.T < 0.01) {
    if (threadIdx.x == 0) a.out[b] = sm.order[0];
    return;
  }
  for (int i = threadIdx.x; i < k; i += kSampThreads) sm.p[i] = snai_exp(__ddiv_rn(sm.val[i], a.T));
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < k; ++i) s = __dadd_rn(s, sm.p[i]);
    sm.cum[0] = s;  // the sum, handed to all threads
  }
  __syncthreads();
  const double sum = sm.cum[0];
  __syncthreads();
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
      if (r <= sm.cum[i]) {
        id = sm.order[i];
        break;
      }
    a.out[b] = id;
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

int check_sample_args(const SampleLaunch &s) {
  if (s.rows < 0) {
    set_error("sampler: rows < 0");
    return -2;
  }
  if (s.V < 1 || s.V > kMaxVocab) {
    set_error("sampler: vocab %d outside [1, %d]", s.V, kMaxVocab);
    return -2;
  }
  if (s.ld < s.V) {
    set_error("sampler: row stride %lld < vocab %d", s.ld, s.V);
    return -2;
  }
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
    if (s.top_k < 1 || s.top_k > kMaxTopK) {
      set_error("sampler variant 1: top_k %d outside [1, %d]", s.top_k, kMaxTopK);
      return -2;
    }
  } else {
    set_error("sampler: unknown variant %d", s.variant);
    return -2;
  }
  return 0;
}

template <int NV4>
static void launch_a(const SampArgs &a, int rows, size_t sm, cudaStream_t st) {
  static unsigned long long done = 0;  // attribute set, one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(done & (1ull << dev))) {
    cudaFuncSetAttribute(sample_a_kernel<NV4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    done |= 1ull << dev;
  }
  sample_a_kernel<NV4><<<rows, kSampThreads, sm, st>>>(a);
}

template <int NV4>
static void launch_b(const SampArgs &a, int rows, size_t sm, cudaStream_t st) {
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(done & (1ull << dev))) {
    cudaFuncSetAttribute(sample_b_kernel<NV4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    done |= 1ull << dev;
  }
  sample_b_kernel<NV4><<<rows, kSampThreads, sm, st>>>(a);
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
  const int layers = (s.V + 2047) / 2048;
  if (s.variant == 0) {
    const size_t sm = sizeof(SmemA) + bitmap;
    if (layers <= 4)
      launch_a<4>(a, s.rows, sm, stream);
    else if (layers <= 8)
      launch_a<8>(a, s.rows, sm, stream);
    else
      launch_a<0>(a, s.rows, sm, stream);
  } else {
    const size_t sm = sizeof(SmemB) + bitmap;
    if (layers <= 4)
      launch_b<4>(a, s.rows, sm, stream);
    else if (layers <= 8)
      launch_b<8>(a, s.rows, sm, stream);
    else if (layers <= 16)
      launch_b<16>(a, s.rows, sm, stream);
    else
      launch_b<0>(a, s.rows, sm, stream);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("sampler launch failed: %s", cudaGetErrorString(e));
    return -4;
  }
  return 0;
}

}  // namespace snai
