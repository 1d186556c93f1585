// sampler.cu - the reference's two logits -> token samplers on sm_100a.
//
// Persistent CTAs of 512 threads, each taking rows b, b+grid, ...; while a row
// is processed the next one is prefetched into L2 (cp.async.bulk.prefetch).
// A row of up to 32768 logits is held in registers (thread t owns the 16-byte
// chunks t, t+512, ...); larger rows are re-read from L2 on every pass.
// Both kernels reproduce the PHP code's double-precision decisions bit for
// bit for given logits and uniform u.  Bulk passes work on the raw fp32
// logits with a few instructions per entry; exact double arithmetic is spent
// only on penalised entries (the history, usually a few hundred) and on the
// handful of entries near a decision.
//
// Variant A (src/snai_inference.php:151-195).
//   t_v = fp32(L_v / T); penalised ids (the unique history, a bitmap in shared
//   memory): t = fp32(t / rep) if t > 0 else fp32(t * rep).  Greedy
//   (T <= 0.01): first index of the maximum.  Otherwise p_v = exp(t_v - max)
//   in double (snai_exp.h), S = sequential sum in vocab order, r = u*S, and
//   the id is the first v whose running sum reaches r.
//   For T > 0, t is monotone in L, so the maximum over unpenalised entries is
//   fp32(max L / T) and only entries within a few ulps of max L can attain it.
//   The sequential running sums are replaced by parallel ones with a proven
//   error bound, and an id is accepted only when r is farther from the running
//   sums around it than the bound ("certified"):
//     tier 1: p_v = 2^(L_v*(log2e/T) - max*log2e) from ex2.approx, one
//             relative bound for the whole row;
//     tier 2: p_v from the contract exponential itself (no exp error);
//     tier 3: warp 0 runs the sequential loop.
//   Each tier is exact whenever it answers, so the id is always the
//   sequential algorithm's id.
//
// Variant B (src/tensor_ffi_adapter.php:168-204).
//   val_v = L_v - rep for ids in the input set, else L_v (double).  The
//   stable descending sort + top_k keeps the k smallest (-val, v).  Fast
//   path: a histogram of fp32 lower bounds of val over distance bins below
//   the row maximum finds the bin of the k-th largest; every entry whose next
//   float above its lower bound reaches that bin is gathered (a superset of
//   the top k), sorted exactly by (val desc, v asc), and the PHP softmax /
//   top-p / draw runs sequentially over the k survivors.  Rows the fast path
//   cannot settle (non-finite values, huge exact ties) take a general radix
//   select.
#include <cfloat>
#include <climits>
#include <cmath>
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "engine.h"
#include "snai_exp.h"

namespace snai {

constexpr int kSampThreads = 512;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kMaxTopK = 1024;
constexpr int kCandCap = 4096;   // exact-sort capacity
constexpr int kFastCand = 2048;  // candidates the fast path accepts
constexpr int kMaxVocab = 1 << 19;
constexpr int kMaxSeg = kMaxVocab / 2048;

struct SampArgs {
  const float *logits;
  long long ld;
  const int *row_map;
  int rows;
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

constexpr int kPenCap = 2048;  // unique history ids listed per row

// Marks the row's history ids (each once, ids outside [0,V) ignored) in a
// shared bitmap of V bits and lists each distinct id once in plist (the
// thread whose atomicOr set the bit lists it).  *npen receives the count
// (possibly above kPenCap: then the list is incomplete).  Starts and ends with
// a barrier.
__device__ void build_bitmap(const SampArgs &a, int mrow, uint32_t *bits, int *plist, int *npen) {
  const int words = (a.V + 31) >> 5;
  __syncthreads();
  for (int i = threadIdx.x; i < words; i += blockDim.x) bits[i] = 0u;
  if (threadIdx.x == 0) *npen = 0;
  __syncthreads();
  int n = a.hist_len ? a.hist_len[mrow] : a.hist_cols;
  n = min(max(n, 0), a.hist_cols);
  const int *hr = a.hist + (size_t)mrow * a.hist_ld;
  const int lane = threadIdx.x & 31;
  for (int i0 = 0; i0 < n; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    const int t = i < n ? hr[i] : -1;
    bool first = false;
    if (t >= 0 && t < a.V) {
      const uint32_t bit = 1u << (t & 31);
      first = !(atomicOr(&bits[t >> 5], bit) & bit);
    }
    const unsigned m = __ballot_sync(0xffffffffu, first);
    int base = 0;
    if (lane == 0 && m) base = atomicAdd(npen, __popc(m));
    base = __shfl_sync(0xffffffffu, base, 0) + __popc(m & ((1u << lane) - 1u));
    if (first && base < kPenCap) plist[base] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ bool in_set(const uint32_t *bits, int v) { return (bits[v >> 5] >> (v & 31)) & 1u; }

// Prefetches a row into L2 (16-byte aligned rows whose size is a multiple of 16).
__device__ __forceinline__ void prefetch_row_l2(const float *p, int V) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) || (V & 3)) return;
  const unsigned bytes = (unsigned)V * 4u;
  for (unsigned off = 0; off < bytes; off += 65536u) {
    const unsigned n = min(65536u, bytes - off);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const char *>(p) + off), "r"(n)
                 : "memory");
  }
}

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

// The penalty of src/snai_inference.php:160-164 applied to a stored value.
__device__ __forceinline__ float penalise_a(float t, double rep) {
  const double d = (double)t;
  return d > 0.0 ? __double2float_rn(__ddiv_rn(d, rep)) : __double2float_rn(__dmul_rn(d, rep));
}

// Variant A's stored value for vocab entry v (src/snai_inference.php:153, 160-164).
__device__ __forceinline__ float tempered(const SampArgs &a, const uint32_t *bits, float x, int v) {
  const float t = div_to_f32(x, a.T, a.Tinv);
  return in_set(bits, v) ? penalise_a(t, a.rep) : t;
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

__device__ __forceinline__ float f4_at(const float4 &f, int j) { return j == 0 ? f.x : j == 1 ? f.y : j == 2 ? f.z : f.w; }
__device__ __forceinline__ void f4_set(float4 &f, int j, float v) {
  if (j == 0) f.x = v;
  else if (j == 1) f.y = v;
  else if (j == 2) f.z = v;
  else f.w = v;
}

// The next float above f (for finite f; +-0 -> the smallest subnormal).
__device__ __forceinline__ float next_up(float f) {
  if (f == 0.f) return 1.401298464e-45f;
  const unsigned u = __float_as_uint(f);
  return __uint_as_float(f > 0.f ? u + 1u : u - 1u);
}

__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// A row of logits, 16-byte chunk i of thread t = entries 4*(t + 512*i) .. +3.
// Entries of the history set are replaced by their exact penalised value
// (variant-specific `pen_value`) and flagged in `pen`.  NV4 > 0: the row
// (V <= 2048*NV4) sits in registers; NV4 == 0: every access re-reads global
// memory and recomputes the penalised values.
template <int NV4>
struct Row {
  const float *L;
  int V;
  bool vec;
  float4 r[NV4 > 0 ? NV4 : 1];
  unsigned long long pen = 0ull;

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
  // Loads (registers) and replaces flagged entries by their penalised value:
  // from the side table penv (indexed by vocab id) when it is given, else
  // computed here by pf.
  template <class PenFn>
  __device__ __forceinline__ void load(const uint32_t *bits, const PenFn &pf, const float *penv) {
    if constexpr (NV4 > 0) {
#pragma unroll
      for (int i = 0; i < NV4; ++i) r[i] = fetch(i);
#pragma unroll
      for (int i = 0; i < NV4; ++i) {
        const int v0 = (threadIdx.x + kSampThreads * i) * 4;
        if (v0 < V) {
          const uint32_t w = (bits[v0 >> 5] >> (v0 & 31)) & 0xFu;
          pen |= (unsigned long long)w << (4 * i);
          if (w) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if ((w >> j) & 1u) f4_set(r[i], j, penv ? penv[v0 + j] : pf(f4_at(r[i], j)));
          }
        }
      }
    }
  }
  // Values and penalty flags of chunk layer i (a run-time i selects among
  // registers with predicated moves, never through local memory).
  template <class PenFn>
  __device__ __forceinline__ float4 get(int i, const uint32_t *bits, const PenFn &pf, uint32_t &pbits) const {
    if constexpr (NV4 > 0) {
      float4 o = r[0];
#pragma unroll
      for (int q = 1; q < NV4; ++q)
        if (q == i) o = r[q];
      pbits = (uint32_t)(pen >> (4 * i)) & 0xFu;
      return o;
    } else {
      float4 o = fetch(i);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      pbits = v0 < V ? (bits[v0 >> 5] >> (v0 & 31)) & 0xFu : 0u;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if ((pbits >> j) & 1u) f4_set(o, j, pf(f4_at(o, j)));
      return o;
    }
  }
};

// ---------------------------------------------------------------------------
// Variant A
// ---------------------------------------------------------------------------

struct SmemA {
  double seg[kMaxSeg];
  double wp[32][kSampWarps];  // per-warp partial sums of 32 segments
  double wsum[kSampWarps];
  float wf[3][kSampWarps];
  int wi[kSampWarps];
  double S, r, seg_base;
  int seg_star;
  int cand;
  double cand_hi, cand_lo;
  int certified;
  float M;
  int flag;
  int npen;
  int plist[kPenCap];
};

// Tier 1 / tier 2 of variant A: returns the id, or -1 if not certified.
// P(i, j) gives p of entry j of this thread's chunk layer i (as a double);
// `eps` bounds |p~ - p| / p for every entry (0 for the contract exp) and
// `eabs` the absolute error of an entry whose p~ underflowed.
template <class PF>
__device__ int certified_draw(SmemA &sm, int V, int nl, double u, double eps, double eabs, const PF &P) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // ---- segment sums (segment i = chunk layer i = 2048 consecutive ids) ----
  for (int g0 = 0; g0 < nl; g0 += 32) {
    const int g1 = min(nl, g0 + 32);
    for (int i = g0; i < g1; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      double c = 0.0;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v0 + j < V) c = __dadd_rn(c, P(i, j));
      c = warp_sum_d(c);
      if (lane == 0) sm.wp[i - g0][warp] = c;
    }
    __syncthreads();
    if (threadIdx.x < g1 - g0) {
      double s = 0.0;
      for (int w = 0; w < kSampWarps; ++w) s = __dadd_rn(s, sm.wp[threadIdx.x][w]);
      sm.seg[g0 + threadIdx.x] = s;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double S = 0.0;
    for (int s = 0; s < nl; ++s) S = __dadd_rn(S, sm.seg[s]);
    const double r = __dmul_rn(u, S);
    int ss = -1;
    double base = 0.0, run = 0.0;
    for (int s = 0; s < nl; ++s) {
      const double nxt = __dadd_rn(run, sm.seg[s]);
      if (nxt >= r) {
        ss = s;
        base = run;
        break;
      }
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
  if (!(isfinite(S) && isfinite(r) && ss >= 0 && u >= 0.0 && u <= 1.0)) return -1;

  // ---- running sums inside the crossing segment ----
  const int v0 = (threadIdx.x + kSampThreads * ss) * 4;
  double p[4] = {0.0, 0.0, 0.0, 0.0};
  double c = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (v0 + j < V) {
      p[j] = P(ss, j);
      c = __dadd_rn(c, p[j]);
    }
  double tot;
  const double ex = block_excl_scan(c, sm.wsum, tot);
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
    double pre = __dadd_rn(sm.seg_base, ex), hi = pre;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < cand - v0) pre = __dadd_rn(pre, p[j]);
      if (j == cand - v0) hi = __dadd_rn(pre, p[j]);
    }
    sm.cand_lo = pre;
    sm.cand_hi = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 0;
    if (cand != INT_MAX) {
      // A summation tree of depth h over non-negative terms is within
      // h 2^-53 (1+o(1)) of the exact sum.  The sequential running sum at v has
      // depth v; ours at most nl + 50 (4 per chunk, 5 + 16 per reduction or
      // scan, nl segments).  Rounding bounds below use 2^-52 (twice the
      // first-order constant).  The p~ of tier 1 are within eps*p of the
      // contract values (eabs for an entry that underflowed), so their running
      // sums are within eps*P(1+2eps) + (v+1)*eabs of the contract's.
      const double slack = (double)(nl + 64);
      const double er = eps * (1.0 + 2.0 * eps) + 1e-12 * (eps > 0.0);
      const double Er = u * (er * S + (double)V * eabs + ((double)V + slack) * 0x1p-52 * S) + 0x1p-52 * r;
      const double hi = sm.cand_hi, lo = sm.cand_lo;
      const double Ehi = er * hi + ((double)cand + 1.0) * eabs + ((double)cand + slack) * 0x1p-52 * hi;
      const double Elo = er * lo + (double)cand * eabs + ((double)cand + slack) * 0x1p-52 * lo;
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
__device__ __noinline__ int sequential_a(const SampArgs &a, const uint32_t *bits, const float *L, double maxv, double u) {
  const int lane = threadIdx.x & 31;
  double sum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const double p = v < a.V ? snai_exp(__dsub_rn((double)tempered(a, bits, L[v], v), maxv)) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) sum = __dadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
  }
  const double r = __dmul_rn(u, sum);
  double cum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const double p = v < a.V ? snai_exp(__dsub_rn((double)tempered(a, bits, L[v], v), maxv)) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) {
      cum = __dadd_rn(cum, __shfl_sync(0xffffffffu, p, j));
      if (cum >= r) return b + j;
    }
  }
  return 0;  // `$best_token = 0` when nothing qualifies (NaN sums)
}

// Exact maximum and first argmax of the stored values, computed entry by
// entry (any T); the rare-case path.
__device__ __noinline__ void exact_max_a(const SampArgs &a, const uint32_t *bits, const float *L, SmemA &sm, float &best, int &bi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  best = -INFINITY;
  bi = INT_MAX;
  for (int v = threadIdx.x; v < a.V; v += kSampThreads) {
    const float t = tempered(a, bits, L[v], v);
    if (t > best) {  // ids ascend per thread: ties keep the first
      best = t;
      bi = v;
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
  __syncthreads();
  if (lane == 0) {
    sm.wf[0][warp] = best;
    sm.wi[warp] = bi;
  }
  __syncthreads();
  best = sm.wf[0][0];
  bi = sm.wi[0];
  for (int w = 1; w < kSampWarps; ++w)
    if (sm.wf[0][w] > best || (sm.wf[0][w] == best && sm.wi[w] < bi)) {
      best = sm.wf[0][w];
      bi = sm.wi[w];
    }
  __syncthreads();
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads, NV4 > 0 && NV4 <= 8 ? 2 : 1) sample_a_kernel(SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemA &sm = *reinterpret_cast<SmemA *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemA));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int V = a.V;
  // side table of exact penalised values, indexed by vocab id (register rows only)
  float *penv = reinterpret_cast<float *>(smem_dyn + sizeof(SmemA) + (((size_t)(V + 31) / 32 * 4 + 15) & ~(size_t)15));
  const bool vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  const double rep = a.rep;
  auto pen_fn = [&](float x) { return penalise_a(div_to_f32(x, a.T, a.Tinv), rep); };

  for (int b = blockIdx.x; b < a.rows; b += gridDim.x) {
    const int mrow = a.row_map ? a.row_map[b] : b;
    const float *L = a.logits + (size_t)mrow * a.ld;
    if (threadIdx.x == 0 && b + (int)gridDim.x < a.rows) {
      const int nrow = a.row_map ? a.row_map[b + gridDim.x] : b + gridDim.x;
      prefetch_row_l2(a.logits + (size_t)nrow * a.ld, V);
    }
    if (a.nan_guard) {
      const float l0 = L[0];
      if (l0 != l0) {  // src/snai_inference.php:146
        if (threadIdx.x == 0) a.out[b] = -1;
        continue;
      }
    }
    build_bitmap(a, mrow, bits, sm.plist, &sm.npen);
    const int np = sm.npen;
    const bool listed = NV4 > 0 && np <= kPenCap;
    if (listed) {
      for (int i = threadIdx.x; i < np; i += kSampThreads) {
        const int h = sm.plist[i];
        penv[h] = pen_fn(L[h]);
      }
      __syncthreads();
    }
    Row<NV4> row;
    row.L = L;
    row.V = V;
    row.vec = vec;
    row.load(bits, pen_fn, listed ? penv : nullptr);
    const int nl = row.layers();

    // ---- maximum: raw logits of unpenalised entries (t is monotone in L for
    // T > 0), exact values of penalised ones ----
    float xmax = -INFINITY, xabs = 0.f, pmax = -INFINITY, pabs = 0.f;
    int pidx = INT_MAX;
#pragma unroll
    for (int i = 0; i < nl; ++i) {
      uint32_t pb;
      const float4 x = row.get(i, bits, pen_fn, pb);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (v0 + j < V) {
          const float f = f4_at(x, j);
          if ((pb >> j) & 1u) {
            if (f > pmax) {
              pmax = f;
              pidx = v0 + j;
            }
            pabs = fmaxf(pabs, fabsf(f));
          } else {
            xmax = fmaxf(xmax, f);
            xabs = fmaxf(xabs, fabsf(f));
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
      xabs = fmaxf(xabs, __shfl_xor_sync(0xffffffffu, xabs, o));
      pabs = fmaxf(pabs, __shfl_xor_sync(0xffffffffu, pabs, o));
      const float ob = __shfl_xor_sync(0xffffffffu, pmax, o);
      const int oi = __shfl_xor_sync(0xffffffffu, pidx, o);
      if (ob > pmax || (ob == pmax && oi < pidx)) {
        pmax = ob;
        pidx = oi;
      }
    }
    if (lane == 0) {
      sm.wf[0][warp] = xmax;
      sm.wf[1][warp] = fmaxf(xabs, pabs);
      sm.wf[2][warp] = pmax;
      sm.wi[warp] = pidx;
    }
    __syncthreads();
    xmax = sm.wf[0][0];
    float tabs_in = sm.wf[1][0];
    pmax = sm.wf[2][0];
    pidx = sm.wi[0];
    for (int w = 1; w < kSampWarps; ++w) {
      xmax = fmaxf(xmax, sm.wf[0][w]);
      tabs_in = fmaxf(tabs_in, sm.wf[1][w]);
      if (sm.wf[2][w] > pmax || (sm.wf[2][w] == pmax && sm.wi[w] < pidx)) {
        pmax = sm.wf[2][w];
        pidx = sm.wi[w];
      }
    }
    __syncthreads();
    const float tmax = (xmax > -INFINITY) ? div_to_f32(xmax, a.T, a.Tinv) : -INFINITY;
    const float M = fmaxf(tmax, pmax);
    const bool simple = a.T > 0.0 && isfinite(M) && isfinite(xmax) && isfinite(tabs_in);

    float best;
    int bi;
    if (simple) {
      // first index attaining M: entries with fp32(x/T) == M have
      // x >= (M - |M| 2^-23) T; check those exactly
      const double lowt = (double)M - fabs((double)M) * 0x1p-22 - 1e-44;
      const float xthr = __double2float_rd(lowt * a.T);
      if (threadIdx.x == 0) sm.cand = (pmax == M) ? pidx : INT_MAX;
      __syncthreads();
#pragma unroll
      for (int i = 0; i < nl; ++i) {
        uint32_t pb;
        const float4 x = row.get(i, bits, pen_fn, pb);
        const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float f = f4_at(x, j);
          if (v0 + j < V && !((pb >> j) & 1u) && f >= xthr && div_to_f32(f, a.T, a.Tinv) == M)
            atomicMin(&sm.cand, v0 + j);
        }
      }
      __syncthreads();
      best = M;
      bi = sm.cand;
      __syncthreads();
    } else {
      exact_max_a(a, bits, L, sm, best, bi);
    }
    // PHP: max starts at -INF and only a strictly larger value moves it.
    const bool any = best > -INFINITY;
    const double maxv = any ? (double)best : -INFINITY;
    if (a.T <= 0.01) {
      if (threadIdx.x == 0) a.out[b] = any ? bi : 0;
      continue;
    }
    const double u = (double)a.uniforms[b];
    int id = -1;
    if (any && simple) {
      // tier 1: p~ = 2^(x c - M log2e), c = fp32(log2e / T); penalised entries
      // use their exact value t: 2^(t log2e - M log2e).
      const float c = (float)(1.4426950408889634 * a.Tinv);
      const float l2e = 1.44269504f;
      const float m2 = M * l2e;
      // |t| <= tabs for every entry (|x/T| rounded up a little)
      const double tabs = (double)tabs_in * fmax(1.0, fabs(a.Tinv)) * (1.0 + 0x1p-20);
      const double eps = (tabs + fabs((double)M) + 1.0) * 0x1p-21 + 0x1p-19;
      auto P1 = [&](int i, int j) {
        uint32_t pb;
        const float4 x = row.get(i, bits, pen_fn, pb);
        const float f = f4_at(x, j);
        const float arg = ((pb >> j) & 1u) ? fmaf(f, l2e, -m2) : fmaf(f, c, -m2);
        return (double)ex2_approx(arg);
      };
      id = certified_draw(sm, V, nl, u, eps, 0x1p-125, P1);
    }
    if (id < 0 && any) {
      // tier 2: the contract exponential of the exact stored values
      auto P2 = [&](int i, int j) {
        uint32_t pb;
        const float4 x = row.get(i, bits, pen_fn, pb);
        const float f = f4_at(x, j);
        const float t = ((pb >> j) & 1u) ? f : div_to_f32(f, a.T, a.Tinv);
        return snai_exp(__dsub_rn((double)t, maxv));
      };
      id = certified_draw(sm, V, nl, u, 0.0, 0.0, P2);
    }
    if (id < 0) {
      // tier 3
      if (warp == 0) {
        const int s = sequential_a(a, bits, L, maxv, u);
        if (lane == 0) a.out[b] = s;
      }
    } else if (threadIdx.x == 0) {
      a.out[b] = id;
    }
  }
}

// ---------------------------------------------------------------------------
// Variant B
// ---------------------------------------------------------------------------

// The histogram and candidate arrays live in the dynamic region after the
// bitmap, where the penalised-value side table lived before the row was
// loaded into registers.
constexpr size_t kBUnionBytes = (size_t)kCandCap * 8 + (size_t)kCandCap * 4 + 4096 * 4;

struct SmemB {
  unsigned int *hist;        // [4096]
  unsigned long long *ckey;  // [kCandCap] exact order key of a candidate
  int *cidx;                 // [kCandCap]
  unsigned int wtot[kSampWarps];
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
  float fw[3][kSampWarps];
  float R;
  int npen;
  int plist[kPenCap];
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

// Fast selection (see the file comment).  The row holds lower bounds (the
// raw logit, or fp32-round-down(L - rep) for penalised entries).  Returns
// false (the same on every thread) when the row needs the general path.
template <int NV4, class PenFn>
__device__ bool fast_select_b(const SampArgs &a, const uint32_t *bits, const Row<NV4> &row, const PenFn &pf,
                              SmemB &sm, int k) {
  const int V = a.V, nl = row.layers();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // pass 1: maximum and spread of the lower bounds
  float mx = -INFINITY, s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < nl; ++i) {
    uint32_t pb;
    const float4 x = row.get(i, bits, pf, pb);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (v0 + j < V) {
        const float f = f4_at(x, j);
        mx = fmaxf(mx, f);
        s1 += f;
        s2 = fmaf(f, f, s2);
      }
    }
  }
  mx = warp_max(mx);
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    sm.fw[0][warp] = mx;
    sm.fw[1][warp] = s1;
    sm.fw[2][warp] = s2;
  }
  __syncthreads();
  mx = -INFINITY;
  s1 = s2 = 0.f;
  for (int w = 0; w < kSampWarps; ++w) {
    mx = fmaxf(mx, sm.fw[0][w]);
    s1 += sm.fw[1][w];
    s2 += sm.fw[2][w];
  }
  __syncthreads();
  // any infinite or NaN entry makes s1 or s2 non-finite: general path
  if (!isfinite(mx) || !isfinite(s1) || !isfinite(s2) || V < k) return false;
  const float mean = s1 / V;
  const float sd = sqrtf(fmaxf(s2 / V - mean * mean, 0.f));
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
      uint32_t pb;
      const float4 x = row.get(i, bits, pf, pb);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d = mx - f4_at(x, j);
        if (v0 + j < V && d < R) atomicAdd(&sm.hist[min((int)(d * inv_w), 254)], 1u);
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

  // pass 3: gather every entry whose next float above its lower bound falls
  // in a bin <= bstar (a penalised entry's value lies below that float)
  if (threadIdx.x == 0) sm.ncand = 0;
  __syncthreads();
  int mine = 0;
#pragma unroll
  for (int i = 0; i < nl; ++i) {
    uint32_t pb;
    const float4 x = row.get(i, bits, pf, pb);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = mx - next_up(f4_at(x, j));
      if (v0 + j < V && d < R && (int)(d * inv_w) <= bstar) ++mine;
    }
  }
  // warp-aggregated slots
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  int base = 0;
  if (lane == 31 && incl) base = atomicAdd(&sm.ncand, incl);
  base = __shfl_sync(0xffffffffu, base, 31) + incl - mine;
  if (mine) {
#pragma unroll
    for (int i = 0; i < nl; ++i) {
      uint32_t pb;
      const float4 x = row.get(i, bits, pf, pb);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f = f4_at(x, j);
        const float d = mx - next_up(f);
        if (v0 + j < V && d < R && (int)(d * inv_w) <= bstar) {
          if (base < kFastCand) {
            // exact value: the logit, or logit - rep for a penalised entry
            const double val = ((pb >> j) & 1u) ? __dsub_rn((double)row.L[v0 + j], a.rep) : (double)f;
            sm.ckey[base] = okey64(val);
            sm.cidx[base] = v0 + j;
          }
          ++base;
        }
      }
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
__device__ __noinline__ bool general_select_b(const SampArgs &a, const uint32_t *bits, const float *L, SmemB &sm, int k) {
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
__global__ void __launch_bounds__(kSampThreads, NV4 > 0 && NV4 <= 8 ? 2 : 1) sample_b_kernel(SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB));
  const int V = a.V;
  const int k = min(a.top_k, V);
  // dynamic union region: the penalised-value side table while the row is
  // loaded, then the candidate keys / indices and the histogram
  uint8_t *uni = smem_dyn + sizeof(SmemB) + (((size_t)(V + 31) / 32 * 4 + 15) & ~(size_t)15);
  float *penv = reinterpret_cast<float *>(uni);
  if (threadIdx.x == 0) {
    sm.ckey = reinterpret_cast<unsigned long long *>(uni);
    sm.cidx = reinterpret_cast<int *>(uni + (size_t)kCandCap * 8);
    sm.hist = reinterpret_cast<unsigned int *>(uni + (size_t)kCandCap * 12);
  }
  const bool vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  const double rep = a.rep;
  auto pen_fn = [&](float x) { return __double2float_rd(__dsub_rn((double)x, rep)); };

  for (int b = blockIdx.x; b < a.rows; b += gridDim.x) {
    const int mrow = a.row_map ? a.row_map[b] : b;
    const float *L = a.logits + (size_t)mrow * a.ld;
    if (threadIdx.x == 0 && b + (int)gridDim.x < a.rows) {
      const int nrow = a.row_map ? a.row_map[b + gridDim.x] : b + gridDim.x;
      prefetch_row_l2(a.logits + (size_t)nrow * a.ld, V);
    }
    build_bitmap(a, mrow, bits, sm.plist, &sm.npen);
    const int np = sm.npen;
    const bool listed = NV4 > 0 && np <= kPenCap;
    if (listed) {
      for (int i = threadIdx.x; i < np; i += kSampThreads) {
        const int h = sm.plist[i];
        penv[h] = pen_fn(L[h]);
      }
      __syncthreads();
    }
    Row<NV4> row;
    row.L = L;
    row.V = V;
    row.vec = vec;
    row.load(bits, pen_fn, listed ? penv : nullptr);
    __syncthreads();  // the side table's space is reused below

    if (!fast_select_b<NV4>(a, bits, row, pen_fn, sm, k)) {
      if (!general_select_b(a, bits, L, sm, k)) {
        if (threadIdx.x == 0) {
          a.out[b] = -2;
          record_error(a.err, kErrSamplerArgs);
        }
        continue;
      }
    }

    // ---- src/tensor_ffi_adapter.php:180-204 over the k survivors ----
    if (a.T < 0.01) {
      if (threadIdx.x == 0) a.out[b] = sm.order[0];
      continue;
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

static int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <class K>
static void launch_persistent(K kern, const SampArgs &a, size_t sm, int per_sm, cudaStream_t st,
                              unsigned long long &done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(done & (1ull << dev))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    done |= 1ull << dev;
  }
  const int grid = std::min(a.rows, sm_count() * per_sm);
  kern<<<grid, kSampThreads, sm, st>>>(a);
}

template <int NV4>
static void launch_a(const SampArgs &a, size_t sm, cudaStream_t st) {
  static unsigned long long done = 0;  // attributes set, one bit per device
  launch_persistent(sample_a_kernel<NV4>, a, sm, NV4 > 0 && NV4 <= 8 ? 2 : 1, st, done);
}

template <int NV4>
static void launch_b(const SampArgs &a, size_t sm, cudaStream_t st) {
  static unsigned long long done = 0;
  launch_persistent(sample_b_kernel<NV4>, a, sm, NV4 > 0 && NV4 <= 8 ? 2 : 1, st, done);
}

int launch_sampler(const SampleLaunch &s, cudaStream_t stream) {
  int rc = check_sample_args(s);
  if (rc) return rc;
  if (s.rows == 0) return 0;
  SampArgs a;
  a.logits = s.logits;
  a.ld = s.ld;
  a.row_map = s.row_map;
  a.rows = s.rows;
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
  const size_t bitmap = ((size_t)((s.V + 31) / 32) * 4 + 15) & ~(size_t)15;
  const int layers = (s.V + 2047) / 2048;
  const size_t side = layers <= 16 ? (size_t)s.V * 4 : 0;  // register rows keep a side table
  if (s.variant == 0) {
    const size_t sm = sizeof(SmemA) + bitmap + side;
    if (layers <= 4)
      launch_a<4>(a, sm, stream);
    else if (layers <= 8)
      launch_a<8>(a, sm, stream);
    else if (layers <= 16)
      launch_a<16>(a, sm, stream);
    else
      launch_a<0>(a, sm, stream);
  } else {
    const size_t sm = sizeof(SmemB) + bitmap + std::max(side, kBUnionBytes);
    if (layers <= 4)
      launch_b<4>(a, sm, stream);
    else if (layers <= 8)
      launch_b<8>(a, sm, stream);
    else if (layers <= 16)
      launch_b<16>(a, sm, stream);
    else
      launch_b<0>(a, sm, stream);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("sampler launch failed: %s", cudaGetErrorString(e));
    return -4;
  }
  return 0;
}

}  // namespace snai
