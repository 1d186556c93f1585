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
constexpr int kMaxTopK = 512;
constexpr int kCandCap = 2048;   // exact-sort capacity
constexpr int kFastCand = kCandCap;  // candidates the fast path accepts
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
  double T, Tinv, rep, repinv, top_p;
  int top_k;
  int nan_guard;
  int *out;
  int *err;
  int redo;  // only the rows whose out[] holds kRedoMark (variant A's CTA-per-row kernel); 2: each staged whole
};

// out[] of a row the one-warp-per-row variant-A kernel could not certify
// (the CTA-per-row kernel's launch that follows redoes exactly these).  The
// redo launch writes its results as -(v + 10) (<= kRedoDone) so that every
// CTA still recognises the marked rows while others finish theirs; a last
// small launch decodes them.
constexpr int kRedoMark = -3;
constexpr int kRedoDone = -8;

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------

constexpr int kPenCap = 1024;  // unique history ids listed per row

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

// build_bitmap for ids already in registers: id (tid + 512 r) of the row is
// h[r] (-1 for none).
template <int HR>
__device__ __forceinline__ void build_bitmap_regs(int V, const int (&h)[HR], uint32_t *bits, int *plist, int *npen) {
  const int words = (V + 31) >> 5;
  __syncthreads();
  for (int i = threadIdx.x; i < words; i += blockDim.x) bits[i] = 0u;
  if (threadIdx.x == 0) *npen = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < HR; ++r) {
    const int t = h[r];
    bool first = false;
    if (t >= 0 && t < V) {
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

constexpr int kHistRegs = 2;  // history ids held per thread (rows of up to 1024 ids)

// Loads the history ids of a row into registers (for build_bitmap_regs).
__device__ __forceinline__ void load_hist_regs(const SampArgs &a, int mrow, int (&h)[kHistRegs]) {
  int n = a.hist_len ? a.hist_len[mrow] : a.hist_cols;
  n = min(max(n, 0), a.hist_cols);
  const int *hr = a.hist + (size_t)mrow * a.hist_ld;
#pragma unroll
  for (int r = 0; r < kHistRegs; ++r) {
    const int i = threadIdx.x + 512 * r;
    h[r] = i < n ? __ldg(hr + i) : -1;
  }
}

// Rows of logits staged one ahead into shared memory by TMA bulk copies.
struct RowFeeder {
  float *stage;
  uint64_t *bar;
  int uses = 0;
  // thread 0: copy row `mrow` into the stage (completion on `bar`)
  __device__ __forceinline__ void issue(const SampArgs &a, int mrow) const {
    const char *src = reinterpret_cast<const char *>(a.logits + (size_t)mrow * a.ld);
    const unsigned bytes = (unsigned)a.V * 4u;
    mbar_arrive_expect_tx(bar, bytes);
    for (unsigned off = 0; off < bytes; off += 32768u) {
      const unsigned n = min(32768u, bytes - off);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(reinterpret_cast<char *>(stage) + off)),
          "l"(src + off), "r"(n), "r"(smem_u32(bar))
          : "memory");
    }
  }
  __device__ __forceinline__ bool wait(int *err) {
    const bool ok = mbar_wait_bounded(bar, (uint32_t)(uses & 1), err, kErrWaitFull);
    ++uses;
    return ok;
  }
};

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

// The penalty of src/snai_inference.php:160-164 applied to a stored value
// (the division as in div_to_f32).
__device__ __forceinline__ float penalise_a(float t, double rep, double repinv) {
  return t > 0.f ? div_to_f32(t, rep, repinv) : __double2float_rn(__dmul_rn((double)t, rep));
}

// Variant A's stored value for vocab entry v (src/snai_inference.php:153, 160-164).
__device__ __forceinline__ float tempered(const SampArgs &a, const uint32_t *bits, float x, int v) {
  const float t = div_to_f32(x, a.T, a.Tinv);
  return in_set(bits, v) ? penalise_a(t, a.rep, a.repinv) : t;
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
  const float *S = nullptr;  // the row staged in shared memory (penalised entries already replaced)
  int V;
  bool vec;
  float4 r[NV4 > 0 ? NV4 : 1];
  unsigned long long pen = 0ull;

  __device__ __forceinline__ int layers() const { return NV4 > 0 ? NV4 : (V + 2047) / 2048; }
  __device__ __forceinline__ float4 fetch(int i) const {
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
    if (S) return v0 < V ? *reinterpret_cast<const float4 *>(S + v0) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (vec && v0 + 3 < V) return __ldg(reinterpret_cast<const float4 *>(L + v0));
    float4 f;
    f.x = v0 < V ? L[v0] : 0.f;
    f.y = v0 + 1 < V ? L[v0 + 1] : 0.f;
    f.z = v0 + 2 < V ? L[v0 + 2] : 0.f;
    f.w = v0 + 3 < V ? L[v0 + 3] : 0.f;
    return f;
  }
  // Loads (registers) and flags penalised entries; their values come
  // substituted from the staged row, or are computed here by pf.
  template <class PenFn>
  __device__ __forceinline__ void load(const uint32_t *bits, const PenFn &pf) {
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
              if (((w >> j) & 1u) && !S) f4_set(r[i], j, pf(f4_at(r[i], j)));
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
      if (!S) {  // a staged row holds the penalised values already
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if ((pbits >> j) & 1u) f4_set(o, j, pf(f4_at(o, j)));
      }
      return o;
    }
  }
};

// Calls f(i) for every chunk layer i: a fully unrolled loop with a literal
// trip count when the row is in registers (so every row.get(i) names a
// fixed register), a plain loop when it streams from memory.
template <int NV4, class F>
__device__ __forceinline__ void for_layers(int nl, const F &f) {
  if constexpr (NV4 > 0) {
#pragma unroll
    for (int i = 0; i < NV4; ++i) f(i);
  } else {
    for (int i = 0; i < nl; ++i) f(i);
  }
}

__device__ __forceinline__ int row_of(const SampArgs &a, int b) { return a.row_map ? a.row_map[b] : b; }

// Start of the staging buffer: after the core struct and the bitmap, rounded
// up to 128 bytes (bulk copies and 16-byte shared loads need 16-byte
// alignment; the host adds kStageAlign bytes of slack).
constexpr size_t kStageAlign = 128;
// (pointer arithmetic on the shared array, so the result stays a known
// shared-memory pointer)
__device__ __forceinline__ float *stage_ptr(uint8_t *smem, size_t core_bytes, int V) {
  const uint32_t off = (uint32_t)(core_bytes + (size_t)((V + 31) / 32) * 4);
  const uint32_t pad = (0u - (smem_u32(smem) + off)) & (uint32_t)(kStageAlign - 1);
  return reinterpret_cast<float *>(smem + off + pad);
}

// Brings row b into `row`: history bitmap and distinct-id list, the staged
// logits with penalised entries replaced in place (pf), registers loaded;
// then starts staging row b + gridDim.x and loading its history ids.
// Returns the raw logit 0 of row b.
template <int NV4, class PenFn>
__device__ __forceinline__ float row_prologue(const SampArgs &a, int b, Row<NV4> &row, uint32_t *bits, int *plist, int *npen,
                              RowFeeder &feed, bool staged, int (&hreg)[kHistRegs], bool hist_in_regs,
                              const PenFn &pf) {
  const int mrow = row_of(a, b);
  const float *L = a.logits + (size_t)mrow * a.ld;
  if (hist_in_regs)
    build_bitmap_regs(a.V, hreg, bits, plist, npen);
  else
    build_bitmap(a, mrow, bits, plist, npen);
  const int np = *npen;
  row.L = L;
  row.V = a.V;
  row.vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  float l0;
  if (staged) {
    feed.wait(a.err);
    float *st = feed.stage;
    l0 = st[0];
    __syncthreads();  // l0 read before the penalty rewrites entry 0
    if (np <= kPenCap) {
      for (int i = threadIdx.x; i < np; i += kSampThreads) {
        const int h = plist[i];
        st[h] = pf(st[h]);
      }
    } else {
      for (int v = threadIdx.x; v < a.V; v += kSampThreads)
        if (in_set(bits, v)) st[v] = pf(st[v]);
    }
    __syncthreads();
    row.S = st;
  } else {
    l0 = L[0];
  }
  row.load(bits, pf);
  __syncthreads();  // the stage has been consumed
  const int nb = b + (int)gridDim.x;
  if (nb < a.rows && !a.redo) {  // a redo pass stages each of its rows itself
    const int nrow = row_of(a, nb);
    if (staged && threadIdx.x == 0) feed.issue(a, nrow);
    if (hist_in_regs) load_hist_regs(a, nrow, hreg);
  }
  return l0;
}

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
  uint64_t bar;  // staging barrier
  int plist[kPenCap];
};

// Tier 1 / tier 2 of variant A: returns the id, or -1 if not certified.
// P(i, j) gives p of entry j of this thread's chunk layer i (as a double);
// `eps` bounds |p~ - p| / p for every entry (0 for the contract exp) and
// `eabs` the absolute error of an entry whose p~ underflowed.
template <int NV4, class PF>
__device__ __forceinline__ int certified_draw(SmemA &sm, int V, int nl, double u, double eps, double eabs, const PF &P) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // ---- segment sums (segment i = chunk layer i = 2048 consecutive ids) ----
  for (int g0 = 0; g0 < nl; g0 += 32) {
    const int g1 = min(nl, g0 + 32);
    auto seg = [&](int i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      const bool full = kSampThreads * 4 * (i + 1) <= V;
      double c = 0.0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const double pj = (full || v0 + j < V) ? P(i, j) : 0.0;
        c = __dadd_rn(c, pj);
      }
      c = warp_sum_d(c);
      if (lane == 0) sm.wp[i - g0][warp] = c;
    };
    if constexpr (NV4 > 0) {
      for_layers<NV4>(nl, seg);  // one group: NV4 <= 32
    } else {
      for (int i = g0; i < g1; ++i) seg(i);
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
__device__ __noinline__ void exact_max_a(const SampArgs &a, const uint32_t *bits, const float *L, float *wf, int *wi,
                                         float &best, int &bi) {
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
    wf[warp] = best;
    wi[warp] = bi;
  }
  __syncthreads();
  best = wf[0];
  bi = wi[0];
  for (int w = 1; w < kSampWarps; ++w)
    if (wf[w] > best || (wf[w] == best && wi[w] < bi)) {
      best = wf[w];
      bi = wi[w];
    }
  __syncthreads();
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads, NV4 > 0 && NV4 <= 8 ? 2 : 1) sample_a_kernel(const __grid_constant__ SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemA &sm = *reinterpret_cast<SmemA *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemA));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int V = a.V;
  const double rep = a.rep;
  auto pen_fn = [&](float x) { return penalise_a(div_to_f32(x, a.T, a.Tinv), rep, a.repinv); };
  RowFeeder feed;
  feed.stage = stage_ptr(smem_dyn, sizeof(SmemA), V);
  feed.bar = &sm.bar;
  // a redo pass takes rows out of order: no history run ahead, and its rows
  // are staged one at a time (redo 2: the launch made room for a row) so that
  // its passes over the row read shared memory instead of L2
  const bool staged = (NV4 > 0 || a.redo == 2) && (a.redo != 1) && (V & 3) == 0 && ((a.ld & 3) == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(feed.stage) & 15) == 0);
  const bool hist_in_regs = !a.redo && a.hist_cols <= 512 * kHistRegs;
  int hreg[kHistRegs];
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // the in-order pipeline stages its first row here; a redo pass issues each
  // of its rows' copies in row_body and waits for it there, so a CTA never
  // leaves with a copy into its shared memory in flight
  if ((int)blockIdx.x < a.rows && !a.redo) {
    const int r0 = row_of(a, blockIdx.x);
    if (staged && threadIdx.x == 0) feed.issue(a, r0);
    if (hist_in_regs) load_hist_regs(a, r0, hreg);
  }

  // a redo launch writes -(v + 10)
  auto put = [&](int b, int v) { a.out[b] = a.redo ? -(v + 10) : v; };
  auto row_body = [&](int b) {
    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;
    if (a.redo && staged && threadIdx.x == 0) {
      // the previous row's penalty writes to the stage come before this copy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      feed.issue(a, row_of(a, b));
    }
    Row<NV4> row;
    const float l0 = row_prologue(a, b, row, bits, sm.plist, &sm.npen, feed, staged, hreg, hist_in_regs, pen_fn);
    if (a.nan_guard && l0 != l0) {  // src/snai_inference.php:146
      if (threadIdx.x == 0) put(b, -1);
      return;
    }
    const int nl = row.layers();

    // ---- maximum: raw logits of unpenalised entries (t is monotone in L for
    // T > 0), exact values of penalised ones ----
    float xmax = -INFINITY, xabs = 0.f, pmax = -INFINITY, pabs = 0.f;
    int pidx = INT_MAX;
    for_layers<NV4>(nl, [&](int i) {
      uint32_t pb;
      const float4 x = row.get(i, bits, pen_fn, pb);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      // a whole layer is valid but the last (uniform test, no per-entry branch)
      const bool full = kSampThreads * 4 * (i + 1) <= V;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f = f4_at(x, j);
        const bool ok = full || v0 + j < V;
        const bool pn = (pb >> j) & 1u;
        const float xf = (ok && !pn) ? f : -INFINITY;
        const float pf = (ok && pn) ? f : -INFINITY;
        xmax = fmaxf(xmax, xf);
        xabs = fmaxf(xabs, (ok && !pn) ? fabsf(f) : 0.f);
        pabs = fmaxf(pabs, (ok && pn) ? fabsf(f) : 0.f);
        const bool up = pf > pmax;  // ids ascend along a thread's chunks: ties keep the first
        pmax = up ? pf : pmax;
        pidx = up ? v0 + j : pidx;
      }
    });
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
      if constexpr (NV4 > 0) {
        // flag the entries that can reach M, then check only those
        unsigned long long cm = 0ull;
        for_layers<NV4>(nl, [&](int i) {
          uint32_t pb;
          const float4 x = row.get(i, bits, pen_fn, pb);
          const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool c = v0 + j < V && !((pb >> j) & 1u) && f4_at(x, j) >= xthr;
            cm |= (unsigned long long)c << (4 * i + j);
          }
        });
        while (cm) {
          const int bit = __ffsll((long long)cm) - 1;
          cm &= cm - 1ull;
          const int i = bit >> 2, j = bit & 3;
          uint32_t pb;
          const float f = f4_at(row.get(i, bits, pen_fn, pb), j);
          if (div_to_f32(f, a.T, a.Tinv) == M) atomicMin(&sm.cand, (threadIdx.x + kSampThreads * i) * 4 + j);
        }
      } else {
        for_layers<NV4>(nl, [&](int i) {
          uint32_t pb;
          const float4 x = row.get(i, bits, pen_fn, pb);
          const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float f = f4_at(x, j);
            if (v0 + j < V && !((pb >> j) & 1u) && f >= xthr) {
              if (div_to_f32(f, a.T, a.Tinv) == M) atomicMin(&sm.cand, v0 + j);
            }
          }
        });
      }
      __syncthreads();
      best = M;
      bi = sm.cand;
      __syncthreads();
    } else {
      exact_max_a(a, bits, L, sm.wf[0], sm.wi, best, bi);
    }
    // PHP: max starts at -INF and only a strictly larger value moves it.
    const bool any = best > -INFINITY;
    const double maxv = any ? (double)best : -INFINITY;
    if (a.T <= 0.01) {
      if (threadIdx.x == 0) put(b, any ? bi : 0);
      return;
    }
    const double u = (double)a.uniforms[b];
    int id = -1;
    if (any && simple && !a.redo) {  // a redo row has failed a tier-1 bound already
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
        const float mult = ((pb >> j) & 1u) ? l2e : c;
        return (double)ex2_approx(fmaf(f4_at(x, j), mult, -m2));
      };
      id = certified_draw<NV4>(sm, V, nl, u, eps, 0x1p-125, P1);
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
      id = certified_draw<NV4>(sm, V, nl, u, 0.0, 0.0, P2);
    }
    if (id < 0) {
      // tier 3
      if (warp == 0) {
        const int s = sequential_a(a, bits, L, maxv, u);
        if (lane == 0) put(b, s);
      }
    } else if (threadIdx.x == 0) {
      put(b, id);
    }
    };
  if (!a.redo) {
    for (int b = blockIdx.x; b < a.rows; b += gridDim.x) row_body(b);
  } else {
    // the marked rows (kRedoMark, or already redone: <= kRedoDone) in id
    // order; this CTA takes those of rank = blockIdx.x (mod gridDim.x)
    __shared__ int redo_cnt[kSampWarps];
    __shared__ int redo_list[kSampThreads];
    int seen = 0;
    for (int b0 = 0; b0 < a.rows; b0 += kSampThreads) {
      const int bb = b0 + (int)threadIdx.x;
      const int ov = bb < a.rows ? a.out[bb] : 0;
      const bool mk = ov == kRedoMark || ov <= kRedoDone;
      const unsigned bal = __ballot_sync(0xffffffffu, mk);
      if (lane == 0) redo_cnt[warp] = __popc(bal);
      __syncthreads();
      int before = 0, tot = 0;
      for (int w = 0; w < kSampWarps; ++w) {
        const int c = redo_cnt[w];
        before += w < warp ? c : 0;
        tot += c;
      }
      const int rank = seen + before + __popc(bal & ((1u << lane) - 1u));
      const bool mine = mk && ov == kRedoMark && rank % (int)gridDim.x == (int)blockIdx.x;
      const unsigned bm2 = __ballot_sync(0xffffffffu, mine);
      __syncthreads();
      if (lane == 0) redo_cnt[warp] = __popc(bm2);
      __syncthreads();
      int b2 = 0, t2 = 0;
      for (int w = 0; w < kSampWarps; ++w) {
        const int c = redo_cnt[w];
        b2 += w < warp ? c : 0;
        t2 += c;
      }
      if (mine) redo_list[b2 + __popc(bm2 & ((1u << lane) - 1u))] = bb;
      __syncthreads();
      for (int q = 0; q < t2; ++q) {
        row_body(redo_list[q]);
        __syncthreads();
      }
      seen += tot;
    }
  }

}

// ---------------------------------------------------------------------------
// Variant B
// ---------------------------------------------------------------------------

struct SmemB {
  unsigned int wtot[kSampWarps];
  int ncand;
  unsigned int prefix, pmask;
  int need;
  int bstar;
  unsigned int bcount;
  int ties_left;
  int overflow;
  float fw[3][kSampWarps];
  float R;
  int npen;
  uint64_t bar;  // staging barrier
  __align__(16) unsigned int hist[256];
  unsigned long long ckey[kCandCap];  // exact order key of a candidate; p[] and cum[] after ranking
  int cidx[kCandCap];
  int order[kMaxTopK];
  double val[kMaxTopK];
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

// Ranks the nc gathered candidates (PHP's arsort order: value descending,
// then id ascending) and keeps the first k: sm.order[rank] = id and
// sm.val[rank] = exp(val / T) (src/tensor_ffi_adapter.php:183-184), or the
// value itself when T < 0.01 (greedy).  G = 2^lg threads share a candidate,
// each counting the candidates that precede it among every G-th one, and add
// their counts by shuffles.
__device__ void rank_candidates(SmemB &sm, int nc, int k, double T) {
  int lg = 0;
  while (lg < 5 && (nc << (lg + 1)) <= kSampThreads) ++lg;
  const int G = 1 << lg, per = kSampThreads >> lg;
  const int sub = threadIdx.x & (G - 1);
  const bool want_p = !(T < 0.01);
  for (int c0 = 0; c0 < nc; c0 += per) {
    const int i = c0 + (threadIdx.x >> lg);
    int rank = 0;
    unsigned long long ki = 0ull;
    int vi = 0;
    if (i < nc) {
      ki = sm.ckey[i];
      vi = sm.cidx[i];
#pragma unroll 4
      for (int j = sub; j < nc; j += G) {
        const unsigned long long kj = sm.ckey[j];
        const int vj = sm.cidx[j];
        rank += (int)((kj > ki) | ((kj == ki) & (vj < vi)));
      }
    }
    for (int o = 1; o < G; o <<= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
    if (i < nc && sub == 0 && rank < k) {
      sm.order[rank] = vi;
      const double val = key_to_double(ki);
      sm.val[rank] = want_p ? snai_exp(__ddiv_rn(val, T)) : val;
    }
  }
  __syncthreads();
}

// Absolute margin of the certified top-p tail.  Against PHP's sequential
// sums, the warp's tree sum, reciprocal and scanned running sums of k <= 512
// terms (each running sum at most 1 + 2^-40) differ by at most
// (2k + 44) 2^-53 <= 1.2e-13; 2^-40 is 7.7 times that.
constexpr double kTailEps = 0x1p-40;

// First index i in [0, k) with C[i] >= x, INT_MAX if none: lane l scans its
// own survivors [i0, i1), the warp takes the minimum.
__device__ __forceinline__ int warp_first_ge(const double *C, int i0, int i1, double x) {
  int f = INT_MAX;
  for (int i = i0; i < i1; ++i)
    if (C[i] >= x) {
      f = i;
      break;
    }
  return __reduce_min_sync(0xffffffffu, f);
}

// src/tensor_ffi_adapter.php:180-204 over k ranked survivors (order[0..k),
// their p in P[0..k)), by one warp; C is scratch for k doubles.  PHP sums p
// in order, divides each p by the sum, accumulates the quotients in order
// until the running sum reaches top_p (crossing term included), takes
// r = u * cum and returns the first survivor whose running sum reaches r.
// The warp computes the same running sums by a tree sum, one reciprocal and
// a lane-then-warp scan, each within kTailEps of PHP's, and accepts the
// result when every decision clears the margin: the first running sum at or
// above top_p - eps is also at or above top_p + eps (or both are the last),
// and for r anywhere in the interval this leaves, the first running sum at
// or above r - eps is also at or above r + eps and lies in the kept prefix.
// Otherwise (a decision within 1e-12, or p infinite, NaN or all zero) lane 0
// redoes PHP's sequential arithmetic exactly.  Returns the id on every lane.
__device__ __forceinline__ int warp_topp(const int *order, const double *P, double *C, int k, double u,
                                         double top_p) {
  const int lane = threadIdx.x & 31;
  const int m = (k + 31) >> 5;
  const int i0 = min(k, lane * m), i1 = min(k, i0 + m);
  double part = 0.0;
  for (int i = i0; i < i1; ++i) part = __dadd_rn(part, P[i]);
  double S = part;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) S = __dadd_rn(S, __shfl_xor_sync(0xffffffffu, S, o));
  int id = -1;
  if (S > 0.0 && S <= DBL_MAX) {
    const double inv = __drcp_rn(S);
    double run = 0.0;
    for (int i = i0; i < i1; ++i) run = __fma_rn(P[i], inv, run);
    double incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = __dadd_rn(incl, n);
    }
    double c = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) c = 0.0;
    for (int i = i0; i < i1; ++i) {
      c = __fma_rn(P[i], inv, c);
      C[i] = c;
    }
    __syncwarp();
    const int jl = min(warp_first_ge(C, i0, i1, top_p - kTailEps), k - 1);
    const int jh = min(warp_first_ge(C, i0, i1, top_p + kTailEps), k - 1);
    const double rl = __dmul_rn(u, C[jl]) - kTailEps, rh = __dmul_rn(u, C[jh]) + kTailEps;
    const int sa = warp_first_ge(C, i0, i1, rl - kTailEps);
    const int sb = warp_first_ge(C, i0, i1, rh + kTailEps);
    if (sa == sb && sa <= jl) id = order[sa];
    __syncwarp();
  }
  if (id < 0) {
    double s = 0.0;
    if (lane == 0)
      for (int i = 0; i < k; ++i) s = __dadd_rn(s, P[i]);
    s = __shfl_sync(0xffffffffu, s, 0);
    for (int i = lane; i < k; i += 32) C[i] = __ddiv_rn(P[i], s);
    __syncwarp();
    if (lane == 0) {
      // $cum_check after i+1 terms is this same running sum
      double cum = 0.0;
      int nf = 0;
      for (int i = 0; i < k; ++i) {
        cum = __dadd_rn(cum, C[i]);
        C[i] = cum;
        nf = i + 1;
        if (cum >= top_p) break;
      }
      const double rr = __dmul_rn(u, cum);
      id = order[0];
      for (int i = 0; i < nf; ++i)
        if (rr <= C[i]) {
          id = order[i];
          break;
        }
    }
    id = __shfl_sync(0xffffffffu, id, 0);
    __syncwarp();
  }
  return id;
}

// The tail of row b over the CTA's ranked survivors (sm.order, p in sm.val),
// by warp 0 alone (the other warps return at once).  Greedy (T < 0.01)
// takes order[0].
__device__ __forceinline__ void topp_tail(const SampArgs &a, SmemB &sm, int k, int b) {
  if (threadIdx.x >= 32) return;
  if (a.T < 0.01) {
    if (threadIdx.x == 0) a.out[b] = sm.order[0];
    return;
  }
  const double u = (double)a.uniforms[b];
  const int id = warp_topp(sm.order, sm.val, reinterpret_cast<double *>(sm.ckey), k, u, a.top_p);
  if (threadIdx.x == 0) a.out[b] = id;
}

// Fast selection (see the file comment).  The row holds lower bounds (the
// raw logit, or fp32-round-down(L - rep) for penalised entries).  Returns
// false (the same on every thread) when the row needs the general path.
template <int NV4, class PenFn>
__device__ __forceinline__ bool fast_select_b(const SampArgs &a, const uint32_t *bits, const Row<NV4> &row, const PenFn &pf,
                              SmemB &sm, int k) {
  const int V = a.V, nl = row.layers();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // pass 1: maximum and spread of the lower bounds
  float mx = -INFINITY, s1 = 0.f, s2 = 0.f;
  for_layers<NV4>(nl, [&](int i) {
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
  });
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
    for_layers<NV4>(nl, [&](int i) {
      uint32_t pb;
      const float4 x = row.get(i, bits, pf, pb);
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d = mx - f4_at(x, j);
        if (v0 + j < V && d < R) atomicAdd(&sm.hist[min((int)(d * inv_w), 254)], 1u);
      }
    });
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
  for_layers<NV4>(nl, [&](int i) {
    uint32_t pb;
    const float4 x = row.get(i, bits, pf, pb);
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = mx - next_up(f4_at(x, j));
      if (v0 + j < V && d < R && (int)(d * inv_w) <= bstar) ++mine;
    }
  });
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
    for_layers<NV4>(nl, [&](int i) {
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
    });
  }
  __syncthreads();
  const int nc = sm.ncand;
  __syncthreads();
  if (nc > kFastCand || nc < k) return false;
  rank_candidates(sm, nc, k, a.T);
  return true;
}
// General selection: radix select on the 32-bit keys of the lower bounds
// (four 8-bit digits), superset gather by the upper bounds, exact sort.
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
  bool exact = false;
  for (int pass = 0; pass < 4; ++pass) {
    const int sh = 24 - 8 * pass, wd = 8;
    const unsigned int bmask = (1u << wd) - 1u;
    for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
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
    exact = (pass == 3);
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
  rank_candidates(sm, sm.ncand, k, a.T);
  return true;
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads, NV4 > 0 && NV4 <= 8 ? 2 : 1) sample_b_kernel(const __grid_constant__ SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  uint32_t *bits = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB));
  const int V = a.V;
  const int k = min(a.top_k, V);
  const double rep = a.rep;
  auto pen_fn = [&](float x) { return __double2float_rd(__dsub_rn((double)x, rep)); };
  RowFeeder feed;
  feed.stage = stage_ptr(smem_dyn, sizeof(SmemB), V);
  feed.bar = &sm.bar;
  const bool staged = NV4 > 0 && (V & 3) == 0 && ((a.ld & 3) == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(feed.stage) & 15) == 0);
  const bool hist_in_regs = a.hist_cols <= 512 * kHistRegs;
  int hreg[kHistRegs];
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if ((int)blockIdx.x < a.rows) {
    const int r0 = row_of(a, blockIdx.x);
    if (staged && threadIdx.x == 0) feed.issue(a, r0);
    if (hist_in_regs) load_hist_regs(a, r0, hreg);
  }

  for (int b = blockIdx.x; b < a.rows; b += gridDim.x) {
    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;
    Row<NV4> row;
    row_prologue(a, b, row, bits, sm.plist, &sm.npen, feed, staged, hreg, hist_in_regs, pen_fn);

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
    topp_tail(a, sm, k, b);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Register-row kernels: rows of at most 2048 * kRegLayers logits with a
// 16-byte aligned start and a length that is a multiple of 4, and at most
// kPenCap history ids.  Row b is staged into shared memory by bulk copies
// while row b - grid is processed, then moved into registers (thread t owns
// the 16-byte chunks t, t + 512, ...), which frees the stage for the next
// row.  Before that, the threads that listed the row's distinct history ids
// settle those entries in the stage: variant A replaces them by -inf (they
// then drop out of the maximum and of every exponential sum) and keeps
// their exact stored values in a side table; variant B replaces them by the
// fp32 lower bound of L - rep.  Bulk passes thus cost one to three
// instructions per entry with no per-entry branches, and only the entries
// near a decision take exact double arithmetic.
//
// Row pipeline (it = this CTA's row counter): the history bitmap and id
// list of row it are built during row it - 1 (three rotating bitmaps, two
// lists), the per-row counters have two copies, and block maxima are
// shared-memory atomics on order-preserving keys, so a greedy row needs
// three block barriers.
// ---------------------------------------------------------------------------

constexpr int kRegLayers = 16;             // chunk layers held in registers at most
constexpr int kSegLen = kSampThreads * 4;  // ids per chunk layer

// 16-byte shared-memory load by shared-window address
__device__ __forceinline__ float4 lds4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float fmax4(const float4 &x) { return fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w)); }
// inverse of okey32 (key 0, NaN's key, maps to -inf)
__device__ __forceinline__ float key_to_float(unsigned int k) {
  if (k == 0u) return -INFINITY;
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// (value, id) key whose maximum is the largest value, then the smallest id
__device__ __forceinline__ unsigned long long argmax_key(float t, int v) {
  return ((unsigned long long)okey32(t) << 32) | (unsigned long long)(0xffffffffu - (unsigned int)v);
}

template <int N>
__device__ __forceinline__ float4 pick_layer(const float4 (&r)[N], int i) {
  float4 o = r[0];
#pragma unroll
  for (int q = 1; q < N; ++q)
    if (q == i) o = r[q];
  return o;
}

template <int N> struct Log2 { static constexpr int v = 1 + Log2<N / 2>::v; };
template <> struct Log2<1> { static constexpr int v = 0; };

// Per-layer warp totals of N per-lane values by a reduce-scatter butterfly
// (plain additions, each one rounding):
// returns the total of layer (lane >> (5 - log2 N)) (every lane of the
// group holds it).  Each total is a tree of depth 5.
template <int N, class T>
__device__ __forceinline__ T warp_reduce_layers(T (&v)[N]) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "power of two");
#pragma unroll
  for (int step = 0; step < Log2<N>::v; ++step) {
    const int o = 16 >> step;
    const int n = N >> step;
    const bool up = (threadIdx.x & o) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; ++k) {
      const T send = up ? v[k] : v[k + n / 2];
      const T keep = up ? v[k + n / 2] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  T s = v[0];
#pragma unroll
  for (int o = 16 >> Log2<N>::v; o > 0; o >>= 1) s = s + __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Per-CTA row pipeline state.  [p] = row parity, bitmaps follow the struct.
struct RowPipe {
  uint64_t bar;  // staging barrier
  int npen[2];   // entries in the row's distinct-id list (variant A)
  unsigned long long pkey[2][kSampWarps];  // per-warp argmax keys of the penalised values
  unsigned int xkey[2];
  int cand[2];
  float l0[2];
  float s1[2], s2[2];
};

__device__ __forceinline__ void pipe_reset(RowPipe &p, int par) {
  p.npen[par] = 0;
  p.xkey[par] = 0u;
  p.cand[par] = INT_MAX;
  p.s1[par] = 0.f;
  p.s2[par] = 0.f;
}

// Marks the history ids in h (each thread's share, -1 for none) that fall in
// [lo, lo + V) in a cleared bitmap of that range; with a list, the thread
// whose atomicOr set a bit also appends the (range-local) id to plist
// (warp-aggregated slots, count in *npen); with `own`, that thread keeps the
// id in own[r] instead (-1 where it set no bit), so every distinct id has
// exactly one owner.
__device__ __forceinline__ void mark_ids(int V, const int (&h)[kHistRegs], uint32_t *bits, int *plist, int *npen,
                                         int lo = 0, int *own = nullptr) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kHistRegs; ++r) {
    const int t = h[r] - lo;
    bool first = false;
    if (t >= 0 && t < V) {
      const uint32_t bit = 1u << (t & 31);
      const uint32_t old = atomicOr(&bits[t >> 5], bit);
      first = !(old & bit);
    }
    if (own) own[r] = first ? t : -1;
    if (plist) {
      const unsigned m = __ballot_sync(0xffffffffu, first);
      int base = 0;
      if (lane == 0 && m) base = atomicAdd(npen, __popc(m));
      base = __shfl_sync(0xffffffffu, base, 0) + __popc(m & ((1u << lane) - 1u));
      if (first && base < kPenCap) plist[base] = t;
    }
  }
}

// Kernel start: clears the three bitmaps and both counter sets, builds the
// bitmap of the CTA's first row and starts its staging.
// (rows b0, b0 + stride, ...: one CTA per row by default; a CTA of a
// cluster handles the ids [lo, lo + a.V) of its cluster's rows)
__device__ __forceinline__ void pipe_start(const SampArgs &a, RowPipe &p, uint32_t *bm, int words, RowFeeder &feed,
                                           int (&hreg)[kHistRegs], int *plist0, int lo = 0, int b0 = -1,
                                           int stride = 0, int *own = nullptr) {
  if (b0 < 0) {
    b0 = blockIdx.x;
    stride = gridDim.x;
  }
  if (threadIdx.x == 0) {
    mbar_init(&p.bar, 1);
    fence_barrier_init();
    pipe_reset(p, 0);
    pipe_reset(p, 1);
  }
  for (int i = threadIdx.x; i < 3 * words; i += kSampThreads) bm[i] = 0u;
  __syncthreads();
  if (b0 < a.rows) {
    const int r0 = row_of(a, b0);
    if (threadIdx.x == 0) feed.issue(a, r0);
    load_hist_regs(a, r0, hreg);
    mark_ids(a.V, hreg, bm, plist0, &p.npen[0], lo, own);
    const int b1 = b0 + stride;
    if (b1 < a.rows) load_hist_regs(a, row_of(a, b1), hreg);
  }
  __syncthreads();
}

// After the first barrier of row `it` (every thread has moved row b into
// registers and finished row it - 1): start staging row b + grid, clear the
// bitmap of row it + 2, mark (and list) row it + 1's history (its bitmap and
// list count were reset at the start of row it: pipe_reset) and load row
// it + 2's.
__device__ __forceinline__ void pipe_advance(const SampArgs &a, RowPipe &p, uint32_t *bm, int words, int it, int b,
                                             RowFeeder &feed, int (&hreg)[kHistRegs], int *plist_next, int lo = 0,
                                             int stride = 0, int *own = nullptr) {
  if (stride == 0) stride = gridDim.x;
  const int nb = b + stride;
  if (nb < a.rows && threadIdx.x == 0) {
    // the stage was written through the generic proxy (settled entries)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    feed.issue(a, row_of(a, nb));
  }
  uint32_t *clr = bm + ((it + 2) % 3) * words;
  for (int i = threadIdx.x; i < words; i += kSampThreads) clr[i] = 0u;
  if (nb < a.rows) {
    mark_ids(a.V, hreg, bm + ((it + 1) % 3) * words, plist_next, &p.npen[(it + 1) & 1], lo, own);
    const int nnb = nb + stride;
    if (nnb < a.rows) load_hist_regs(a, row_of(a, nnb), hreg);
  }
}

struct SmemRA {
  RowPipe pipe;
  double wp[kRegLayers][kSampWarps];  // per-warp totals of each chunk layer
  double wsum[kSampWarps];
  double segpen[kSegLen];             // p of the penalised entries of the crossing layer
  double S, r, base;
  int ss, dcand;
  int plist[2][kPenCap];
  float pval[2][kPenCap];  // exact stored value of plist[.][s]
};

// Certified draw (tiers 1 and 2 of variant A) over a row read through
// acc(i) (chunk layer i of this thread: raw logits, -inf for penalised
// entries and past the vocab).  pe(x) gives p of an unpenalised raw value x
// (0 for -inf; float in tier 1, whose chunk sums and per-warp layer sums are
// then taken in fp32, double in tier 2); pp(s) gives p of penalised entry
// plist[s] (same type), added to its layer's partial sum by the thread that
// holds slot s.  Returns the id, or -1 if not certified.
template <int NV4, class ACC, class PE, class PP>
__device__ __forceinline__ int draw_reg(SmemRA &sm, const uint32_t *bits, const int *plist, const ACC &acc, int V,
                                        int np, double u, double eps, double eabs, const PE &pe, const PP &pp) {
  using PT = decltype(pe(0.f));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int SH = 5 - Log2<NV4>::v;
  PT part[NV4];
#pragma unroll
  for (int i = 0; i < NV4; ++i) {
    const float4 x = acc(i);
    part[i] = (pe(x.x) + pe(x.y)) + (pe(x.z) + pe(x.w));
  }
  PT pq[kPenCap / kSampThreads];
#pragma unroll
  for (int q = 0; q < kPenCap / kSampThreads; ++q) {
    const int s = threadIdx.x + q * kSampThreads;
    pq[q] = PT(0);
    if (s < np) {
      pq[q] = pp(s);
      const int sg = plist[s] / kSegLen;
#pragma unroll
      for (int i = 0; i < NV4; ++i) part[i] = part[i] + (i == sg ? pq[q] : PT(0));
    }
  }
  const PT lt = warp_reduce_layers<NV4>(part);
  if ((lane & ((1 << SH) - 1)) == 0) sm.wp[lane >> SH][warp] = (double)lt;
  __syncthreads();
  if (warp == 0) {
    double seg = 0.0;
    if (lane < NV4)
      for (int w = 0; w < kSampWarps; ++w) seg = __dadd_rn(seg, sm.wp[lane][w]);
    double incl = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = __dadd_rn(incl, n);
    }
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = 0.0;
    const double S = __shfl_sync(0xffffffffu, incl, 31);
    const double rr = __dmul_rn(u, S);
    const unsigned hit = __ballot_sync(0xffffffffu, lane < NV4 && incl >= rr);
    const int ss = hit ? __ffs(hit) - 1 : 0;
    const double base = __shfl_sync(0xffffffffu, excl, ss);
    if (lane == 0) {
      sm.S = S;
      sm.r = rr;
      sm.base = base;
      sm.ss = (isfinite(S) && isfinite(rr) && hit && u >= 0.0 && u <= 1.0) ? ss : -1;
      sm.dcand = INT_MAX;
    }
  }
  __syncthreads();
  const int ss = sm.ss;
  if (ss < 0) return -1;
#pragma unroll
  for (int q = 0; q < kPenCap / kSampThreads; ++q) {
    const int s = threadIdx.x + q * kSampThreads;
    if (s < np) {
      const int h = plist[s];
      if (h / kSegLen == ss) sm.segpen[h % kSegLen] = (double)pq[q];
    }
  }
  __syncthreads();
  // ---- running sums inside the crossing layer ----
  const double S = sm.S, rr = sm.r;
  const int v0 = (threadIdx.x + kSampThreads * ss) * 4;
  const float4 x = acc(ss);
  const uint32_t pw = v0 < V ? (bits[v0 >> 5] >> (v0 & 31)) & 0xFu : 0u;
  double p[4];
  double c = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float f = f4_at(x, j);
    p[j] = v0 + j >= V ? 0.0 : ((pw >> j) & 1u) ? sm.segpen[(v0 + j) % kSegLen] : (double)pe(f);
    c = __dadd_rn(c, p[j]);
  }
  // exclusive block scan of c in thread order: warp Kogge-Stone, then the
  // warp totals scanned by every warp with shuffles
  double incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl = __dadd_rn(incl, n);
  }
  if (lane == 31) sm.wsum[warp] = incl;
  __syncthreads();
  double wt = lane < kSampWarps ? sm.wsum[lane] : 0.0;
#pragma unroll
  for (int o = 1; o < kSampWarps; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, wt, o);
    if (lane >= o) wt = __dadd_rn(wt, n);
  }
  double wbase = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
  if (warp == 0) wbase = 0.0;
  double ex = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) ex = 0.0;
  ex = __dadd_rn(wbase, ex);
  double prev = __dadd_rn(sm.base, ex);
  int mine = -1;
  double lo = prev, hi = prev;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const double cur = __dadd_rn(prev, p[j]);
    if (mine < 0 && v0 + j < V && cur >= rr) {
      mine = j;
      lo = prev;
      hi = cur;
    }
    prev = cur;
  }
  if (mine >= 0) {
    // A crossing thread certifies its own candidate; the smallest candidate
    // (the first crossing) wins, with its verdict in the low bit.
    // Error model: every p~ is within eps*p (+ eabs if it underflowed) of
    // the contract value; every computed sum is a tree over non-negative
    // terms of depth at most nl + 64 (chunk, penalised, butterfly, warp,
    // layer, scan) against the sequential sum's depth of at most
    // V; 2^-52 per level is twice the first-order rounding constant.
    const int cand = v0 + mine;
    const double slack = (double)(NV4 + 64);
    const double er = eps * (1.0 + 2.0 * eps) + 1e-12 * (eps > 0.0);
    const double Er = u * (er * S + (double)V * eabs + ((double)V + slack) * 0x1p-52 * S) + 0x1p-52 * rr;
    const double Ehi = er * hi + ((double)cand + 1.0) * eabs + ((double)cand + slack) * 0x1p-52 * hi;
    const double Elo = er * lo + (double)cand * eabs + ((double)cand + slack) * 0x1p-52 * lo;
    const bool up = hi - Ehi >= rr + Er;
    const bool dn = cand == 0 || lo + Elo < rr - Er;
    atomicMin(&sm.dcand, 2 * cand + ((up && dn) ? 0 : 1));
  }
  __syncthreads();
  const int key = sm.dcand;
  return (key != INT_MAX && !(key & 1)) ? key >> 1 : -1;
}

// Tier 2 of the register-row kernel: the contract exponential of the exact
// stored values, reading the raw row from global memory (a rare path, kept
// out of line so it does not weigh on the register row's allocation).
template <int NV4>
__device__ __noinline__ int tier2_a(const SampArgs &a, const uint32_t *bits, const float *L, SmemRA &sm,
                                    const int *plist, const float *pval, int np, double u, double maxv) {
  const int V = a.V;
  auto acc = [&](int i) {
    const int v0 = (threadIdx.x + kSampThreads * i) * 4;
    float4 x = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (v0 < V) {
      x = __ldg(reinterpret_cast<const float4 *>(L + v0));
      const uint32_t w = (bits[v0 >> 5] >> (v0 & 31)) & 0xFu;
      if (w & 1u) x.x = -INFINITY;
      if (w & 2u) x.y = -INFINITY;
      if (w & 4u) x.z = -INFINITY;
      if (w & 8u) x.w = -INFINITY;
    }
    return x;
  };
  return draw_reg<NV4>(
      sm, bits, plist, acc, V, np, u, 0.0, 0.0,
      [&](float x) { return snai_exp(__dsub_rn((double)div_to_f32(x, a.T, a.Tinv), maxv)); },
      [&](int s) { return snai_exp(__dsub_rn((double)pval[s], maxv)); });
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads, NV4 <= 8 ? 2 : 1) sample_a_reg(const __grid_constant__ SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemRA &sm = *reinterpret_cast<SmemRA *>(smem_dyn);
  RowPipe &pp = sm.pipe;
  const int V = a.V;
  const int words = (V + 31) >> 5;
  uint32_t *bm = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemRA));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool greedy = a.T <= 0.01;
  RowFeeder feed;
  feed.stage = stage_ptr(smem_dyn, sizeof(SmemRA) + (size_t)8 * words, V);
  feed.bar = &pp.bar;
  int hreg[kHistRegs];
  pipe_start(a, pp, bm, words, feed, hreg, sm.plist[0]);

  // Every row ends with a block barrier, so at a row's start the previous
  // row has finished with everything of the other parity.
  int it = 0;
  for (int b = blockIdx.x; b < a.rows; b += gridDim.x, ++it) {
    const int par = it & 1;
    const uint32_t *bits = bm + (it % 3) * words;
    int *plist = sm.plist[par];
    float *pval = sm.pval[par];
    if (threadIdx.x == 0) pipe_reset(pp, par ^ 1);
    const bool ok = feed.wait(a.err);
    const int np = min(pp.npen[par], kPenCap);
    // exact stored values of the penalised entries, by the threads that
    // listed them (-inf left in the stage); their (value, id) argmax per warp
    unsigned long long pk = 0ull;
    if (warp * 32 < np) {
#pragma unroll
      for (int q = 0; q < kPenCap / kSampThreads; ++q) {
        const int s = threadIdx.x + q * kSampThreads;
        if (s < np) {
          const int h = plist[s];
          const float raw = feed.stage[h];
          if (h == 0) pp.l0[par] = raw;
          const float t = penalise_a(div_to_f32(raw, a.T, a.Tinv), a.rep, a.repinv);
          pval[s] = t;
          feed.stage[h] = -INFINITY;
          const unsigned long long key = argmax_key(t, h);
          pk = key > pk ? key : pk;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, pk, o);
        pk = ok2 > pk ? ok2 : pk;
      }
    }
    if (lane == 0) pp.pkey[par][warp] = pk;
    __syncthreads();

    // ---- registers; maximum of the unpenalised raw logits ----
    float4 r[NV4];
    float xmax = -INFINITY;
    const uint32_t st_u32 = smem_u32(feed.stage);
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      r[i] = v0 < V ? lds4(st_u32 + 4u * v0) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      xmax = fmaxf(xmax, fmax4(r[i]));
    }
    if (threadIdx.x == 0 && !(bits[0] & 1u)) pp.l0[par] = r[0].x;
    const float my_xmax = xmax;
    xmax = warp_max(xmax);
    if (lane == 0) atomicMax(&pp.xkey[par], okey32(xmax));
    if (!__syncthreads_and(ok)) break;
    pipe_advance(a, pp, bm, words, it, b, feed, hreg, sm.plist[par ^ 1]);

    if (a.nan_guard && pp.l0[par] != pp.l0[par]) {  // src/snai_inference.php:146
      if (threadIdx.x == 0) a.out[b] = -1;
      __syncthreads();
      continue;
    }
    xmax = key_to_float(pp.xkey[par]);
    pk = pp.pkey[par][lane & (kSampWarps - 1)];
#pragma unroll
    for (int o = kSampWarps / 2; o > 0; o >>= 1) {
      const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, pk, o);
      pk = ok2 > pk ? ok2 : pk;
    }
    const float pmax = key_to_float((unsigned int)(pk >> 32));
    const int pidx = pk ? (int)(0xffffffffu - (unsigned int)pk) : INT_MAX;
    const float tmax = (xmax > -INFINITY) ? div_to_f32(xmax, a.T, a.Tinv) : -INFINITY;
    const float M = fmaxf(tmax, pmax);
    const bool simple = a.T > 0.0 && isfinite(M) && isfinite(xmax);
    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;

    if (greedy && simple) {
      // first index attaining M: entries with fp32(x/T) == M have
      // x >= (M - |M| 2^-23) T; only threads holding one look
      const double lowt = (double)M - fabs((double)M) * 0x1p-22 - 1e-44;
      const float xthr = __double2float_rd(lowt * a.T);
      int mc = INT_MAX;
      if (my_xmax >= xthr) {
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
          if (fmax4(r[i]) >= xthr) {
            const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float f = f4_at(r[i], j);
              if (f >= xthr && div_to_f32(f, a.T, a.Tinv) == M) mc = min(mc, v0 + j);
            }
          }
        }
      }
      if (threadIdx.x == 0 && pmax == M) mc = min(mc, pidx);
      if (mc != INT_MAX) atomicMin(&pp.cand[par], mc);
      __syncthreads();
      if (threadIdx.x == 0) a.out[b] = pp.cand[par];
      continue;
    }

    float best = M;
    int bi = INT_MAX;
    if (!simple) exact_max_a(a, bits, L, reinterpret_cast<float *>(sm.wsum), reinterpret_cast<int *>(sm.wsum) + 16,
                             best, bi);
    // PHP: max starts at -INF and only a strictly larger value moves it.
    const bool any = best > -INFINITY;
    if (greedy) {
      if (threadIdx.x == 0) a.out[b] = any ? bi : 0;
      __syncthreads();
      continue;
    }
    const double maxv = any ? (double)best : -INFINITY;
    const double u = (double)a.uniforms[b];
    int id = -1;
    if (any && simple) {
      // tier 1: p~ = 2^(x c - M log2e), c = fp32(log2e / T); penalised entries
      // use their exact value t: 2^(t log2e - M log2e).  Rounding of c, of
      // fp32(M log2e) and of the fma moves the exponent by at most
      // 3 (|t| + |M|) log2e 2^-24, and ex2.approx adds a relative 2^-22.
      // Entries with t < M - 91 have p < 2^-131 and p~ < 2^-125 (flushed or
      // tiny): an absolute error of eabs = 2^-125 each.  Every other entry
      // has |t| <= |M| + 91, whence the relative bound below.  A NaN logit
      // makes S NaN and the row falls through to tier 3; -inf entries give 0
      // in both.  The fp32 sums (4 entries, up to 2 penalised ones, then a
      // depth-5 warp tree) add at most 9 * 2^-24 (1 + 2^-20) < 2^-20.
      const float c = (float)(1.4426950408889634 * a.Tinv);
      const float l2e = 1.44269504f;
      const float m2 = M * l2e;
      const double tabs = fabs((double)M) + 91.0;
      const double eps = (tabs + fabs((double)M) + 1.0) * 0x1p-21 + 0x1p-19 + 0x1p-20;
      id = draw_reg<NV4>(
          sm, bits, plist, [&](int i) { return pick_layer(r, i); }, V, np, u, eps, 0x1p-125,
          [&](float x) { return ex2_approx(fmaf(x, c, -m2)); },
          [&](int s) { return ex2_approx(fmaf(pval[s], l2e, -m2)); });
      if (id < 0) id = tier2_a<NV4>(a, bits, L, sm, plist, pval, np, u, maxv);
    }
    if (id < 0) {
      // tier 3 (also every row with a NaN logit)
      if (warp == 0) {
        const int s = sequential_a(a, bits, L, maxv, u);
        if (lane == 0) a.out[b] = s;
      }
    } else if (threadIdx.x == 0) {
      a.out[b] = id;
    }
    __syncthreads();
  }
}

// Variant B over the register row: the maximum of the lower bounds (one
// fmaxf per entry), the spread estimated from chunk layer 0, a histogram of
// the distance below the maximum, and a gather by one threshold.
template <int NV4>
__global__ void __launch_bounds__(kSampThreads, NV4 <= 8 ? 2 : 1) sample_b_reg(const __grid_constant__ SampArgs a) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  RowPipe &pp = *reinterpret_cast<RowPipe *>(smem_dyn + sizeof(SmemB));
  const int V = a.V;
  const int words = (V + 31) >> 5;
  uint32_t *bm = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB) + sizeof(RowPipe));
  const int lane = threadIdx.x & 31;
  const int k = min(a.top_k, V);
  const double rep = a.rep;
  RowFeeder feed;
  feed.stage = stage_ptr(smem_dyn, sizeof(SmemB) + sizeof(RowPipe) + (size_t)8 * words, V);
  feed.bar = &pp.bar;
  int hreg[kHistRegs];
  // distinct history ids this thread owns in the next row, 16 bits each
  // (0xFFFF: none; register rows hold at most 32768 ids)
  static_assert(kHistRegs == 2, "two owned ids per thread");
  int own_tmp[kHistRegs];
  pipe_start(a, pp, bm, words, feed, hreg, nullptr, 0, -1, 0, own_tmp);
  unsigned own_next = (own_tmp[0] & 0xFFFFu) | ((unsigned)own_tmp[1] << 16);
  float *po = reinterpret_cast<float *>(sm.plist);  // stored logit of an owned id, [q][thread]

  int it = 0;
  for (int b = blockIdx.x; b < a.rows; b += gridDim.x, ++it) {
    const int par = it & 1;
    const uint32_t *bits = bm + (it % 3) * words;
    const unsigned own = own_next;
    if (threadIdx.x == 0) pipe_reset(pp, par ^ 1);
    const bool ok = feed.wait(a.err);
    // penalised entries -> fp32 lower bound of L - rep, in the stage (each
    // by its owner, which keeps the stored value)
#pragma unroll
    for (int q = 0; q < kHistRegs; ++q) {
      const unsigned v = (own >> (16 * q)) & 0xFFFFu;
      if (v != 0xFFFFu) {
        const float x = feed.stage[v];
        po[q * kSampThreads + threadIdx.x] = x;
        feed.stage[v] = __double2float_rd(__dsub_rn((double)x, rep));
      }
    }
    __syncthreads();

    // ---- registers; maximum; spread of chunk layer 0 ----
    float4 r[NV4];
    float mx = -INFINITY, s1 = 0.f, s2 = 0.f;
    const uint32_t st_u32 = smem_u32(feed.stage);
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      r[i] = v0 < V ? lds4(st_u32 + 4u * v0) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (i == 0 && v0 < V) {
        const float4 x = r[0];
        s1 = (x.x + x.y) + (x.z + x.w);
        s2 = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, x.w * x.w)));
      }
      mx = fmaxf(mx, fmax4(r[i]));
    }
    const float my_mx = mx;
    mx = warp_max(mx);
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      atomicMax(&pp.xkey[par], okey32(mx));
      atomicAdd(&pp.s1[par], s1);
      atomicAdd(&pp.s2[par], s2);
    }
    for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
    if (threadIdx.x == 0) sm.ncand = 0;
    if (!__syncthreads_and(ok)) break;
    pipe_advance(a, pp, bm, words, it, b, feed, hreg, nullptr, 0, 0, own_tmp);
    if (b + (int)gridDim.x < a.rows) own_next = (own_tmp[0] & 0xFFFFu) | ((unsigned)own_tmp[1] << 16);

    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;
    mx = key_to_float(pp.xkey[par]);
    s1 = pp.s1[par];
    s2 = pp.s2[par];
    const int n0 = min(V, kSegLen);
    bool fast = isfinite(mx) && isfinite(s1) && isfinite(s2) && V >= k;
    float R = 0.f;
    if (fast) {
      const float mean = s1 / n0;
      const float sd = sqrtf(fmaxf(s2 / n0 - mean * mean, 0.f));
      R = 2.5f * sd;
      fast = R > 0.f && isfinite(R);
    }
    int bstar = 255;
    // ---- histogram of the distance below the maximum, 255 bins over [0, R);
    // every warp finds the first bin whose running count reaches k
    for (int attempt = 0; fast && attempt < 3 && bstar >= 255; ++attempt) {
      if (attempt > 0) {
        __syncthreads();
        for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
        __syncthreads();
      }
      const float inv_w = 255.f / R;
#pragma unroll
      for (int i = 0; i < NV4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float d = mx - f4_at(r[i], j);
          if (d < R) atomicAdd(&sm.hist[min((int)(d * inv_w), 254)], 1u);
        }
      }
      __syncthreads();
      const uint4 h0 = *reinterpret_cast<const uint4 *>(&sm.hist[lane * 8]);
      const uint4 h1 = *reinterpret_cast<const uint4 *>(&sm.hist[lane * 8 + 4]);
      const unsigned int run = (h0.x + h0.y) + (h0.z + h0.w) + ((h1.x + h1.y) + (h1.z + h1.w));
      unsigned int incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      // the first of this lane's bins whose running count reaches k
      int bs = 255;
      if (incl >= (unsigned)k) {
        unsigned int acc = incl - run;
        const unsigned int hb[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        bs = lane * 8 + 7;
#pragma unroll
        for (int q = 0; q < 7; ++q) {
          acc += hb[q];
          if (acc >= (unsigned)k) {
            bs = lane * 8 + q;
            break;
          }
        }
      }
      bstar = __reduce_min_sync(0xffffffffu, bs);
      if (bstar >= 255) R *= 8.f;
    }
    fast = fast && bstar < 255;
    if (fast) {
      // ---- gather.  An entry lands in a bin <= bstar only if its lower
      // bound exceeds mx - (bstar+1) (R/255) (1 + 2^-21), so at least k
      // lower bounds reach g; every entry whose exact value reaches the
      // least of them has a lower bound (its value rounded down) at least
      // that large, so `g` admits a superset of the top k.  Unpenalised
      // entries come from the registers, penalised ones (exact value
      // L - rep) from their owners.
      const double gd = (double)mx - (double)(bstar + 1) * ((double)R / 255.0) * (1.0 + 0x1p-20);
      float g = __double2float_rd(gd);
      g = (g == -INFINITY) ? g : __uint_as_float(g > 0.f ? __float_as_uint(g) - 1u
                                                          : (g == 0.f ? 0x80000001u : __float_as_uint(g) + 1u));
#pragma unroll
      for (int q = 0; q < kHistRegs; ++q) {
        const unsigned v = (own >> (16 * q)) & 0xFFFFu;
        if (v != 0xFFFFu) {
          const double val = __dsub_rn((double)po[q * kSampThreads + threadIdx.x], rep);
          if (__double2float_rd(val) >= g) {
            const int slot = atomicAdd(&sm.ncand, 1);
            if (slot < kFastCand) {
              sm.ckey[slot] = okey64(val);
              sm.cidx[slot] = (int)v;
            }
          }
        }
      }
      if (my_mx >= g) {
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
          if (fmax4(r[i]) >= g) {
            const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float f = f4_at(r[i], j);
              if (f >= g && !in_set(bits, v0 + j)) {
                const int slot = atomicAdd(&sm.ncand, 1);
                if (slot < kFastCand) {
                  sm.ckey[slot] = okey64((double)f);
                  sm.cidx[slot] = v0 + j;
                }
              }
            }
          }
        }
      }
      __syncthreads();
      const int nc = sm.ncand;
      fast = nc <= kFastCand && nc >= k;
      if (fast) rank_candidates(sm, nc, k, a.T);
    }
    if (!fast) {
      __syncthreads();
      if (!general_select_b(a, bits, L, sm, k)) {
        if (threadIdx.x == 0) {
          a.out[b] = -2;
          record_error(a.err, kErrSamplerArgs);
        }
        __syncthreads();
        continue;
      }
    }
    // ---- src/tensor_ffi_adapter.php:180-204 over the k survivors, by warp
    // 0 (the other warps wait at the barrier: letting them run ahead into
    // the next row measured slower)
    topp_tail(a, sm, k, b);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Streaming variant B: one warp per row, no block barriers.
//
// A warp streams its rows' logits through a ring of shared-memory chunks
// filled by cp.async (kStreamSlots in flight, running on into the warp's
// next row) and keeps
// a buffer of candidates whose lower bound lb (the logit, or fp32 round-down
// of L - rep for a penalised id) reaches a threshold t.  t starts at -inf;
// when the buffer fills, a radix select over the buffer's lb keys finds its
// k-th largest lb, which becomes t, and the buffer keeps the entries at or
// above it.  t never exceeds the row's k-th largest lb, and every entry of
// the top k by exact value (L or L - rep, in double) has lb >= t, so the
// buffer always holds the top k.  At the row's end a last select cuts the
// buffer to the entries at or above the k-th largest lb, those are ranked
// by (exact value descending, id ascending) and the warp runs the top-p tail.
// Rows whose candidates cannot be cut (more ties than the buffer holds, or
// fewer than k comparable entries, e.g. NaN) take an exact warp-level radix
// select over 64-bit keys of the exact values, streaming the row again.
//
// At a row's start the warp marks the row's history ids in its bitmap,
// reading them straight from global memory (eight loads in flight per lane).
// ---------------------------------------------------------------------------

constexpr int kStreamCapMax = 1024;   // candidate buffer entries per warp at most (top-k 256)
constexpr int kStreamSlots = 2;       // staged chunks in flight per warp
constexpr int kStreamPer = 8;         // 16-byte words per lane per chunk (variant A: 32 ids, one bitmap word)
constexpr int kStreamChunk = 32 * kStreamPer;  // 16-byte words per chunk
constexpr int kStreamBPer = 8;        // variant B: 16-byte words per lane per chunk (4 and 6 measured slower at V=16384)
constexpr int kStreamBChunk = 32 * kStreamBPer;
static_assert(kStreamBPer * 4 <= 64, "one mask bit per staged entry of a lane");
constexpr int kStreamMaxK = 256;      // top-k the buffer supports
constexpr int kStreamWarps = 20;      // warps per CTA at most

// Per-warp shared-memory carve (the same on host and device); every region
// starts on a 16-byte boundary (cp.async destinations, uint4 reads).
struct StreamLayout {
  int words, cap;  // cap: candidate buffer entries (room for 2k + 128, at least 256)
  unsigned off_val, off_bm, off_id, off_rh, off_p, off_ord, bytes;  // ring at 0
};
__host__ __device__ inline StreamLayout stream_layout(int V, int k) {
  auto up16 = [](unsigned x) { return (x + 15u) & ~15u; };
  StreamLayout L;
  L.words = (V + 31) / 32;
  L.cap = (2 * k + 128 + 31) / 32 * 32;
  if (L.cap < 256) L.cap = 256;
  if (L.cap > kStreamCapMax) L.cap = kStreamCapMax;
  unsigned o = up16(kStreamSlots * kStreamBChunk * 16);  // staged chunks
  L.off_val = o;
  o = up16(o + (unsigned)L.cap * 8u);  // double values (then 64-bit keys, then running sums)
  L.off_bm = o;
  o = up16(o + (unsigned)L.words * 4u);
  L.off_id = o;
  o = up16(o + (unsigned)L.cap * 4u);
  L.off_rh = o;
  o = up16(o + 256 * 4);
  L.off_p = o;
  o = up16(o + (unsigned)k * 8u);
  L.off_ord = o;
  o = up16(o + (unsigned)k * 4u);
  L.bytes = o;
  return L;
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Largest digit d with (count of keys whose digit is >= d) >= need, from a
// 256-bin histogram; `above` = count of digits > d.  -1 if all bins hold
// fewer than `need`.  Every lane returns the same values.
__device__ __forceinline__ int warp_top_digit(const unsigned *rh, unsigned need, unsigned &above) {
  const int lane = threadIdx.x & 31;
  const uint4 h0 = reinterpret_cast<const uint4 *>(rh)[lane * 2];
  const uint4 h1 = reinterpret_cast<const uint4 *>(rh)[lane * 2 + 1];
  const unsigned b[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const unsigned sum = ((b[0] + b[1]) + (b[2] + b[3])) + ((b[4] + b[5]) + (b[6] + b[7]));
  unsigned incl = sum;  // this lane's bins and every higher lane's
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned n = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += n;
  }
  int d = -1;
  unsigned ab = 0u;
  if (incl >= need && incl - sum < need) {
    unsigned acc = incl - sum;
#pragma unroll
    for (int q = 7; q >= 0; --q) {
      if (d < 0 && acc + b[q] >= need) {
        d = lane * 8 + q;
        ab = acc;
      }
      acc += b[q];
    }
  }
  d = __reduce_max_sync(0xffffffffu, d);
  above = d >= 0 ? __shfl_sync(0xffffffffu, ab, d >> 3) : 0u;
  return d;
}

__device__ __forceinline__ unsigned lb_key(double val) { return okey32(__double2float_rd(val)); }

// Cuts the buffer to the entries whose lb key has the top 16 bits of the
// k-th largest or more (two 8-bit radix rounds); returns the new count
// (>= k) and sets t to the lowest float of that 16-bit bucket.  Needs
// cnt >= k.
__device__ __noinline__ int stream_compact(double *bval, int *bid, unsigned *rh, int cnt, int k, float &t) {
  const int lane = threadIdx.x & 31;
  unsigned prefix = 0u, need = (unsigned)k;
  for (int shift = 24; shift >= 16; shift -= 8) {
    for (int i = lane; i < 256; i += 32) rh[i] = 0u;
    __syncwarp();
    const unsigned hm = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int i = lane; i < cnt; i += 32) {
      const unsigned key = lb_key(bval[i]);
      if ((key & hm) == (prefix & hm)) atomicAdd(&rh[(key >> shift) & 255u], 1u);
    }
    __syncwarp();
    unsigned above;
    const int d = warp_top_digit(rh, need, above);
    __syncwarp();
    need -= above;
    prefix |= (unsigned)d << shift;
  }
  int w = 0;
  for (int i0 = 0; i0 < cnt; i0 += 32) {
    const int i = i0 + lane;
    double v = 0.0;
    int id = 0;
    bool keep = false;
    if (i < cnt) {
      v = bval[i];
      id = bid[i];
      keep = lb_key(v) >= prefix;
    }
    __syncwarp();
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    if (keep) {
      const int slot = w + __popc(m & ((1u << lane) - 1u));
      bval[slot] = v;
      bid[slot] = id;
    }
    w += __popc(m);
    __syncwarp();
  }
  t = key_to_float(prefix);
  if (t != t) t = -INFINITY;  // the bucket of -inf starts at NaN patterns
  return w;
}

// Raw-logit threshold admitting every entry with lb >= t.
__device__ __forceinline__ float stream_traw(float t, double rep) {
  if (rep >= 0.0 || t == -INFINITY) return t;
  const double x = (double)t + rep - 0x1p-50 * (fabs((double)t) + fabs(rep));
  const float f = __double2float_rd(x);
  return f == -INFINITY ? f : __uint_as_float(f > 0.f ? __float_as_uint(f) - 1u
                                                      : (f == 0.f ? 0x80000001u : __float_as_uint(f) + 1u));
}

struct StreamState {
  int cnt;
  int ovf;
  float t, traw;
};

// Marks the history ids of logits row `mrow` (the first hist_len[mrow], or
// all hist_cols) in the warp's bitmap, loading them from global memory.
__device__ __forceinline__ void mark_history(const SampArgs &a, int mrow, uint32_t *bm) {
  const int lane = threadIdx.x & 31;
  if (a.hist == nullptr || a.hist_cols <= 0 || mrow < 0) return;
  const int *hr = a.hist + (size_t)mrow * a.hist_ld;
  const int n = min(max(a.hist_len ? a.hist_len[mrow] : a.hist_cols, 0), a.hist_cols);
  for (int c0 = 0; c0 < n; c0 += 32 * 8) {
    int t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + 32 * j + lane;
      t[j] = c < n ? __ldg(hr + c) : -1;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (t[j] >= 0 && t[j] < a.V) atomicOr(&bm[t[j] >> 5], 1u << (t[j] & 31));
  }
  __syncwarp();
}

// Entries of this lane's chunk words marked in `bits` (bit 4r + j: word r,
// element j; a superset of those with raw logit >= traw) whose lb reaches t
// join the buffer.  Slots come from one warp scan; a batch that does not fit
// is taken word by word, the buffer cut whenever the next word could
// overflow it.  rf: the staged chunk, c0: its first word.
__device__ __forceinline__ unsigned long long stream_filter(const float *rf, unsigned long long bits, int c0,
                                                            const uint32_t *bm, double rep, float t) {
  const int lane = threadIdx.x & 31;
  unsigned long long keep = 0ull;
  while (bits) {
    const int b = __ffsll((long long)bits) - 1;
    bits &= bits - 1ull;
    const int r = b >> 2, j = b & 3;
    const float f = rf[(32 * r + lane) * 4 + j];
    const int v = (c0 + 32 * r + lane) * 4 + j;
    // an unpenalised entry's lower bound is its float (fp32 -> double -> fp32
    // rounds back to it): only penalised ids need the double subtraction
    const bool ok = in_set(bm, v) ? __double2float_rd(__dsub_rn((double)f, rep)) >= t : f >= t;
    if (ok) keep |= 1ull << b;
  }
  return keep;
}
__device__ __forceinline__ void stream_write(const float *rf, unsigned long long keep, int c0, int slot,
                                             const uint32_t *bm, double rep, double *bval, int *bid) {
  const int lane = threadIdx.x & 31;
  while (keep) {
    const int b = __ffsll((long long)keep) - 1;
    keep &= keep - 1ull;
    const int r = b >> 2, j = b & 3;
    const float f = rf[(32 * r + lane) * 4 + j];
    const int v = (c0 + 32 * r + lane) * 4 + j;
    bval[slot] = in_set(bm, v) ? __dsub_rn((double)f, rep) : (double)f;
    bid[slot] = v;
    ++slot;
  }
}
__device__ __forceinline__ int warp_excl_scan(int c, int &tot) {
  const int lane = threadIdx.x & 31;
  int incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  tot = __shfl_sync(0xffffffffu, incl, 31);
  return incl - c;
}
__device__ __forceinline__ void stream_take(const float *rf, unsigned long long bits, int c0, StreamState &st,
                                            double *bval, int *bid, const uint32_t *bm, unsigned *rh, int k,
                                            double rep, int cut_at, int cap) {
  if (st.ovf) return;
  unsigned long long keep = stream_filter(rf, bits, c0, bm, rep, st.t);
  int tot;
  int ex = warp_excl_scan(__popcll(keep), tot);
  if (st.cnt + tot <= cap) {
    stream_write(rf, keep, c0, st.cnt + ex, bm, rep, bval, bid);
    st.cnt += tot;
  } else {
#pragma unroll 1
    for (int r = 0; r < kStreamBPer; ++r) {
      unsigned long long kr = keep & (0xFull << (4 * r));
      if (st.cnt > cap - 128) {
        st.cnt = stream_compact(bval, bid, rh, st.cnt, k, st.t);
        st.traw = stream_traw(st.t, rep);
        if (st.cnt > cap - 128) {
          st.ovf = 1;
          return;
        }
        kr = stream_filter(rf, kr, c0, bm, rep, st.t);
      }
      ex = warp_excl_scan(__popcll(kr), tot);
      stream_write(rf, kr, c0, st.cnt + ex, bm, rep, bval, bid);
      st.cnt += tot;
    }
  }
  if (st.cnt > cut_at) {
    st.cnt = stream_compact(bval, bid, rh, st.cnt, k, st.t);
    st.traw = stream_traw(st.t, rep);
    if (st.cnt > cap - 128) st.ovf = 1;
  }
}

// A row whose buffer came up short: two radix rounds over the row's lb keys
// find the 16-bit bucket of the k-th largest, and the entries at or above
// it are gathered (exact values) into the buffer.  Returns their count, or
// 0 if they do not fit (or the row has fewer than k comparable entries).
__device__ __noinline__ int stream_regather(const float *Lrow, int V, const uint32_t *bm, double *bval, int *bid,
                                            unsigned *rh, int k, double rep, int cap) {
  const int lane = threadIdx.x & 31;
  const int n4 = V >> 2;
  const float4 *L4 = reinterpret_cast<const float4 *>(Lrow);
  auto val_of = [&](float f, int v) { return in_set(bm, v) ? __dsub_rn((double)f, rep) : (double)f; };
  unsigned prefix = 0u, need = (unsigned)k;
  for (int shift = 24; shift >= 16; shift -= 8) {
    for (int i = lane; i < 256; i += 32) rh[i] = 0u;
    __syncwarp();
    const unsigned hm = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int idx = lane; idx < n4; idx += 32) {
      const float4 x = __ldg(L4 + idx);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f = f4_at(x, j);
        if (f == f) {
          const unsigned key = lb_key(val_of(f, idx * 4 + j));
          if ((key & hm) == (prefix & hm)) atomicAdd(&rh[(key >> shift) & 255u], 1u);
        }
      }
    }
    __syncwarp();
    unsigned above;
    const int d = warp_top_digit(rh, need, above);
    __syncwarp();
    if (d < 0) return 0;
    need -= above;
    prefix |= (unsigned)d << shift;
  }
  int cnt = 0;
  for (int idx0 = 0; idx0 < n4; idx0 += 32) {
    const int idx = idx0 + lane;
    float4 x = make_float4(NAN, NAN, NAN, NAN);
    if (idx < n4) x = __ldg(L4 + idx);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = f4_at(x, j);
      const double val = val_of(f, idx * 4 + j);
      const bool take = f == f && lb_key(val) >= prefix;
      const unsigned m = __ballot_sync(0xffffffffu, take);
      const int slot = cnt + __popc(m & ((1u << lane) - 1u));
      if (take && slot < cap) {
        bval[slot] = val;
        bid[slot] = idx * 4 + j;
      }
      cnt += __popc(m);
    }
  }
  __syncwarp();
  return cnt <= cap ? cnt : 0;
}

// Exact top-k of a row by a radix select over 64-bit keys of the exact
// values (the row streamed once per digit), then the entries above the k-th
// key and, of those equal to it, the first in id order, gathered in id
// order: exactly k entries.  Returns k, or 0 if the row has fewer entries.
__device__ __noinline__ int stream_exact(const float *Lrow, int V, const uint32_t *bm, double *bval, int *bid,
                                         unsigned *rh, int k, double rep) {
  const int lane = threadIdx.x & 31;
  const int n4 = V >> 2;
  const float4 *L4 = reinterpret_cast<const float4 *>(Lrow);
  auto key_of = [&](float f, int v) { return okey64(in_set(bm, v) ? __dsub_rn((double)f, rep) : (double)f); };
  unsigned long long prefix = 0ull;
  unsigned need = (unsigned)k;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = lane; i < 256; i += 32) rh[i] = 0u;
    __syncwarp();
    const unsigned long long hm = shift == 56 ? 0ull : (~0ull << (shift + 8));
    for (int idx = lane; idx < n4; idx += 32) {
      const float4 x = __ldg(L4 + idx);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned long long key = key_of(f4_at(x, j), idx * 4 + j);
        if ((key & hm) == (prefix & hm)) atomicAdd(&rh[(unsigned)(key >> shift) & 255u], 1u);
      }
    }
    __syncwarp();
    unsigned above;
    const int d = warp_top_digit(rh, need, above);
    __syncwarp();
    if (d < 0) return 0;
    need -= above;
    prefix |= (unsigned long long)d << shift;
  }
  // `need` entries equal to the k-th key are taken, in id order
  int cnt = 0;
  unsigned eq_left = need;
  for (int idx0 = 0; idx0 < n4; idx0 += 32) {
    const int idx = idx0 + lane;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (idx < n4) x = __ldg(L4 + idx);
    unsigned long long key[4];
    int gt = 0, eq = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      key[j] = idx < n4 ? key_of(f4_at(x, j), idx * 4 + j) : 0ull;
      const bool valid = idx < n4;
      gt += valid && key[j] > prefix;
      eq += valid && key[j] == prefix;
    }
    int eq_ex = eq, take_ex;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, eq_ex, o);
      if (lane >= o) eq_ex += n;
    }
    const int eq_tot = __shfl_sync(0xffffffffu, eq_ex, 31);
    eq_ex -= eq;  // equal entries before this lane's
    int take = gt;
    {
      int e = eq_ex;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (idx < n4 && key[j] == prefix) {
          take += (unsigned)e < eq_left;
          ++e;
        }
    }
    take_ex = take;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, take_ex, o);
      if (lane >= o) take_ex += n;
    }
    const int take_tot = __shfl_sync(0xffffffffu, take_ex, 31);
    int slot = cnt + take_ex - take;
    int e = eq_ex;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (idx < n4) {
        const int v = idx * 4 + j;
        bool t = key[j] > prefix;
        if (key[j] == prefix) {
          t = (unsigned)e < eq_left;
          ++e;
        }
        if (t) {
          bval[slot] = key_to_double(key[j]);
          bid[slot] = v;
          ++slot;
        }
      }
    }
    cnt += take_tot;
    eq_left -= (unsigned)min(eq_tot, (int)eq_left);
    __syncwarp();
  }
  return cnt;
}

// Row end: cut, rank, top-p tail; writes out[b].
__device__ __noinline__ void stream_finish(const SampArgs &a, int b, StreamState st, double *bval, int *bid,
                                           const uint32_t *bm, unsigned *rh, double *P, int *ord, int k, int cap) {
  const int lane = threadIdx.x & 31;
  int M = 0;
  if (!st.ovf && st.cnt >= k) {
    float t = st.t;
    M = stream_compact(bval, bid, rh, st.cnt, k, t);
  } else {
    const float *Lrow = a.logits + (size_t)row_of(a, b) * a.ld;
    M = st.ovf ? 0 : stream_regather(Lrow, a.V, bm, bval, bid, rh, k, a.rep, cap);
    if (M < k) M = stream_exact(Lrow, a.V, bm, bval, bid, rh, k, a.rep);
    if (M < k) {
      if (lane == 0) {
        a.out[b] = -2;
        record_error(a.err, kErrSamplerArgs);
      }
      return;
    }
  }
  // exact order keys in place, then ranks (value descending, id ascending)
  unsigned long long *bkey = reinterpret_cast<unsigned long long *>(bval);
  for (int i = lane; i < M; i += 32) bkey[i] = okey64(bval[i]);
  __syncwarp();
  const bool want_p = !(a.T < 0.01);
  for (int i = lane; i < M; i += 32) {
    const unsigned long long ki = bkey[i];
    const int vi = bid[i];
    int rank = 0;
#pragma unroll 4
    for (int j = 0; j < M; ++j) {
      const unsigned long long kj = bkey[j];
      const int vj = bid[j];
      rank += (int)((kj > ki) | ((kj == ki) & (vj < vi)));
    }
    if (rank < k) {
      ord[rank] = vi;
      const double val = key_to_double(ki);
      P[rank] = want_p ? snai_exp(__ddiv_rn(val, a.T)) : val;
    }
  }
  __syncwarp();
  int id;
  if (!want_p) {
    id = ord[0];
  } else {
    const double u = (double)a.uniforms[b];
    id = warp_topp(ord, P, bval, k, u, a.top_p);
  }
  if (lane == 0) a.out[b] = id;
  __syncwarp();
}

__global__ void __launch_bounds__(kStreamWarps * 32, 1) sample_b_stream(const __grid_constant__ SampArgs a, int W) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int V = a.V, n4 = V >> 2, S = (n4 + kStreamBChunk - 1) / kStreamBChunk;
  const int k = a.T < 0.01 ? 1 : min(a.top_k, V);
  const StreamLayout Ly = stream_layout(V, k);
  const int cap = Ly.cap;
  uint8_t *base = smem_dyn + (size_t)warp * Ly.bytes;
  float4 *ring = reinterpret_cast<float4 *>(base);
  double *bval = reinterpret_cast<double *>(base + Ly.off_val);
  uint32_t *bm = reinterpret_cast<uint32_t *>(base + Ly.off_bm);
  int *bid = reinterpret_cast<int *>(base + Ly.off_id);
  unsigned *rh = reinterpret_cast<unsigned *>(base + Ly.off_rh);
  double *P = reinterpret_cast<double *>(base + Ly.off_p);
  int *ord = reinterpret_cast<int *>(base + Ly.off_ord);
  // warp-major numbering: row r goes to CTA r % grid, so every SM gets an
  // equal share of the rows (to within one); the warps of an SM share its
  // issue slots, so the SM with the most rows sets the kernel's time
  const int NW = gridDim.x * W, gw = warp * gridDim.x + blockIdx.x;
  if (warp >= W || gw >= a.rows) return;
  const int nrows = (a.rows - 1 - gw) / NW + 1;
  // logits / history row of the warp's i-th row (-1 past the last)
  auto mrow_of = [&](int i) -> int { return i < nrows ? row_of(a, gw + i * NW) : -1; };
  for (int w = lane; w < Ly.words; w += 32) bm[w] = 0u;
  __syncwarp();
  int mp = mrow_of(0), mq = mrow_of(1);
  // the first row's history is marked before any chunk is staged
  mark_history(a, mp, bm);

  // Chunk q of the warp's stream (row q / S, chunk q % S of it) is staged
  // in slot q % kStreamSlots, each lane copying (cp.async, one group per
  // chunk) and later reading the same two 16-byte words; the copy position
  // (pi, ps) runs kStreamSlots chunks ahead of the consumed one, and mq,
  // the row after pi, is loaded a whole row before it is needed.
  int pi = 0, ps = 0;
  const float4 *Lp = mp >= 0 ? reinterpret_cast<const float4 *>(a.logits + (size_t)mp * a.ld) : nullptr;
  auto issue = [&](int slot) {
    if (Lp != nullptr) {
      const int c0 = ps * kStreamBChunk + lane;
#pragma unroll
      for (int r = 0; r < kStreamBPer; ++r)
        if (c0 + 32 * r < n4) cp_async16(ring + slot * kStreamBChunk + 32 * r + lane, Lp + c0 + 32 * r);
    }
    cp_async_commit();
    if (++ps == S) {
      ps = 0;
      ++pi;
      Lp = mq >= 0 ? reinterpret_cast<const float4 *>(a.logits + (size_t)mq * a.ld) : nullptr;
      mq = mrow_of(pi + 1);
    }
  };
  for (int q = 0; q < kStreamSlots; ++q) issue(q);

  StreamState st{0, 0, -INFINITY, -INFINITY};
  // the buffer is cut once it holds more than cut_at entries (at most
  // cap - 128, so one more chunk word per lane always fits); cutting early in
  // the row raises t sooner and spares later chunks their pushes
  const int cut_at = min(cap - 128, max(2 * k, 128));
  // G groups of gl lanes for the opening threshold: one group (the chunk's
  // maximum, a true bound) for k = 1; else G >= 8 groups and G >= 2.5 x
  // (x = top-k entries expected in one chunk), so that for a row in random
  // order a group maximum exceeds the k-th largest with probability
  // 1 - exp(-x/G) <= 1/3 and all G of them do so in ~1e-4 of the rows (those
  // take the three-pass path).  G >= k makes it a true bound.
  int gl = 32;
  if (k > 1) {
    const float x = (float)k * (float)(kStreamBChunk * 4) / (float)V;
    int G = 8;
    while (G < 32 && G < k && (float)G < 2.5f * x) G <<= 1;
    gl = 32 / G;
  }
  const long long total = (long long)nrows * S;
  int ci = 0, cs = 0;
  for (long long q = 0; q < total; ++q) {
    const int slot = (int)(q % kStreamSlots);
    cp_async_wait<kStreamSlots - 1>();  // this chunk
    if (cs == 0 && ci > 0) mark_history(a, mrow_of(ci), bm);
    const int c0 = cs * kStreamBChunk;
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    float4 x[kStreamBPer];
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < kStreamBPer; ++r) {
      x[r] = c0 + 32 * r + lane < n4 ? ring[slot * kStreamBChunk + 32 * r + lane] : ninf;
      m = fmaxf(m, fmax4(x[r]));
    }
    if (cs == 0) {
      // Opening threshold: the least of G group maxima of the row's first
      // chunk.  At least G entries reach it; when fewer than k entries end
      // up at or above it, the row is redone exactly (rows where it lands
      // above the k-th largest: ~1e-4 for the group count chosen).
      float g = m;
      for (int o = 1; o < gl; o <<= 1) g = fmaxf(g, __shfl_xor_sync(0xffffffffu, g, o));
      for (int o = gl; o < 32; o <<= 1) g = fminf(g, __shfl_xor_sync(0xffffffffu, g, o));
      if (!(g == g)) g = -INFINITY;
      // a penalised group maximum has lb >= raw - rep
      if (a.rep > 0.0 && g != -INFINITY) {
        const float f = __double2float_rd((double)g - a.rep);
        g = f == -INFINITY ? f : __uint_as_float(f > 0.f ? __float_as_uint(f) - 1u
                                                         : (f == 0.f ? 0x80000001u : __float_as_uint(f) + 1u));
      }
      st.t = g;
      st.traw = stream_traw(g, a.rep);
    }
    if (__any_sync(0xffffffffu, m >= st.traw)) {
      unsigned long long bits = 0ull;
#pragma unroll
      for (int r = 0; r < kStreamBPer; ++r) {
        const bool valid = c0 + 32 * r + lane < n4;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (valid && f4_at(x[r], j) >= st.traw) bits |= 1ull << (4 * r + j);
      }
      stream_take(reinterpret_cast<const float *>(ring + slot * kStreamBChunk), bits, c0, st, bval, bid, bm, rh, k,
                  a.rep, cut_at, cap);
    }
    issue(slot);  // the slot's next chunk (this lane's words were read above)
    if (++cs == S) {
      stream_finish(a, gw + ci * NW, st, bval, bid, bm, rh, P, ord, k, cap);
      for (int w = lane; w < Ly.words; w += 32) bm[w] = 0u;
      __syncwarp();
      st = StreamState{0, 0, -INFINITY, -INFINITY};
      cs = 0;
      ++ci;
    }
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Streaming variant A: one warp per row, no block barriers.  (Greedy, T <=
// 0.01: the chunks keep their maximum only, and the row's end looks for the
// first id attaining M in the chunks that can hold one.)
//
// The warp streams the row through the same cp.async ring as the variant-B
// kernel.  Lane l reads the chunk's 16-byte words 8l .. 8l + 7 (in a rotated
// order, so the shared-memory reads do not conflict): its 32 entries are
// contiguous ids, covered by one 32-bit word of the history bitmap.  Per
// 1024-entry chunk the warp takes the maximum mu of y = x c (x the raw
// logit, c = fp32(log2e / T); penalised ids excluded) and the fp32 sum s of
// 2^(y - mu), the penalised ids contributing 2^(t log2e - mu) with their
// exact stored value t; (mu, s) go to a per-warp table.  At the row's end
// the exact maximum M (the tempered maximum raw logit, or a penalised t)
// fixes m2 = fp32(M log2e); the chunk totals s 2^(mu - m2) give S and the
// chunk where u S is crossed; that chunk is read again, each lane sums the
// p~ = 2^(x c - m2) (penalised: 2^(t log2e - m2)) of its 32 ids, a warp
// scan finds the lane where the running sum crosses u S and that lane walks
// its ids.  The draw is accepted when r is farther from the running sums at
// the chosen id and its predecessor than the error bound of the register-row
// kernel's tier 1 (widened for the two-step exponent and the fp32 chunk
// sums); otherwise the contract exponential redoes the same search exactly
// (tier 2), and rows it cannot settle (or NaN rows) run PHP's sequential
// loop (tier 3).
// ---------------------------------------------------------------------------

constexpr int kStreamAWarps = 16;  // warps per CTA at most (128 registers a thread)

struct StreamALayout {
  int words, nch;
  unsigned off_bm, off_ch, off_pv, bytes;  // ring at 0
};
__host__ __device__ inline StreamALayout stream_a_layout(int V) {
  auto up16 = [](unsigned x) { return (x + 15u) & ~15u; };
  StreamALayout L;
  L.words = (V + 31) / 32;
  L.nch = ((V >> 2) + kStreamChunk - 1) / kStreamChunk;
  unsigned o = up16(kStreamSlots * kStreamChunk * 16);
  L.off_bm = o;
  o = up16(o + (unsigned)L.words * 4u);
  L.off_ch = o;  // per chunk: (mu, s, s of the penalised ids, -) floats
  o = up16(o + (unsigned)L.nch * 16u);
  L.off_pv = o;  // the crossing chunk: 32 values of each lane, [e][lane]
  o = up16(o + 32u * 32u * 4u);
  L.bytes = o;
  return L;
}

// Prefix of the chunk totals tot(c) in chunk order: S, and the first chunk
// whose inclusive prefix reaches rr = u S with the prefix before it.
template <class TOT>
__device__ __forceinline__ int chunk_prefix(int nch, double u, const TOT &tot, double &S, double &rr, double &before) {
  const int lane = threadIdx.x & 31;
  S = 0.0;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const double t = c0 + lane < nch ? tot(c0 + lane) : 0.0;
    S = __dadd_rn(S, warp_sum_d(t));
  }
  rr = __dmul_rn(u, S);
  double carry = 0.0;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const double t = c0 + lane < nch ? tot(c0 + lane) : 0.0;
    double incl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = __dadd_rn(incl, n);
    }
    double ex = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) ex = 0.0;
    const unsigned m = __ballot_sync(0xffffffffu, c0 + lane < nch && __dadd_rn(carry, incl) >= rr);
    if (m) {
      const int src = __ffs(m) - 1;
      before = __dadd_rn(carry, __shfl_sync(0xffffffffu, ex, src));
      return c0 + src;
    }
    carry = __dadd_rn(carry, __shfl_sync(0xffffffffu, incl, 31));
  }
  before = carry;
  return nch - 1;
}

// Running sums over chunk cs in id order, from `base`: lane l owns ids
// 32l .. 32l + 31 of the chunk, pf(e) gives p of its e-th one.  Returns the
// first id whose running sum reaches rr (INT_MAX if none) with the running
// sums before (lo) and after (hi) it.
template <class PF>
__device__ __forceinline__ int chunk_crossing(const PF &pf, int cs, int V, double base, double rr, double &lo,
                                              double &hi) {
  const int lane = threadIdx.x & 31;
  double w = 0.0;
#pragma unroll 4
  for (int e = 0; e < 32; ++e) w = __dadd_rn(w, pf(e));
  double incl = w;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl = __dadd_rn(incl, n);
  }
  double ex = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) ex = 0.0;
  const unsigned m = __ballot_sync(0xffffffffu, __dadd_rn(base, incl) >= rr);
  if (!m) return INT_MAX;
  const int src = __ffs(m) - 1;
  int cand = INT_MAX;
  double mlo = 0.0, mhi = 0.0;
  if (lane == src) {
    double run = __dadd_rn(base, ex);
    const int v0 = cs * kStreamChunk * 4 + 32 * lane;
    for (int e = 0; e < 32 && v0 + e < V; ++e) {
      const double cur = __dadd_rn(run, pf(e));
      if (cur >= rr) {
        cand = v0 + e;
        mlo = run;
        mhi = cur;
        break;
      }
      run = cur;
    }
  }
  cand = __shfl_sync(0xffffffffu, cand, src);
  lo = __shfl_sync(0xffffffffu, mlo, src);
  hi = __shfl_sync(0xffffffffu, mhi, src);
  return cand;
}

// Certificate of the crossing id `cand` (running sums lo, hi around it)
// against r, for sums whose entries are within er*p + eabs of the contract
// values, plus at most `eadd` over all entries together, and whose depth is
// at most `slack` beyond PHP's sequential one.
__device__ __forceinline__ bool certify_cross(int cand, double lo, double hi, double S, double rr, double u, int V,
                                              double er, double eabs, double eadd, double slack) {
  const double Er = u * (er * S + eadd + (double)V * eabs + ((double)V + slack) * 0x1p-52 * S) + 0x1p-52 * rr;
  const double Ehi = er * hi + eadd + ((double)cand + 1.0) * eabs + ((double)cand + slack) * 0x1p-52 * hi;
  const double Elo = er * lo + eadd + (double)cand * eabs + ((double)cand + slack) * 0x1p-52 * lo;
  return hi - Ehi >= rr + Er && (cand == 0 || lo + Elo < rr - Er);
}

// This lane's 32 raw logits of chunk cs (-inf past the row), loaded at once.
__device__ __forceinline__ void lane_block(const float *Lrow, int cs, int V, float4 (&xw)[8]) {
  const int lane = threadIdx.x & 31;
  const int n4 = V >> 2;
  const float4 *L4 = reinterpret_cast<const float4 *>(Lrow);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int wd = cs * kStreamChunk + 8 * lane + k;
    xw[k] = wd < n4 ? __ldg(L4 + wd) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
}

// Row end of the variant-A stream: M, tier 1 (then 2, then 3); writes out[b].
__device__ __noinline__ void stream_a_finish(const SampArgs &a, int b, float xmax, float pmax, int pidx, float l0,
                                             int ovf, float4 *tab, const uint32_t *bm, float *pv, int nch, float cexp) {
  const int lane = threadIdx.x & 31;
  const int V = a.V;
  xmax = warp_max(xmax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {  // the largest penalised value, its first id
    const float ob = __shfl_xor_sync(0xffffffffu, pmax, o);
    const int oi = __shfl_xor_sync(0xffffffffu, pidx, o);
    if (ob > pmax || (ob == pmax && oi < pidx)) {
      pmax = ob;
      pidx = oi;
    }
  }
  l0 = __shfl_sync(0xffffffffu, l0, 0);
  ovf = __any_sync(0xffffffffu, ovf);
  if (a.nan_guard && l0 != l0) {  // src/snai_inference.php:146
    if (lane == 0) a.out[b] = -1;
    return;
  }
  if (a.T <= 0.01) {
    // greedy: the first id attaining M.  An unpenalised entry with
    // fp32(x/T) == M has x >= (M - |M| 2^-22) T; only the chunks whose
    // maximum reaches that bound are read again, in id order.
    const float tmax = xmax > -INFINITY ? div_to_f32(xmax, a.T, a.Tinv) : -INFINITY;
    const float M = fmaxf(tmax, pmax);
    int best = 0;  // PHP: max starts at -INF and only a strictly larger value moves it
    if (M > -INFINITY && !(isfinite(M) && isfinite(xmax))) {
      best = kRedoMark;  // the CTA-per-row kernel's exact maximum
    } else if (M > -INFINITY) {
      best = pmax == M ? pidx : INT_MAX;
      const double lowt = (double)M - fabs((double)M) * 0x1p-22 - 1e-44;
      const float xthr = __double2float_rd(lowt * a.T);
      const float *Lrow = a.logits + (size_t)row_of(a, b) * a.ld;
      const int words = (V + 31) / 32;
      for (int c = 0; c < nch; ++c) {
        if (!(tab[c].x >= xthr)) continue;  // the same value on every lane
        float4 xw[8];
        lane_block(Lrow, c, V, xw);
        const int bw = c * kStreamPer * 4 + lane;
        const unsigned pm = bw < words ? bm[bw] : 0u;
        const int v0 = c * kStreamChunk * 4 + 32 * lane;
        int f = INT_MAX;
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = 4 * k + j;
            const float x = f4_at(xw[k], j);
            if (v0 + e < V && !((pm >> e) & 1u) && x >= xthr && f == INT_MAX && div_to_f32(x, a.T, a.Tinv) == M)
              f = v0 + e;
          }
        f = __reduce_min_sync(0xffffffffu, f);
        best = min(best, f);
        if (f != INT_MAX) break;
      }
    }
    if (lane == 0) a.out[b] = best;
    __syncwarp();
    return;
  }
  const float tmax = xmax > -INFINITY ? div_to_f32(xmax, a.T, a.Tinv) : -INFINITY;
  const float M = fmaxf(tmax, pmax);
  // PHP: max starts at -INF and only a strictly larger value moves it
  const bool any = M > -INFINITY;
  const double u = (double)a.uniforms[b];
  const float *Lrow = a.logits + (size_t)row_of(a, b) * a.ld;
  int id = -1;
  if (any && isfinite(M) && !ovf) {
    const float l2e = 1.44269504f;
    const float m2 = M * l2e;
    double S, rr, before;
    const int cs = chunk_prefix(
        nch, u, [&](int c) { const float4 e = tab[c]; return (double)e.y * (double)ex2_approx(e.x - m2); }, S, rr,
        before);
    // the penalised ids' share Sp and its distance-weighted sum Wp
    double Sp = 0.0, Wp = 0.0;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      double sp = 0.0, wp = 0.0;
      if (c0 + lane < nch) {
        const float4 e = tab[c0 + lane];
        sp = (double)e.z * (double)ex2_approx(e.x - m2);
        wp = fabs((double)m2 - (double)e.x) * sp;
      }
      Sp = __dadd_rn(Sp, warp_sum_d(sp));
      Wp = __dadd_rn(Wp, warp_sum_d(wp));
    }
    if (isfinite(S) && isfinite(rr) && S > 0.0 && u >= 0.0 && u <= 1.0) {
      const int v0 = cs * kStreamChunk * 4 + 32 * lane;
      const int bw = cs * kStreamPer * 4 + lane;  // the bitmap word of this lane's 32 ids
      const unsigned pm = bw < (V + 31) / 32 ? bm[bw] : 0u;
      {
        // p~ of this lane's 32 ids to the scratch: unpenalised ones from the
        // loaded words, then the penalised ones over them
        float4 xw[8];
        lane_block(Lrow, cs, V, xw);
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float f = f4_at(xw[k], j);
            pv[(4 * k + j) * 32 + lane] = v0 + 4 * k + j < V ? ex2_approx(fmaf(f, cexp, -m2)) : 0.f;
          }
        for (unsigned bits = pm; bits; bits &= bits - 1u) {
          const int e = __ffs(bits) - 1;
          const float f = Lrow[v0 + e];
          pv[e * 32 + lane] = ex2_approx(fmaf(penalise_a(div_to_f32(f, a.T, a.Tinv), a.rep, a.repinv), l2e, -m2));
        }
      }
      __syncwarp();
      double lo = 0.0, hi = 0.0;
      const int cand = chunk_crossing([&](int e) { return (double)pv[e * 32 + lane]; }, cs, V, before, rr, lo, hi);
      __syncwarp();
      // p~ against the contract value p = 2^-dist, dist = (M - t) log2e >= 0.
      // The draw only compares running sums with u S, so a factor common to
      // every p~ cancels: the roundings of c and of m2 shift every
      // unpenalised exponent by the same M log2e (dc - dm) plus at most
      // 2^-24 dist each (penalised exponents: the same with log2e's rounding;
      // the two groups differ by at most 2.9 |M| 2^-24, charged on Sp).
      // Per entry there remain t's rounding (2^-24 (1.443 |M| + dist)), the
      // fma and mu - m2 (mu between an unpenalised entry's x c and m2: 2^-24
      // dist each): a relative 2^-24 (|M| + 2.77 dist), with 2^-22 per
      // ex2.approx (two per chunk-total entry).  Summed over the entries,
      // 2.77 dist p adds up to at most 2.77 S log2 V (the entropy of p / S
      // is at most log2 V, and S >= 1).  A penalised id's fma works against
      // its chunk's unpenalised mu: 2^-24 |m2 - mu| more on its p (Wp).
      // fp32 sums: 16 levels for an unpenalised chunk total, 38 for the
      // penalised part.  Entries that underflow count as an absolute 2^-125.
      const double er = (1.5 * fabs((double)M) + 16.0) * 0x1p-24 + 0x1p-21 + 1e-12;
      const double eadd = 0x1p-24 *
                          (2.78 * log2((double)V) * S * (1.0 + 1e-3) + 0.7 * Wp + (38.0 + 3.0 * fabs((double)M)) * Sp) *
                          (1.0 + 2.0 * er);
      if (cand != INT_MAX && certify_cross(cand, lo, hi, S, rr, u, V, er, 0x1p-125, eadd, 80.0 + nch)) id = cand;
    }
  }
  // not certified (or not finite, or a NaN logit): the CTA-per-row kernel's
  // exact tiers take the row in the launch that follows
  if (lane == 0) a.out[b] = id >= 0 ? id : kRedoMark;
  __syncwarp();
}

template <bool GREEDY>
__global__ void __launch_bounds__(kStreamAWarps * 32, 1) sample_a_stream(const __grid_constant__ SampArgs a, int W) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int V = a.V, n4 = V >> 2, S = (n4 + kStreamChunk - 1) / kStreamChunk;
  const StreamALayout Ly = stream_a_layout(V);
  uint8_t *base = smem_dyn + (size_t)warp * Ly.bytes;
  float4 *ring = reinterpret_cast<float4 *>(base);
  uint32_t *bm = reinterpret_cast<uint32_t *>(base + Ly.off_bm);
  float4 *tab = reinterpret_cast<float4 *>(base + Ly.off_ch);
  float *pv = reinterpret_cast<float *>(base + Ly.off_pv);
  // warp-major numbering: row r goes to CTA r % grid, so every SM gets an
  // equal share of the rows (to within one); the warps of an SM share its
  // issue slots, so the SM with the most rows sets the kernel's time
  const int NW = gridDim.x * W, gw = warp * gridDim.x + blockIdx.x;
  if (warp >= W || gw >= a.rows) return;
  const int nrows = (a.rows - 1 - gw) / NW + 1;
  const float cexp = (float)(1.4426950408889634 * a.Tinv);
  const float l2e = 1.44269504f;
  auto mrow_of = [&](int i) -> int { return i < nrows ? row_of(a, gw + i * NW) : -1; };
  for (int w = lane; w < Ly.words; w += 32) bm[w] = 0u;
  __syncwarp();
  int mp = mrow_of(0), mq = mrow_of(1);
  mark_history(a, mp, bm);
  int pi = 0, ps = 0;
  const float4 *Lp = mp >= 0 ? reinterpret_cast<const float4 *>(a.logits + (size_t)mp * a.ld) : nullptr;
  auto issue = [&](int slot) {
    if (Lp != nullptr) {
      const int c0 = ps * kStreamChunk + lane;
#pragma unroll
      for (int r = 0; r < kStreamPer; ++r)
        if (c0 + 32 * r < n4) cp_async16(ring + slot * kStreamChunk + 32 * r + lane, Lp + c0 + 32 * r);
    }
    cp_async_commit();
    if (++ps == S) {
      ps = 0;
      ++pi;
      Lp = mq >= 0 ? reinterpret_cast<const float4 *>(a.logits + (size_t)mq * a.ld) : nullptr;
      mq = mrow_of(pi + 1);
    }
  };
  for (int q = 0; q < kStreamSlots; ++q) issue(q);

  float xmax = -INFINITY, pmax = -INFINITY, l0 = 0.f;
  int pidx = INT_MAX, ovf = 0;
  constexpr bool greedy = GREEDY;
  const long long total = (long long)nrows * S;
  int ci = 0, cs = 0;
  for (long long q = 0; q < total; ++q) {
    const int slot = (int)(q % kStreamSlots);
    cp_async_wait<kStreamSlots - 1>();
    if (cs == 0 && ci > 0) mark_history(a, mrow_of(ci), bm);
    // every lane's copies of this chunk are complete: the lanes read across
    __syncwarp();
    const float4 *rs = ring + slot * kStreamChunk + 8 * lane;  // this lane's eight words
    const int wd0 = cs * kStreamChunk + 8 * lane;
    const int bw = cs * kStreamPer * 4 + lane;
    const unsigned pm = bw < Ly.words ? bm[bw] : 0u;
    float4 x[8];
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int k = (r + lane) & 7;  // rotated: the eight lanes of a phase hit distinct banks
      x[r] = wd0 + k < n4 ? rs[k] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const unsigned nib = (pm >> (4 * k)) & 0xFu;
      if (nib & 1u) x[r].x = -INFINITY;
      if (nib & 2u) x[r].y = -INFINITY;
      if (nib & 4u) x[r].z = -INFINITY;
      if (nib & 8u) x[r].w = -INFINITY;
      m = fmaxf(m, fmax4(x[r]));
    }
    if (cs == 0 && lane == 0) l0 = reinterpret_cast<const float *>(rs)[0];  // the raw logit 0
    xmax = fmaxf(xmax, m);
    const float wm = warp_max(m);
    const float mu = wm > -INFINITY ? wm * cexp : 0.f;
    float sum = 0.f, sump = 0.f;
    // penalised ids of this lane, their stored values from the staged words
    for (unsigned bits = pm; bits; bits &= bits - 1u) {
      const int e = __ffs(bits) - 1;
      const float t =
          penalise_a(div_to_f32(reinterpret_cast<const float *>(rs)[e], a.T, a.Tinv), a.rep, a.repinv);
      if (t > pmax) {  // this lane's ids ascend: ties keep the first
        pmax = t;
        pidx = cs * kStreamChunk * 4 + 32 * lane + e;
      }
      const float y = fmaf(t, l2e, -mu);
      ovf |= y > 120.f;
      sump += greedy ? 0.f : ex2_approx(y);
    }
    __syncwarp();  // every lane has read the slot
    issue(slot);
    if (!greedy) {
#pragma unroll
      for (int r = 0; r < 8; ++r)
        sum += (ex2_approx(fmaf(x[r].x, cexp, -mu)) + ex2_approx(fmaf(x[r].y, cexp, -mu))) +
               (ex2_approx(fmaf(x[r].z, cexp, -mu)) + ex2_approx(fmaf(x[r].w, cexp, -mu)));
      sum = warp_sum(sum);
      sump = warp_sum(sump);
    }
    if (lane == 0) tab[cs] = greedy ? make_float4(wm, 0.f, 0.f, 0.f) : make_float4(mu, sum + sump, sump, 0.f);
    if (++cs == S) {
      __syncwarp();
      stream_a_finish(a, gw + ci * NW, xmax, pmax, pidx, l0, ovf, tab, bm, pv, S, cexp);
      for (int w = lane; w < Ly.words; w += 32) bm[w] = 0u;
      __syncwarp();
      xmax = -INFINITY;
      pmax = -INFINITY;
      pidx = INT_MAX;
      ovf = 0;
      cs = 0;
      ++ci;
    }
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Cluster kernels: rows longer than one CTA's register row.  A cluster of C
// CTAs (C = ceil(V / 32768), at most 8) takes a row; CTA r holds the ids
// [32768 r, 32768 (r + 1)) in registers through the same staged-row
// pipeline, and the row's decisions combine the CTAs' partial results
// through distributed shared memory (each CTA publishes into its own
// exchange area, a cluster barrier, then every CTA reads all C entries in
// rank order, so every CTA derives the same values).
// ---------------------------------------------------------------------------

constexpr int kSliceLen = kSegLen * kRegLayers;  // ids per CTA of a cluster row
constexpr int kMaxCluster = 8;

struct XchgA {
  unsigned int xkey;         // maximum of the slice's unpenalised raw logits (okey32)
  float l0;                  // raw logit 0 (rank 0)
  unsigned long long pkey;   // argmax key of the slice's penalised values (global ids)
  unsigned long long ekey;   // exact-maximum key (rare path)
  int cand;                  // first global id attaining M in the slice
  int verdict;               // rank 0: the draw's id or -1
  double seg[kRegLayers];    // the slice's layer totals of the current draw
};

__device__ __forceinline__ uint32_t xc_addr(const void *field, uint32_t rank) { return mapa_shared(smem_u32(field), rank); }

// The sequential algorithm of src/snai_inference.php:178-194 over a cluster
// row, by warp 0 of one CTA; the penalty set is read from the owning CTA's
// bitmap (bits_u32: this CTA's shared address of the row's bitmap, the same
// offset in every CTA).
__device__ __noinline__ int sequential_a_cluster(const SampArgs &a, uint32_t bits_u32, const float *L, double maxv,
                                                 double u) {
  const int lane = threadIdx.x & 31;
  auto pvalue = [&](int v, uint32_t w) -> double {
    const float t = div_to_f32(L[v], a.T, a.Tinv);
    const float tt = ((w >> (v & 31)) & 1u) ? penalise_a(t, a.rep, a.repinv) : t;
    return snai_exp(__dsub_rn((double)tt, maxv));
  };
  double sum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const uint32_t w = ld_cluster_u32(mapa_shared(bits_u32 + (uint32_t)((b % kSliceLen) >> 5) * 4u, b / kSliceLen));
    const double p = v < a.V ? pvalue(v, w) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) sum = __dadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
  }
  const double r = __dmul_rn(u, sum);
  double cum = 0.0;
  for (int b = 0; b < a.V; b += 32) {
    const int v = b + lane;
    const uint32_t w = ld_cluster_u32(mapa_shared(bits_u32 + (uint32_t)((b % kSliceLen) >> 5) * 4u, b / kSliceLen));
    const double p = v < a.V ? pvalue(v, w) : 0.0;
    const int cnt = min(32, a.V - b);
    for (int j = 0; j < cnt; ++j) {
      cum = __dadd_rn(cum, __shfl_sync(0xffffffffu, p, j));
      if (cum >= r) return b + j;
    }
  }
  return 0;
}

// Certified draw over a cluster row (tiers 1 and 2 of variant A): the
// per-CTA part of draw_reg, the layer totals of all CTAs scanned in id order
// by every CTA, the crossing layer scanned and certified by its CTA, whose
// verdict reaches every CTA through rank 0's exchange area.
template <class ACC, class PE, class PP>
__device__ __forceinline__ int draw_cluster(SmemRA &sm, XchgA *xc, uint32_t rank, uint32_t C, int lo, int Vtot,
                                            const uint32_t *bits, const int *plist, const ACC &acc, int Vl, int np,
                                            double u, double eps, double eabs, const PE &pe, const PP &pp) {
  constexpr int NV4 = kRegLayers;
  using PT = decltype(pe(0.f));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int SH = 5 - Log2<NV4>::v;
  PT part[NV4];
#pragma unroll
  for (int i = 0; i < NV4; ++i) {
    const float4 x = acc(i);
    part[i] = (pe(x.x) + pe(x.y)) + (pe(x.z) + pe(x.w));
  }
  PT pq[kPenCap / kSampThreads];
#pragma unroll
  for (int q = 0; q < kPenCap / kSampThreads; ++q) {
    const int s = threadIdx.x + q * kSampThreads;
    pq[q] = PT(0);
    if (s < np) {
      pq[q] = pp(s);
      const int sg = plist[s] / kSegLen;
#pragma unroll
      for (int i = 0; i < NV4; ++i) part[i] = part[i] + (i == sg ? pq[q] : PT(0));
    }
  }
  const PT lt = warp_reduce_layers<NV4>(part);
  if ((lane & ((1 << SH) - 1)) == 0) sm.wp[lane >> SH][warp] = (double)lt;
  __syncthreads();
  if (warp == 0 && lane < NV4) {
    double seg = 0.0;
    for (int w = 0; w < kSampWarps; ++w) seg = __dadd_rn(seg, sm.wp[lane][w]);
    xc->seg[lane] = seg;
  }
  cluster_sync_all();
  if (warp == 0) {
    // lane l: global layers 4l .. 4l+3 (layer g = 16 rank + local layer)
    const int nl = (int)C * NV4;
    double t[4], run = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int g = 4 * lane + j;
      t[j] = g < nl ? ld_cluster_f64(xc_addr(&xc->seg[g % NV4], (uint32_t)(g / NV4))) : 0.0;
      run = __dadd_rn(run, t[j]);
    }
    double incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = __dadd_rn(incl, n);
    }
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = 0.0;
    const double S = __shfl_sync(0xffffffffu, incl, 31);
    const double rr = __dmul_rn(u, S);
    int first = -1;
    double base = 0.0, p = excl;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const double nx = __dadd_rn(p, t[j]);
      if (first < 0 && 4 * lane + j < nl && nx >= rr) {
        first = 4 * lane + j;
        base = p;
      }
      p = nx;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, first >= 0);
    const int src = hit ? __ffs(hit) - 1 : 0;
    const int g = __shfl_sync(0xffffffffu, first, src);
    base = __shfl_sync(0xffffffffu, base, src);
    if (lane == 0) {
      sm.S = S;
      sm.r = rr;
      sm.base = base;
      sm.ss = (isfinite(S) && isfinite(rr) && hit && u >= 0.0 && u <= 1.0) ? g : -1;
      sm.dcand = INT_MAX;
    }
  }
  __syncthreads();
  const int gs = sm.ss;
  if (gs < 0) return -1;  // the same on every CTA: all read the same totals in the same order
  const int sc = gs / NV4, ss = gs % NV4;
  if ((int)rank == sc) {
#pragma unroll
    for (int q = 0; q < kPenCap / kSampThreads; ++q) {
      const int s = threadIdx.x + q * kSampThreads;
      if (s < np) {
        const int h = plist[s];
        if (h / kSegLen == ss) sm.segpen[h % kSegLen] = (double)pq[q];
      }
    }
    __syncthreads();
    const double S = sm.S, rr = sm.r;
    const int v0 = (threadIdx.x + kSampThreads * ss) * 4;
    const float4 x = acc(ss);
    const uint32_t pw = v0 < Vl ? (bits[v0 >> 5] >> (v0 & 31)) & 0xFu : 0u;
    double pr[4];
    double c = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = f4_at(x, j);
      pr[j] = v0 + j >= Vl ? 0.0 : ((pw >> j) & 1u) ? sm.segpen[(v0 + j) % kSegLen] : (double)pe(f);
      c = __dadd_rn(c, pr[j]);
    }
    double incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = __dadd_rn(incl, n);
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    double wt = lane < kSampWarps ? sm.wsum[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < kSampWarps; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, wt, o);
      if (lane >= o) wt = __dadd_rn(wt, n);
    }
    double wbase = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
    if (warp == 0) wbase = 0.0;
    double ex = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) ex = 0.0;
    ex = __dadd_rn(wbase, ex);
    double prev = __dadd_rn(sm.base, ex);
    int mine = -1;
    double lo_s = prev, hi_s = prev;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const double cur = __dadd_rn(prev, pr[j]);
      if (mine < 0 && v0 + j < Vl && cur >= rr) {
        mine = j;
        lo_s = prev;
        hi_s = cur;
      }
      prev = cur;
    }
    if (mine >= 0) {
      // the error model of draw_reg, with every CTA's layers in the depth
      const int cand = lo + v0 + mine;
      const double slack = (double)((int)C * NV4 + 64);
      const double er = eps * (1.0 + 2.0 * eps) + 1e-12 * (eps > 0.0);
      const double Er = u * (er * S + (double)Vtot * eabs + ((double)Vtot + slack) * 0x1p-52 * S) + 0x1p-52 * rr;
      const double Ehi = er * hi_s + ((double)cand + 1.0) * eabs + ((double)cand + slack) * 0x1p-52 * hi_s;
      const double Elo = er * lo_s + (double)cand * eabs + ((double)cand + slack) * 0x1p-52 * lo_s;
      const bool up = hi_s - Ehi >= rr + Er;
      const bool dn = cand == 0 || lo_s + Elo < rr - Er;
      atomicMin(&sm.dcand, 2 * cand + ((up && dn) ? 0 : 1));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const int key = sm.dcand;
      const int v = (key != INT_MAX && !(key & 1)) ? key >> 1 : -1;
      st_cluster_u32(xc_addr(&xc->verdict, 0), (uint32_t)v);
    }
  }
  cluster_sync_all();
  return (int)ld_cluster_u32(xc_addr(&xc->verdict, 0));
}

template <int NV4>
__global__ void __launch_bounds__(kSampThreads, 1) sample_a_cluster(const __grid_constant__ SampArgs a) {
  static_assert(NV4 == kRegLayers, "one slice per CTA");
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemRA &sm = *reinterpret_cast<SmemRA *>(smem_dyn);
  RowPipe &pp = sm.pipe;
  XchgA *xcs = reinterpret_cast<XchgA *>(smem_dyn + sizeof(SmemRA));  // [2], row parity
  const uint32_t rank = cluster_ctarank(), C = cluster_nctarank();
  const int lo = (int)rank * kSliceLen;
  const int Vl = min(a.V - lo, kSliceLen);
  SampArgs va = a;  // this CTA's slice of every row
  va.logits = a.logits + lo;
  va.V = Vl;
  const int words = kSliceLen / 32;  // bitmap copies at the same offsets in every CTA
  uint32_t *bm = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemRA) + 2 * sizeof(XchgA));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool greedy = a.T <= 0.01;
  RowFeeder feed;
  feed.stage = stage_ptr(smem_dyn, sizeof(SmemRA) + 2 * sizeof(XchgA) + (size_t)8 * words, kSliceLen);
  feed.bar = &pp.bar;
  int hreg[kHistRegs];
  const int cid = (int)(blockIdx.x / C), ncl = (int)(gridDim.x / C);
  pipe_start(va, pp, bm, words, feed, hreg, sm.plist[0], lo, cid, ncl);
  cluster_sync_all();  // every CTA's exchange area exists before the first remote access

  int it = 0;
  for (int b = cid; b < a.rows; b += ncl, ++it) {
    const int par = it & 1;
    XchgA *xc = &xcs[par];
    const uint32_t *bits = bm + (it % 3) * words;
    int *plist = sm.plist[par];
    float *pval = sm.pval[par];
    if (threadIdx.x == 0) pipe_reset(pp, par ^ 1);
    const bool ok = feed.wait(a.err);  // a timeout is recorded; the cluster keeps its barrier sequence
    const int np = min(pp.npen[par], kPenCap);
    unsigned long long pk = 0ull;
    if (warp * 32 < np) {
#pragma unroll
      for (int q = 0; q < kPenCap / kSampThreads; ++q) {
        const int s = threadIdx.x + q * kSampThreads;
        if (s < np) {
          const int h = plist[s];
          const float raw = feed.stage[h];
          if (h == 0) pp.l0[par] = raw;
          const float t = penalise_a(div_to_f32(raw, a.T, a.Tinv), a.rep, a.repinv);
          pval[s] = t;
          feed.stage[h] = -INFINITY;
          const unsigned long long key = argmax_key(t, lo + h);
          pk = key > pk ? key : pk;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, pk, o);
        pk = o2 > pk ? o2 : pk;
      }
    }
    if (lane == 0) pp.pkey[par][warp] = pk;
    __syncthreads();
    float4 r[NV4];
    float xmax = -INFINITY;
    const uint32_t st_u32 = smem_u32(feed.stage);
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      r[i] = v0 < Vl ? lds4(st_u32 + 4u * v0) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      xmax = fmaxf(xmax, fmax4(r[i]));
    }
    if (threadIdx.x == 0 && !(bits[0] & 1u)) pp.l0[par] = r[0].x;
    const float my_xmax = xmax;
    xmax = warp_max(xmax);
    if (lane == 0) atomicMax(&pp.xkey[par], okey32(xmax));
    __syncthreads();
    (void)ok;
    pipe_advance(va, pp, bm, words, it, b, feed, hreg, sm.plist[par ^ 1], lo, ncl);

    // ---- publish the slice's maxima, then combine over the cluster ----
    pk = pp.pkey[par][lane & (kSampWarps - 1)];
#pragma unroll
    for (int o = kSampWarps / 2; o > 0; o >>= 1) {
      const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, pk, o);
      pk = o2 > pk ? o2 : pk;
    }
    if (threadIdx.x == 0) {
      xc->xkey = pp.xkey[par];
      xc->pkey = pk;
      xc->l0 = pp.l0[par];
      xc->cand = INT_MAX;
    }
    cluster_sync_all();
    unsigned int xk = 0u;
    unsigned long long gpk = 0ull;
    for (uint32_t c = 0; c < C; ++c) {
      xk = max(xk, ld_cluster_u32(xc_addr(&xc->xkey, c)));
      const unsigned long long o2 = ld_cluster_u64(xc_addr(&xc->pkey, c));
      gpk = o2 > gpk ? o2 : gpk;
    }
    const float l0 = __uint_as_float(ld_cluster_u32(xc_addr(&xc->l0, 0)));
    if (a.nan_guard && l0 != l0) {  // src/snai_inference.php:146
      if (rank == 0 && threadIdx.x == 0) a.out[b] = -1;
      continue;
    }
    xmax = key_to_float(xk);
    const float pmax = key_to_float((unsigned int)(gpk >> 32));
    const int pidx = gpk ? (int)(0xffffffffu - (unsigned int)gpk) : INT_MAX;
    const float tmax = (xmax > -INFINITY) ? div_to_f32(xmax, a.T, a.Tinv) : -INFINITY;
    const float M = fmaxf(tmax, pmax);
    const bool simple = a.T > 0.0 && isfinite(M) && isfinite(xmax);
    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;

    if (greedy && simple) {
      const double lowt = (double)M - fabs((double)M) * 0x1p-22 - 1e-44;
      const float xthr = __double2float_rd(lowt * a.T);
      int mc = INT_MAX;
      if (my_xmax >= xthr) {
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
          if (fmax4(r[i]) >= xthr) {
            const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float f = f4_at(r[i], j);
              if (f >= xthr && div_to_f32(f, a.T, a.Tinv) == M) mc = min(mc, lo + v0 + j);
            }
          }
        }
      }
      if (rank == 0 && threadIdx.x == 0 && pmax == M) mc = min(mc, pidx);
      if (mc != INT_MAX) atomicMin(&xc->cand, mc);
      cluster_sync_all();
      if (rank == 0 && threadIdx.x == 0) {
        int best = INT_MAX;
        for (uint32_t c = 0; c < C; ++c) best = min(best, (int)ld_cluster_u32(xc_addr(&xc->cand, c)));
        a.out[b] = best;
      }
      continue;
    }

    float best = M;
    int bi = INT_MAX;
    if (!simple) {
      // exact maximum of the slice's stored values (from global memory), combined over the cluster
      float lb;
      int li;
      exact_max_a(va, bits, L + lo, reinterpret_cast<float *>(sm.wsum), reinterpret_cast<int *>(sm.wsum) + 16, lb,
                  li);
      if (threadIdx.x == 0) xc->ekey = li == INT_MAX ? 0ull : argmax_key(lb, lo + li);
      cluster_sync_all();
      unsigned long long ek = 0ull;
      for (uint32_t c = 0; c < C; ++c) {
        const unsigned long long o2 = ld_cluster_u64(xc_addr(&xc->ekey, c));
        ek = o2 > ek ? o2 : ek;
      }
      best = key_to_float((unsigned int)(ek >> 32));
      bi = ek ? (int)(0xffffffffu - (unsigned int)ek) : INT_MAX;
    }
    const bool any = best > -INFINITY;
    if (greedy) {
      if (rank == 0 && threadIdx.x == 0) a.out[b] = any ? bi : 0;
      continue;
    }
    const double maxv = any ? (double)best : -INFINITY;
    const double u = (double)a.uniforms[b];
    int id = -1;
    if (any && simple) {
      const float c = (float)(1.4426950408889634 * a.Tinv);
      const float l2e = 1.44269504f;
      const float m2 = M * l2e;
      const double tabs = fabs((double)M) + 91.0;
      const double eps = (tabs + fabs((double)M) + 1.0) * 0x1p-21 + 0x1p-19 + 0x1p-20;
      id = draw_cluster(
          sm, xc, rank, C, lo, a.V, bits, plist, [&](int i) { return pick_layer(r, i); }, Vl, np, u, eps, 0x1p-125,
          [&](float x) { return ex2_approx(fmaf(x, c, -m2)); },
          [&](int s) { return ex2_approx(fmaf(pval[s], l2e, -m2)); });
      if (id < 0) {
        // tier 2: the contract exponential, the slice read from global memory
        const float *Ls = L + lo;
        auto acc = [&](int i) {
          const int v0 = (threadIdx.x + kSampThreads * i) * 4;
          float4 x = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          if (v0 < Vl) {
            x = __ldg(reinterpret_cast<const float4 *>(Ls + v0));
            const uint32_t w = (bits[v0 >> 5] >> (v0 & 31)) & 0xFu;
            if (w & 1u) x.x = -INFINITY;
            if (w & 2u) x.y = -INFINITY;
            if (w & 4u) x.z = -INFINITY;
            if (w & 8u) x.w = -INFINITY;
          }
          return x;
        };
        id = draw_cluster(
            sm, xc, rank, C, lo, a.V, bits, plist, acc, Vl, np, u, 0.0, 0.0,
            [&](float x) { return snai_exp(__dsub_rn((double)div_to_f32(x, a.T, a.Tinv), maxv)); },
            [&](int s) { return snai_exp(__dsub_rn((double)pval[s], maxv)); });
      }
    }
    if (id < 0) {
      // tier 3 on rank 0, reading every CTA's bitmap: the cluster waits
      if (rank == 0 && warp == 0) {
        const int s = sequential_a_cluster(a, smem_u32(bits), L, maxv, u);
        if (lane == 0) a.out[b] = s;
      }
      cluster_sync_all();
    } else if (rank == 0 && threadIdx.x == 0) {
      a.out[b] = id;
    }
    __syncthreads();
  }
  cluster_sync_all();  // no CTA leaves while another may still read its shared memory
}

struct XchgB {
  unsigned int xkey;  // maximum of the slice's lower bounds (okey32)
  float s1, s2;       // spread statistics of rank 0's chunk layer 0
  int bstar;          // rank 0 -> every CTA: the histogram's threshold bin
};

// Variant B over a cluster row: the fast selection of sample_b_reg with the
// maximum and the histogram combined over the cluster (rank 0 sums the
// CTAs' histograms), every CTA gathering its candidates into rank 0's
// candidate table, and rank 0 ranking them and running the top-p tail.  Rows
// the fast path cannot settle take general_select_b on rank 0 over the whole
// row, with a whole-row history bitmap built for them.
__global__ void __launch_bounds__(kSampThreads, 1) sample_b_cluster(const __grid_constant__ SampArgs a) {
  constexpr int NV4 = kRegLayers;
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  SmemB &sm = *reinterpret_cast<SmemB *>(smem_dyn);
  RowPipe &pp = *reinterpret_cast<RowPipe *>(smem_dyn + sizeof(SmemB));
  XchgB *xcs = reinterpret_cast<XchgB *>(smem_dyn + sizeof(SmemB) + sizeof(RowPipe));  // [2]
  const uint32_t rank = cluster_ctarank(), C = cluster_nctarank();
  const int lo = (int)rank * kSliceLen;
  const int Vl = min(a.V - lo, kSliceLen);
  SampArgs va = a;
  va.logits = a.logits + lo;
  va.V = Vl;
  const int words = kSliceLen / 32;
  uint32_t *bm = reinterpret_cast<uint32_t *>(smem_dyn + sizeof(SmemB) + sizeof(RowPipe) + 2 * sizeof(XchgB));
  uint32_t *fullbits = bm + 3 * (kSliceLen / 32);  // rank 0: whole-row bitmap for the general path
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k = min(a.top_k, a.V);
  const double rep = a.rep;
  RowFeeder feed;
  // stage_ptr adds one bitmap of `words` words: the core, three slice
  // bitmaps and the whole-row bitmap come before the stage
  feed.stage = stage_ptr(smem_dyn,
                         sizeof(SmemB) + sizeof(RowPipe) + 2 * sizeof(XchgB) + (size_t)8 * words +
                             (size_t)((a.V + 31) / 32) * 4,
                         kSliceLen);
  feed.bar = &pp.bar;
  int hreg[kHistRegs];
  const int cid = (int)(blockIdx.x / C), ncl = (int)(gridDim.x / C);
  pipe_start(va, pp, bm, words, feed, hreg, sm.plist, lo, cid, ncl);
  cluster_sync_all();
  const uint32_t ncand0 = xc_addr(&sm.ncand, 0);

  int it = 0;
  for (int b = cid; b < a.rows; b += ncl, ++it) {
    const int par = it & 1;
    XchgB *xc = &xcs[par];
    const uint32_t *bits = bm + (it % 3) * words;
    if (threadIdx.x == 0) pipe_reset(pp, par ^ 1);
    const bool ok = feed.wait(a.err);
    (void)ok;
    const int np = min(pp.npen[par], kPenCap);
    for (int s = threadIdx.x; s < np; s += kSampThreads) {
      const int h = sm.plist[s];
      feed.stage[h] = __double2float_rd(__dsub_rn((double)feed.stage[h], rep));
    }
    __syncthreads();
    float4 r[NV4];
    float mx = -INFINITY, s1 = 0.f, s2 = 0.f;
    const uint32_t st_u32 = smem_u32(feed.stage);
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int v0 = (threadIdx.x + kSampThreads * i) * 4;
      r[i] = v0 < Vl ? lds4(st_u32 + 4u * v0) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (i == 0 && v0 < Vl && rank == 0) {
        const float4 x = r[0];
        s1 = (x.x + x.y) + (x.z + x.w);
        s2 = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, x.w * x.w)));
      }
      mx = fmaxf(mx, fmax4(r[i]));
    }
    const float my_mx = mx;
    mx = warp_max(mx);
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      atomicMax(&pp.xkey[par], okey32(mx));
      atomicAdd(&pp.s1[par], s1);
      atomicAdd(&pp.s2[par], s2);
    }
    for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
    if (threadIdx.x == 0) sm.ncand = 0;
    __syncthreads();
    pipe_advance(va, pp, bm, words, it, b, feed, hreg, sm.plist, lo, ncl);
    if (threadIdx.x == 0) {
      xc->xkey = pp.xkey[par];
      xc->s1 = pp.s1[par];
      xc->s2 = pp.s2[par];
    }
    cluster_sync_all();
    unsigned int xk = 0u;
    for (uint32_t c = 0; c < C; ++c) xk = max(xk, ld_cluster_u32(xc_addr(&xc->xkey, c)));
    mx = key_to_float(xk);
    s1 = __uint_as_float(ld_cluster_u32(xc_addr(&xc->s1, 0)));
    s2 = __uint_as_float(ld_cluster_u32(xc_addr(&xc->s2, 0)));
    const float *L = a.logits + (size_t)row_of(a, b) * a.ld;
    const int n0 = min(a.V, kSegLen);
    bool fast = isfinite(mx) && isfinite(s1) && isfinite(s2) && a.V >= k;
    float R = 0.f;
    if (fast) {
      const float mean = s1 / n0;
      const float sd = sqrtf(fmaxf(s2 / n0 - mean * mean, 0.f));
      R = 2.5f * sd;
      fast = R > 0.f && isfinite(R);
    }
    int bstar = 255;
    for (int attempt = 0; fast && attempt < 3 && bstar >= 255; ++attempt) {
      if (attempt > 0) {
        for (int i = threadIdx.x; i < 256; i += kSampThreads) sm.hist[i] = 0u;
        __syncthreads();
      }
      const float inv_w = 255.f / R;
#pragma unroll
      for (int i = 0; i < NV4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float d = mx - f4_at(r[i], j);
          if (d < R) atomicAdd(&sm.hist[min((int)(d * inv_w), 254)], 1u);
        }
      }
      cluster_sync_all();
      if (rank == 0 && warp == 0) {
        unsigned int c8[8], run = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          unsigned int h = 0;
          for (uint32_t c = 0; c < C; ++c) h += ld_cluster_u32(xc_addr(&sm.hist[lane * 8 + q], c));
          run += h;
          c8[q] = run;
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
          if (before + c8[q] >= (unsigned)k) bs = lane * 8 + q;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bs = min(bs, __shfl_xor_sync(0xffffffffu, bs, o));
        if (lane < (int)C) st_cluster_u32(xc_addr(&xc->bstar, (uint32_t)lane), (uint32_t)bs);
      }
      cluster_sync_all();
      bstar = xc->bstar;
      if (bstar >= 255) R *= 8.f;
    }
    fast = fast && bstar < 255;
    if (fast) {
      // gather (the superset threshold of sample_b_reg) into rank 0's table
      const double gd = (double)mx - (double)(bstar + 1) * ((double)R / 255.0) * (1.0 + 0x1p-20);
      float g = __double2float_rd(gd);
      g = (g == -INFINITY) ? g : __uint_as_float(g > 0.f ? __float_as_uint(g) - 1u
                                                          : (g == 0.f ? 0x80000001u : __float_as_uint(g) + 1u));
      if (my_mx >= g) {
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
          if (fmax4(r[i]) >= g) {
            const int v0 = (threadIdx.x + kSampThreads * i) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float f = f4_at(r[i], j);
              if (f >= g) {
                const int v = v0 + j;
                const double val = in_set(bits, v) ? __dsub_rn((double)L[lo + v], rep) : (double)f;
                const uint32_t slot = atom_cluster_add_u32(ncand0, 1u);
                if (slot < (uint32_t)kFastCand) {
                  st_cluster_u64(xc_addr(&sm.ckey[slot], 0), okey64(val));
                  st_cluster_u32(xc_addr(&sm.cidx[slot], 0), (uint32_t)(lo + v));
                }
              }
            }
          }
        }
      }
    }
    cluster_sync_all();
    if (rank != 0) continue;
    // ---- rank 0: selection and the top-p tail (the other CTAs go on) ----
    if (fast) {
      const int nc = sm.ncand;
      fast = nc <= kFastCand && nc >= k;
      if (fast) rank_candidates(sm, nc, k, a.T);
    }
    if (!fast) {
      // whole-row history bitmap for the general path
      const int fw = (a.V + 31) >> 5;
      for (int i = threadIdx.x; i < fw; i += kSampThreads) fullbits[i] = 0u;
      __syncthreads();
      {
        const int mrow = row_of(a, b);
        int n = a.hist_len ? a.hist_len[mrow] : a.hist_cols;
        n = min(max(n, 0), a.hist_cols);
        const int *hr = a.hist + (size_t)mrow * a.hist_ld;
        for (int i = threadIdx.x; i < n; i += kSampThreads) {
          const int t = hr[i];
          if (t >= 0 && t < a.V) atomicOr(&fullbits[t >> 5], 1u << (t & 31));
        }
      }
      __syncthreads();
      if (!general_select_b(a, fullbits, L, sm, k)) {
        if (threadIdx.x == 0) {
          a.out[b] = -2;
          record_error(a.err, kErrSamplerArgs);
        }
        __syncthreads();
        continue;
      }
    }
    if (a.T < 0.01) {
      if (threadIdx.x == 0) a.out[b] = sm.order[0];
      __syncthreads();
      continue;
    }
    topp_tail(a, sm, k, b);
    __syncthreads();
  }
  cluster_sync_all();
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
  int dev = 0;
  cudaGetDevice(&dev);
  return device_sm_count(dev);
}

// The full 227 KB of dynamic shared memory and the largest carve-out.
template <class K>
static bool set_smem_attrs(K kern) {
  const bool ok = set_dyn_smem(kern, 227 * 1024);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return ok;
}

template <class K>
static void launch_persistent(K kern, const SampArgs &a, size_t sm, int per_sm, cudaStream_t st,
                              DeviceOnce &done) {
  int dev = 0;
  cudaGetDevice(&dev);
  done.run(dev, [&] { return set_smem_attrs(kern); });
  const int grid = std::min(a.rows, sm_count() * per_sm);
  kern<<<grid, kSampThreads, sm, st>>>(a);
}

// One cluster of C CTAs per row, clusters walking the rows; returns false if
// the cluster shape cannot be scheduled (the caller falls back).
template <class K>
static bool launch_cluster(K kern, const SampArgs &a, size_t sm, int C, cudaStream_t st, DeviceOnce &done) {
  int dev = 0;
  cudaGetDevice(&dev);
  done.run(dev, [&] { return set_smem_attrs(kern); });
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)C;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = sm;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)C);
  int fit = 0;
  if (cudaOccupancyMaxActiveClusters(&fit, kern, &cfg) != cudaSuccess || fit < 1) {
    cudaGetLastError();
    return false;
  }
  const int clusters = std::max(1, std::min(a.rows, fit));
  cfg.gridDim = dim3((unsigned)(clusters * C));
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess;
}

template <int NV4>
static void launch_a(const SampArgs &a, size_t sm, cudaStream_t st) {
  static DeviceOnce done;  // attributes set, per device
  if constexpr (NV4 == 0)
    launch_persistent(sample_a_kernel<0>, a, sm, 1, st, done);
  else
    launch_persistent(sample_a_reg<NV4>, a, sm, NV4 <= 8 ? 2 : 1, st, done);
}

// Last step of a variant-A redo: the redone rows' -(v + 10) back to v.
__global__ void redo_decode_kernel(int *out, int rows) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < rows && out[b] <= kRedoDone) out[b] = -out[b] - 10;
}

template <int NV4>
static void launch_b(const SampArgs &a, size_t sm, cudaStream_t st) {
  static DeviceOnce done;
  if constexpr (NV4 == 0)
    launch_persistent(sample_b_kernel<0>, a, sm, 1, st, done);
  else
    launch_persistent(sample_b_reg<NV4>, a, sm, NV4 <= 8 ? 2 : 1, st, done);
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
  a.repinv = 1.0 / s.rep;
  a.top_p = s.top_p;
  a.top_k = s.top_k;
  a.nan_guard = s.nan_guard;
  a.out = s.out_ids;
  a.err = s.err;
  a.redo = 0;
  // The one-warp-per-row kernels pay off from a few rows per SM on; a
  // smaller batch is quicker with a whole CTA per row.  Warps per CTA: at
  // most what the rows fill across all SMs.
  const bool many = s.rows >= 4 * sm_count();
  const int wrows = (s.rows + sm_count() - 1) / sm_count();
  // variant A over 16-byte aligned rows: the streaming kernel (greedy only for
  // rows longer than a register row, where it beats the CTA clusters)
  if (many && s.variant == 0 && (s.temperature > 0.01 || s.V > kSliceLen) && (s.V & 3) == 0 && (s.ld & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(s.logits) & 15) == 0) {
    const StreamALayout Ly = stream_a_layout(s.V);
    const int W = std::min<int>({kStreamAWarps, (int)((227u * 1024u) / Ly.bytes), wrows});
    if (W >= 2) {
      static DeviceOnce done;
      int dev = 0;
      cudaGetDevice(&dev);
      done.run(dev, [] {
        const bool a = set_dyn_smem(sample_a_stream<false>, 227 * 1024);
        return set_dyn_smem(sample_a_stream<true>, 227 * 1024) && a;
      });
      const int grid = std::min(sm_count(), (s.rows + W - 1) / W);
      if (s.temperature <= 0.01)
        sample_a_stream<true><<<grid, W * 32, (size_t)W * Ly.bytes, stream>>>(a, W);
      else
        sample_a_stream<false><<<grid, W * 32, (size_t)W * Ly.bytes, stream>>>(a, W);
      // the rows it could not certify, exactly, by the CTA-per-row kernel
      SampArgs r = a;
      const size_t core = sizeof(SmemA) + (((size_t)((s.V + 31) / 32) * 4 + 15) & ~(size_t)15);
      const size_t staged = core + (size_t)s.V * 4 + kStageAlign;
      r.redo = staged <= 227u * 1024u ? 2 : 1;  // room to stage a whole row: its passes read shared memory
      launch_a<0>(r, r.redo == 2 ? staged : core, stream);
      redo_decode_kernel<<<(s.rows + 255) / 256, 256, 0, stream>>>(a.out, s.rows);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) {
        set_error("sampler launch failed: %s", cudaGetErrorString(e));
        return -4;
      }
      return 0;
    }
  }
  // variant B over 16-byte aligned rows: the streaming kernel, one warp per row
  if (many && s.variant != 0 && (s.V & 3) == 0 && (s.ld & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(s.logits) & 15) == 0) {
    const int kk = s.temperature < 0.01 ? 1 : std::min(s.top_k, s.V);
    const StreamLayout Ly = stream_layout(s.V, kk);
    const int W = std::min<int>({kStreamWarps, (int)((227u * 1024u) / Ly.bytes), wrows});
    if (kk <= kStreamMaxK && W >= 2) {
      static DeviceOnce done;
      int dev = 0;
      cudaGetDevice(&dev);
      done.run(dev, [] { return set_dyn_smem(sample_b_stream, 227 * 1024); });
      const int grid = std::min(sm_count(), (s.rows + W - 1) / W);
      sample_b_stream<<<grid, W * 32, (size_t)W * Ly.bytes, stream>>>(a, W);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) {
        set_error("sampler launch failed: %s", cudaGetErrorString(e));
        return -4;
      }
      return 0;
    }
  }
  const size_t bitmap = ((size_t)((s.V + 31) / 32) * 4 + 15) & ~(size_t)15;
  const int layers = (s.V + kSegLen - 1) / kSegLen;
  // register rows: whole 16-byte chunks from 16-byte aligned row starts, and
  // a history that fits the per-row id list
  const bool reg = layers <= kRegLayers && (s.V & 3) == 0 && (s.ld & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(s.logits) & 15) == 0 && s.hist_cols <= kPenCap;
  const int nv4 = !reg ? 0 : layers <= 4 ? 4 : layers <= 8 ? 8 : 16;
  // rows of up to 8 slices: a cluster of CTAs per row
  const int C = (s.V + kSliceLen - 1) / kSliceLen;
  const bool clus = !reg && C >= 2 && C <= kMaxCluster && (s.V & 3) == 0 && (s.ld & 3) == 0 &&
                    (reinterpret_cast<uintptr_t>(s.logits) & 15) == 0 && s.hist_cols <= kPenCap;
  if (clus) {
    const size_t maps = 3 * (size_t)(kSliceLen / 32) * 4 + (size_t)kSliceLen * 4 + kStageAlign;
    bool launched;
    if (s.variant == 0) {
      static DeviceOnce done;
      launched = launch_cluster(sample_a_cluster<kRegLayers>, a, sizeof(SmemRA) + 2 * sizeof(XchgA) + maps, C,
                                stream, done);
    } else {
      static DeviceOnce done;
      launched = launch_cluster(sample_b_cluster, a,
                                sizeof(SmemB) + sizeof(RowPipe) + 2 * sizeof(XchgB) + maps +
                                    (size_t)((s.V + 31) / 32) * 4,
                                C, stream, done);
    }
    if (launched) {
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) {
        set_error("sampler launch failed: %s", cudaGetErrorString(e));
        return -4;
      }
      return 0;
    }
  }
  // register rows: three bitmaps, then the staging buffer (+ alignment slack)
  const size_t rsm = reg ? 3 * (size_t)((s.V + 31) / 32) * 4 + (size_t)s.V * 4 + kStageAlign : 0;
  if (s.variant == 0) {
    const size_t sm = reg ? sizeof(SmemRA) + rsm : sizeof(SmemA) + bitmap;
    if (nv4 == 4)
      launch_a<4>(a, sm, stream);
    else if (nv4 == 8)
      launch_a<8>(a, sm, stream);
    else if (nv4 == 16)
      launch_a<16>(a, sm, stream);
    else
      launch_a<0>(a, sm, stream);
  } else {
    const size_t sm = reg ? sizeof(SmemB) + sizeof(RowPipe) + rsm : sizeof(SmemB) + bitmap;
    if (nv4 == 4)
      launch_b<4>(a, sm, stream);
    else if (nv4 == 8)
      launch_b<8>(a, sm, stream);
    else if (nv4 == 16)
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
