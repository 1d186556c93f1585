// epilogue.cuh - what a projection does with its fp32 results.
//
// store(m, n, v, cnt) receives v[0..cnt) = C[m][n .. n+cnt) for an even n
// (up to 16 columns of one row); store4(m, n, v, cnt, pre) receives up to 4
// columns from n, a multiple of 4 (the tensor-core drains hand consecutive
// lanes consecutive 4-column groups of one row, so these stores coalesce),
// with pre = load4(m, n, cnt), which the drains issue ahead of time (the
// residual's old values; nothing for the others), and ri = row(m), loaded
// once per tile by the lane that owns row m.  prefetch(m, n, cols) warms L2
// with what a tile's drain will read (called before the accumulator is
// ready).
// The element-wise arithmetic mirrors core/cortex.nim operation for
// operation (explicit _rn intrinsics: no contraction into FMA), so the only
// differences from the reference are the dot products' summation order.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "engine.h"

namespace snai {

// Q|K|V = x * [Wq;Wk;Wv]^T.  RoPE on q and k (core/cortex.nim:74-87, applied
// at :504 and :509), q to a row buffer, k and v appended to the cache at the
// row's position (:506-510).  Channels >= heads*hs are never read by
// attention and are dropped.
struct EpiQKV {
  const RowDesc *rows;
  float *q;
  float *kv;
  const float2 *rope;
  int D, att_ch, hs;
  size_t slot_stride, layer_off, part_stride, head_stride;
  // non-null: K and V go to this row-major [M, 2, att_ch] staging buffer and
  // the attention kernel appends them to the cache (one row per slot); it
  // also applies RoPE to q and k then (one position per block there, where a
  // decode step's rows, all at one position, would otherwise hammer one
  // table row from every SM at once)
  float *kvs;
  // tma != 0 (staging mode with att_ch == D): q [M][att_ch] and the staging
  // buffer [M][2 att_ch] as fp32 tensors (16 x 32 boxes, 64-byte swizzle);
  // the drains store their runs by TMA
  int tma;
  CUtensorMap tq, tkv;

  static constexpr bool kTmaStore = true;
  __device__ __forceinline__ const CUtensorMap *tma_out(int n, int &x) const {
    if (!tma) return nullptr;
    x = n < D ? n : n - D;
    return n < D ? &tq : &tkv;
  }

  __device__ __forceinline__ float *kv_dst(const RowDesc &rd, int m, int part, int head, int j) const {
    if (kvs) return kvs + ((size_t)m * 2 + (part - 1)) * att_ch + (size_t)head * hs + j;
    return kv + (size_t)rd.slot * slot_stride + layer_off + (size_t)(part - 1) * part_stride +
           (size_t)head * head_stride + (size_t)rd.pos * hs + j;
  }

  __device__ __forceinline__ void pair(const RowDesc &rd, int m, int n, float a, float b) const {
    const int part = n / D;
    const int ch = n - part * D;
    if (ch >= att_ch) return;
    const int head = ch / hs;
    const int j = ch - head * hs;
    if (part < 2 && !kvs) {
      const float2 cs = rope[(size_t)rd.pos * (hs >> 1) + (j >> 1)];
      const float a2 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
      const float b2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
      a = a2;
      b = b2;
    }
    if (part == 0) {
      *reinterpret_cast<float2 *>(q + (size_t)m * att_ch + ch) = make_float2(a, b);
    } else {
      *reinterpret_cast<float2 *>(kv_dst(rd, m, part, head, j)) = make_float2(a, b);
    }
  }

  static constexpr bool kTmaReduce = false;
  struct Pre {};
  using Row = RowDesc;
  __device__ __forceinline__ Row row(int m) const { return rows[m]; }
  __device__ __forceinline__ void prefetch(int, int, int) const {}
  __device__ __forceinline__ Pre load4(int, int, int) const { return Pre{}; }
  __device__ __forceinline__ void store4(int m, int n, float4 v, int cnt, Pre, const RowDesc &rd) const {
    if (cnt == 4 && (hs & 3) == 0 && (D & 3) == 0) {
      const int part = (n >= D) + (n >= 2 * D);
      const int ch = n - part * D;
      if (ch >= att_ch) return;
      const int head = (hs & (hs - 1)) == 0 ? ch >> (__ffs(hs) - 1) : ch / hs;
      const int j = ch - head * hs;
      float4 o = v;
      if (part < 2 && !kvs) {
        const float4 c = *reinterpret_cast<const float4 *>(rope + (size_t)rd.pos * (hs >> 1) + (j >> 1));
        o.x = __fsub_rn(__fmul_rn(v.x, c.x), __fmul_rn(v.y, c.y));
        o.y = __fadd_rn(__fmul_rn(v.x, c.y), __fmul_rn(v.y, c.x));
        o.z = __fsub_rn(__fmul_rn(v.z, c.z), __fmul_rn(v.w, c.w));
        o.w = __fadd_rn(__fmul_rn(v.z, c.w), __fmul_rn(v.w, c.z));
      }
      float *dst = part == 0 ? q + (size_t)m * att_ch + ch : kv_dst(rd, m, part, head, j);
      *reinterpret_cast<float4 *>(dst) = o;
      return;
    }
    const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i + 1 < 4; i += 2)
      if (i + 1 < cnt) pair(rd, m, n + i, a[i], a[i + 1]);
  }

  __device__ __forceinline__ void store(int m, int n, const float *v, int cnt) const {
    // a staged row needs no descriptor here (RoPE and the append happen in
    // attention)
    const RowDesc rd = kvs ? RowDesc{} : rows[m];
    if (cnt == 16 && (hs & 15) == 0 && (D & 15) == 0) {
      // 16 channels of one head of one part (n is a multiple of 16)
      const int part = n / D;
      const int ch = n - part * D;
      if (ch >= att_ch) return;
      const int head = ch / hs;
      const int j = ch - head * hs;
      float o[16];
      if (part < 2 && !kvs) {
        const float4 *cs = reinterpret_cast<const float4 *>(rope + (size_t)rd.pos * (hs >> 1) + (j >> 1));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 c = cs[i];  // (cos, sin) of two consecutive pairs
          const float a0 = v[4 * i], b0 = v[4 * i + 1], a1 = v[4 * i + 2], b1 = v[4 * i + 3];
          o[4 * i] = __fsub_rn(__fmul_rn(a0, c.x), __fmul_rn(b0, c.y));
          o[4 * i + 1] = __fadd_rn(__fmul_rn(a0, c.y), __fmul_rn(b0, c.x));
          o[4 * i + 2] = __fsub_rn(__fmul_rn(a1, c.z), __fmul_rn(b1, c.w));
          o[4 * i + 3] = __fadd_rn(__fmul_rn(a1, c.w), __fmul_rn(b1, c.z));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = v[i];
      }
      float *dst = part == 0 ? q + (size_t)m * att_ch + ch : kv_dst(rd, m, part, head, j);
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
      return;
    }
#pragma unroll
    for (int i = 0; i + 1 < 16; i += 2)
      if (i + 1 < cnt) pair(rd, m, n + i, v[i], v[i + 1]);
  }
};

// h += C  (residual adds after Wo and W_down, core/cortex.nim:541-542, 550-551)
struct EpiResidual {
  float *h;
  int ld;
  // h as a [M][ld] fp32 tensor, 16 x 32 boxes, 64-byte swizzle: the
  // tensor-core drains add their staged 32-row x 16-column runs into h with
  // TMA reduce-adds (the add happens at L2, the SM does not wait for h)
  CUtensorMap tmap;
  static constexpr bool kTmaReduce = true;
  static constexpr bool kTmaStore = false;
  using Pre = float4;
  struct Row {};
  __device__ __forceinline__ Row row(int) const { return Row{}; }
  __device__ __forceinline__ void prefetch(int m, int n, int cols) const {
    const char *p = reinterpret_cast<const char *>(h + (size_t)m * ld + n);
    for (int b = 0; b < cols * 4; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + b));
  }
  __device__ __forceinline__ Pre load4(int m, int n, int cnt) const {
    const float *p = h + (size_t)m * ld + n;
    if (cnt == 4 && (ld & 3) == 0) return __ldcg(reinterpret_cast<const float4 *>(p));
    return make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __device__ __forceinline__ void store4(int m, int n, float4 v, int cnt, Pre pre, Row) const {
    float *p = h + (size_t)m * ld + n;
    if (cnt == 4 && (ld & 3) == 0) {
      float4 o = pre;
      o.x = __fadd_rn(o.x, v.x);
      o.y = __fadd_rn(o.y, v.y);
      o.z = __fadd_rn(o.z, v.z);
      o.w = __fadd_rn(o.w, v.w);
      *reinterpret_cast<float4 *>(p) = o;
      return;
    }
    const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < cnt) p[i] = __fadd_rn(p[i], a[i]);
  }
  __device__ __forceinline__ void store(int m, int n, const float *v, int cnt) const {
    float *p = h + (size_t)m * ld + n;
    if (cnt == 16 && (ld & 3) == 0) {
      float4 o[4];  // all four loads in flight before any store
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = __ldcg(reinterpret_cast<const float4 *>(p + 4 * i));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[i].x = __fadd_rn(o[i].x, v[4 * i]);
        o[i].y = __fadd_rn(o[i].y, v[4 * i + 1]);
        o[i].z = __fadd_rn(o[i].z, v[4 * i + 2]);
        o[i].w = __fadd_rn(o[i].w, v[4 * i + 3]);
        *reinterpret_cast<float4 *>(p + 4 * i) = o[i];
      }
    } else {
      // partial runs (the GEMV's row pairs): a reduction at L2 instead of a
      // load the thread would wait for; each element has this one addend, so
      // h + v is rounded once, as in the loaded form (the atomic flushes
      // subnormal sums to zero)
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < cnt) atomicAdd(p + i, v[i]);
    }
  }
};

// u = SiLU(C) = C * (1 / (1 + exp(-C)))  (core/cortex.nim:545-548).  A bf16
// u (the BF16 tensor-core mode) is rounded to 8 bits of mantissa, so there
// the exponential and the quotient are the hardware approximations (a few
// fp32 ulps, far below the bf16 rounding); an fp32 u keeps the IEEE steps.
template <typename TA>
struct EpiSilu {
  TA *u;
  int ld;
  __device__ static __forceinline__ float silu(float x) {
    if constexpr (sizeof(TA) == 2) return __fdividef(x, __fadd_rn(1.0f, __expf(-x)));
    return __fmul_rn(x, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))));
  }
  static constexpr bool kTmaReduce = false;
  static constexpr bool kTmaStore = false;
  struct Pre {};
  struct Row {};
  __device__ __forceinline__ Row row(int) const { return Row{}; }
  __device__ __forceinline__ void prefetch(int, int, int) const {}
  __device__ __forceinline__ Pre load4(int, int, int) const { return Pre{}; }
  __device__ __forceinline__ void store4(int m, int n, float4 v, int cnt, Pre, Row) const {
    TA *p = u + (size_t)m * ld + n;
    if (cnt == 4 && (ld & 3) == 0) {
      if constexpr (sizeof(TA) == 2) {
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(silu(v.x), silu(v.y));
        const __nv_bfloat162 h1 = __floats2bfloat162_rn(silu(v.z), silu(v.w));
        *reinterpret_cast<uint2 *>(p) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
      } else {
        *reinterpret_cast<float4 *>(p) = make_float4(silu(v.x), silu(v.y), silu(v.z), silu(v.w));
      }
      return;
    }
    const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < cnt) ActIO<TA>::store(p + i, silu(a[i]));
  }
  __device__ __forceinline__ void store(int m, int n, const float *v, int cnt) const {
    TA *p = u + (size_t)m * ld + n;
    if (cnt == 16 && (ld & 15) == 0) {
      if constexpr (sizeof(TA) == 2) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(silu(v[2 * i]), silu(v[2 * i + 1]));
          w[i] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        reinterpret_cast<uint4 *>(p)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4 *>(p)[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4 *>(p + i) = make_float4(silu(v[i]), silu(v[i + 1]), silu(v[i + 2]), silu(v[i + 3]));
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < cnt) ActIO<TA>::store(p + i, silu(v[i]));
  }
};

// logits[out slot][n] = C  (core/cortex.nim:555-561)
struct EpiLogits {
  float *logits;
  const int2 *outrows;  // chunk-local logits row -> (chunk row, slot)
  long long ld;
  static constexpr bool kTmaReduce = false;
  static constexpr bool kTmaStore = false;
  struct Pre {};
  using Row = int;
  __device__ __forceinline__ Row row(int m) const { return outrows[m].y; }
  __device__ __forceinline__ void prefetch(int, int, int) const {}
  __device__ __forceinline__ Pre load4(int, int, int) const { return Pre{}; }
  __device__ __forceinline__ void store4(int m, int n, float4 v, int cnt, Pre, int orow) const {
    float *p = logits + (size_t)orow * ld + n;
    if (cnt == 4 && (ld & 3) == 0) {
      *reinterpret_cast<float4 *>(p) = v;
      return;
    }
    const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < cnt) p[i] = a[i];
  }
  __device__ __forceinline__ void store(int m, int n, const float *v, int cnt) const {
    float *p = logits + (size_t)outrows[m].y * ld + n;
    if (cnt == 16 && (ld & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < cnt) p[i] = v[i];
    }
  }
};

// ---- the training step's products on the tensor cores (train.cu) ----
//
// C = acc, C = R + acc (a residual into a new buffer), the MLP's SiLU (fin =
// acc and fout = SiLU(acc)) and its derivative (C = acc * s (1 + x (1 - s)),
// s = 1 / (1 + exp(-x)), x = fin; core/cortex.nim:678-681), row-major with
// leading dimension ld, in the reference's float operations.
struct EpiTrain {
  enum Kind { kStore = 0, kAdd = 1, kSilu = 2, kSiluBack = 3 };
  int kind;
  float *C;         // output (fin for kSilu)
  float *C2;        // fout (kSilu)
  const float *R;   // residual (kAdd) or fin (kSiluBack)
  long long ld;
  static constexpr bool kTmaReduce = false;
  static constexpr bool kTmaStore = false;
  using Pre = float4;
  struct Row {};
  __device__ __forceinline__ Row row(int) const { return Row{}; }
  __device__ __forceinline__ void prefetch(int, int, int) const {}
  __device__ __forceinline__ Pre load4(int m, int n, int cnt) const {
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kind == kAdd || kind == kSiluBack) {
      const float *p = R + (size_t)m * ld + n;
      if (cnt == 4 && (ld & 3) == 0) return __ldg(reinterpret_cast<const float4 *>(p));
      r.x = p[0];
      if (cnt > 1) r.y = p[1];
      if (cnt > 2) r.z = p[2];
      if (cnt > 3) r.w = p[3];
    }
    return r;
  }
  __device__ static __forceinline__ float silu(float x) {
    return __fmul_rn(x, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))));
  }
  __device__ static __forceinline__ float silu_back(float d, float x) {
    const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    return __fmul_rn(d, __fmul_rn(s, __fadd_rn(1.0f, __fmul_rn(x, __fsub_rn(1.0f, s)))));
  }
  __device__ __forceinline__ void store4(int m, int n, float4 v, int cnt, Pre pre, Row) const {
    float a[4] = {v.x, v.y, v.z, v.w};
    const float r[4] = {pre.x, pre.y, pre.z, pre.w};
    float b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (kind == kAdd) a[i] = __fadd_rn(r[i], a[i]);
      if (kind == kSiluBack) a[i] = silu_back(a[i], r[i]);
      b[i] = kind == kSilu ? silu(a[i]) : 0.f;
    }
    float *p = C + (size_t)m * ld + n;
    float *q = C2 + (size_t)m * ld + n;
    if (cnt == 4 && (ld & 3) == 0) {
      *reinterpret_cast<float4 *>(p) = make_float4(a[0], a[1], a[2], a[3]);
      if (kind == kSilu) *reinterpret_cast<float4 *>(q) = make_float4(b[0], b[1], b[2], b[3]);
      return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < cnt) {
        p[i] = a[i];
        if (kind == kSilu) q[i] = b[i];
      }
  }
  __device__ __forceinline__ void store(int, int, const float *, int) const {}
};

}  // namespace snai
