// train.cu - the training step of core/cortex.nim:565-822 on sm_100a.
//
// cortex_train_step runs one sequence of `act` = min(n, ctx) tokens: a
// forward pass over all positions at once that keeps every activation the
// backward pass needs, the softmax cross-entropy of every position, BPTT,
// the global gradient-norm clip (core/cortex.nim:230-258) and Adam
// (:145-207).  The reference walks the positions one at a time; the only
// thing that crosses positions is attention, whose backward pass is the
// transposed products dK = dS^T Q and dV = P^T dO, so here every step is a
// GEMM over all positions (positions are GEMM rows) plus row kernels:
//
//   forward, per layer l (rows = positions 0..act-1):
//     na   = RMSNorm(hid_l, rms_att)            qkv = na Wqkv^T, RoPE on q, k
//     S_h  = Q_h K_h^T (causal tiles)           P = softmax(S / sqrtf(hs)), max from -9999
//     att_h = P_h V_h                           hf = hid_l + att Wo^T
//     nf   = RMSNorm(hf, rms_ffn)               fin = nf Wup^T, fout = SiLU(fin)
//     hid_{l+1} = hf + fout Wdown^T
//   nfinal = RMSNorm(hid_L, rms_final), logits = nfinal Wout^T,
//   p = softmax (max from -9999), loss_i = -ln(p[target] + 1e-7), dlogits = p - onehot
//   backward: the transposes of each product (dX = dY W as an NN GEMM, the
//   weight gradient dY^T X as a TN GEMM), the SiLU derivative in the epilogue
//   of dffn, attention from the recomputed scores (multiplied by 1/sqrtf(hs),
//   as the reference's backward does), RMSNorm backward per row with the
//   weight gradient summed over positions by a deterministic two-level sum,
//   inverse RoPE on dq, dk, and the embedding gradient summed per token in
//   descending position order, as the reference adds it.
//
// Precision: FP32 engines compute in fp32 throughout, as the reference (every
// GEMM an fp32 SIMT GEMM with fp32 accumulation; only the summation order
// differs from the reference's sequential sums).  TF32 and BF16 engines run
// the projections' products on the TF32 tensor cores (fp32 operands, fp32
// accumulation); everything else stays fp32.  Adam is element-wise and
// rounds exactly as the reference (IEEE division and square root), so given
// the same gradients and clip factor its result is bit-for-bit the
// reference's.
//
// Every gradient is written (not accumulated) by exactly one kernel per step,
// except the embedding gradient, which is zeroed first; gradients, the Adam
// moments and the weights share one layout (the engine's weight block), so
// the clip and Adam are single passes over the whole block.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "common.cuh"
#include "engine.h"
#include "epilogue.cuh"

namespace snai {

// ============================================================================
// fp32 SIMT GEMM, three operand layouts, batched, with causal tile limits
// ============================================================================
//
// C(m, n) = sum_k A(m, k) B(n, k) over a 128 x 128 (or 128 x 64) tile per
// CTA, 256 threads, 8 x 8 (8 x 4) outputs per thread (rows ty*4..+3 and
// 64+ty*4..+3, columns tx*4..+3 and 64+tx*4..+3, so every shared-memory read
// is a broadcast or a conflict-free float4), k in steps of 8 through a
// two-stage shared-memory ring fed from registers.
//   A_KC: A stored [m][k] (k contiguous), else [k][m] (m contiguous)
//   B_KC: B stored [n][k] (k contiguous), else [k][n] (n contiguous)
// so NT (X W^T) is <true, true>, NN (dY W) is <true, false> and TN (dY^T X)
// is <false, false>.
// VEC: every operand row start is 16-byte aligned and a float4 that starts
// inside an operand's contiguous extent may read up to three elements past it
// (allocated, finite: the buffers are padded); otherwise scalar loads.
// causal: 1 skips tiles with n0 > m0 + 127 (scores of later positions);
// 2 ends k at m0 + 128 (A(m, k) = 0 for k > m); 3 starts k at m0 (A(m, k) = 0
// for k < m).
constexpr int kGBM = 128, kGBK = 8, kGThreads = 256;  // tile rows, k step, threads (tile width: 128 or 64)
constexpr int kGLd = kGBM + 4;  // shared row stride: the transposing stores of the two k halves hit distinct banks

struct GemmArgs {
  int M, N, K;
  const float *A;
  long long lda, sA;  // row stride, batch stride (elements)
  const float *B;
  long long ldb, sB;
  int causal;
  int splits = 1, kchunk = 0;  // split-K: blockIdx.z = batch * splits + split; split s takes k in [s kchunk, (s+1) kchunk)
};

// Stores v[0..cnt) at p (a float4 store when it can).
__device__ __forceinline__ void store_run(float *p, const float *v, int cnt) {
  if (cnt == 4 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    for (int i = 0; i < cnt; ++i) p[i] = v[i];
  }
}

struct SimtStore {  // C = acc
  float *C;
  long long ldc, sC;
  __device__ __forceinline__ void operator()(int z, int m, int n, const float *v, int cnt) const {
    store_run(C + z * sC + (long long)m * ldc + n, v, cnt);
  }
};

struct SimtAdd {  // C = R + acc (a residual into a new buffer)
  float *C;
  const float *R;
  long long ld;
  __device__ __forceinline__ void operator()(int, int m, int n, const float *v, int cnt) const {
    const float *r = R + (long long)m * ld + n;
    float o[4];
    for (int i = 0; i < cnt; ++i) o[i] = __fadd_rn(r[i], v[i]);
    store_run(C + (long long)m * ld + n, o, cnt);
  }
};

// fin = acc, fout = fin * (1 / (1 + exp(-fin)))  (core/cortex.nim:624-627)
struct SimtSilu {
  float *fin, *fout;
  long long ld;
  __device__ __forceinline__ void operator()(int, int m, int n, const float *v, int cnt) const {
    float o[4];
    for (int i = 0; i < cnt; ++i) o[i] = __fmul_rn(v[i], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[i]))));
    store_run(fin + (long long)m * ld + n, v, cnt);
    store_run(fout + (long long)m * ld + n, o, cnt);
  }
};

// dffn = acc * (sig * (1 + x * (1 - sig))), sig = 1 / (1 + exp(-x)), x = fin  (:678-681)
struct SimtSiluBack {
  float *C;
  const float *X;
  long long ld;
  __device__ __forceinline__ void operator()(int, int m, int n, const float *v, int cnt) const {
    const float *x = X + (long long)m * ld + n;
    float o[4];
    for (int i = 0; i < cnt; ++i) {
      const float xv = x[i];
      const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-xv)));
      const float f = __fmul_rn(sig, __fadd_rn(1.0f, __fmul_rn(xv, __fsub_rn(1.0f, sig))));
      o[i] = __fmul_rn(v[i], f);
    }
    store_run(C + (long long)m * ld + n, o, cnt);
  }
};

template <bool A_KC, bool B_KC, bool VEC, int BN, class Epi>
__global__ void __launch_bounds__(kGThreads, 2) snai_train_sgemm(const GemmArgs g, const Epi epi) {
  constexpr int NH = BN / 64;       // 64-column halves of the tile
  constexpr int BLd = BN + 4;       // B's shared row stride
  __shared__ __align__(16) float As[2][kGBK][kGLd];
  __shared__ __align__(16) float Bs[2][kGBK][BLd];
  const int z = blockIdx.z;  // the epilogue's batch index (batch * splits + split when split)
  const int zb = z / g.splits, sp = z % g.splits;
  const int m0 = blockIdx.y * kGBM, n0 = blockIdx.x * BN;
  if (g.causal == 1 && n0 > m0 + kGBM - 1) return;
  const float *__restrict__ A = g.A + zb * g.sA;
  const float *__restrict__ B = g.B + zb * g.sB;
  int kb = 0, ke = g.K;
  if (g.causal == 2) ke = min(g.K, m0 + kGBM);
  if (g.causal == 3) kb = min(m0, g.K);
  if (g.splits > 1) {  // kchunk is a multiple of kGBK, so every split starts on a tile
    kb = max(kb, sp * g.kchunk);
    ke = min(ke, (sp + 1) * g.kchunk);
  }
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

  // one float4 (or four scalars) per operand of width W per k step
  // [r][k] operand: r = tid >> 1, k = (tid & 1) * 4 (threads with r < W);
  // [k][r] operand: k = tid / (W / 4), r = (tid % (W / 4)) * 4 (threads with k < kGBK)
  auto load = [&](const float *__restrict__ P, long long ld, int r0, int R, bool kc, int k0, int W) -> float4 {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kc) {
      if ((tid >> 1) >= W) return v;
      const int r = r0 + (tid >> 1), k = k0 + (tid & 1) * 4;
      if (r < R) {
        const float *p = P + (long long)r * ld + k;
        if (VEC) {
          if (k < ke) v = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
          if (k < ke) v.x = __ldg(p);
          if (k + 1 < ke) v.y = __ldg(p + 1);
          if (k + 2 < ke) v.z = __ldg(p + 2);
          if (k + 3 < ke) v.w = __ldg(p + 3);
        }
      }
    } else {
      const int q = W / 4;
      if (tid / q >= kGBK) return v;
      const int k = k0 + tid / q, r = r0 + (tid % q) * 4;
      if (k < ke && r < R) {
        const float *p = P + (long long)k * ld + r;
        if (VEC) {
          v = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
          v.x = __ldg(p);
          if (r + 1 < R) v.y = __ldg(p + 1);
          if (r + 2 < R) v.z = __ldg(p + 2);
          if (r + 3 < R) v.w = __ldg(p + 3);
        }
      }
    }
    return v;
  };
  auto store = [&](float *S, int ld, float4 v, bool kc, int W) {
    if (kc) {
      if ((tid >> 1) >= W) return;
      const int r = tid >> 1, k = (tid & 1) * 4;
      S[k * ld + r] = v.x;
      S[(k + 1) * ld + r] = v.y;
      S[(k + 2) * ld + r] = v.z;
      S[(k + 3) * ld + r] = v.w;
    } else {
      const int q = W / 4;
      if (tid / q >= kGBK) return;
      *reinterpret_cast<float4 *>(&S[(tid / q) * ld + (tid % q) * 4]) = v;
    }
  };

  float acc[8][4 * NH];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4 * NH; ++j) acc[i][j] = 0.f;

  const int nt = ke > kb ? (ke - kb + kGBK - 1) / kGBK : 0;
  if (nt > 0) {
    store(&As[0][0][0], kGLd, load(A, g.lda, m0, g.M, A_KC, kb, kGBM), A_KC, kGBM);
    store(&Bs[0][0][0], BLd, load(B, g.ldb, n0, g.N, B_KC, kb, BN), B_KC, BN);
  }
  __syncthreads();
  for (int t = 0; t < nt; ++t) {
    const int cur = t & 1;
    float4 na = make_float4(0.f, 0.f, 0.f, 0.f), nb = na;
    if (t + 1 < nt) {
      na = load(A, g.lda, m0, g.M, A_KC, kb + (t + 1) * kGBK, kGBM);
      nb = load(B, g.ldb, n0, g.N, B_KC, kb + (t + 1) * kGBK, BN);
    }
#pragma unroll
    for (int kk = 0; kk < kGBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[cur][kk][64 + ty * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float b[4 * NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float4 bh = *reinterpret_cast<const float4 *>(&Bs[cur][kk][h * 64 + tx * 4]);
        b[4 * h] = bh.x;
        b[4 * h + 1] = bh.y;
        b[4 * h + 2] = bh.z;
        b[4 * h + 3] = bh.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4 * NH; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < nt) {
      store(&As[cur ^ 1][0][0], kGLd, na, A_KC, kGBM);
      store(&Bs[cur ^ 1][0][0], BLd, nb, B_KC, BN);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= g.M) continue;
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const int n = n0 + h * 64 + tx * 4;
      if (n >= g.N) continue;
      const int cnt = min(4, g.N - n);
      epi(z, m, n, &acc[i][h * 4], cnt);
    }
  }
}

// Split-K: C = sum over splits s of P[z][s] (in split order), then the
// GEMM's epilogue; P is [batch][splits][M][N].
template <class Epi>
__global__ void __launch_bounds__(256) snai_train_splitk_reduce(const float *__restrict__ P, int splits, int M, int N,
                                                               int batch, const Epi epi) {
  const int N4 = (N + 3) / 4;
  const long long total = (long long)batch * M * N4;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const int z = (int)(i / ((long long)M * N4));
    const long long r = i % ((long long)M * N4);
    const int m = (int)(r / N4), n = (int)(r % N4) * 4;
    const int cnt = min(4, N - n);
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < splits; ++s) {
      const float *p = P + (((size_t)z * splits + s) * M + m) * (size_t)N + n;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < cnt) v[j] = __fadd_rn(v[j], p[j]);
    }
    epi(z, m, n, v, cnt);
  }
}

// ============================================================================
// row kernels
// ============================================================================

constexpr int kRowThreads = 256;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block sum / max over kRowThreads threads (all threads get the result).
__device__ __forceinline__ float block_sum_f(float v, float *red) {
  v = warp_sum_f(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kRowThreads / 32; ++w) t = __fadd_rn(t, red[w]);
  __syncthreads();
  return t;
}
__device__ __forceinline__ float block_max_f(float v, float *red) {
  v = warp_max_f(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < kRowThreads / 32; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// 1 / sqrt(ss / D + 1e-5) in the reference's float operations (core/cortex.nim:121).
__device__ __forceinline__ float train_rms_inv(float ss, int D) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
}

// hid0[i] = emb[tok[i]] with ids outside [0, V) reading row 0 (:592-600).
__global__ void __launch_bounds__(kRowThreads) snai_train_embed(const int *__restrict__ tok, const float *__restrict__ emb,
                                                               float *__restrict__ out, int V, int D) {
  const int i = blockIdx.x;
  int t = tok[i];
  if (t < 0 || t >= V) t = 0;
  const float4 *s = reinterpret_cast<const float4 *>(emb + (size_t)t * D);
  float4 *d = reinterpret_cast<float4 *>(out + (size_t)i * D);
  for (int k = threadIdx.x; k < D / 4; k += kRowThreads) d[k] = s[k];
}

// out[i] = x[i] * inv * w (applyRMSNorm, :117-123), one row per CTA.
__global__ void __launch_bounds__(kRowThreads) snai_train_rmsnorm(const float *__restrict__ x, const float *__restrict__ w,
                                                                 float *__restrict__ out, int D) {
  __shared__ float red[kRowThreads / 32];
  const float *xr = x + (size_t)blockIdx.x * D;
  float s = 0.f;
  for (int k = threadIdx.x; k < D; k += kRowThreads) s = __fmaf_rn(xr[k], xr[k], s);
  const float inv = train_rms_inv(block_sum_f(s, red), D);
  float *o = out + (size_t)blockIdx.x * D;
  for (int k = threadIdx.x; k < D; k += kRowThreads) o[k] = __fmul_rn(__fmul_rn(xr[k], inv), w[k]);
}

// RoPE (applyRoPE, :74-87) of channels [0, 2D) of the [M, ld] rows (q and k),
// row i at position i; every head of D / hs is rotated, as the reference does.
// sign -1 rotates backwards (the backward pass, :786-787).
__global__ void snai_train_rope(float *__restrict__ x, long long ld, int M, int D, int hs, const float2 *__restrict__ rope,
                                float sign) {
  const int i = blockIdx.y;
  const int nh = D / hs, half = hs / 2;
  const int pairs = 2 * nh * half;  // q and k
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
    const int part = p / (nh * half), r = p % (nh * half);
    const int h = r / half, j = r % half;
    float *v = x + (long long)i * ld + (long long)part * D + h * hs + 2 * j;
    const float2 cs = rope[(size_t)i * half + j];
    const float c = cs.x, s = __fmul_rn(sign, cs.y);
    const float v0 = v[0], v1 = v[1];
    v[0] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    v[1] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
  }
}

// Forward softmax of row i of head h (:515-534): s_t = S[t] / sqrtf(hs) for
// t <= i, max from -9999, e_t = exp(s_t - max), w_t = e_t / sum; zeros for
// i < t < ldS.  One warp per row.
__global__ void snai_train_softmax_fwd(float *__restrict__ S, int M, int ldS, float sqrt_hs) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int i = warp;
  float *row = S + ((size_t)blockIdx.y * M + i) * ldS;
  float mx = -9999.0f;
  for (int t = lane; t <= i; t += 32) {
    const float s = __fdiv_rn(row[t], sqrt_hs);
    row[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max_f(mx);
  float sum = 0.f;
  for (int t = lane; t <= i; t += 32) {
    const float e = expf(__fsub_rn(row[t], mx));
    row[t] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = warp_sum_f(sum);
  for (int t = lane; t < ldS; t += 32) row[t] = t <= i ? __fdiv_rn(row[t], sum) : 0.f;
}

// Backward softmax of row i of head h (:712-746): w_t from the recomputed
// scores S'[t] * (1 / sqrtf(hs)) (max from -9999), sum_w_dw = sum_t w_t dP[t],
// dS[t] = w_t (dP[t] - sum_w_dw) * scale.  S' becomes w, dP becomes dS;
// zeros for i < t < ldS.  One warp per row.
__global__ void snai_train_softmax_bwd(float *__restrict__ S, float *__restrict__ dP, int M, int ldS, float scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int i = warp;
  const size_t off = ((size_t)blockIdx.y * M + i) * ldS;
  float *row = S + off, *drow = dP + off;
  float mx = -9999.0f;
  for (int t = lane; t <= i; t += 32) {
    const float s = __fmul_rn(row[t], scale);
    row[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max_f(mx);
  float sum = 0.f;
  for (int t = lane; t <= i; t += 32) {
    const float e = expf(__fsub_rn(row[t], mx));
    row[t] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = warp_sum_f(sum);
  float swd = 0.f;
  for (int t = lane; t <= i; t += 32) {
    const float w = __fdiv_rn(row[t], sum);
    row[t] = w;
    swd = __fadd_rn(swd, __fmul_rn(w, drow[t]));
  }
  swd = warp_sum_f(swd);
  for (int t = lane; t < ldS; t += 32) {
    if (t <= i) {
      drow[t] = __fmul_rn(__fmul_rn(row[t], __fsub_rn(drow[t], swd)), scale);
    } else {
      row[t] = 0.f;
      drow[t] = 0.f;
    }
  }
}

// Logits row i -> probabilities (max from -9999, exp, sum, divide; :606-615),
// loss_i = -ln(p[target] + 1e-7) (:616) and dlogits = p - onehot(target)
// (:624-625) in place; the row's padding [V, Vp) is zeroed.
__global__ void __launch_bounds__(kRowThreads) snai_train_xent(float *__restrict__ L, int V, int Vp,
                                                              const int *__restrict__ tgt, float *__restrict__ loss) {
  __shared__ float red[kRowThreads / 32];
  __shared__ float ptg;
  float *row = L + (size_t)blockIdx.x * Vp;
  int tg = tgt[blockIdx.x];
  if (tg < 0 || tg >= V) tg = 0;
  float mx = -9999.0f;
  for (int v = threadIdx.x; v < V; v += kRowThreads) mx = fmaxf(mx, row[v]);
  mx = block_max_f(mx, red);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += kRowThreads) {
    const float e = expf(__fsub_rn(row[v], mx));
    row[v] = e;
    s = __fadd_rn(s, e);
  }
  const float sum = block_sum_f(s, red);
  for (int v = threadIdx.x; v < Vp; v += kRowThreads) {
    if (v < V) {
      const float p = __fdiv_rn(row[v], sum);
      if (v == tg) {
        ptg = p;
        row[v] = __fsub_rn(p, 1.0f);
      } else {
        row[v] = p;
      }
    } else {
      row[v] = 0.f;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) loss[blockIdx.x] = -logf(__fadd_rn(ptg, 1e-7f));
}

// total = sum_i loss_i in position order, out = total / act (:616, :821).
__global__ void snai_train_loss_sum(const float *__restrict__ loss, int act, float *__restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float t = 0.f;
  for (int i = 0; i < act; ++i) t = __fadd_rn(t, loss[i]);
  out[0] = __fdiv_rn(t, (float)act);
}

// applyRMSNormBackwardAcc (:125-143) on row i: dn (the gradient of the norm's
// output) and a (its input) give dx; dh = dx (first) or dh + dx; gprod[i] =
// dn * nx for the weight gradient.
__global__ void __launch_bounds__(kRowThreads) snai_train_rmsnorm_bwd(const float *__restrict__ dn,
                                                                     const float *__restrict__ a,
                                                                     const float *__restrict__ w, int D,
                                                                     float *__restrict__ dh, int first,
                                                                     float *__restrict__ gprod) {
  __shared__ float red[kRowThreads / 32];
  const size_t off = (size_t)blockIdx.x * D;
  const float *ar = a + off, *dr = dn + off;
  float s = 0.f;
  for (int k = threadIdx.x; k < D; k += kRowThreads) s = __fmaf_rn(ar[k], ar[k], s);
  const float inv = train_rms_inv(block_sum_f(s, red), D);
  float sd = 0.f;
  for (int k = threadIdx.x; k < D; k += kRowThreads)
    sd = __fadd_rn(sd, __fmul_rn(__fmul_rn(dr[k], w[k]), __fmul_rn(ar[k], inv)));
  const float mean = __fdiv_rn(block_sum_f(sd, red), (float)D);
  for (int k = threadIdx.x; k < D; k += kRowThreads) {
    const float nx = __fmul_rn(ar[k], inv);
    gprod[off + k] = __fmul_rn(dr[k], nx);
    const float dx = __fmul_rn(__fsub_rn(__fmul_rn(dr[k], w[k]), __fmul_rn(nx, mean)), inv);
    dh[off + k] = first ? dx : __fadd_rn(dh[off + k], dx);
  }
}

// g[d] = sum over rows i of gprod[i][d] (the RMSNorm weight gradient summed
// over positions), deterministic in two launches: CTA (c, r) sums the rows of
// chunk r for 32 columns (8 row slices combined in slice order) into
// part[r][d]; then the chunks are added in chunk order.
constexpr int kColChunks = 32;

__global__ void __launch_bounds__(256) snai_train_colsum_part(const float *__restrict__ gprod, int M, int D,
                                                             float *__restrict__ part) {
  __shared__ float red[8][33];
  const int d = blockIdx.x * 32 + threadIdx.x, r = blockIdx.y;
  const int rows = (M + kColChunks - 1) / kColChunks, i0 = r * rows, i1 = min(M, i0 + rows);
  float s = 0.f;
  if (d < D)
    for (int i = i0 + threadIdx.y; i < i1; i += 8) s = __fadd_rn(s, gprod[(size_t)i * D + d]);
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && d < D) {
    float t = 0.f;
    for (int y = 0; y < 8; ++y) t = __fadd_rn(t, red[y][threadIdx.x]);
    part[(size_t)r * D + d] = t;
  }
}

__global__ void snai_train_colsum_fin(const float *__restrict__ part, int D, float *__restrict__ g) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
#pragma unroll 8
  for (int r = 0; r < kColChunks; ++r) s = __fadd_rn(s, part[(size_t)r * D + d]);
  g[d] = s;
}

// Token links of the sequence: prev[i] = the last position j < i holding the
// same (clamped) token, or -1; last[i] = 1 when no later position holds it.
// One CTA; the first kLinkMax clamped ids are staged in shared memory.
constexpr int kLinkMax = 8192;

__global__ void __launch_bounds__(1024) snai_train_tok_links(const int *__restrict__ tok, int act, int V,
                                                            int *__restrict__ prev, int *__restrict__ last) {
  __shared__ int ids[kLinkMax];
  auto clamp = [&](int t) { return (t < 0 || t >= V) ? 0 : t; };
  for (int i = threadIdx.x; i < act && i < kLinkMax; i += blockDim.x) ids[i] = clamp(tok[i]);
  __syncthreads();
  auto id = [&](int j) { return j < kLinkMax ? ids[j] : clamp(tok[j]); };
  for (int i = threadIdx.x; i < act; i += blockDim.x) {
    const int t = id(i);
    int p = -1;
    for (int j = i - 1; j >= 0; --j)
      if (id(j) == t) {
        p = j;
        break;
      }
    prev[i] = p;
    int l = 1;
    for (int j = i + 1; j < act; ++j)
      if (id(j) == t) {
        l = 0;
        break;
      }
    last[i] = l;
  }
}

// g_emb[tok] += dh[i] over positions i in descending order (:817-818): the
// CTA of the last position holding a token walks that token's positions
// backwards through prev and sums their rows in that order.
__global__ void __launch_bounds__(kRowThreads) snai_train_emb_grad(const float *__restrict__ dh, const int *__restrict__ tok,
                                                                  const int *__restrict__ prev,
                                                                  const int *__restrict__ last, int V, int D,
                                                                  float *__restrict__ gemb) {
  const int i = blockIdx.x;
  if (!last[i]) return;
  int t = tok[i];
  if (t < 0 || t >= V) t = 0;
  float *g = gemb + (size_t)t * D;
  for (int k = threadIdx.x; k < D; k += kRowThreads) {
    float s = g[k];
    for (int j = i; j >= 0; j = prev[j]) s = __fadd_rn(s, dh[(size_t)j * D + k]);
    g[k] = s;
  }
}

// K (rotated) and V of positions 0..act-1, heads < H, into slot 0's cache:
// the reference's training forward writes its KV cache rows (:509-510).
__global__ void snai_train_kv_publish(const float *__restrict__ qkv, long long ld, int act, int D, int H, int hs,
                                      float *__restrict__ kv, size_t part_stride, size_t head_stride) {
  const int i = blockIdx.x;
  for (int c = threadIdx.x; c < 2 * H * hs; c += blockDim.x) {
    const int part = c / (H * hs), r = c % (H * hs), h = r / hs, j = r % hs;
    kv[part * part_stride + h * head_stride + (size_t)i * hs + j] = qkv[(long long)i * ld + (1 + part) * D + h * hs + j];
  }
}

// out[c][r] = in[r][c] for r < R, c < C, and out[c][r] = 0 for R <= r < Rp:
// the K-major operands of the tensor-core form of the NN and TN products
// (32 x 32 tiles through shared memory, both sides coalesced).
__global__ void __launch_bounds__(256) snai_train_transpose(const float *__restrict__ in, long long ldi, int R, int C,
                                                           float *__restrict__ out, int Rp) {
  __shared__ float t[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int y = threadIdx.y; y < 32; y += 8) {
    const int r = r0 + y, c = c0 + threadIdx.x;
    t[y][threadIdx.x] = (r < R && c < C) ? in[(long long)r * ldi + c] : 0.f;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += 8) {
    const int c = c0 + y, r = r0 + threadIdx.x;
    if (c < C && r < Rp) out[(long long)c * Rp + r] = t[threadIdx.x][y];
  }
}

// ============================================================================
// global-norm clip and Adam over the whole gradient block
// ============================================================================

constexpr int kClipBlocks = 592;  // 4 x 148 SMs

// Partial sums of squares (double) per CTA over g[0..n).
__global__ void __launch_bounds__(kRowThreads) snai_train_sumsq(const float *__restrict__ g, size_t n,
                                                               double *__restrict__ part) {
  __shared__ double red[kRowThreads / 32];
  double s = 0.0;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  const size_t n4 = n / 4;
  for (size_t i = (size_t)blockIdx.x * kRowThreads + threadIdx.x; i < n4; i += (size_t)gridDim.x * kRowThreads) {
    const float4 v = g4[i];
    s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kRowThreads / 32; ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

// clip[0] = the factor, clip[1] = 1 when it applies (clipGlobalGradientNorm
// with max_norm 1: norm NaN or > 1 -> 1 / norm, or 0 when the norm is NaN or
// 0), clip[2] = the norm.
__global__ void snai_train_clip_factor(const double *__restrict__ part, int nparts, float *__restrict__ clip) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double t = 0.0;
  for (int i = 0; i < nparts; ++i) t += part[i];
  const float gn = __fsqrt_rn((float)t);
  const float max_norm = 1.0f;
  const bool nan = gn != gn;
  clip[2] = gn;
  if (nan || gn > max_norm) {
    clip[0] = (nan || gn == 0.0f) ? 0.0f : __fdiv_rn(max_norm, gn);
    clip[1] = 1.0f;
  } else {
    clip[0] = 1.0f;
    clip[1] = 0.0f;
  }
}

struct AdamArgs {
  float *w, *m, *v;
  const float *g;
  size_t n, sparse_end;  // elements [0, sparse_end) follow the sparse rule (the embedding)
  float lr, b1, b2, omb1, omb2, b1t, b2t, scale;
  const float *clip;
};

// adamStep (:145-160) per element, after the clip factor (:255-258).
__device__ __forceinline__ void adam_elem(const AdamArgs &a, size_t i, bool apply, float cf, float g, float &w,
                                          float &m, float &v) {
  float gg = g;
  if (apply) gg = __fmul_rn(gg, cf);
  const float grad = __fdiv_rn(gg, a.scale);
  if (i < a.sparse_end && grad == 0.0f) return;
  if (grad != grad || grad > 9999.0f || grad < -9999.0f) return;
  m = __fadd_rn(__fmul_rn(a.b1, m), __fmul_rn(a.omb1, grad));
  v = __fadd_rn(__fmul_rn(a.b2, v), __fmul_rn(__fmul_rn(a.omb2, grad), grad));
  const float mh = __fdiv_rn(m, a.b1t), vh = __fdiv_rn(v, a.b2t);
  w = __fsub_rn(w, __fdiv_rn(__fmul_rn(a.lr, mh), __fadd_rn(__fsqrt_rn(vh), 1e-8f)));
}

// Four elements per thread (the weight block is a multiple of 64 floats);
// w, m, v are read and written only where the gradient is not zero or the
// element is outside the embedding, as the sparse rule leaves the others.
__global__ void __launch_bounds__(kRowThreads) snai_train_adam(const AdamArgs a) {
  const bool apply = a.clip[1] != 0.0f;
  const float cf = a.clip[0];
  const size_t n4 = a.n / 4;
  const float4 *g4 = reinterpret_cast<const float4 *>(a.g);
  float4 *w4 = reinterpret_cast<float4 *>(a.w), *m4 = reinterpret_cast<float4 *>(a.m),
         *v4 = reinterpret_cast<float4 *>(a.v);
  for (size_t j = (size_t)blockIdx.x * kRowThreads + threadIdx.x; j < n4; j += (size_t)gridDim.x * kRowThreads) {
    const float4 g = __ldcs(g4 + j);
    const size_t i = 4 * j;
    if (i + 4 <= a.sparse_end && g.x == 0.f && g.y == 0.f && g.z == 0.f && g.w == 0.f) continue;
    float4 w = w4[j], m = m4[j], v = v4[j];
    adam_elem(a, i, apply, cf, g.x, w.x, m.x, v.x);
    adam_elem(a, i + 1, apply, cf, g.y, w.y, m.y, v.y);
    adam_elem(a, i + 2, apply, cf, g.z, w.z, m.z, v.z);
    adam_elem(a, i + 3, apply, cf, g.w, w.w, m.w, v.w);
    w4[j] = w;
    m4[j] = m;
    v4[j] = v;
  }
}

// ============================================================================
// host side
// ============================================================================

struct TrainState {
  int cap = 0;      // rows (= ctx)
  int Vp = 0;       // vocab padded to a multiple of 4
  int ldS = 0;      // attention row stride (ctx padded to a multiple of 4)
  void *mom = nullptr;    // Adam first and second moments, each a mirror of the weight block
  void *grad = nullptr;   // gradients, a mirror of the weight block
  void *act = nullptr;    // activations and scratch
  float *m = nullptr, *v = nullptr, *g = nullptr;
  int adam_t = 0;
  int *tin = nullptr, *ttg = nullptr;
  std::vector<float *> hid, na, qkv, att, hf, nf, fin, fout;
  float *nfinal = nullptr, *probs = nullptr, *S = nullptr, *dP = nullptr;
  float *dh = nullptr, *dn = nullptr, *dffn = nullptr, *datt = nullptr, *dqkv = nullptr, *gprod = nullptr;
  float *loss_rows = nullptr, *loss = nullptr, *clip = nullptr, *colpart = nullptr;
  int *prev = nullptr, *last = nullptr;
  double *clip_part = nullptr;
  // tensor-core engines (TF32 / BF16): transposed operands of the NN and TN
  // products -- a weight W^T, dY^T and X^T with the positions padded to Mp
  float *wt = nullptr, *yt = nullptr, *xt = nullptr;
  float *split = nullptr;  // split-K partials
};
constexpr size_t kSplitFloats = size_t(16) << 20;  // 64 MB of split-K partials

namespace {

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Device mirror of a weight pointer inside another block of the same layout.
float *mirror(const Engine &e, void *block, const float *w) {
  return reinterpret_cast<float *>(static_cast<char *>(block) +
                                   (reinterpret_cast<const char *>(w) - static_cast<const char *>(e.wblock)));
}

int launch_rc(const char *what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(err));
    return -1;
  }
  return 0;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <bool A_KC, bool B_KC, int BN, class Epi>
int gemm_bn(Engine &e, const GemmArgs &g0, int batch, const Epi &epi, bool vec) {
  GemmArgs g = g0;
  const int gx = (g.N + BN - 1) / BN, gy = (g.M + kGBM - 1) / kGBM;
  vec = vec && aligned16(g.A) && aligned16(g.B) && g.lda % 4 == 0 && g.ldb % 4 == 0 && g.sA % 4 == 0 && g.sB % 4 == 0;
  const long long tiles = (long long)gx * gy * batch;
  const int sms = device_sm_count(e.device);
  int splits = 1;
  if (e.train && e.train->split && g.causal != 1 && tiles < 2 * sms && g.K >= 1024) {
    splits = (int)std::min<long long>({(2 * sms + tiles - 1) / tiles, (long long)g.K / 256,
                                       (long long)(kSplitFloats / ((size_t)batch * g.M * g.N))});
    if (splits < 2) splits = 1;
  }
  if (splits > 1) {
    g.splits = splits;
    g.kchunk = ((g.K + splits - 1) / splits + kGBK - 1) / kGBK * kGBK;
    const SimtStore part{e.train->split, (long long)g.N, (long long)g.M * g.N};
    const dim3 grid(gx, gy, batch * splits);
    if (vec)
      snai_train_sgemm<A_KC, B_KC, true, BN, SimtStore><<<grid, kGThreads, 0, e.stream>>>(g, part);
    else
      snai_train_sgemm<A_KC, B_KC, false, BN, SimtStore><<<grid, kGThreads, 0, e.stream>>>(g, part);
    const long long n4 = (long long)batch * g.M * ((g.N + 3) / 4);
    const int rb = (int)std::min<long long>((n4 + 255) / 256, (long long)sms * 8);
    snai_train_splitk_reduce<Epi><<<rb, 256, 0, e.stream>>>(e.train->split, splits, g.M, g.N, batch, epi);
    e.launches += 2;
    return launch_rc("training GEMM");
  }
  const dim3 grid(gx, gy, batch);
  if (vec)
    snai_train_sgemm<A_KC, B_KC, true, BN, Epi><<<grid, kGThreads, 0, e.stream>>>(g, epi);
  else
    snai_train_sgemm<A_KC, B_KC, false, BN, Epi><<<grid, kGThreads, 0, e.stream>>>(g, epi);
  e.launches++;
  return launch_rc("training GEMM");
}

// One GEMM launch; VEC when every operand row start is 16-byte aligned.  A
// grid of fewer tiles than twice the SMs with a long k range is split over k
// (partials in `split`, summed in split order by a second launch that runs
// the epilogue), so that every SM gets work.  Products at most 64 columns
// wide (the per-head attention products) take 128 x 64 tiles.
template <bool A_KC, bool B_KC, class Epi>
int gemm(Engine &e, const GemmArgs &g, int batch, const Epi &epi, bool vec) {
  if (g.M <= 0 || g.N <= 0) return 0;
  if (g.N <= 64) return gemm_bn<A_KC, B_KC, 64>(e, g, batch, epi, vec);
  return gemm_bn<A_KC, B_KC, 128>(e, g, batch, epi, vec);
}

GemmArgs args(int M, int N, int K, const float *A, long long lda, const float *B, long long ldb, int causal = 0,
              long long sA = 0, long long sB = 0) {
  GemmArgs g;
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = A;
  g.lda = lda;
  g.sA = sA;
  g.B = B;
  g.ldb = ldb;
  g.sB = sB;
  g.causal = causal;
  return g;
}

}  // namespace

int train_moments(Engine &e) {
  if (!e.train) e.train = new TrainState();
  TrainState &t = *e.train;
  if (t.mom) return 0;
  if (cudaMalloc(&t.mom, 2 * e.wblock_bytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("device allocation of the Adam moments failed (%zu B)", 2 * e.wblock_bytes);
    return -1;
  }
  t.m = static_cast<float *>(t.mom);
  t.v = reinterpret_cast<float *>(static_cast<char *>(t.mom) + e.wblock_bytes);
  cudaMemsetAsync(t.mom, 0, 2 * e.wblock_bytes, e.stream);  // fresh moments are zero (allocShared0)
  return 0;
}

static int train_alloc(Engine &e) {
  if (train_moments(e)) return -1;
  TrainState &t = *e.train;
  if (t.act) return 0;
  const Dims &d = e.d;
  const size_t C = d.ctx, D = d.D, F = d.F, L = d.L;
  t.cap = d.ctx;
  t.Vp = (d.V + 3) / 4 * 4;
  t.ldS = (d.ctx + 3) / 4 * 4;
  std::vector<std::pair<float **, size_t>> items;  // (pointer, floats)
  t.hid.assign(L + 1, nullptr);
  for (auto *v : {&t.na, &t.qkv, &t.att, &t.hf, &t.nf, &t.fin, &t.fout}) v->assign(L, nullptr);
  for (size_t l = 0; l <= L; ++l) items.push_back({&t.hid[l], C * D});
  for (size_t l = 0; l < L; ++l) {
    items.push_back({&t.na[l], C * D});
    items.push_back({&t.qkv[l], C * 3 * D});
    items.push_back({&t.att[l], C * D});
    items.push_back({&t.hf[l], C * D});
    items.push_back({&t.nf[l], C * D});
    items.push_back({&t.fin[l], C * F});
    items.push_back({&t.fout[l], C * F});
  }
  items.push_back({&t.nfinal, C * D});
  items.push_back({&t.probs, C * (size_t)t.Vp});
  items.push_back({&t.S, (size_t)d.heads * C * t.ldS});
  items.push_back({&t.dP, (size_t)d.heads * C * t.ldS});
  items.push_back({&t.dh, C * D});
  items.push_back({&t.dn, C * D});
  items.push_back({&t.dffn, C * F});
  items.push_back({&t.datt, C * D});
  items.push_back({&t.dqkv, C * 3 * D});
  items.push_back({&t.gprod, C * D});
  items.push_back({&t.loss_rows, C});
  items.push_back({&t.loss, 4});
  items.push_back({&t.clip, 4});
  items.push_back({&t.colpart, (size_t)kColChunks * D});
  items.push_back({&t.split, kSplitFloats});
  if (e.precision != kFP32) {
    const size_t Cp = (C + 3) / 4 * 4, Nmax = (std::max({(size_t)d.V, 3 * D, F}) + 3) / 4 * 4;
    items.push_back({&t.wt, Nmax * std::max(D, F)});
    items.push_back({&t.yt, Nmax * Cp});
    items.push_back({&t.xt, std::max(D, F) * Cp});
  }
  size_t off = 0;
  std::vector<size_t> offs;
  for (auto &it : items) {
    offs.push_back(off);
    off = align256(off + it.second * sizeof(float));
  }
  const size_t tok_off = off;
  off = align256(off + 4 * C * sizeof(int));
  const size_t part_off = off;
  off = align256(off + kClipBlocks * sizeof(double));
  if (cudaMalloc(&t.act, off) != cudaSuccess || cudaMalloc(&t.grad, e.wblock_bytes) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(t.act);
    t.act = nullptr;
    set_error("device allocation of the training buffers failed (%zu B + %zu B)", off, e.wblock_bytes);
    return -1;
  }
  char *base = static_cast<char *>(t.act);
  for (size_t i = 0; i < items.size(); ++i) *items[i].first = reinterpret_cast<float *>(base + offs[i]);
  t.tin = reinterpret_cast<int *>(base + tok_off);
  t.ttg = t.tin + C;
  t.prev = t.ttg + C;
  t.last = t.prev + C;
  t.clip_part = reinterpret_cast<double *>(base + part_off);
  t.g = static_cast<float *>(t.grad);
  // zero everything once: columns never written (q/k/v/att channels past
  // heads * hs, padding of the score and logits rows, the weight block's
  // alignment gaps) stay zero
  cudaMemsetAsync(t.act, 0, off, e.stream);
  cudaMemsetAsync(t.grad, 0, e.wblock_bytes, e.stream);
  return launch_rc("training buffers");
}

void train_free(Engine &e) {
  if (!e.train) return;
  cudaFree(e.train->mom);
  cudaFree(e.train->grad);
  cudaFree(e.train->act);
  delete e.train;
  e.train = nullptr;
}

float *train_tensor(Engine &e, int which, const float *w) {
  if (which == 0) {
    if (train_alloc(e)) return nullptr;
    return mirror(e, e.train->grad, w);
  }
  if (train_moments(e)) return nullptr;
  return mirror(e, which == 1 ? static_cast<void *>(e.train->m) : static_cast<void *>(e.train->v), w);
}

int train_adam_steps(const Engine &e) { return e.train ? e.train->adam_t : 0; }

// Forward, loss and backward of one sequence (act >= 1 tokens, host arrays);
// gradients are left in the gradient block; the mean loss goes to *loss_out.
int train_grads(Engine &e, const int *tin, const int *ttg, int act, float *loss_out) {
  if (train_alloc(e)) return -1;
  TrainState &t = *e.train;
  const Dims &d = e.d;
  const int D = d.D, F = d.F, V = d.V, L = d.L, H = d.heads, hs = d.hs, M = act;
  const long long D3 = 3LL * D;
  cudaStream_t st = e.stream;
  int rc = 0;
  rc |= cudaMemcpyAsync(t.tin, tin, sizeof(int) * act, cudaMemcpyHostToDevice, st) != cudaSuccess;
  rc |= cudaMemcpyAsync(t.ttg, ttg, sizeof(int) * act, cudaMemcpyHostToDevice, st) != cudaSuccess;
  // the embedding gradient is accumulated; every other gradient is stored
  rc |= cudaMemsetAsync(mirror(e, t.grad, e.emb), 0, sizeof(float) * (size_t)V * D, st) != cudaSuccess;
  if (rc) {
    set_error("training step: copy to the device failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  const bool hvec = hs % 4 == 0;  // head slices of the q/k/v rows are 16-byte aligned
  const float inv_sqrt = 1.0f / std::sqrt((float)hs);  // the backward's scale (:706), host float as the reference
  const int rw_blocks = (M * 32 + 255) / 256;          // warp-per-row kernels: 8 rows per CTA

  // The projections' three products.  FP32 engines run them as fp32 SIMT
  // GEMMs; TF32 / BF16 engines on the TF32 tensor cores (fp32 operands),
  // whose tiles take K-major operands only, so the NN product uses W^T and
  // the TN product dY^T and X^T (positions padded to Mp with zeros).
  const bool tc = e.precision != kFP32;
  const int Mp = (M + 3) / 4 * 4;
  using ET = EpiTrain;
  auto transpose = [&](const float *in, long long ldi, int R, int Cc, float *out, int Rp) {
    snai_train_transpose<<<dim3((Cc + 31) / 32, (Rp + 31) / 32), dim3(32, 8), 0, st>>>(in, ldi, R, Cc, out, Rp);
    e.launches++;
  };
  // C[M, N] = A[M, K] W[N, K]^T (A rows dense)
  auto nt = [&](int N, int K, const float *A, const float *W, const ET &te, auto simt) -> int {
    if (tc) return train_gemm_tc(e, M, N, K, A, W, te);
    return gemm<true, true>(e, args(M, N, K, A, K, W, K), 1, simt, true);
  };
  // C[M, N] = A[M, K] W[K, N] (W a weight [K, N]; A's rows are K rounded up to 4)
  auto nn = [&](int N, int K, const float *A, long long lda, const float *W, const ET &te, auto simt) -> int {
    if (!tc) return gemm<true, false>(e, args(M, N, K, A, lda, W, N), 1, simt, true);
    const int Kp = (K + 3) / 4 * 4;
    if (lda != Kp) {  // the tensor-core tiles read dense rows
      set_error("training step: NN operand rows of %lld floats, %d expected", lda, Kp);
      return -1;
    }
    transpose(W, N, K, N, t.wt, Kp);
    return train_gemm_tc(e, M, N, Kp, A, t.wt, te);
  };
  // C[R, Cc] = sum over positions i of Y[i][r] X[i][c] (a weight gradient)
  auto tn = [&](int R, int Cc, const float *Y, long long ldy, const float *X, long long ldx, float *C) -> int {
    if (!tc) return gemm<false, false>(e, args(R, Cc, M, Y, ldy, X, ldx), 1, SimtStore{C, Cc, 0}, true);
    transpose(Y, ldy, M, R, t.yt, Mp);
    transpose(X, ldx, M, Cc, t.xt, Mp);
    return train_gemm_tc(e, R, Cc, Mp, t.yt, t.xt, ET{ET::kStore, C, nullptr, nullptr, Cc});
  };

  // ---------------- forward ----------------
  snai_train_embed<<<M, kRowThreads, 0, st>>>(t.tin, e.emb, t.hid[0], V, D);
  e.launches++;
  for (int l = 0; l < L; ++l) {
    const LayerWeights &w = e.layers[l];
    snai_train_rmsnorm<<<M, kRowThreads, 0, st>>>(t.hid[l], w.rms_att, t.na[l], D);
    e.launches++;
    rc |= nt(3 * D, D, t.na[l], w.wqkv, ET{ET::kStore, t.qkv[l], nullptr, nullptr, D3}, SimtStore{t.qkv[l], D3, 0});
    snai_train_rope<<<dim3((D + 255) / 256, M), 256, 0, st>>>(t.qkv[l], D3, M, D, hs,
                                                                                                   e.rope, 1.0f);
    e.launches++;
    // S_h = Q_h K_h^T, then P = softmax
    rc |= gemm<true, true>(e, args(M, M, hs, t.qkv[l], D3, t.qkv[l] + D, D3, 1, hs, hs), H,
                           SimtStore{t.S, t.ldS, (long long)M * t.ldS}, hvec);
    snai_train_softmax_fwd<<<dim3(rw_blocks, H), 256, 0, st>>>(t.S, M, t.ldS, e.sqrt_hs);
    e.launches++;
    // att_h = P_h V_h
    rc |= gemm<true, false>(e, args(M, hs, M, t.S, t.ldS, t.qkv[l] + 2 * D, D3, 2, (long long)M * t.ldS, hs), H,
                            SimtStore{t.att[l], D, hs}, hvec);
    rc |= nt(D, D, t.att[l], w.wo, ET{ET::kAdd, t.hf[l], nullptr, t.hid[l], D}, SimtAdd{t.hf[l], t.hid[l], D});
    snai_train_rmsnorm<<<M, kRowThreads, 0, st>>>(t.hf[l], w.rms_ffn, t.nf[l], D);
    e.launches++;
    rc |= nt(F, D, t.nf[l], w.wup, ET{ET::kSilu, t.fin[l], t.fout[l], nullptr, F}, SimtSilu{t.fin[l], t.fout[l], F});
    rc |= nt(D, F, t.fout[l], w.wdown, ET{ET::kAdd, t.hid[l + 1], nullptr, t.hf[l], D},
             SimtAdd{t.hid[l + 1], t.hf[l], D});
  }
  snai_train_rmsnorm<<<M, kRowThreads, 0, st>>>(t.hid[L], e.rms_final, t.nfinal, D);
  e.launches++;
  rc |= nt(V, D, t.nfinal, e.w_out, ET{ET::kStore, t.probs, nullptr, nullptr, t.Vp}, SimtStore{t.probs, t.Vp, 0});
  snai_train_xent<<<M, kRowThreads, 0, st>>>(t.probs, V, t.Vp, t.ttg, t.loss_rows);
  snai_train_loss_sum<<<1, 32, 0, st>>>(t.loss_rows, M, t.loss);
  e.launches += 2;
  // the reference's training forward leaves its K/V rows in the cache
  for (int l = 0; l < L; ++l) {
    snai_train_kv_publish<<<M, 256, 0, st>>>(t.qkv[l], D3, M, D, H, hs, e.kv + l * e.kv_layer_stride,
                                             e.kv_part_stride, e.kv_head_stride);
    e.launches++;
  }
  if (rc || launch_rc("training forward")) return -1;

  // ---------------- backward ----------------
  auto G = [&](const float *w) { return mirror(e, t.grad, w); };
  auto colsum = [&](float *g) {
    snai_train_colsum_part<<<dim3((D + 31) / 32, kColChunks), dim3(32, 8), 0, st>>>(t.gprod, M, D, t.colpart);
    snai_train_colsum_fin<<<(D + 255) / 256, 256, 0, st>>>(t.colpart, D, g);
    e.launches += 2;
  };
  rc |= nn(D, V, t.probs, t.Vp, e.w_out, ET{ET::kStore, t.dn, nullptr, nullptr, D}, SimtStore{t.dn, D, 0});
  rc |= tn(V, D, t.probs, t.Vp, t.nfinal, D, G(e.w_out));
  snai_train_rmsnorm_bwd<<<M, kRowThreads, 0, st>>>(t.dn, t.hid[L], e.rms_final, D, t.dh, 1, t.gprod);
  e.launches++;
  colsum(G(e.rms_final));
  for (int l = L - 1; l >= 0; --l) {
    const LayerWeights &w = e.layers[l];
    // MLP
    rc |= nn(F, D, t.dh, D, w.wdown, ET{ET::kSiluBack, t.dffn, nullptr, t.fin[l], F},
             SimtSiluBack{t.dffn, t.fin[l], F});
    rc |= tn(D, F, t.dh, D, t.fout[l], F, G(w.wdown));
    rc |= nn(D, F, t.dffn, F, w.wup, ET{ET::kStore, t.dn, nullptr, nullptr, D}, SimtStore{t.dn, D, 0});
    rc |= tn(F, D, t.dffn, F, t.nf[l], D, G(w.wup));
    snai_train_rmsnorm_bwd<<<M, kRowThreads, 0, st>>>(t.dn, t.hf[l], w.rms_ffn, D, t.dh, 0, t.gprod);
    e.launches++;
    colsum(G(w.rms_ffn));
    // Wo
    rc |= nn(D, D, t.dh, D, w.wo, ET{ET::kStore, t.datt, nullptr, nullptr, D}, SimtStore{t.datt, D, 0});
    rc |= tn(D, D, t.dh, D, t.att[l], D, G(w.wo));
    // attention: recomputed scores, dP = dO V^T, then dS, dQ, dK, dV
    const long long sS = (long long)M * t.ldS;
    rc |= gemm<true, true>(e, args(M, M, hs, t.qkv[l], D3, t.qkv[l] + D, D3, 1, hs, hs), H, SimtStore{t.S, t.ldS, sS},
                           hvec);
    rc |= gemm<true, true>(e, args(M, M, hs, t.datt, D, t.qkv[l] + 2 * D, D3, 1, hs, hs), H,
                           SimtStore{t.dP, t.ldS, sS}, hvec);
    snai_train_softmax_bwd<<<dim3(rw_blocks, H), 256, 0, st>>>(t.S, t.dP, M, t.ldS, inv_sqrt);
    e.launches++;
    rc |= gemm<true, false>(e, args(M, hs, M, t.dP, t.ldS, t.qkv[l] + D, D3, 2, sS, hs), H, SimtStore{t.dqkv, D3, hs},
                            hvec);
    rc |= gemm<false, false>(e, args(M, hs, M, t.dP, t.ldS, t.qkv[l], D3, 3, sS, hs), H,
                             SimtStore{t.dqkv + D, D3, hs}, hvec);
    rc |= gemm<false, false>(e, args(M, hs, M, t.S, t.ldS, t.datt, D, 3, sS, hs), H,
                             SimtStore{t.dqkv + 2 * D, D3, hs}, hvec);
    snai_train_rope<<<dim3((D + 255) / 256, M), 256, 0, st>>>(t.dqkv, D3, M, D, hs, e.rope,
                                                                                          -1.0f);
    e.launches++;
    // Wq, Wk, Wv (one stacked [3D, D] matrix)
    rc |= nn(D, 3 * D, t.dqkv, D3, w.wqkv, ET{ET::kStore, t.dn, nullptr, nullptr, D}, SimtStore{t.dn, D, 0});
    rc |= tn(3 * D, D, t.dqkv, D3, t.na[l], D, G(w.wqkv));
    snai_train_rmsnorm_bwd<<<M, kRowThreads, 0, st>>>(t.dn, t.hid[l], w.rms_att, D, t.dh, 0, t.gprod);
    e.launches++;
    colsum(G(w.rms_att));
  }
  snai_train_tok_links<<<1, 1024, 0, st>>>(t.tin, M, V, t.prev, t.last);
  snai_train_emb_grad<<<M, kRowThreads, 0, st>>>(t.dh, t.tin, t.prev, t.last, V, D, G(e.emb));
  e.launches += 2;
  if (rc || launch_rc("training backward")) return -1;
  if (cudaMemcpyAsync(loss_out, t.loss, sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    set_error("training step: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  return 0;
}

// clipGlobalGradientNorm(1.0) then applyGlobalAdamUpdate(lr, scale) on the
// device (no host synchronisation).
int train_apply(Engine &e, float lr, float scale) {
  if (train_alloc(e)) return -1;
  TrainState &t = *e.train;
  cudaStream_t st = e.stream;
  const size_t n = e.wblock_bytes / sizeof(float);
  snai_train_sumsq<<<kClipBlocks, kRowThreads, 0, st>>>(t.g, n, t.clip_part);
  snai_train_clip_factor<<<1, 32, 0, st>>>(t.clip_part, kClipBlocks, t.clip);
  e.launches += 2;
  t.adam_t += 1;
  AdamArgs a;
  a.w = static_cast<float *>(e.wblock);
  a.m = t.m;
  a.v = t.v;
  a.g = t.g;
  a.n = n;
  a.sparse_end = (size_t)(e.emb - static_cast<float *>(e.wblock)) + (size_t)e.d.V * e.d.D;
  a.lr = lr;
  a.b1 = 0.9f;
  a.b2 = 0.999f;
  a.omb1 = 1.0f - a.b1;
  a.omb2 = 1.0f - a.b2;
  // b1t = 1 - pow(b1, t) in float (:166-167)
  a.b1t = 1.0f - ::powf(a.b1, (float)t.adam_t);
  a.b2t = 1.0f - ::powf(a.b2, (float)t.adam_t);
  a.scale = scale;
  a.clip = t.clip;
  const int blocks = (int)std::min<size_t>((n / 4 + kRowThreads - 1) / kRowThreads, (size_t)device_sm_count(e.device) * 8);
  if (scale != 0.0f) {  // adamStep returns at once when scale == 0 (:147)
    snai_train_adam<<<blocks, kRowThreads, 0, st>>>(a);
    e.launches++;
  }
  return launch_rc("training update");
}

// Clip factor and norm of the last train_apply (host copy; synchronises).
int train_clip_info(Engine &e, float *factor, float *norm, int *applied) {
  if (!e.train || !e.train->clip) return -1;
  float c[3];
  if (cudaMemcpyAsync(c, e.train->clip, sizeof c, cudaMemcpyDeviceToHost, e.stream) != cudaSuccess ||
      cudaStreamSynchronize(e.stream) != cudaSuccess)
    return -1;
  *factor = c[0];
  *applied = c[1] != 0.0f;
  *norm = c[2];
  return 0;
}

}  // namespace snai
