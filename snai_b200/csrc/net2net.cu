// net2net.cu - model merging, averaging and Net2Net upscaling on the GPU.
//
// The reference does these in PHP, one float at a time:
//   src/net2net_forge.php:29-102   merge_models: element-wise mean of N models
//   src/train_cluster.php:144-224  average_models_stream: the same mean (the
//                                  federated average of the training workers)
//   src/net2net_forge.php:108-214  upscale_model: d -> target, ffn -> 4 target,
//                                  ctx x 2, layers x 2, old entries copied
//                                  (x 0.01 for Wo / W_down of the new layers),
//                                  new entries uniform noise in [-0.005, 0.005]
// Arithmetic kept from the PHP code: the mean sums the models' fp32 values as
// doubles in model order and divides by N in double, then rounds to fp32
// (pack("g")); a copied entry is fp32(double(x) * scale); a noise entry is
// fp32(((u * 2) - 1) * 0.005) in double.  PHP draws u from mt_rand(); here u
// comes from a counter-based generator (SplitMix64, Steele, Lea and Flood
// 2014) keyed by (seed, tensor, element), so a seeded upscale is the same on
// any device and in the test oracle.
#include <cuda_runtime.h>

#include <cstdint>

#include "engine.h"

namespace snai {

// Element-wise mean of n arrays (n <= kMergeMaxSources): out[j] =
// fp32((sum_i double(src_i[j])) / n), summed in source order.  Sources may be
// another GPU's memory (peer loads over NVLink).
__global__ void merge_mean_kernel(const MergeSources srcs, float *__restrict__ out, size_t count, bool vec) {
  const double n = (double)srcs.n;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  size_t done = 0;
  if (vec) {  // 16-byte aligned sources and output: four floats per load
    const size_t n4 = count / 4;
    for (size_t j = tid; j < n4; j += stride) {
      double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
      for (int i = 0; i < srcs.n; ++i) {
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(srcs.src[i]) + j);
        s0 += (double)v.x;
        s1 += (double)v.y;
        s2 += (double)v.z;
        s3 += (double)v.w;
      }
      reinterpret_cast<float4 *>(out)[j] = make_float4((float)(s0 / n), (float)(s1 / n), (float)(s2 / n),
                                                       (float)(s3 / n));
    }
    done = n4 * 4;
  }
  for (size_t j = done + tid; j < count; j += stride) {
    double s = 0.0;
    for (int i = 0; i < srcs.n; ++i) s += (double)__ldcs(srcs.src[i] + j);
    out[j] = (float)(s / n);
  }
}

int launch_merge_mean(const MergeSources &srcs, float *out, size_t count, int device, cudaStream_t stream) {
  if (count == 0) return 0;
  bool vec = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  for (int i = 0; i < srcs.n; ++i) vec = vec && (reinterpret_cast<uintptr_t>(srcs.src[i]) & 15) == 0;
  merge_mean_kernel<<<4 * device_sm_count(device), 256, 0, stream>>>(srcs, out, count, vec);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// The noise draw of element j of output tensor `stream` in [0, 1): 53 bits of
// SplitMix64 of (seed, stream, j).
__host__ __device__ inline double net2net_uniform(uint64_t seed, uint64_t stream, uint64_t j) {
  const uint64_t z = splitmix64(seed ^ splitmix64((stream << 40) + j));
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

// One upscaled tensor (src/net2net_forge.php:108-147): out[r][c] =
// fp32(double(old[r][c]) * scale) inside the old shape, noise elsewhere.
__global__ void upscale_tensor_kernel(const float *__restrict__ old, int old_r, int old_c, float *__restrict__ out,
                                      int new_r, int new_c, double scale, uint64_t seed, uint64_t stream) {
  const size_t total = (size_t)new_r * new_c;
  for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < total; j += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(j / new_c), c = (int)(j % new_c);
    double v;
    if (r < old_r && c < old_c)
      v = (double)old[(size_t)r * old_c + c] * scale;
    else
      v = (net2net_uniform(seed, stream, j) * 2.0 - 1.0) * 0.005;
    out[j] = (float)v;
  }
}

int launch_upscale_tensor(const float *old, int old_r, int old_c, float *out, int new_r, int new_c, double scale,
                          uint64_t seed, uint64_t stream, int device, cudaStream_t st) {
  upscale_tensor_kernel<<<4 * device_sm_count(device), 256, 0, st>>>(old, old_r, old_c, out, new_r, new_c, scale,
                                                                     seed, stream);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace snai
