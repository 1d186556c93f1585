// engine.h - internal state of a libcortex decode engine (host side).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>

#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>
#include <vector>

namespace snai {

enum Precision { kFP32 = 0, kTF32 = 1, kBF16 = 2 };

// One-time set-up per device (kernel attributes), safe when several host
// threads drive engines at once (one thread per GPU, or several on one GPU)
// and for any device number: the set-up runs under the lock, so no thread
// launches before the attribute it needs is in place.
class DeviceOnce {
 public:
  // Runs f() (returning true on success) the first time `dev` asks and
  // returns its result; later calls return true at once.
  template <class F>
  bool run(int dev, F &&f) {
    std::lock_guard<std::mutex> g(mu_);
    if (done_.count(dev)) return true;
    done_.insert(dev);
    return f();
  }

 private:
  std::mutex mu_;
  std::set<int> done_;
};

// Multiprocessor count of a device (queried once per device, thread-safe).
int device_sm_count(int dev);

// Raises a kernel's dynamic shared-memory limit to `bytes`, less the
// kernel's static shared memory (a CTA may use 227 KB in all).  A failure is
// cleared from the runtime's error state, so that it cannot surface as the
// error of a later launch, and returned as false.
template <class K>
bool set_dyn_smem(K kern, int bytes) {
  const void *fn = reinterpret_cast<const void *>(kern);
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const int limit = 227 * 1024 - (int)fa.sharedSizeBytes;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes < limit ? bytes : limit) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

// Shape of a model.  Rules of core/cortex.nim:261-271: ffn = 4*dim whatever
// the file header says; head size hs = dim/heads forced even and >= 2; RoPE
// rotates dim/hs heads (core/cortex.nim:75); attention uses `heads` heads, so
// only the first heads*hs channels of q, k, v are ever read.
struct Dims {
  int V = 0, D = 0, F = 0, ctx = 0, L = 0;
  int heads = 0, hs = 0;
  int att_ch = 0;  // heads * hs
};

// One row of a forward pass: a token at a cache position of a slot.
// `out` >= 0 asks for the logits of this row in logits slot `out`.
// When the pass takes tokens from a device array, `token` is the index into it.
struct RowDesc {
  int slot, pos, token, out;
};

struct LayerWeights {
  float *rms_att = nullptr, *rms_ffn = nullptr;
  float *wqkv = nullptr;  // [3D, D]: Wq, Wk, Wv stacked (their file order)
  float *wo = nullptr;    // [D, D]
  float *wup = nullptr;   // [F, D]
  float *wdown = nullptr; // [D, F]
  __nv_bfloat16 *wqkv_h = nullptr, *wo_h = nullptr, *wup_h = nullptr, *wdown_h = nullptr;
};

// One layer's fp32 weights for the persistent one-row pass kernel (a device
// table of these is made with the engine).
struct PassLayer {
  const float *rms_att, *rms_ffn, *wqkv, *wo, *wup, *wdown;
};

struct TrainState;  // train.cu

struct Engine {
  Dims d;
  int device = 0;
  int precision = kFP32;
  int max_seqs = 1;
  int m_max = 0;  // rows per forward chunk
  bool att_split = true;  // split-position attention for passes of few rows (SNAI_ATTENTION_SPLIT=0: off)
  bool pass_kernel = false;  // one persistent kernel for FP32 passes of 1-2 rows (SNAI_PASS_KERNEL=1: on)
  PassLayer *pass_layers = nullptr;  // [L] on the device
  unsigned *pass_bar = nullptr;      // [2] grid-barrier counters of the pass kernel, zero between launches
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;

  // weights (fp32 masters; bf16 copies in BF16 mode)
  void *wblock = nullptr;
  size_t wblock_bytes = 0;
  void *avg_tmp = nullptr;  // this engine's shard of a cross-engine average (kept for the next one)
  size_t avg_tmp_bytes = 0;
  void *hblock = nullptr;
  float *emb = nullptr, *w_out = nullptr, *rms_final = nullptr;
  __nv_bfloat16 *w_out_h = nullptr;
  std::vector<LayerWeights> layers;

  // KV cache: kv[slot][layer][k|v][head][ctx][hs] fp32
  float *kv = nullptr;
  size_t kv_slot_stride = 0, kv_layer_stride = 0, kv_part_stride = 0, kv_head_stride = 0;

  // RoPE table [ctx][hs/2] of (cos, sin), computed on the host with the
  // reference's float expressions (core/cortex.nim:79-82).
  float2 *rope = nullptr;
  float sqrt_hs = 1.f;  // sqrtf(hs), the attention score divisor (:521)

  // activations for m_max rows
  void *ablock = nullptr;
  RowDesc *rows_d = nullptr;
  int2 *outrows_d = nullptr;  // (chunk row, logits slot)
  float *h = nullptr;         // [m_max, D] residual stream
  void *x = nullptr;          // [m_max, D] normed input of a projection (fp32 or bf16)
  float *q = nullptr;         // [m_max, att_ch]
  float *kvs = nullptr;       // [m_max, 2, att_ch] K and V of the new position, when appended by attention
  void *att = nullptr;        // [m_max, D]
  void *u = nullptr;          // [m_max, F]
  void *xo = nullptr;         // [m_max, D] normed rows that need logits
  float *att_part = nullptr;    // split attention: chunk partials [att_part_entries][68]
  size_t att_part_entries = 0;  // SMs x min(ceil(ctx / 64), 128)
  int *att_cnt = nullptr;       // split attention: arrival counters [256], zero between launches
  float *logits = nullptr;    // [max_seqs, V], per slot
  int *hist = nullptr;        // [max_seqs, ctx] every token fed to the slot
  int *seq_len_d = nullptr;   // [max_seqs] tokens fed (device copy of pos)
  int *ids_d = nullptr;       // [max_seqs]
  float *unif_d = nullptr;    // [max_seqs]
  int *slots_d = nullptr;     // [max_seqs]
  int *err_d = nullptr;       // device error word

  // decode-step graph (cortex_decode_steps): one captured decode step of
  // `batch` slots, replayed per step; a device step counter indexes the
  // per-step uniforms and ids
  struct DecodeGraph {
    cudaGraphExec_t exec = nullptr;
    int batch = 0, variant = 0, top_k = 0, nan_guard = 0;
    long long kernels = 0;        // kernels in one replay
    double temperature = 0, rep = 0, top_p = 0;
    const float *unif = nullptr;  // [steps, batch] read through *step_d
    int *ids = nullptr;           // [steps, batch] written through *step_d
  } graph;
  int *step_d = nullptr;          // device step counter of a graph replay
  float *unif_all = nullptr;      // [cap, ...] per-step uniforms staged for a replay
  int *ids_all = nullptr;         // [cap, ...] per-step ids of a replay
  size_t all_cap = 0;             // elements of unif_all / ids_all

  // host staging of a chunk's rows.  Pageable on purpose: cudaMemcpyAsync
  // from pageable memory returns once the source has been consumed, so the
  // buffers can be refilled by the next call without waiting for the GPU.
  std::vector<RowDesc> rows_stage;
  std::vector<char> slot_seen;  // per slot, for the one-row-per-slot test of a chunk
  std::vector<int2> out_stage;

  // host mirrors
  std::vector<int> pos;            // per slot
  std::vector<char> logits_valid;  // per slot
  TrainState *train = nullptr;     // gradients, Adam moments, training activations (made on first use)
  long long launches = 0;

  // optional per-kernel-class timing (CUDA events on the engine stream)
  bool prof = false;
  struct ProfPending {
    int kind;
    cudaEvent_t a, b;
    double bytes, flops;
  };
  std::vector<ProfPending> prof_pending;
  std::vector<cudaEvent_t> prof_free;
  long long prof_count[16] = {};
  double prof_ms[16] = {}, prof_bytes[16] = {}, prof_flops[16] = {};
};

// Kernel classes of the profiler (cortex_profile_read `kind`).
enum ProfKind : int {
  kProfEmbed = 0, kProfNorm = 1, kProfQKV = 2, kProfAttention = 3, kProfWo = 4, kProfUp = 5, kProfDown = 6,
  kProfLogits = 7, kProfSampler = 8, kProfPass = 9, kProfKinds = 10
};
// Brackets one launch: returns a token for prof_end (or -1 when off).
int prof_begin(Engine &e);
void prof_end(Engine &e, int token, int kind, double bytes, double flops);
// Folds finished events into the totals (synchronizes the stream).
void prof_collect(Engine &e);

// ---- error reporting (cortex_api.cu) ----
void set_error(const char *fmt, ...);
void clear_error();

// ---- forward pass (forward.cu) ----
// Runs rows[0..n) (each slot's positions ascending) through the model in
// chunks of at most e.m_max rows.  If tokens_d is not null, row tokens are
// tokens_d[row.token].  Returns 0 or a negative error.
int run_rows(Engine &e, const RowDesc *rows, int n, const int *tokens_d);

// fp32 -> bf16 copy of a weight tensor on e.stream.
int convert_bf16(Engine &e, const float *src, __nv_bfloat16 *dst, size_t n);
// fp32 -> bf16 copies of up to 64 tensors (each a multiple of 4 elements,
// 16-byte aligned) in one launch on e.stream.
struct Bf16Segments {
  struct Seg {
    const float *src;
    __nv_bfloat16 *dst;
    size_t n;
  } seg[64];
  int count = 0;
};
int convert_bf16_segments(Engine &e, const Bf16Segments &segs);
// Fills n floats with a value on e.stream.
int fill_f32(Engine &e, float *dst, size_t n, float v);

// ---- sampler (sampler.cu) ----
struct SampleLaunch {
  const float *logits = nullptr;
  long long ld = 0;
  const int *row_map = nullptr;  // row b reads logits/hist/hist_len row row_map[b]
  int rows = 0, V = 0;
  const int *hist = nullptr;
  long long hist_ld = 0;
  int hist_cols = 0;
  const int *hist_len = nullptr;
  const float *uniforms = nullptr;
  int variant = 0;
  double temperature = 1.0, rep = 1.0, top_p = 1.0;
  int top_k = 1;
  int nan_guard = 0;
  int *out_ids = nullptr;
  int *err = nullptr;
};
// Checks the arguments; returns 0 or a negative error (with set_error).
int check_sample_args(const SampleLaunch &a);
// One decode step of `batch` slots with everything on the device (the body of
// a graph): per-step uniforms from unif_all[*step_d], the sampler, the rows
// built from seq_len_d, the forward pass with tokens ids_d, ids copied to
// ids_all[*step_d] and the counter advanced.  No host synchronization, no
// host-to-device copies.  Returns 0 or a negative error.
int decode_step_device(Engine &e, int batch, const SampleLaunch &sampler);
int launch_sampler(const SampleLaunch &a, cudaStream_t stream);

// ---- merging and Net2Net (net2net.cu) ----
constexpr int kMergeMaxSources = 64;
struct MergeSources {
  const float *src[kMergeMaxSources];
  int n = 0;
};
// out[j] = fp32((sum_i double(src_i[j])) / n), sources summed in order (any
// GPU's memory the device can read).
int launch_merge_mean(const MergeSources &srcs, float *out, size_t count, int device, cudaStream_t stream);
// One Net2Net-upscaled tensor: old values (x scale) inside [old_r, old_c),
// seeded noise in [-0.005, 0.005] elsewhere.
int launch_upscale_tensor(const float *old, int old_r, int old_c, float *out, int new_r, int new_c, double scale,
                          uint64_t seed, uint64_t stream, int device, cudaStream_t st);

// ---- training step (train.cu) ----
// Allocates the Adam moments (zero) if they do not exist yet.
int train_moments(Engine &e);
// Device address of the gradient (which 0), first (1) or second (2) Adam
// moment of the weight at w (a pointer into the weight block); allocates the
// buffers on first use (nullptr on failure).
float *train_tensor(Engine &e, int which, const float *w);
// Forward, loss and backward of core/cortex.nim:565-818 for act >= 1 tokens
// (host arrays); gradients left in the gradient block, the mean loss in
// *loss_out (synchronises).  Returns 0 or a negative error.
int train_grads(Engine &e, const int *tin, const int *ttg, int act, float *loss_out);
// Global-norm clip (1.0) and one Adam step with gradient divisor `scale`,
// queued on e.stream.  Returns 0 or a negative error.
int train_apply(Engine &e, float lr, float scale);
int train_clip_info(Engine &e, float *factor, float *norm, int *applied);
int train_adam_steps(const Engine &e);
void train_free(Engine &e);
struct EpiTrain;  // epilogue.cuh
// C[M, N] = A[M, K] W[N, K]^T on the TF32 tensor cores with a training
// epilogue (forward.cu).  Returns 0 or a negative error.
int train_gemm_tc(Engine &e, int M, int N, int K, const float *A, const float *W, const EpiTrain &epi);

// Bounded-wait self-test (forward.cu): a kernel whose mbarrier wait never
// completes gives up after limit_ns and records an error in e.err_d; the id
// buffer's first entry becomes 1.  Returns 0 once queued.
int wait_selftest(Engine &e, long long limit_ns);

}  // namespace snai
