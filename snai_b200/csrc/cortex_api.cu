// cortex_api.cu - the C ABI of libcortex.so (include/cortex.h).
//
// Host side of the engine: model loading (SNAI_V4), device memory layout,
// the reference's thirteen entry points and the batched extension.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <chrono>
#include <condition_variable>
#include <functional>
#include <limits>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/cortex.h"
#include "engine.h"

namespace snai {

static thread_local std::string g_err;

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

void clear_error() { g_err.clear(); }

namespace {

int env_int(const char *name, int def) {
  const char *v = getenv(name);
  if (!v || !*v) return def;
  return atoi(v);
}

struct DeviceGuard {
  int prev = -1, want;
  explicit DeviceGuard(int d) : want(d) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() {
    if (prev >= 0 && prev != want) cudaSetDevice(prev);
  }
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Carves aligned sub-buffers out of one allocation.
struct Carver {
  size_t off = 0;
  std::vector<std::pair<void **, size_t>> items;
  void add(void **p, size_t bytes) {
    items.push_back({p, off});
    off = align_up(off + std::max<size_t>(bytes, 1), 256);
  }
  template <typename T>
  void add(T **p, size_t n) {
    add(reinterpret_cast<void **>(p), n * sizeof(T));
  }
  void place(void *base) {
    for (auto &it : items) *it.first = static_cast<char *>(base) + it.second;
  }
};

// Shape rules of core/cortex.nim:261-271 plus this engine's limits.
bool make_dims(int vocab, int dim, int ctx, int layers, int heads, Dims *d) {
  if (vocab < 1 || dim < 4 || ctx < 1 || layers < 1) {
    set_error("unsupported shape: vocab=%d dim=%d ctx=%d layers=%d (need vocab>=1, dim>=4, ctx>=1, layers>=1)", vocab,
              dim, ctx, layers);
    return false;
  }
  if (dim % 4 != 0) {
    set_error("hidden_dim %d is not a multiple of 4 (this engine reads activations in 16-byte units)", dim);
    return false;
  }
  d->V = vocab;
  d->D = dim;
  d->F = dim * 4;
  d->ctx = ctx;
  d->L = layers;
  d->heads = std::max(1, heads);
  int hs = dim / d->heads;
  if (hs % 2 != 0) hs -= 1;
  if (hs < 2) hs = 2;
  d->hs = hs;
  d->att_ch = d->heads * hs;
  if (d->att_ch > dim) {
    // core/cortex.nim:515-538 would read past the end of each cache row
    set_error("num_heads %d gives head size %d: %d heads x %d > hidden_dim %d", heads, hs, d->heads, hs, dim);
    return false;
  }
  // attention keeps a score per position and two head vectors in shared memory
  if (((size_t)ctx + 2 * (size_t)hs) * sizeof(float) + 2048 > 200 * 1024) {
    set_error("ctx_size %d with head size %d exceeds this engine's attention limit (%d positions)", ctx, hs,
              (200 * 1024 - 2048) / 4 - 2 * hs);
    return false;
  }
  return true;
}

void free_engine(Engine *e) {
  if (!e) return;
  DeviceGuard g(e->device);
  if (e->own_stream) cudaStreamSynchronize(e->own_stream);
  cudaFree(e->wblock);
  cudaFree(e->hblock);
  cudaFree(e->kv);
  cudaFree(e->ablock);
  if (e->graph.exec) cudaGraphExecDestroy(e->graph.exec);
  cudaFree(e->unif_all);
  cudaFree(e->ids_all);
  cudaFree(e->avg_tmp);
  train_free(*e);
  if (e->own_stream) cudaStreamDestroy(e->own_stream);
  delete e;
}

Engine *create_engine(const Dims &d, int max_seqs, int device, int precision) {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    set_error("no CUDA device available (libcortex runs on the GPU only)");
    return nullptr;
  }
  if (device < 0 || device >= ndev) {
    set_error("device %d out of range (%d devices)", device, ndev);
    return nullptr;
  }
  if (max_seqs < 1) {
    set_error("max_seqs must be >= 1");
    return nullptr;
  }
  if (precision < kFP32 || precision > kBF16) {
    set_error("unknown precision %d", precision);
    return nullptr;
  }
  DeviceGuard g(device);
  Engine *e = new Engine();
  e->d = d;
  e->device = device;
  e->precision = precision;
  e->max_seqs = max_seqs;
  int chunk = env_int("SNAI_CHUNK_ROWS", 0);
  if (chunk <= 0) chunk = std::max(max_seqs, std::min(8192, std::max(d.ctx, 256)));
  e->m_max = (int)align_up((size_t)std::max(chunk, max_seqs), 128);
  e->att_split = env_int("SNAI_ATTENTION_SPLIT", 1) != 0;
  e->pass_kernel = env_int("SNAI_PASS_KERNEL", 0) != 0;

  const size_t D = d.D, F = d.F, V = d.V;
  // ---- weights ----
  Carver w;
  w.add(&e->emb, V * D);
  w.add(&e->w_out, V * D);
  w.add(&e->rms_final, D);
  e->layers.resize(d.L);
  for (auto &l : e->layers) {
    w.add(&l.rms_att, D);
    w.add(&l.rms_ffn, D);
    w.add(&l.wqkv, 3 * D * D);
    w.add(&l.wo, D * D);
    w.add(&l.wup, F * D);
    w.add(&l.wdown, D * F);
  }
  Carver hw;
  if (precision == kBF16) {
    hw.add(&e->w_out_h, V * D);
    for (auto &l : e->layers) {
      hw.add(&l.wqkv_h, 3 * D * D);
      hw.add(&l.wo_h, D * D);
      hw.add(&l.wup_h, F * D);
      hw.add(&l.wdown_h, D * F);
    }
  }
  // ---- activations and per-slot state ----
  const size_t M = e->m_max;
  Carver a;
  a.add(&e->rows_d, M);
  a.add(&e->outrows_d, M);
  a.add(&e->h, M * D);
  a.add(&e->x, M * D * sizeof(float));
  a.add(&e->q, M * (size_t)d.att_ch);
  a.add(&e->kvs, M * 2 * (size_t)d.att_ch);
  a.add(&e->att, M * D * sizeof(float));
  a.add(&e->u, M * F * sizeof(float));
  a.add(&e->xo, M * D * sizeof(float));
  e->att_part_entries = (size_t)device_sm_count(device) * std::min((d.ctx + 63) / 64, 128);
  a.add(&e->att_part, e->att_part_entries * 68);
  a.add(&e->att_cnt, 256);
  a.add(&e->logits, (size_t)max_seqs * V);
  a.add(&e->hist, (size_t)max_seqs * d.ctx);
  a.add(&e->seq_len_d, (size_t)max_seqs);
  a.add(&e->ids_d, (size_t)max_seqs);
  a.add(&e->unif_d, (size_t)max_seqs);
  a.add(&e->slots_d, (size_t)max_seqs);
  a.add(&e->rope, (size_t)d.ctx * (d.hs / 2));
  a.add(&e->err_d, 4);
  a.add(&e->step_d, 4);
  a.add(&e->pass_layers, (size_t)d.L);
  a.add(&e->pass_bar, 2);

  e->kv_head_stride = (size_t)d.ctx * d.hs;
  e->kv_part_stride = e->kv_head_stride * d.heads;
  e->kv_layer_stride = 2 * e->kv_part_stride;
  e->kv_slot_stride = e->kv_layer_stride * d.L;
  const size_t kv_bytes = e->kv_slot_stride * max_seqs * sizeof(float);

  cudaError_t err = cudaMalloc(&e->wblock, w.off);
  if (err == cudaSuccess && hw.off) err = cudaMalloc(&e->hblock, hw.off);
  if (err == cudaSuccess) err = cudaMalloc(&e->ablock, a.off);
  if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void **>(&e->kv), kv_bytes);
  if (err != cudaSuccess) {
    set_error("device allocation failed (weights %zu B, activations %zu B, kv cache %zu B): %s", w.off, a.off,
              kv_bytes, cudaGetErrorString(err));
    cudaGetLastError();
    free_engine(e);
    return nullptr;
  }
  w.place(e->wblock);
  e->wblock_bytes = w.off;
  if (hw.off) hw.place(e->hblock);
  a.place(e->ablock);
  if (cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    free_engine(e);
    return nullptr;
  }
  e->stream = e->own_stream;
  cudaMemsetAsync(e->wblock, 0, w.off, e->stream);
  if (hw.off) cudaMemsetAsync(e->hblock, 0, hw.off, e->stream);
  cudaMemsetAsync(e->ablock, 0, a.off, e->stream);
  cudaMemsetAsync(e->kv, 0, kv_bytes, e->stream);
  // RMSNorm weights start at 1 (core/cortex.nim:433-438)
  fill_f32(*e, e->rms_final, D, 1.0f);
  for (auto &l : e->layers) {
    fill_f32(*e, l.rms_att, D, 1.0f);
    fill_f32(*e, l.rms_ffn, D, 1.0f);
  }
  // RoPE table, with the reference's float expressions (core/cortex.nim:79-82)
  std::vector<float2> rope((size_t)d.ctx * (d.hs / 2));
  for (int p = 0; p < d.ctx; ++p)
    for (int i = 0; i + 1 < d.hs; i += 2) {
      const float freq = 1.0f / ::powf(10000.0f, (float)i / (float)d.hs);
      const float theta = (float)p * freq;
      rope[(size_t)p * (d.hs / 2) + i / 2] = make_float2(::cosf(theta), 1.0f * ::sinf(theta));
    }
  cudaMemcpyAsync(e->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice, e->stream);
  std::vector<PassLayer> pl(d.L);
  for (int l = 0; l < d.L; ++l) {
    const LayerWeights &w = e->layers[l];
    pl[l] = PassLayer{w.rms_att, w.rms_ffn, w.wqkv, w.wo, w.wup, w.wdown};
  }
  cudaMemcpyAsync(e->pass_layers, pl.data(), pl.size() * sizeof(PassLayer), cudaMemcpyHostToDevice, e->stream);
  e->sqrt_hs = ::sqrtf((float)d.hs);
  e->pos.assign(max_seqs, 0);
  e->logits_valid.assign(max_seqs, 0);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) {
    set_error("engine initialisation failed: %s", cudaGetErrorString(cudaGetLastError()));
    free_engine(e);
    return nullptr;
  }
  return e;
}

// fp32 -> bf16 copies of every projection weight (BF16 mode).
// Every projection weight in one launch per 64 tensors.
int refresh_bf16(Engine &e) {
  if (e.precision != kBF16) return 0;
  const size_t D = e.d.D, F = e.d.F, V = e.d.V;
  Bf16Segments segs;
  int rc = 0;
  auto add = [&](const float *s, __nv_bfloat16 *d, size_t n) {
    if (segs.count == 64) {
      rc |= convert_bf16_segments(e, segs);
      segs.count = 0;
    }
    segs.seg[segs.count++] = Bf16Segments::Seg{s, d, n};
  };
  add(e.w_out, e.w_out_h, V * D);
  for (auto &l : e.layers) {
    add(l.wqkv, l.wqkv_h, 3 * D * D);
    add(l.wo, l.wo_h, D * D);
    add(l.wup, l.wup_h, F * D);
    add(l.wdown, l.wdown_h, D * F);
  }
  return rc | convert_bf16_segments(e, segs);
}

// Device pointer and element count of a tensor (core/cortex.nim:439-462).
float *tensor_ptr(Engine &e, int layer, int type, size_t *n) {
  const size_t D = e.d.D, F = e.d.F, V = e.d.V;
  if (layer >= e.d.L || layer < -1) return nullptr;
  if (layer == -1) {
    if (type == 0) { *n = V * D; return e.emb; }
    if (type == 1) { *n = V * D; return e.w_out; }
    if (type == 2) { *n = D; return e.rms_final; }
    return nullptr;
  }
  LayerWeights &l = e.layers[layer];
  switch (type) {
    case 10: *n = D; return l.rms_att;
    case 11: *n = D; return l.rms_ffn;
    case 12: *n = D * D; return l.wqkv;
    case 13: *n = D * D; return l.wqkv + D * D;
    case 14: *n = D * D; return l.wqkv + 2 * D * D;
    case 15: *n = D * D; return l.wo;
    case 16: *n = F * D; return l.wup;
    case 17: *n = D * F; return l.wdown;
  }
  return nullptr;
}

// bf16 copy of a tensor, if it has one.
__nv_bfloat16 *tensor_ptr_h(Engine &e, int layer, int type) {
  if (e.precision != kBF16) return nullptr;
  const size_t D = e.d.D;
  if (layer == -1) return type == 1 ? e.w_out_h : nullptr;
  if (layer < 0 || layer >= e.d.L) return nullptr;
  LayerWeights &l = e.layers[layer];
  switch (type) {
    case 12: return l.wqkv_h;
    case 13: return l.wqkv_h + D * D;
    case 14: return l.wqkv_h + 2 * D * D;
    case 15: return l.wo_h;
    case 16: return l.wup_h;
    case 17: return l.wdown_h;
  }
  return nullptr;
}

int check_device_error(Engine &e) {
  int code = 0;
  if (cudaMemcpy(&code, e.err_d, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    set_error("CUDA error: %s", cudaGetErrorString(cudaGetLastError()));
    return -4;
  }
  if (code) {
    cudaMemset(e.err_d, 0, sizeof(int));
    // a kernel that gave up may have left its arrival counters mid-way
    cudaMemset(e.pass_bar, 0, 2 * sizeof(unsigned));
    cudaMemset(e.att_cnt, 0, 256 * sizeof(int));
    set_error("device-side error %d (%s)", code,
              code == 6   ? "the bounded-wait self-test's wait expired"
              : code == 5 ? "the sampler saw an impossible row"
                          : "a bounded wait in a kernel expired");
    return -6;
  }
  return 0;
}

int finish(Engine &e, bool wait) {
  if (!wait) {
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      set_error("CUDA error: %s", cudaGetErrorString(le));
      return -4;
    }
    return 0;
  }
  if (cudaStreamSynchronize(e.stream) != cudaSuccess) {
    set_error("CUDA error: %s", cudaGetErrorString(cudaGetLastError()));
    return -4;
  }
  return check_device_error(e);
}

bool slots_ok(Engine &e, const int *slots, int batch) {
  std::vector<char> seen(e.max_seqs, 0);
  for (int b = 0; b < batch; ++b) {
    const int s = slots ? slots[b] : b;
    if (s < 0 || s >= e.max_seqs) {
      set_error("slot %d out of range [0, %d)", s, e.max_seqs);
      return false;
    }
    if (seen[s]) {
      set_error("slot %d appears twice in one batch", s);
      return false;
    }
    seen[s] = 1;
  }
  return true;
}

int upload_seq_len(Engine &e) {
  return cudaMemcpyAsync(e.seq_len_d, e.pos.data(), sizeof(int) * e.max_seqs, cudaMemcpyHostToDevice, e.stream) ==
                 cudaSuccess
             ? 0
             : -4;
}

int forward_batch(Engine &e, const int *tokens, int batch, int n_tok, const int *slots, float *logits, int flags) {
  clear_error();
  if (batch < 0 || n_tok < 0) {
    set_error("negative batch or token count");
    return -2;
  }
  if (batch == 0 || n_tok == 0) return 0;
  if (!tokens) {
    set_error("tokens is NULL");
    return -2;
  }
  if (!slots_ok(e, slots, batch)) return -2;
  const bool dev = flags & SNAI_DEVICE_PTRS;
  DeviceGuard g(e.device);
  std::vector<RowDesc> rows;
  rows.reserve((size_t)batch * n_tok);
  std::vector<int> done(batch, 0);
  for (int b = 0; b < batch; ++b) {
    const int s = slots ? slots[b] : b;
    const int p0 = e.pos[s];
    for (int i = 0; i < n_tok; ++i) {
      if (p0 + i >= e.d.ctx) break;  // core/cortex.nim:495
      const int idx = b * n_tok + i;
      rows.push_back(RowDesc{s, p0 + i, dev ? idx : tokens[idx], i == n_tok - 1 ? s : -1});
      done[b]++;
    }
  }
  int rc = run_rows(e, rows.data(), (int)rows.size(), dev ? tokens : nullptr);
  if (rc) return rc;
  for (int b = 0; b < batch; ++b) {
    const int s = slots ? slots[b] : b;
    e.pos[s] += done[b];
    if (done[b] == n_tok) e.logits_valid[s] = 1;
  }
  if (logits) {
    for (int b = 0; b < batch; ++b) {
      const int s = slots ? slots[b] : b;
      if (done[b] != n_tok) continue;  // reference leaves the buffer untouched
      if (cudaMemcpyAsync(logits + (size_t)b * e.d.V, e.logits + (size_t)s * e.d.V, sizeof(float) * e.d.V,
                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, e.stream) != cudaSuccess) {
        set_error("logits copy failed");
        return -4;
      }
    }
  }
  return finish(e, !dev);
}

// SNAI_V4 header (src/tensor_io.php:22-59, core/cortex.nim:969-996) and the
// engine shape it gives; the file is left at the first tensor.  NULL (with
// the error set) on a bad open, magic or header.
FILE *open_snai(const char *path, int num_heads, Dims *d, uint32_t *ffn_out) {
  if (!path) {
    set_error("filepath is NULL");
    return nullptr;
  }
  FILE *f = fopen(path, "rb");
  if (!f) {
    set_error("cannot open %s", path);
    return nullptr;
  }
  unsigned char hdr[28];
  if (fread(hdr, 1, 28, f) != 28) {
    fclose(f);
    set_error("%s: short header", path);
    return nullptr;
  }
  // magic: the non-NUL characters of the first 8 bytes (core/cortex.nim:986-990)
  std::string magic;
  for (int i = 0; i < 8; ++i)
    if (hdr[i]) magic.push_back((char)hdr[i]);
  if (magic != "SNAI_V4") {
    fclose(f);
    set_error("%s: magic is not SNAI_V4", path);
    return nullptr;
  }
  uint32_t p[5];
  for (int i = 0; i < 5; ++i)
    p[i] = (uint32_t)hdr[8 + 4 * i] | ((uint32_t)hdr[9 + 4 * i] << 8) | ((uint32_t)hdr[10 + 4 * i] << 16) |
           ((uint32_t)hdr[11 + 4 * i] << 24);
  const uint32_t vocab = p[0], dim = p[1], ffn = p[2], ctx = p[3], layers = p[4];
  if (vocab > (uint32_t)std::numeric_limits<int>::max() || dim > 65536 || ctx > (1u << 24) || layers > 4096) {
    fclose(f);
    set_error("%s: header values out of range", path);
    return nullptr;
  }
  if ((uint64_t)ffn > 4ull * dim) {
    // the reference would read ffn*dim floats into a 4*dim*dim buffer
    fclose(f);
    set_error("%s: ffn_dim %u > 4 * hidden_dim %u", path, ffn, dim);
    return nullptr;
  }
  if (!make_dims((int)vocab, (int)dim, (int)ctx, (int)layers, num_heads, d)) {
    fclose(f);
    return nullptr;
  }
  *ffn_out = ffn;
  return f;
}

// Reads every tensor of an open SNAI_V4 file straight into the engine's
// fp32 weights, in file order (core/cortex.nim:998-1041: read n floats or
// fail).  Two pinned staging buffers alternate: the file is read into one
// while the other's host-to-device copy runs on the engine's stream.
bool read_weights(Engine *e, FILE *f, uint32_t ffn) {
  constexpr size_t kStage = 8u << 20;  // floats per staging buffer (32 MB)
  float *stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool ok = cudaHostAlloc(reinterpret_cast<void **>(&stage[0]), kStage * 4, cudaHostAllocDefault) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void **>(&stage[1]), kStage * 4, cudaHostAllocDefault) == cudaSuccess &&
            cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) set_error("pinned staging buffers for the loader: %s", cudaGetErrorString(cudaGetLastError()));
  int b = 0;
  bool used[2] = {false, false};
  auto blast = [&](float *dst, size_t n) {
    for (size_t at = 0; ok && at < n;) {
      const size_t c = std::min(kStage, n - at);
      if (used[b] && cudaEventSynchronize(done[b]) != cudaSuccess) {  // its last copy has left the buffer
        ok = false;
        set_error("loader copy failed: %s", cudaGetErrorString(cudaGetLastError()));
        break;
      }
      if (fread(stage[b], sizeof(float), c, f) != c) {
        ok = false;
        set_error("file ends before all tensors were read");
        break;
      }
      if (cudaMemcpyAsync(dst + at, stage[b], c * sizeof(float), cudaMemcpyHostToDevice, e->stream) != cudaSuccess ||
          cudaEventRecord(done[b], e->stream) != cudaSuccess) {
        ok = false;
        set_error("loader copy failed: %s", cudaGetErrorString(cudaGetLastError()));
        break;
      }
      used[b] = true;
      b ^= 1;
      at += c;
    }
  };
  const size_t D = e->d.D, V = e->d.V, FF = (size_t)ffn * D;
  blast(e->emb, V * D);
  blast(e->w_out, V * D);
  blast(e->rms_final, D);
  for (int l = 0; ok && l < e->d.L; ++l) {
    LayerWeights &w = e->layers[l];
    blast(w.rms_att, D);
    blast(w.rms_ffn, D);
    blast(w.wqkv, D * D);
    blast(w.wqkv + D * D, D * D);
    blast(w.wqkv + 2 * D * D, D * D);
    blast(w.wo, D * D);
    blast(w.wup, FF);
    blast(w.wdown, FF);
  }
  if (cudaStreamSynchronize(e->stream) != cudaSuccess && ok) {
    ok = false;
    set_error("loader copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  }
  for (int i = 0; i < 2; ++i) {
    if (stage[i]) cudaFreeHost(stage[i]);
    if (done[i]) cudaEventDestroy(done[i]);
  }
  return ok;
}

Engine *load_stream(const char *path, int num_heads, int max_seqs, int device, int precision) {
  clear_error();
  Dims d;
  uint32_t ffn = 0;
  FILE *f = open_snai(path, num_heads, &d, &ffn);
  if (!f) return nullptr;
  Engine *e = create_engine(d, max_seqs, device, precision);
  if (!e) {
    fclose(f);
    return nullptr;
  }
  DeviceGuard g(e->device);
  const bool ok = read_weights(e, f, ffn);
  fclose(f);
  if (!ok) {
    set_error("%s: %s", path, g_err.c_str());
    free_engine(e);
    return nullptr;
  }
  if (refresh_bf16(*e) || cudaStreamSynchronize(e->stream) != cudaSuccess) {
    set_error("weight conversion failed: %s", cudaGetErrorString(cudaGetLastError()));
    free_engine(e);
    return nullptr;
  }
  return e;
}

int legacy_device() {
  int d = env_int("SNAI_DEVICE", -1);
  if (d >= 0) return d;
  if (cudaGetDevice(&d) != cudaSuccess) d = 0;
  return d;
}

int legacy_precision() { return env_int("SNAI_PRECISION", kFP32); }

}  // namespace
}  // namespace snai

using namespace snai;

// ============================================================================
// Part 1 - reference boundary
// ============================================================================

extern "C" void *cortex_init(int vocab_size, int hidden_dim, int ctx_size, int num_layers, int num_heads) {
  return cortex_init_ex(vocab_size, hidden_dim, ctx_size, num_layers, num_heads, 1, legacy_device(),
                        legacy_precision());
}

extern "C" void *cortex_load_stream(const char *filepath, int num_heads) {
  return load_stream(filepath, num_heads, 1, legacy_device(), legacy_precision());
}

extern "C" void cortex_forward(void *state, int *raw_tokens, int num_tokens, float *raw_logits) {
  if (!state) return;
  Engine &e = *static_cast<Engine *>(state);
  const int zero = 0;
  // logits are copied only if the call's last token was processed (:555)
  const int rc = forward_batch(e, raw_tokens, 1, num_tokens, &zero, raw_logits, SNAI_HOST_PTRS);
  if (rc != 0) {
    fprintf(stderr, "libcortex: cortex_forward failed: %s\n", g_err.c_str());
    if (raw_logits)
      for (int v = 0; v < e.d.V; ++v) raw_logits[v] = std::numeric_limits<float>::quiet_NaN();
  }
}

extern "C" void cortex_reset_cache(void *state) {
  if (!state) return;
  const int zero = 0;
  cortex_seq_reset(state, &zero, 1);
}

extern "C" void cortex_free(void *state) { free_engine(static_cast<Engine *>(state)); }

extern "C" void cortex_init_gpu(void) {
  clear_error();
  int ndev = 0;
  cudaError_t err = cudaGetDeviceCount(&ndev);
  if (err != cudaSuccess || ndev == 0) {
    set_error("cortex_init_gpu: no CUDA device (%s)", cudaGetErrorString(err));
    fprintf(stderr, "libcortex: %s\n", g_err.c_str());
    return;
  }
  const int d = env_int("SNAI_DEVICE", 0);
  err = cudaSetDevice(d);
  if (err == cudaSuccess) err = cudaFree(nullptr);
  if (err != cudaSuccess) {
    set_error("cortex_init_gpu: device %d: %s", d, cudaGetErrorString(err));
    fprintf(stderr, "libcortex: %s\n", g_err.c_str());
  }
}

extern "C" int get_vocab_size(void *state) { return state ? static_cast<Engine *>(state)->d.V : 0; }
extern "C" int get_ctx_size(void *state) { return state ? static_cast<Engine *>(state)->d.ctx : 0; }

extern "C" void cortex_load_layer(void *state, int layer_idx, int tensor_type, float *raw_weights, int num_weights) {
  if (!state || !raw_weights) return;
  Engine &e = *static_cast<Engine *>(state);
  size_t n = 0;
  float *p = tensor_ptr(e, layer_idx, tensor_type, &n);
  if (!p || (size_t)num_weights != n) return;  // core/cortex.nim:465: silent on mismatch
  DeviceGuard g(e.device);
  cudaStreamSynchronize(e.stream);
  cudaMemcpy(p, raw_weights, n * sizeof(float), cudaMemcpyHostToDevice);
  if (__nv_bfloat16 *h = tensor_ptr_h(e, layer_idx, tensor_type)) {
    convert_bf16(e, p, h, n);
    cudaStreamSynchronize(e.stream);
  }
}

extern "C" void cortex_extract_layer(void *state, int layer_idx, int tensor_type, float *raw_weights,
                                     int num_weights) {
  if (!state || !raw_weights) return;
  Engine &e = *static_cast<Engine *>(state);
  size_t n = 0;
  float *p = tensor_ptr(e, layer_idx, tensor_type, &n);
  if (!p || (size_t)num_weights != n) return;
  DeviceGuard g(e.device);
  cudaStreamSynchronize(e.stream);
  cudaMemcpy(raw_weights, p, n * sizeof(float), cudaMemcpyDeviceToHost);
}

// Copies one gradient / moment tensor in or out (which: 0 gradient, 1 m, 2 v).
static void train_tensor_copy(void *state, int which, int layer_idx, int tensor_type, float *raw, int size, bool in) {
  if (!state || !raw) return;
  Engine &e = *static_cast<Engine *>(state);
  size_t n = 0;
  float *w = tensor_ptr(e, layer_idx, tensor_type, &n);
  if (!w || (size_t)size != n) return;  // silent on mismatch, as :465
  DeviceGuard g(e.device);
  float *p = train_tensor(e, which, w);
  if (!p) {
    fprintf(stderr, "libcortex: %s\n", g_err.c_str());
    if (!in) std::fill(raw, raw + n, std::numeric_limits<float>::quiet_NaN());
    return;
  }
  cudaStreamSynchronize(e.stream);
  if (in)
    cudaMemcpy(p, raw, n * sizeof(float), cudaMemcpyHostToDevice);
  else
    cudaMemcpy(raw, p, n * sizeof(float), cudaMemcpyDeviceToHost);
}

extern "C" void cortex_load_adam_layer(void *state, int layer_idx, int tensor_type, bool is_variance, float *raw,
                                       int size) {
  train_tensor_copy(state, is_variance ? 2 : 1, layer_idx, tensor_type, raw, size, true);
}

extern "C" void cortex_extract_adam_layer(void *state, int layer_idx, int tensor_type, bool is_variance, float *raw,
                                          int size) {
  train_tensor_copy(state, is_variance ? 2 : 1, layer_idx, tensor_type, raw, size, false);
}

extern "C" void cortex_load_grad_layer(void *state, int layer_idx, int tensor_type, const float *raw, int size) {
  train_tensor_copy(state, 0, layer_idx, tensor_type, const_cast<float *>(raw), size, true);
}

extern "C" void cortex_extract_grad_layer(void *state, int layer_idx, int tensor_type, float *raw, int size) {
  train_tensor_copy(state, 0, layer_idx, tensor_type, raw, size, false);
}

extern "C" int cortex_train_grads(void *state, const int *raw_inputs, const int *raw_targets, int num_tokens,
                                  float *loss) {
  clear_error();
  if (!state || !loss) {
    set_error("cortex_train_grads: NULL state or loss");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  const int act = std::min(num_tokens, e.d.ctx);  // core/cortex.nim:566-567
  *loss = 0.0f;
  if (act <= 0) return 0;
  if (!raw_inputs || !raw_targets) {
    set_error("cortex_train_grads: NULL token arrays");
    return -1;
  }
  DeviceGuard g(e.device);
  const int rc = train_grads(e, raw_inputs, raw_targets, act, loss);
  return rc ? rc : check_device_error(e);
}

extern "C" int cortex_train_apply(void *state, float lr, float scale) {
  clear_error();
  if (!state) {
    set_error("cortex_train_apply: NULL state");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  if (train_apply(e, lr, scale)) return -1;
  return refresh_bf16(e);  // the tensor-core copies follow the updated weights
}

extern "C" int cortex_train_info(void *state, int *adam_steps, float *clip_factor, float *grad_norm, int *clipped) {
  if (!state) return -1;
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  float f = 0.f, n = 0.f;
  int a = 0;
  const int rc = train_clip_info(e, &f, &n, &a);
  if (adam_steps) *adam_steps = train_adam_steps(e);
  if (rc) return -1;
  if (clip_factor) *clip_factor = f;
  if (grad_norm) *grad_norm = n;
  if (clipped) *clipped = a;
  return 0;
}

// core/cortex.nim:565-822: gradients, clip, Adam; the mean loss.
extern "C" float cortex_train_step(void *state, int *raw_inputs, int *raw_targets, int num_tokens, float lr) {
  if (!state) {
    set_error("cortex_train_step: NULL state");
    return std::numeric_limits<float>::quiet_NaN();
  }
  Engine &e = *static_cast<Engine *>(state);
  const int act = std::min(num_tokens, e.d.ctx);
  if (act <= 0) return 0.0f;  // :567
  float loss = 0.0f;
  int rc = cortex_train_grads(state, raw_inputs, raw_targets, num_tokens, &loss);
  if (rc == 0) rc = cortex_train_apply(state, lr, (float)act);
  if (rc == 0) {
    DeviceGuard g(e.device);
    if (cudaStreamSynchronize(e.stream) != cudaSuccess) {
      set_error("cortex_train_step: %s", cudaGetErrorString(cudaGetLastError()));
      rc = -1;
    } else {
      rc = check_device_error(e);
    }
  }
  if (rc != 0) {
    fprintf(stderr, "libcortex: cortex_train_step failed: %s\n", g_err.c_str());
    return std::numeric_limits<float>::quiet_NaN();
  }
  return loss;
}

// ============================================================================
// Part 2 - batched extension
// ============================================================================

extern "C" const char *cortex_last_error(void) { return g_err.c_str(); }

extern "C" void *cortex_load_stream_ex(const char *filepath, int num_heads, int max_seqs, int device, int precision) {
  return load_stream(filepath, num_heads, max_seqs, device, precision);
}

extern "C" void *cortex_init_ex(int vocab_size, int hidden_dim, int ctx_size, int num_layers, int num_heads,
                                int max_seqs, int device, int precision) {
  clear_error();
  Dims d;
  if (!make_dims(vocab_size, hidden_dim, ctx_size, num_layers, num_heads, &d)) return nullptr;
  Engine *e = create_engine(d, max_seqs, device, precision);
  if (e && refresh_bf16(*e)) {
    free_engine(e);
    return nullptr;
  }
  return e;
}

extern "C" int cortex_num_slots(void *state) { return state ? static_cast<Engine *>(state)->max_seqs : 0; }
extern "C" int cortex_head_size(void *state) { return state ? static_cast<Engine *>(state)->d.hs : 0; }
extern "C" int cortex_num_heads(void *state) { return state ? static_cast<Engine *>(state)->d.heads : 0; }

extern "C" int cortex_seq_reset(void *state, const int *slots, int n) {
  clear_error();
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  if (!slots) {
    std::fill(e.pos.begin(), e.pos.end(), 0);
    std::fill(e.logits_valid.begin(), e.logits_valid.end(), 0);
  } else {
    for (int i = 0; i < n; ++i) {
      if (slots[i] < 0 || slots[i] >= e.max_seqs) {
        set_error("slot %d out of range", slots[i]);
        return -2;
      }
      e.pos[slots[i]] = 0;
      e.logits_valid[slots[i]] = 0;
    }
  }
  DeviceGuard g(e.device);
  if (upload_seq_len(e)) {
    set_error("cudaMemcpy failed");
    return -4;
  }
  return finish(e, true);
}

extern "C" int cortex_seq_pos(void *state, int slot) {
  if (!state) return -1;
  Engine &e = *static_cast<Engine *>(state);
  if (slot < 0 || slot >= e.max_seqs) return -1;
  return e.pos[slot];
}

extern "C" int cortex_forward_batch(void *state, const int *tokens, int batch, int n_tok, const int *slots,
                                    float *logits, int flags) {
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  return forward_batch(*static_cast<Engine *>(state), tokens, batch, n_tok, slots, logits, flags);
}

extern "C" int cortex_decode_batch(void *state, const int *slots, int batch, const float *uniforms,
                                   const snai_sample_params *params, int *out_ids, int flags) {
  clear_error();
  if (!state || !params || !out_ids) {
    set_error("state, params and out_ids must not be NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  if (batch < 0 || batch > e.max_seqs) {
    set_error("batch %d outside [0, %d]", batch, e.max_seqs);
    return -2;
  }
  if (batch == 0) return 0;
  if (!slots_ok(e, slots, batch)) return -2;
  for (int b = 0; b < batch; ++b) {
    const int s = slots ? slots[b] : b;
    if (!e.logits_valid[s]) {
      set_error("slot %d has no logits yet (feed its prompt first)", s);
      return -2;
    }
  }
  const bool dev = flags & SNAI_DEVICE_PTRS;
  DeviceGuard g(e.device);
  std::vector<int> sl(batch);
  for (int b = 0; b < batch; ++b) sl[b] = slots ? slots[b] : b;
  if (cudaMemcpyAsync(e.slots_d, sl.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, e.stream) != cudaSuccess) {
    set_error("slot upload failed");
    return -4;
  }
  const float *u = uniforms;
  if (uniforms && !dev) {
    if (cudaMemcpyAsync(e.unif_d, uniforms, sizeof(float) * batch, cudaMemcpyHostToDevice, e.stream) !=
        cudaSuccess) {
      set_error("uniform upload failed");
      return -4;
    }
    u = e.unif_d;
  }
  SampleLaunch s;
  s.logits = e.logits;
  s.ld = e.d.V;
  s.row_map = e.slots_d;
  s.rows = batch;
  s.V = e.d.V;
  s.hist = e.hist;
  s.hist_ld = e.d.ctx;
  s.hist_cols = e.d.ctx;
  s.hist_len = e.seq_len_d;
  s.uniforms = u;
  s.variant = params->variant;
  s.temperature = params->temperature;
  s.rep = params->rep_penalty;
  s.top_k = params->top_k;
  s.top_p = params->top_p;
  s.nan_guard = params->nan_guard;
  s.out_ids = e.ids_d;
  s.err = e.err_d;
  double hist_total = 0;
  for (int b = 0; b < batch; ++b) hist_total += e.pos[sl[b]];
  const int ptok = prof_begin(e);
  int rc = launch_sampler(s, e.stream);
  if (rc) return rc;
  e.launches++;
  prof_end(e, ptok, kProfSampler, 4.0 * batch * e.d.V + 4.0 * hist_total + 12.0 * batch, 0.0);
  std::vector<RowDesc> rows;
  rows.reserve(batch);
  for (int b = 0; b < batch; ++b) {
    const int sl_b = sl[b];
    if (e.pos[sl_b] >= e.d.ctx) continue;
    rows.push_back(RowDesc{sl_b, e.pos[sl_b], b, sl_b});
  }
  rc = run_rows(e, rows.data(), (int)rows.size(), e.ids_d);
  if (rc) return rc;
  for (const RowDesc &r : rows) e.pos[r.slot] += 1;
  if (cudaMemcpyAsync(out_ids, e.ids_d, sizeof(int) * batch, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                      e.stream) != cudaSuccess) {
    set_error("id copy failed");
    return -4;
  }
  return finish(e, !dev);
}

// `steps` decode steps of `batch` slots: step k samples with uniforms[k] and
// writes out_ids[k] (both [steps, batch]).  One step is captured as a CUDA
// graph (the rows, uniforms and ids live on the device, indexed by a device
// step counter) and replayed, so a step costs one graph launch instead of
// one host launch per kernel.  Falls back to cortex_decode_batch per step
// when the profiler is on or a slot would reach the context limit.
extern "C" int cortex_decode_steps(void *state, const int *slots, int batch, int steps, const float *uniforms,
                                   const snai_sample_params *params, int *out_ids, int flags) {
  clear_error();
  if (!state || !params || !out_ids) {
    set_error("state, params and out_ids must not be NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  if (batch < 0 || batch > e.max_seqs || steps < 0) {
    set_error("batch %d outside [0, %d] or negative steps %d", batch, e.max_seqs, steps);
    return -2;
  }
  if (batch == 0 || steps == 0) return 0;
  if (!uniforms && params->temperature > 0.01) {
    set_error("uniforms must not be NULL for a sampling temperature");
    return -2;
  }
  if (!slots_ok(e, slots, batch)) return -2;
  const bool dev = flags & SNAI_DEVICE_PTRS;
  std::vector<int> sl(batch);
  bool graph_ok = !e.prof;
  for (int b = 0; b < batch; ++b) {
    sl[b] = slots ? slots[b] : b;
    if (!e.logits_valid[sl[b]]) {
      set_error("slot %d has no logits yet (feed its prompt first)", sl[b]);
      return -2;
    }
    if (e.pos[sl[b]] + steps > e.d.ctx) graph_ok = false;
  }
  if (!graph_ok) {
    for (int k = 0; k < steps; ++k) {
      const int rc = cortex_decode_batch(state, slots, batch, uniforms ? uniforms + (size_t)k * batch : nullptr,
                                         params, out_ids + (size_t)k * batch, flags);
      if (rc) return rc;
    }
    return 0;
  }
  DeviceGuard g(e.device);
  const size_t need = (size_t)steps * batch;
  if (need > e.all_cap) {
    // room for a whole context of steps of every slot (at most 8 M entries),
    // so that later calls with more steps keep the captured graph
    const size_t want = std::max(need, std::min<size_t>((size_t)e.d.ctx * e.max_seqs, 8u << 20));
    cudaFree(e.unif_all);
    cudaFree(e.ids_all);
    e.unif_all = nullptr;
    e.ids_all = nullptr;
    e.all_cap = 0;
    if (cudaMalloc(&e.unif_all, want * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&e.ids_all, want * sizeof(int)) != cudaSuccess) {
      set_error("out of device memory for %zu staged uniforms", want);
      return -3;
    }
    e.all_cap = want;
  }
  const cudaMemcpyKind in = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (cudaMemcpyAsync(e.slots_d, sl.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, e.stream) != cudaSuccess ||
      (uniforms && cudaMemcpyAsync(e.unif_all, uniforms, sizeof(float) * need, in, e.stream) != cudaSuccess) ||
      (!uniforms && cudaMemsetAsync(e.unif_all, 0, sizeof(float) * need, e.stream) != cudaSuccess) ||
      cudaMemsetAsync(e.step_d, 0, sizeof(int), e.stream) != cudaSuccess) {
    set_error("decode-steps upload failed: %s", cudaGetErrorString(cudaGetLastError()));
    return -4;
  }
  SampleLaunch s;
  s.logits = e.logits;
  s.ld = e.d.V;
  s.row_map = e.slots_d;
  s.rows = batch;
  s.V = e.d.V;
  s.hist = e.hist;
  s.hist_ld = e.d.ctx;
  s.hist_cols = e.d.ctx;
  s.hist_len = e.seq_len_d;
  s.uniforms = e.unif_d;
  s.variant = params->variant;
  s.temperature = params->temperature;
  s.rep = params->rep_penalty;
  s.top_k = params->top_k;
  s.top_p = params->top_p;
  s.nan_guard = params->nan_guard;
  s.out_ids = e.ids_d;
  s.err = e.err_d;
  int rc = check_sample_args(s);
  if (rc) return rc;
  Engine::DecodeGraph &gr = e.graph;
  const bool same = gr.exec && gr.batch == batch && gr.variant == s.variant && gr.temperature == s.temperature &&
                    gr.rep == s.rep && gr.top_k == s.top_k && gr.top_p == s.top_p &&
                    gr.nan_guard == s.nan_guard && gr.unif == e.unif_all && gr.ids == e.ids_all;
  int k0 = 0;
  if (!same) {
    // first step eagerly (sets every kernel's attributes outside a capture),
    // then capture one step for this and later calls
    if (gr.exec) cudaGraphExecDestroy(gr.exec);
    gr.exec = nullptr;
    rc = decode_step_device(e, batch, s);
    if (rc) return rc;
    k0 = 1;
    {
      const long long l0 = e.launches;
      if (cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        set_error("stream capture failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -4;
      }
      rc = decode_step_device(e, batch, s);
      cudaGraph_t graph = nullptr;
      const cudaError_t ce = cudaStreamEndCapture(e.stream, &graph);
      gr.kernels = e.launches - l0;
      e.launches = l0;  // captured, not launched
      if (rc || ce != cudaSuccess || !graph) {
        if (graph) cudaGraphDestroy(graph);
        if (!rc) set_error("stream capture failed: %s", cudaGetErrorString(ce));
        return rc ? rc : -4;
      }
      const cudaError_t ie = cudaGraphInstantiate(&gr.exec, graph, 0);
      cudaGraphDestroy(graph);
      if (ie != cudaSuccess) {
        gr.exec = nullptr;
        set_error("graph instantiation failed: %s", cudaGetErrorString(ie));
        return -4;
      }
      gr.batch = batch;
      gr.variant = s.variant;
      gr.temperature = s.temperature;
      gr.rep = s.rep;
      gr.top_k = s.top_k;
      gr.top_p = s.top_p;
      gr.nan_guard = s.nan_guard;
      gr.unif = e.unif_all;
      gr.ids = e.ids_all;
    }
  }
  const long long per_step = gr.kernels;
  for (int k = k0; k < steps; ++k) {
    if (cudaGraphLaunch(gr.exec, e.stream) != cudaSuccess) {
      set_error("graph launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return -4;
    }
    e.launches += per_step;
  }
  for (int b = 0; b < batch; ++b) e.pos[sl[b]] += steps;
  if (cudaMemcpyAsync(out_ids, e.ids_all, sizeof(int) * need, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                      e.stream) != cudaSuccess) {
    set_error("id copy failed");
    return -4;
  }
  return finish(e, !dev);
}

extern "C" int cortex_get_logits(void *state, const int *slots, int n, float *out) {
  clear_error();
  if (!state || !out) {
    set_error("state and out must not be NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  for (int i = 0; i < n; ++i) {
    const int s = slots ? slots[i] : i;
    if (s < 0 || s >= e.max_seqs) {
      set_error("slot %d out of range", s);
      return -2;
    }
    cudaMemcpyAsync(out + (size_t)i * e.d.V, e.logits + (size_t)s * e.d.V, sizeof(float) * e.d.V,
                    cudaMemcpyDeviceToHost, e.stream);
  }
  return finish(e, true);
}

extern "C" int cortex_sample(const float *logits, int rows, int vocab, long long ld, const int *hist, int hist_cols,
                             const int *hist_len, const float *uniforms, const snai_sample_params *params,
                             int *out_ids, void *stream) {
  clear_error();
  if (!params) {
    set_error("params is NULL");
    return -1;
  }
  SampleLaunch s;
  s.logits = logits;
  s.ld = ld;
  s.rows = rows;
  s.V = vocab;
  s.hist = hist;
  s.hist_ld = hist_cols;
  s.hist_cols = hist_cols;
  s.hist_len = hist_len;
  s.uniforms = uniforms;
  s.variant = params->variant;
  s.temperature = params->temperature;
  s.rep = params->rep_penalty;
  s.top_k = params->top_k;
  s.top_p = params->top_p;
  s.nan_guard = params->nan_guard;
  s.out_ids = out_ids;
  return launch_sampler(s, static_cast<cudaStream_t>(stream));
}

extern "C" int cortex_set_stream(void *state, void *stream) {
  if (!state) return -1;
  Engine &e = *static_cast<Engine *>(state);
  e.stream = stream ? static_cast<cudaStream_t>(stream) : e.own_stream;
  return 0;
}

extern "C" int cortex_synchronize(void *state) {
  clear_error();
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  return finish(e, true);
}

extern "C" int cortex_seq_rewind(void *state, const int *slots, int n, int pos) {
  clear_error();
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  for (int i = 0; i < n; ++i) {
    const int s = slots ? slots[i] : i;
    if (s < 0 || s >= e.max_seqs) {
      set_error("slot %d out of range", s);
      return -2;
    }
    if (pos < 0 || pos > e.pos[s]) {
      set_error("slot %d: cannot rewind from %d to %d", s, e.pos[s], pos);
      return -2;
    }
  }
  for (int i = 0; i < n; ++i) e.pos[slots ? slots[i] : i] = pos;
  DeviceGuard g(e.device);
  if (upload_seq_len(e)) {
    set_error("cudaMemcpy failed");
    return -4;
  }
  return finish(e, false);
}

extern "C" int cortex_profile_enable(void *state, int on) {
  if (!state) return -1;
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  prof_collect(e);
  for (int k = 0; k < 16; ++k) {
    e.prof_count[k] = 0;
    e.prof_ms[k] = e.prof_bytes[k] = e.prof_flops[k] = 0.0;
  }
  e.prof = on != 0;
  return 0;
}

extern "C" int cortex_profile_read(void *state, int kind, long long *launches, double *ms, double *bytes,
                                   double *flops) {
  if (!state || kind < 0 || kind >= kProfKinds) return -1;
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  prof_collect(e);
  if (launches) *launches = e.prof_count[kind];
  if (ms) *ms = e.prof_ms[kind];
  if (bytes) *bytes = e.prof_bytes[kind];
  if (flops) *flops = e.prof_flops[kind];
  return 0;
}

extern "C" int cortex_selftest_wait_timeout(void *state, long long limit_ns) {
  clear_error();
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  if (limit_ns < 1000 || limit_ns > 2000000000ll) {
    set_error("limit_ns %lld outside [1 us, 2 s]", limit_ns);
    return -2;
  }
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  return wait_selftest(e, limit_ns);
}

extern "C" long long cortex_kernel_launches(void *state) {
  return state ? static_cast<Engine *>(state)->launches : 0;
}

// ============================================================================
// Engine groups: one process driving several GPUs
// ============================================================================
//
// Sequences are independent (core/cortex.nim:487-563 shares nothing between
// them), so a group splits `total` sequences into contiguous shards, one
// engine per listed device, and never exchanges tensors between them.  The
// model file is read once: into the first engine, then its fp32 weight
// block is copied to every other engine by peer copies over NVLink (the
// engines' weight layouts are identical), and each GPU packs its own bf16
// copies.  Calls run one worker thread per engine; ids and logits are
// gathered into the caller's host arrays.
namespace snai {
namespace {

struct Group {
  std::vector<Engine *> engines;
  std::vector<int> first, count;  // shard of each engine
  int total = 0;
  double load_s = 0.0;
  // worker pool: one thread per engine
  std::vector<std::thread> workers;
  std::mutex mu;
  std::condition_variable cv_go, cv_done;
  std::function<int(int)> task;
  long long generation = 0;
  int pending = 0;
  bool quit = false;
  std::vector<int> rc;
  std::vector<std::string> err;

  void start() {
    rc.assign(engines.size(), 0);
    err.assign(engines.size(), std::string());
    for (size_t i = 0; i < engines.size(); ++i)
      workers.emplace_back([this, i] {
        long long seen = 0;
        for (;;) {
          std::function<int(int)> t;
          {
            std::unique_lock<std::mutex> lk(mu);
            cv_go.wait(lk, [&] { return quit || generation != seen; });
            if (quit) return;
            seen = generation;
            t = task;
          }
          clear_error();
          const int r = t((int)i);
          std::string msg = r ? g_err : std::string();
          std::lock_guard<std::mutex> lk(mu);
          rc[i] = r;
          err[i] = msg;
          if (--pending == 0) cv_done.notify_all();
        }
      });
  }
  // Runs f(i) for every engine on its worker; returns the first failure.
  int run(std::function<int(int)> f) {
    std::unique_lock<std::mutex> lk(mu);
    task = std::move(f);
    pending = (int)engines.size();
    ++generation;
    cv_go.notify_all();
    cv_done.wait(lk, [&] { return pending == 0; });
    for (size_t i = 0; i < engines.size(); ++i)
      if (rc[i]) {
        set_error("engine %zu (device %d): %s", i, engines[i]->device, err[i].c_str());
        return rc[i];
      }
    return 0;
  }
  ~Group() {
    {
      std::lock_guard<std::mutex> lk(mu);
      quit = true;
    }
    cv_go.notify_all();
    for (auto &t : workers) t.join();
    for (Engine *e : engines) free_engine(e);
  }
};

Group *load_group(const char *path, int num_heads, int total, const int *devices, int n, int precision) {
  clear_error();
  if (!devices || n < 1 || total < n) {
    set_error("a group needs at least one device and one sequence per device (devices=%d, sequences=%d)", n, total);
    return nullptr;
  }
  const auto t0 = std::chrono::steady_clock::now();
  Dims d;
  uint32_t ffn = 0;
  FILE *f = open_snai(path, num_heads, &d, &ffn);
  if (!f) return nullptr;
  Group *g = new Group();
  g->total = total;
  for (int i = 0; i < n; ++i) {
    const int a = (int)((long long)total * i / n), b = (int)((long long)total * (i + 1) / n);
    Engine *e = create_engine(d, b - a, devices[i], precision);
    if (!e) {
      fclose(f);
      delete g;
      return nullptr;
    }
    g->engines.push_back(e);
    g->first.push_back(a);
    g->count.push_back(b - a);
  }
  Engine *e0 = g->engines[0];
  bool ok;
  {
    DeviceGuard dg(e0->device);
    ok = read_weights(e0, f, ffn);
  }
  fclose(f);
  if (!ok) {
    set_error("%s: %s", path, g_err.c_str());
    delete g;
    return nullptr;
  }
  // fan the fp32 weights out from the first engine by peer copies
  for (int i = 1; ok && i < n; ++i) {
    Engine *e = g->engines[i];
    DeviceGuard dg(e->device);
    if (e->device != e0->device) {
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, e->device, e0->device) == cudaSuccess && can) {
        const cudaError_t pe = cudaDeviceEnablePeerAccess(e0->device, 0);
        if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) ok = false;
        cudaGetLastError();
      }
    }
    if (ok && cudaMemcpyPeerAsync(e->wblock, e->device, e0->wblock, e0->device, e0->wblock_bytes, e->stream) !=
                  cudaSuccess)
      ok = false;
    if (!ok) set_error("weight copy to device %d failed: %s", e->device, cudaGetErrorString(cudaGetLastError()));
  }
  for (int i = 0; ok && i < n; ++i) {
    Engine *e = g->engines[i];
    DeviceGuard dg(e->device);
    if (refresh_bf16(*e) || cudaStreamSynchronize(e->stream) != cudaSuccess) {
      ok = false;
      set_error("weight conversion on device %d failed: %s", e->device, cudaGetErrorString(cudaGetLastError()));
    }
  }
  if (!ok) {
    delete g;
    return nullptr;
  }
  g->start();
  g->load_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return g;
}

}  // namespace
}  // namespace snai

extern "C" void *cortex_group_load(const char *filepath, int num_heads, int total_seqs, const int *devices,
                                   int n_devices, int precision) {
  return load_group(filepath, num_heads, total_seqs, devices, n_devices, precision);
}

extern "C" void cortex_group_free(void *group) { delete static_cast<Group *>(group); }

extern "C" int cortex_group_size(void *group) {
  return group ? (int)static_cast<Group *>(group)->engines.size() : 0;
}

extern "C" void *cortex_group_engine(void *group, int i) {
  Group *g = static_cast<Group *>(group);
  if (!g || i < 0 || i >= (int)g->engines.size()) return nullptr;
  return g->engines[i];
}

extern "C" int cortex_group_shard(void *group, int i, int *first, int *count) {
  Group *g = static_cast<Group *>(group);
  if (!g || i < 0 || i >= (int)g->engines.size()) return -1;
  if (first) *first = g->first[i];
  if (count) *count = g->count[i];
  return 0;
}

extern "C" double cortex_group_load_seconds(void *group) {
  return group ? static_cast<Group *>(group)->load_s : 0.0;
}

extern "C" int cortex_group_forward(void *group, const int *tokens, int n_tok, float *logits) {
  clear_error();
  Group *g = static_cast<Group *>(group);
  if (!g || !tokens) {
    set_error("group and tokens must not be NULL");
    return -1;
  }
  const long long V = g->engines[0]->d.V;
  return g->run([&](int i) {
    Engine &e = *g->engines[i];
    return forward_batch(e, tokens + (size_t)g->first[i] * n_tok, g->count[i], n_tok, nullptr,
                         logits ? logits + (size_t)g->first[i] * V : nullptr, SNAI_HOST_PTRS);
  });
}

extern "C" int cortex_group_decode_steps(void *group, int steps, const float *uniforms,
                                         const snai_sample_params *params, int *out_ids) {
  clear_error();
  Group *g = static_cast<Group *>(group);
  if (!g || !params || !out_ids || steps < 0) {
    set_error("group, params and out_ids must not be NULL, steps >= 0");
    return -1;
  }
  if (steps == 0) return 0;
  const size_t T = (size_t)g->total;
  return g->run([&](int i) {
    const int a = g->first[i], B = g->count[i];
    // this shard's columns of [steps][total], contiguous
    std::vector<float> u(uniforms ? (size_t)steps * B : 0);
    for (int k = 0; uniforms && k < steps; ++k)
      std::copy(uniforms + k * T + a, uniforms + k * T + a + B, u.begin() + (size_t)k * B);
    std::vector<int> ids((size_t)steps * B);
    const int r = cortex_decode_steps(g->engines[i], nullptr, B, steps, uniforms ? u.data() : nullptr, params,
                                      ids.data(), SNAI_HOST_PTRS);
    if (r) return r;
    for (int k = 0; k < steps; ++k) std::copy(ids.begin() + (size_t)k * B, ids.begin() + (size_t)(k + 1) * B,
                                              out_ids + k * T + a);
    return 0;
  });
}

// ============================================================================
// Merging, federated averaging and Net2Net upscaling (net2net.cu kernels)
// ============================================================================
namespace snai {
namespace {

// Reads up to n bytes; returns the count (short only at the end of the file).
size_t read_full(FILE *f, void *dst, size_t n) {
  size_t got = 0;
  while (got < n) {
    const size_t r = fread(static_cast<char *>(dst) + got, 1, n - got, f);
    if (r == 0) break;
    got += r;
  }
  return got;
}

struct Files {
  std::vector<FILE *> f;
  ~Files() {
    for (FILE *x : f)
      if (x) fclose(x);
  }
};

struct DevBuf {
  void *p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};
struct HostBuf {
  void *p = nullptr;
  ~HostBuf() {
    if (p) cudaFreeHost(p);
  }
};

// src/net2net_forge.php:29-102 (merge_models) and src/train_cluster.php:144-224
// (average_models_stream): the first file's header (every header must equal
// it), then float j = fp32((sum_i double(x_i[j])) / n) for every float of
// the first file; a shorter file contributes 0.0 past its end.
int merge_files(const char *const *paths, int n, const char *out_path, int device) {
  clear_error();
  if (!paths || n < 1 || n > kMergeMaxSources || !out_path) {
    set_error("merge needs 1..%d input files and an output path", kMergeMaxSources);
    return -2;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    set_error("device %d not available", device);
    return -2;
  }
  DeviceGuard g(device);
  Files in;
  unsigned char hdr0[28];
  for (int i = 0; i < n; ++i) {
    FILE *f = paths[i] ? fopen(paths[i], "rb") : nullptr;
    if (!f) {
      set_error("cannot read %s", paths[i] ? paths[i] : "(null)");
      return -2;
    }
    in.f.push_back(f);
    unsigned char h[28];
    const size_t got = read_full(f, h, 28);
    if (i == 0) {
      memcpy(hdr0, h, 28);
      if (got != 28) {
        set_error("%s: short header", paths[0]);
        return -2;
      }
    } else if (got != 28 || memcmp(h, hdr0, 28) != 0) {
      set_error("%s: header differs from %s (model shapes do not match)", paths[i], paths[0]);
      return -2;
    }
  }
  FILE *out = fopen(out_path, "wb");
  if (!out) {
    set_error("cannot write %s", out_path);
    return -2;
  }
  Files outf;
  outf.f.push_back(out);
  if (fwrite(hdr0, 1, 28, out) != 28) {
    set_error("write to %s failed", out_path);
    return -2;
  }
  constexpr size_t kChunk = 4u << 20;  // floats per file per round
  HostBuf hin, hout;
  DevBuf din, dout;
  cudaStream_t st = nullptr;
  if (cudaHostAlloc(&hin.p, kChunk * 4 * n, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(&hout.p, kChunk * 4, cudaHostAllocDefault) != cudaSuccess ||
      cudaMalloc(&din.p, kChunk * 4 * n) != cudaSuccess || cudaMalloc(&dout.p, kChunk * 4) != cudaSuccess ||
      cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("merge buffers: %s", cudaGetErrorString(cudaGetLastError()));
    if (st) cudaStreamDestroy(st);
    return -3;
  }
  float *hi = static_cast<float *>(hin.p), *ho = static_cast<float *>(hout.p);
  float *di = static_cast<float *>(din.p), *dd = static_cast<float *>(dout.p);
  int rc = 0;
  for (;;) {
    const size_t got0 = read_full(in.f[0], hi, kChunk * 4);
    const size_t nf = got0 / 4;  // whole floats of the first file (intval(strlen / 4))
    if (got0 == 0) break;
    for (int i = 1; i < n; ++i) {
      const size_t gi = read_full(in.f[i], hi + (size_t)i * kChunk, nf * 4) / 4;
      std::fill(hi + (size_t)i * kChunk + gi, hi + (size_t)i * kChunk + nf, 0.0f);  // past the end: 0.0
    }
    MergeSources srcs;
    srcs.n = n;
    for (int i = 0; i < n; ++i) srcs.src[i] = di + (size_t)i * kChunk;
    bool ok = true;
    for (int i = 0; ok && i < n; ++i)
      ok = cudaMemcpyAsync(di + (size_t)i * kChunk, hi + (size_t)i * kChunk, nf * 4, cudaMemcpyHostToDevice, st) ==
           cudaSuccess;
    ok = ok && launch_merge_mean(srcs, dd, nf, device, st) == 0 &&
         cudaMemcpyAsync(ho, dd, nf * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
         cudaStreamSynchronize(st) == cudaSuccess;
    if (!ok) {
      set_error("merge on device %d failed: %s", device, cudaGetErrorString(cudaGetLastError()));
      rc = -4;
      break;
    }
    if (fwrite(ho, 4, nf, out) != nf) {
      set_error("write to %s failed", out_path);
      rc = -2;
      break;
    }
    if (got0 < kChunk * 4) break;
  }
  cudaStreamDestroy(st);
  return rc;
}

// src/net2net_forge.php:149-214 upscale_model on the GPU.
int upscale_file(const char *in_path, const char *out_path, int target_dim, uint64_t seed, int device) {
  clear_error();
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    set_error("device %d not available", device);
    return -2;
  }
  FILE *f = in_path ? fopen(in_path, "rb") : nullptr;
  if (!f) {
    set_error("input file not found: %s", in_path ? in_path : "(null)");
    return -2;
  }
  Files in;
  in.f.push_back(f);
  unsigned char hdr[28];
  if (read_full(f, hdr, 28) != 28) {
    set_error("%s: short header", in_path);
    return -2;
  }
  uint32_t p[5];
  for (int i = 0; i < 5; ++i)
    p[i] = (uint32_t)hdr[8 + 4 * i] | ((uint32_t)hdr[9 + 4 * i] << 8) | ((uint32_t)hdr[10 + 4 * i] << 16) |
           ((uint32_t)hdr[11 + 4 * i] << 24);
  const int64_t vocab = p[0], old_dim = p[1], old_ffn = p[2], old_ctx = p[3], old_layers = p[4];
  if (target_dim <= old_dim) {
    set_error("target dimension %d must be larger than the current %lld", target_dim, (long long)old_dim);
    return -2;
  }
  if (vocab < 1 || old_dim < 1 || old_layers < 1 || target_dim > 65536 || vocab * (int64_t)target_dim > (1ll << 33)) {
    set_error("%s: unsupported shape", in_path);
    return -2;
  }
  const int64_t new_dim = target_dim, new_ffn = 4 * new_dim, new_ctx = old_ctx * 2, new_layers = old_layers * 2;
  // the whole input (missing floats of a short file read as 0.0, like the reference's unpack of a short row)
  const int64_t layer_floats = 2 * old_dim + 4 * old_dim * old_dim + 2 * old_dim * old_ffn;
  const int64_t in_floats = 2 * vocab * old_dim + old_dim + old_layers * layer_floats;
  std::vector<float> src((size_t)in_floats, 0.0f);
  read_full(f, src.data(), (size_t)in_floats * 4);
  FILE *out = out_path ? fopen(out_path, "wb") : nullptr;
  if (!out) {
    set_error("cannot write %s", out_path ? out_path : "(null)");
    return -2;
  }
  Files outf;
  outf.f.push_back(out);
  unsigned char oh[28];
  memcpy(oh, hdr, 8);  // the input's magic
  const uint32_t np[5] = {(uint32_t)vocab, (uint32_t)new_dim, (uint32_t)new_ffn, (uint32_t)new_ctx,
                          (uint32_t)new_layers};
  for (int i = 0; i < 5; ++i)
    for (int b = 0; b < 4; ++b) oh[8 + 4 * i + b] = (unsigned char)(np[i] >> (8 * b));
  if (fwrite(oh, 1, 28, out) != 28) {
    set_error("write to %s failed", out_path);
    return -2;
  }
  DeviceGuard g(device);
  const size_t max_new = (size_t)std::max<int64_t>({vocab * new_dim, new_ffn * new_dim});
  const size_t max_old = (size_t)std::max<int64_t>({vocab * old_dim, old_ffn * old_dim, old_dim * old_dim});
  DevBuf dold, dnew;
  std::vector<float> host(max_new);
  if (cudaMalloc(&dold.p, max_old * 4) != cudaSuccess || cudaMalloc(&dnew.p, max_new * 4) != cudaSuccess) {
    set_error("upscale buffers: %s", cudaGetErrorString(cudaGetLastError()));
    return -3;
  }
  uint64_t stream = 0;  // output tensor index: keys the noise
  auto grow = [&](const float *old, int64_t orr, int64_t oc, int64_t nr, int64_t nc, double scale) -> int {
    if (cudaMemcpy(dold.p, old, (size_t)(orr * oc) * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_upscale_tensor(static_cast<float *>(dold.p), (int)orr, (int)oc, static_cast<float *>(dnew.p), (int)nr,
                              (int)nc, scale, seed, stream++, device, nullptr) != 0 ||
        cudaMemcpy(host.data(), dnew.p, (size_t)(nr * nc) * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
      set_error("upscale on device %d failed: %s", device, cudaGetErrorString(cudaGetLastError()));
      return -4;
    }
    if (fwrite(host.data(), 4, (size_t)(nr * nc), out) != (size_t)(nr * nc)) {
      set_error("write to %s failed", out_path);
      return -2;
    }
    return 0;
  };
  const float *at = src.data();
  int rc = grow(at, vocab, old_dim, vocab, new_dim, 1.0);  // embeddings
  at += vocab * old_dim;
  if (!rc) rc = grow(at, vocab, old_dim, vocab, new_dim, 1.0);  // w_out
  at += vocab * old_dim;
  if (!rc) rc = grow(at, 1, old_dim, 1, new_dim, 1.0);  // rms_final
  at += old_dim;
  const float *layer0 = at;
  for (int64_t l = 0; !rc && l < new_layers; ++l) {
    const float *q = layer0 + (l % old_layers) * layer_floats;  // new layers repeat l % old_layers
    const double os = l >= old_layers ? 0.01 : 1.0;              // Wo and W_down of a new layer
    const int64_t dd = old_dim * old_dim;
    if (!rc) rc = grow(q, 1, old_dim, 1, new_dim, 1.0);
    if (!rc) rc = grow(q + old_dim, 1, old_dim, 1, new_dim, 1.0);
    if (!rc) rc = grow(q + 2 * old_dim, old_dim, old_dim, new_dim, new_dim, 1.0);
    if (!rc) rc = grow(q + 2 * old_dim + dd, old_dim, old_dim, new_dim, new_dim, 1.0);
    if (!rc) rc = grow(q + 2 * old_dim + 2 * dd, old_dim, old_dim, new_dim, new_dim, 1.0);
    if (!rc) rc = grow(q + 2 * old_dim + 3 * dd, old_dim, old_dim, new_dim, new_dim, os);
    if (!rc) rc = grow(q + 2 * old_dim + 4 * dd, old_ffn, old_dim, new_ffn, new_dim, 1.0);
    if (!rc) rc = grow(q + 2 * old_dim + 4 * dd + old_ffn * old_dim, old_dim, old_ffn, new_dim, new_ffn, os);
  }
  return rc;
}

// The federated average of engines' weights in GPU memory: every engine ends
// with fp32((sum_i double(w_i)) / n), summed in engine order.  Device g
// computes shard g of the weight block from every engine's copy (peer loads
// over NVLink where the copies are on other GPUs) into a buffer of its own;
// once all shards exist, every engine copies them into its weights (peer
// copies) and packs its bf16 copies.
int average_engines(Engine *const *es, int n) {
  if (n < 1 || n > kMergeMaxSources) {
    set_error("averaging needs 1..%d engines", kMergeMaxSources);
    return -2;
  }
  for (int i = 0; i < n; ++i) {
    if (!es[i]) {
      set_error("engine %d is NULL", i);
      return -1;
    }
    const Dims &a = es[0]->d, &b = es[i]->d;
    if (a.V != b.V || a.D != b.D || a.L != b.L || es[i]->wblock_bytes != es[0]->wblock_bytes) {
      set_error("engine %d has another model shape than engine 0", i);
      return -2;
    }
  }
  const size_t E = es[0]->wblock_bytes / 4;
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(es[i]->device);
    cudaStreamSynchronize(es[i]->stream);
    for (int j = 0; j < n; ++j) {
      if (es[j]->device == es[i]->device) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, es[i]->device, es[j]->device) != cudaSuccess || !can) {
        set_error("device %d cannot read device %d's memory", es[i]->device, es[j]->device);
        return -5;
      }
      const cudaError_t pe = cudaDeviceEnablePeerAccess(es[j]->device, 0);
      if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) {
        set_error("peer access %d -> %d: %s", es[i]->device, es[j]->device, cudaGetErrorString(pe));
        return -5;
      }
      cudaGetLastError();
    }
  }
  std::vector<float *> part(n);
  std::vector<size_t> a0(n), cnt(n);
  for (int i = 0; i <= n; ++i) {  // shard boundaries on 64-float (256-byte) multiples
    const size_t b = i == n ? E : E * i / n / 64 * 64;
    if (i < n) a0[i] = b;
    if (i > 0) cnt[i - 1] = b - a0[i - 1];
  }
  MergeSources srcs;
  srcs.n = n;
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(es[i]->device);
    for (int j = 0; j < n; ++j) srcs.src[j] = static_cast<const float *>(es[j]->wblock) + a0[i];
    Engine &e = *es[i];
    const size_t need = std::max<size_t>(cnt[i], 1) * 4;
    if (e.avg_tmp_bytes < need) {  // a shard buffer per engine, kept for later averages
      cudaFree(e.avg_tmp);
      e.avg_tmp = nullptr;
      e.avg_tmp_bytes = 0;
      if (cudaMalloc(&e.avg_tmp, need) != cudaSuccess) {
        set_error("average buffer on device %d: %s", e.device, cudaGetErrorString(cudaGetLastError()));
        return -3;
      }
      e.avg_tmp_bytes = need;
    }
    part[i] = static_cast<float *>(e.avg_tmp);
    if (launch_merge_mean(srcs, part[i], cnt[i], es[i]->device, es[i]->stream) != 0) {
      set_error("average on device %d failed: %s", es[i]->device, cudaGetErrorString(cudaGetLastError()));
      return -4;
    }
  }
  for (int i = 0; i < n; ++i) {  // every shard is done before any engine's weights change
    DeviceGuard g(es[i]->device);
    if (cudaStreamSynchronize(es[i]->stream) != cudaSuccess) {
      set_error("average on device %d failed: %s", es[i]->device, cudaGetErrorString(cudaGetLastError()));
      return -4;
    }
  }
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(es[i]->device);
    for (int j = 0; j < n; ++j)
      if (cudaMemcpyPeerAsync(static_cast<float *>(es[i]->wblock) + a0[j], es[i]->device, part[j], es[j]->device,
                              cnt[j] * 4, es[i]->stream) != cudaSuccess) {
        set_error("shard copy %d -> %d failed: %s", es[j]->device, es[i]->device,
                  cudaGetErrorString(cudaGetLastError()));
        return -4;
      }
    if (refresh_bf16(*es[i])) {
      set_error("bf16 packing on device %d failed", es[i]->device);
      return -4;
    }
  }
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(es[i]->device);
    if (cudaStreamSynchronize(es[i]->stream) != cudaSuccess) {
      set_error("average on device %d failed: %s", es[i]->device, cudaGetErrorString(cudaGetLastError()));
      return -4;
    }
  }
  return 0;
}

}  // namespace
}  // namespace snai

extern "C" int cortex_merge_files(const char *const *paths, int n, const char *out_path, int device) {
  return merge_files(paths, n, out_path, device);
}

extern "C" int cortex_upscale_file(const char *in_path, const char *out_path, int target_dim,
                                   unsigned long long seed, int device) {
  return upscale_file(in_path, out_path, target_dim, seed, device);
}

extern "C" int cortex_average_states(void *const *states, int n) {
  clear_error();
  if (!states) {
    set_error("states is NULL");
    return -1;
  }
  std::vector<Engine *> es(n > 0 ? n : 0);
  for (int i = 0; i < n; ++i) es[i] = static_cast<Engine *>(states[i]);
  return average_engines(es.data(), n);
}

extern "C" int cortex_group_average(void *group) {
  clear_error();
  Group *g = static_cast<Group *>(group);
  if (!g) {
    set_error("group is NULL");
    return -1;
  }
  return average_engines(g->engines.data(), (int)g->engines.size());
}

// ============================================================================
// Forward pass without allocation
// ============================================================================
//
// Some callers must not allocate GPU memory while they run: hosts whose
// device memory is owned by another allocator (a framework's caching
// allocator, a fixed pool handed out at start-up) or code paths where a
// cudaMalloc would stall or fail.  cortex_forward_batch_noalloc runs the same
// forward pass as cortex_forward_batch, but keeps the pass's activation
// scratch (row lists, hidden states, normed inputs, q, attention output, MLP
// intermediate) in the file-scope device array below instead of buffers the
// state owns.  The array is kNoAllocScratchBytes on every GPU that loads this
// library and stays resident until the process exits.
namespace snai {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  The host-side
// name is only a stand-in for the symbol, so the address is looked up with
// the state's device current.  It is looked up on every call (cheap once
// the module is loaded, and no allocation), so a context that was reset and
// made again never sees a stale address.
int noalloc_scratch(int dev, void **out) {
  void *p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (err != cudaSuccess || !p) {
    set_error("cudaGetSymbolAddress(no-alloc scratch) failed on device %d: %s", dev, cudaGetErrorString(err));
    cudaGetLastError();
    return -4;
  }
  *out = p;
  return 0;
}

// Lays the per-row activation buffers of `rows` rows out in `base`; returns
// the bytes used (the same buffers create_engine carves for m_max rows).
size_t carve_rows(Engine &e, int rows, void *base) {
  const size_t M = rows, D = e.d.D, F = e.d.F;
  Carver a;
  a.add(&e.rows_d, M);
  a.add(&e.outrows_d, M);
  a.add(&e.h, M * D);
  a.add(&e.x, M * D * sizeof(float));
  a.add(&e.q, M * (size_t)e.d.att_ch);
  a.add(&e.kvs, M * 2 * (size_t)e.d.att_ch);
  a.add(&e.att, M * D * sizeof(float));
  a.add(&e.u, M * F * sizeof(float));
  a.add(&e.xo, M * D * sizeof(float));
  if (base) a.place(base);
  return a.off;
}

}  // namespace
}  // namespace snai

extern "C" int cortex_forward_batch_noalloc(void *state, const int *tokens, int batch, int n_tok, const int *slots,
                                            float *logits, int flags) {
  clear_error();
  if (!state) {
    set_error("state is NULL");
    return -1;
  }
  Engine &e = *static_cast<Engine *>(state);
  DeviceGuard g(e.device);
  void *scratch = nullptr;
  int rc = noalloc_scratch(e.device, &scratch);
  if (rc) return rc;
  // rows per chunk that fit the scratch (chunks of any count keep batches unlimited)
  Engine probe = {};
  probe.d = e.d;
  const size_t one = carve_rows(probe, 1, nullptr);
  int rows = (int)std::min<size_t>((size_t)e.m_max, kNoAllocScratchBytes / std::max<size_t>(one, 1));
  while (rows > 0 && carve_rows(probe, rows, nullptr) > kNoAllocScratchBytes) --rows;
  // whole 128-row tensor-core tiles per chunk when the array holds them (the
  // state's own chunks are multiples of 128 rows too)
  if (rows > 128) rows = rows / 128 * 128;
  if (rows < 1) {
    set_error("no-alloc forward: one row of this model needs %zu bytes of scratch, more than the %zu-byte array",
              one, kNoAllocScratchBytes);
    return -2;
  }
  // Point the pass at the static scratch, run it, restore the state's own buffers.
  RowDesc *rows_d = e.rows_d;
  int2 *outrows_d = e.outrows_d;
  float *h = e.h, *q = e.q, *kvs = e.kvs;
  void *x = e.x, *att = e.att, *u = e.u, *xo = e.xo;
  const int m_max = e.m_max;
  carve_rows(e, rows, scratch);
  e.m_max = rows;
  rc = forward_batch(e, tokens, batch, n_tok, slots, logits, flags);
  e.rows_d = rows_d;
  e.outrows_d = outrows_d;
  e.h = h;
  e.q = q;
  e.kvs = kvs;
  e.x = x;
  e.att = att;
  e.u = u;
  e.xo = xo;
  e.m_max = m_max;
  return rc;
}
