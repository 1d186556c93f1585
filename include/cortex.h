/*
 * cortex.h - C ABI of libcortex.so, the B200 (sm_100a) decode engine.
 *
 * Part 1 is the reference's boundary: the thirteen symbols core/cortex.nim
 * exports with {.exportc, dynlib, cdecl.} (core/cortex.nim:16) and that the
 * PHP host binds with FFI::cdef (src/tensor_ffi_adapter.php:46-61,
 * src/snai_inference.php:84-91).  Names, argument types, argument meaning,
 * ownership and error behaviour are the reference's; each declaration names
 * the line it replaces.  PHP resolves every declared symbol when it parses
 * the cdef block, so all of them exist, including the training ones.
 *
 * Part 2 is an additive batched API (the PHP host does not need it): many
 * independent sequences ("slots") per state, token ids sampled on the GPU
 * with the reference's two samplers, and a stateless sampler over device
 * logits.  All functions of part 2 return 0 on success and a negative code on
 * failure; cortex_last_error() then describes the failure.
 *
 * Threading: a state is used by one host thread at a time (the reference is
 * single-threaded too, core/cortex.nim:61).  Different states may live on
 * different GPUs and be driven from different threads.
 */
#ifndef SNAI_CORTEX_H
#define SNAI_CORTEX_H

#include <stdbool.h>

#if defined(__GNUC__)
#define CORTEX_API __attribute__((visibility("default")))
#else
#define CORTEX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== */
/* Part 1 - reference boundary                                              */
/* ======================================================================== */

/* core/cortex.nim:261 cortex_init.  Allocates a state of the given shape with
 * zero weights and unit RMSNorm weights (core/cortex.nim:433-438).  ffn is
 * 4*dim; head size is dim/heads forced even and >= 2 (:267-271).  NULL on
 * failure (no GPU, out of memory, unsupported shape). */
CORTEX_API void *cortex_init(int vocab_size, int hidden_dim, int ctx_size, int num_layers, int num_heads);

/* core/cortex.nim:978 cortex_load_stream.  Reads a SNAI_V4 file (28-byte
 * header: magic[8], vocab, hidden, ffn, ctx, layers as u32 LE, then fp32 LE
 * tensors in the order of core/cortex.nim:1002-1041).  NULL when the file
 * cannot be opened, the magic is not "SNAI_V4" or a read comes up short. */
CORTEX_API void *cortex_load_stream(const char *filepath, int num_heads);

/* core/cortex.nim:487 cortex_forward.  Feeds num_tokens ids (out-of-range ids
 * read as 0, :493) at the next cache positions; stops silently at ctx
 * (:495).  Writes vocab fp32 logits of the last token into the caller's
 * buffer, before returning, only if that token was processed.  If the GPU
 * fails, the logits are set to NaN (which the PHP host's NaN check at
 * src/snai_inference.php:146 turns into a stop) and cortex_last_error() says
 * why. */
CORTEX_API void cortex_forward(void *state, int *raw_tokens, int num_tokens, float *raw_logits);

/* core/cortex.nim:484 cortex_reset_cache: the next token goes to position 0. */
CORTEX_API void cortex_reset_cache(void *state);

/* core/cortex.nim:824 cortex_free.  NULL-safe. */
CORTEX_API void cortex_free(void *state);

/* core/cortex.nim:1046 cortex_init_gpu.  Selects and initialises the CUDA
 * device (SNAI_DEVICE, default 0).  Unlike the reference it does not claim
 * success on failure: the failure is kept in cortex_last_error(). */
CORTEX_API void cortex_init_gpu(void);

/* core/cortex.nim:1050 / :1054.  0 for a NULL state. */
CORTEX_API int get_vocab_size(void *state);
CORTEX_API int get_ctx_size(void *state);

/* core/cortex.nim:464 / :469.  Copies one tensor in or out by (layer, type):
 * layer -1: 0 embeddings [V,d], 1 w_out [V,d], 2 rms_final [d];
 * layer l : 10 rms_att, 11 rms_ffn [d], 12 Wq, 13 Wk, 14 Wv, 15 Wo [d,d],
 *           16 W_up [4d,d], 17 W_down [d,4d]  (fp32, row-major).
 * A size mismatch or unknown (layer, type) is a silent no-op (:465). */
CORTEX_API void cortex_load_layer(void *state, int layer_idx, int tensor_type, float *raw_weights, int num_weights);
CORTEX_API void cortex_extract_layer(void *state, int layer_idx, int tensor_type, float *raw_weights, int num_weights);

/* core/cortex.nim:474 / :479.  Adam moment storage per tensor (m when
 * is_variance is false, v otherwise), in device memory beside the weights;
 * zero until loaded or trained (allocShared0). */
CORTEX_API void cortex_load_adam_layer(void *state, int layer_idx, int tensor_type, bool is_variance, float *raw, int size);
CORTEX_API void cortex_extract_adam_layer(void *state, int layer_idx, int tensor_type, bool is_variance, float *raw, int size);

/* core/cortex.nim:565 cortex_train_step.  One sequence of act =
 * min(num_tokens, ctx) input ids and their targets (ids outside [0, V) read
 * as 0): forward over every position with the activations kept, softmax
 * cross-entropy, backpropagation through every position, the global
 * gradient-norm clip at 1.0 (:230-258) and one Adam step (b1 0.9, b2 0.999,
 * eps 1e-8, gradients divided by act; the embedding skips rows whose
 * gradient is 0, :145-207).  Returns the mean loss (0 when act <= 0, with
 * nothing changed).  Like the reference it leaves the K/V rows of positions
 * 0..act-1 in the sequence's (slot 0's) cache and its position unchanged.
 * fp32 arithmetic throughout (the GEMMs sum in another order than the
 * reference's sequential loops).  On failure returns NaN (the PHP worker
 * stops on a NaN loss, src/train_worker.php:152-155) and sets
 * cortex_last_error(). */
CORTEX_API float cortex_train_step(void *state, int *raw_inputs, int *raw_targets, int num_tokens, float lr);

/* ======================================================================== */
/* Part 2 - batched extension                                               */
/* ======================================================================== */

/* GEMM operand precision.  FP32 runs every projection as fp32 FFMA GEMV
 * (closest to the reference).  TF32 / BF16 run every projection on tcgen05
 * tensor cores (fp32 accumulate), whatever the number of rows in a pass, so
 * a sequence's results do not depend on the other sequences of its pass. */
#define SNAI_PREC_FP32 0
#define SNAI_PREC_TF32 1
#define SNAI_PREC_BF16 2

/* Pointer-location flag for the batched calls. */
#define SNAI_HOST_PTRS 0   /* tokens, uniforms, ids, logits are host memory; the call returns when done */
#define SNAI_DEVICE_PTRS 1 /* device memory; work is queued on the state's stream, no host wait */

/* The two samplers of the reference.
 * variant 0 = src/snai_inference.php:151-195: logits /= temperature (stored as
 *   fp32), repetition penalty over the unique history (L>0: /= rep, else *= rep,
 *   stored as fp32), greedy iff temperature <= 0.01, else softmax (double) and
 *   the first id whose running sum reaches u*sum.
 * variant 1 = src/tensor_ffi_adapter.php:168-204: subtract rep from the logits
 *   of ids in the history, stable descending order, keep top_k, greedy iff
 *   temperature < 0.01, else exp(v/T) (no max shift), keep the prefix whose
 *   running sum reaches top_p, then the first id with u*cum <= running sum.
 * u comes from the caller (one fp32 uniform per row) in place of
 * mt_rand()/mt_getrandmax().  nan_guard (variant 0 only): a row whose logit 0
 * is NaN yields id -1, as the host loop's NaN check stops there
 * (src/snai_inference.php:146). */
typedef struct snai_sample_params {
  int variant;
  double temperature;
  double rep_penalty;
  int top_k;    /* variant 1; 1 <= top_k <= 512 */
  double top_p; /* variant 1 */
  int nan_guard;
} snai_sample_params;

/* Last error of the calling thread ("" if none). */
CORTEX_API const char *cortex_last_error(void);

/* cortex_load_stream with max_seqs independent sequence slots on CUDA device
 * `device`, using the given GEMM precision. */
CORTEX_API void *cortex_load_stream_ex(const char *filepath, int num_heads, int max_seqs, int device, int precision);

/* cortex_init with slots, device and precision. */
CORTEX_API void *cortex_init_ex(int vocab_size, int hidden_dim, int ctx_size, int num_layers, int num_heads, int max_seqs,
                     int device, int precision);

CORTEX_API int cortex_num_slots(void *state);
CORTEX_API int cortex_head_size(void *state);
CORTEX_API int cortex_num_heads(void *state);

/* Resets the given slots (all slots when slots is NULL) to position 0. */
CORTEX_API int cortex_seq_reset(void *state, const int *slots, int n);

/* Current cache position of a slot (-1 on error). */
CORTEX_API int cortex_seq_pos(void *state, int slot);

/* Feeds n_tok tokens to each of `batch` slots (tokens row-major [batch][n_tok];
 * slots[b], or b when slots is NULL).  Each slot behaves as cortex_forward on
 * its own cache (ctx cut-off per slot).  The logits of each slot's last token
 * stay on the device for cortex_decode_batch; if `logits` is not NULL they are
 * also copied to logits[b][vocab] for the slots whose last token was
 * processed.  flags: SNAI_HOST_PTRS or SNAI_DEVICE_PTRS. */
CORTEX_API int cortex_forward_batch(void *state, const int *tokens, int batch, int n_tok, const int *slots, float *logits,
                         int flags);

/* One step of the host loop of src/snai_inference.php:139-215 for `batch`
 * slots at once: sample an id per slot from its current logits (history =
 * every token fed to the slot so far), then feed that id.  uniforms[b] is the
 * draw of row b; out_ids[b] receives the sampled id. */
CORTEX_API int cortex_decode_batch(void *state, const int *slots, int batch, const float *uniforms,
                        const snai_sample_params *params, int *out_ids, int flags);

/* `steps` consecutive cortex_decode_batch steps: step k uses uniforms[k][b]
 * and writes out_ids[k][b] (both [steps][batch]).  One step is captured once
 * as a CUDA graph whose rows, uniforms and ids live on the device, and
 * replayed: a launch-bound small batch pays one graph launch per step.  The
 * result equals `steps` calls of cortex_decode_batch.  Falls back to those
 * calls while the profiler is on or when a slot would reach the context
 * limit within the steps.  No reference counterpart (the PHP host samples one
 * token per FFI call). */
CORTEX_API int cortex_decode_steps(void *state, const int *slots, int batch, int steps, const float *uniforms,
                                   const snai_sample_params *params, int *out_ids, int flags);

/* Copies the current device logits of the given slots to host memory
 * out[n][vocab]. */
CORTEX_API int cortex_get_logits(void *state, const int *slots, int n, float *out);

/* Stateless sampler over device memory: logits[rows][ld] (row stride ld >=
 * vocab), history ids hist[rows][hist_cols] of which hist_len[r] (all
 * hist_cols when hist_len is NULL) are used, uniforms[rows], out_ids[rows].
 * Queued on `stream` (a cudaStream_t; NULL = legacy default stream). */
CORTEX_API int cortex_sample(const float *logits, int rows, int vocab, long long ld, const int *hist, int hist_cols,
                  const int *hist_len, const float *uniforms, const snai_sample_params *params, int *out_ids,
                  void *stream);

/* Makes the state queue its work on `stream` (a cudaStream_t of the state's
 * device; NULL restores the state's own stream). */
CORTEX_API int cortex_set_stream(void *state, void *stream);

/* Waits for the state's queued work; reports a device-side error if any. */
CORTEX_API int cortex_synchronize(void *state);

/* Moves the given slots (all when slots is NULL) back to cache position
 * `pos` (<= their current position): later tokens are forgotten and will be
 * overwritten.  The slots' current logits are kept. */
CORTEX_API int cortex_seq_rewind(void *state, const int *slots, int n, int pos);

/* Kernel-class profiler.  When on, every launch is bracketed by CUDA events
 * on the state's stream and its algorithmic bytes and FLOPs are counted.
 * kind: 0 embedding+norm, 1 rmsnorm, 2 QKV projection, 3 attention,
 * 4 Wo projection, 5 W_up, 6 W_down, 7 logits projection, 8 sampler,
 * 9 the persistent kernel of a whole one- or two-row fp32 decode pass.
 * Enabling (or disabling) clears the counters; reading waits for the
 * stream. */
CORTEX_API int cortex_profile_enable(void *state, int on);
CORTEX_API int cortex_profile_read(void *state, int kind, long long *launches, double *ms, double *bytes,
                                   double *flops);

/* cortex_forward_batch for callers that must not allocate GPU memory during
 * the call (their device memory belongs to another allocator or a fixed
 * pool, or an allocation would stall a latency-critical path).  No
 * counterpart in the reference.  Same arguments, results and per-slot
 * effects as cortex_forward_batch; the pass's activation scratch lives in
 * one 8 MiB array in the library's device image instead of the state's
 * buffers, and the call makes no cudaMalloc/cudaFree or other allocating
 * GPU call.  Rows are processed in chunks that fit the array (whole 128-row
 * tiles when more than 128 rows fit); a model whose single row needs more
 * than 8 MiB of scratch is rejected with an error.  Every call looks the
 * array's device address up with the state's device current (the first
 * call on a device may load the library's device code, so make it before
 * any stream capture).  While the kernel profiler (cortex_profile_enable)
 * is on, its first calls create the CUDA events it brackets launches with;
 * with the profiler off nothing is created.  All calls on a device share
 * the array: calls that overlap on the GPU (two streams, two threads) race.
 * Nothing in the array has to start at zero: every byte a call reads it
 * wrote first. */
CORTEX_API int cortex_forward_batch_noalloc(void *state, const int *tokens, int batch, int n_tok, const int *slots,
                                            float *logits, int flags);

/* ------------------------------------------------------------------------ */
/* Engine groups: one process, several GPUs.  No counterpart in the          */
/* reference (one sequence per CortexState, core/cortex.nim:24-59); this is  */
/* how a single host process (the PHP host has no launcher) uses several     */
/* GPUs.  Sequences are independent, so a group splits total_seqs into      */
/* contiguous shards, shard i = [total*i/n, total*(i+1)/n) on devices[i]     */
/* (a device may be listed more than once), with no tensor exchanged         */
/* between the engines.                                                      */
/* ------------------------------------------------------------------------ */

/* Reads the SNAI_V4 file once (pinned double-buffered reads into the first
 * engine), copies the fp32 weights from the first GPU to the others by peer
 * copies, and packs the bf16 copies on every GPU.  NULL on failure (the
 * reasons of cortex_load_stream, or a device that cannot be used). */
CORTEX_API void *cortex_group_load(const char *filepath, int num_heads, int total_seqs, const int *devices,
                                   int n_devices, int precision);
CORTEX_API void cortex_group_free(void *group);
/* Number of engines; the i-th engine's state (usable with every cortex_*
 * call of part 2, e.g. cortex_seq_rewind); its shard. */
CORTEX_API int cortex_group_size(void *group);
CORTEX_API void *cortex_group_engine(void *group, int i);
CORTEX_API int cortex_group_shard(void *group, int i, int *first, int *count);
/* Wall seconds cortex_group_load took (file read, copies, packing). */
CORTEX_API double cortex_group_load_seconds(void *group);
/* cortex_forward_batch for every sequence of the group at once (host
 * memory): tokens [total][n_tok], logits [total][vocab] or NULL.  One host
 * thread per engine; returns when every engine is done. */
CORTEX_API int cortex_group_forward(void *group, const int *tokens, int n_tok, float *logits);
/* cortex_decode_steps for every sequence of the group (host memory):
 * uniforms [steps][total], out_ids [steps][total], gathered from the
 * engines by their threads. */
CORTEX_API int cortex_group_decode_steps(void *group, int steps, const float *uniforms,
                                         const snai_sample_params *params, int *out_ids);

/* ------------------------------------------------------------------------ */
/* Merging, federated averaging and Net2Net upscaling on the GPU.  The      */
/* reference does these in PHP outside the engine; here they are library    */
/* calls.  Return 0, or a negative code with cortex_last_error().           */
/* ------------------------------------------------------------------------ */

/* src/net2net_forge.php:29-102 merge_models / src/train_cluster.php:144-224
 * average_models_stream: writes out_path = the first file's 28-byte header
 * (every header must equal it, else -2) followed by, for every float j of
 * the first file, fp32((sum_i double(x_i[j])) / n) summed in file order (a
 * shorter file contributes 0.0 past its end).  1 <= n <= 64; the sums run
 * on `device`. */
CORTEX_API int cortex_merge_files(const char *const *paths, int n, const char *out_path, int device);

/* src/net2net_forge.php:149-214 upscale_model on `device`: hidden_dim ->
 * target_dim (> hidden_dim, else -2), ffn -> 4 * target_dim, ctx x 2,
 * layers x 2 (new layer l repeats l % old_layers, its Wo and W_down scaled
 * by 0.01); old entries fp32(double(x) * scale), new entries
 * fp32(((u * 2) - 1) * 0.005).  The reference draws u from mt_rand(); here
 * u comes from SplitMix64 keyed by (seed, output tensor, element), so the
 * same seed gives the same file. */
CORTEX_API int cortex_upscale_file(const char *in_path, const char *out_path, int target_dim, unsigned long long seed,
                                   int device);

/* The federated average (the arithmetic of src/train_cluster.php:144-224)
 * of n engine states' weights in GPU memory, typically one engine per GPU:
 * afterwards every state holds fp32((sum_i double(w_i)) / n), summed in
 * state order.  Each GPU computes its shard of the weights reading the
 * other GPUs' copies with peer loads over NVLink, then every GPU copies the
 * shards in (peer copies) and repacks its bf16 copies.  Same model shape
 * everywhere; 1 <= n <= 64.  KV caches and positions are untouched. */
CORTEX_API int cortex_average_states(void *const *states, int n);
/* cortex_average_states over a group's engines. */
CORTEX_API int cortex_group_average(void *group);

/* ------------------------------------------------------------------------ */
/* The reference's BPE tokenizer (src/snai_tokenizer.php) as library calls. */
/* ------------------------------------------------------------------------ */

/* src/snai_tokenizer.php:23-38: loads the HF-style vocabulary JSON
 * (model.vocab, model.merges; e.g. lib/symbio_vocab.json).  NULL on failure.
 * A tokenizer may be shared by threads (its merge cache is locked). */
CORTEX_API void *cortex_tokenizer_load(const char *vocab_json);
CORTEX_API void cortex_tokenizer_free(void *tok);
/* src/snai_tokenizer.php:41-43 getVocabSize. */
CORTEX_API int cortex_tokenizer_vocab_size(void *tok);
/* src/snai_tokenizer.php:118-185 encode of text_len bytes (strlen when
 * text_len < 0): invalid UTF-8 -> '?', a leading ' ' unless the text starts
 * with ' ', '[' or '<', the special tokens split out, BPE per U+2581 chunk,
 * unknown pieces -> <unk>.  No NFKC (the PHP code applies it only when its
 * intl extension is loaded).  Writes up to max_ids ids and returns how many
 * the text has (negative on error). */
CORTEX_API int cortex_tokenizer_encode(void *tok, const char *text, int text_len, int *ids, int max_ids);
/* src/snai_tokenizer.php:187-199 decode: the ids' strings (unknown ids
 * skipped), U+2581 -> ' ', trimmed when trim != 0.  Writes at most
 * max_bytes - 1 bytes and a NUL; returns the full length in bytes. */
CORTEX_API int cortex_tokenizer_decode(void *tok, const int *ids, int n, int trim, char *out, int max_bytes);

/* Self-test of the failure path every kernel wait takes.  No counterpart in
 * the reference (whose engine has no device waits).  Queues one kernel on
 * the state's stream that waits on an mbarrier nothing completes; the wait
 * gives up after limit_ns (1 us .. 2 s) of GPU time, records its error code
 * in the state's device error word and returns, so the GPU context stays
 * usable.  The next cortex_synchronize then returns -6 and
 * cortex_last_error() names the expired wait; the error word is cleared by
 * that report.  Returns 0 once queued. */
CORTEX_API int cortex_selftest_wait_timeout(void *state, long long limit_ns);

/* ------------------------------------------------------------------------ */
/* The two halves of cortex_train_step, and its gradients.  No counterpart   */
/* in the reference (whose step is one call); for inspecting and testing a   */
/* step, and for callers that combine gradients before the update.           */
/* ------------------------------------------------------------------------ */

/* Forward, loss and backward of cortex_train_step (gradients of the summed
 * loss left in the state's gradient block, the weights unchanged).  Writes
 * the mean loss to *loss (0 when act <= 0).  Returns 0 or a negative code. */
CORTEX_API int cortex_train_grads(void *state, const int *raw_inputs, const int *raw_targets, int num_tokens,
                                  float *loss);
/* The clip and the Adam step of cortex_train_step on the current gradients,
 * with Adam's gradient divisor `scale` (cortex_train_step passes act).
 * Counts one Adam step.  Queued on the state's stream (no host wait). */
CORTEX_API int cortex_train_apply(void *state, float lr, float scale);
/* Gradient tensor by (layer, type) as cortex_load_layer / extract_layer;
 * a size mismatch is a silent no-op. */
CORTEX_API void cortex_load_grad_layer(void *state, int layer_idx, int tensor_type, const float *raw, int size);
CORTEX_API void cortex_extract_grad_layer(void *state, int layer_idx, int tensor_type, float *raw, int size);
/* Adam steps taken (the reference's adam_t), and the clip of the last
 * cortex_train_apply: its factor, the gradient norm and whether it applied.
 * Returns 0, or -1 before the first update. */
CORTEX_API int cortex_train_info(void *state, int *adam_steps, float *clip_factor, float *grad_norm, int *clipped);

/* Number of kernels the state has launched since it was created. */
CORTEX_API long long cortex_kernel_launches(void *state);

#ifdef __cplusplus
}
#endif

#endif /* SNAI_CORTEX_H */
