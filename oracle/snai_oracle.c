/*
 * snai_oracle.c - TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of the reference's decode path, used as the checker by
 * tests/, __graft_entry__.smoke() and the cpu_baseline / reference arm of
 * bench.py.  Nothing in the product (snai_b200/, libcortex.so) links, loads
 * or calls this file.
 *
 * PARITY UNPINNED: the reference engine is Nim (core/cortex.nim) and its host
 * is PHP (src/snai_inference.php, src/tensor_ffi_adapter.php).  Neither
 * toolchain exists on this machine or on the GPU machines, and the reference
 * ships no tests, fixtures or golden vectors, so this restatement is checked
 * only against hand-derived known-answer cases (tests/golden/).
 *
 * What is restated, line by line:
 *   core/cortex.nim:261-271   shape rules of cortex_init (ffn = 4*dim, head size)
 *   core/cortex.nim:74-87     applyRoPE   (powf / cosf / sinf in float32)
 *   core/cortex.nim:89-98     matVecMul   (CPU branch: sequential float sum)
 *   core/cortex.nim:117-123   applyRMSNorm (eps 1e-5, float32)
 *   core/cortex.nim:484-485   cortex_reset_cache
 *   core/cortex.nim:487-563   cortex_forward (token clamp, ctx break, KV append,
 *                             attention with max initialised to -9999, SiLU MLP,
 *                             logits for the last token only)
 *   core/cortex.nim:439-482   tensor type codes of load/extract layer
 *   core/cortex.nim:969-1044  cortex_load_stream (SNAI_V4 header + tensor order)
 *   core/cortex.nim:565-822   cortex_train_step (forward with saved activations,
 *                             softmax cross-entropy, BPTT in reverse position
 *                             order, global gradient-norm clip :230-258, Adam
 *                             :145-207 with the sparse embedding rule)
 *   core/cortex.nim:474-482   load/extract of the Adam moments
 *   src/snai_inference.php:151-195     sampler "variant A"
 *   src/tensor_ffi_adapter.php:168-204 sampler "variant B"
 *
 * Floating point: build with -O2 -ffp-contract=off and no -ffast-math, so every
 * float operation is rounded as the Nim-generated C rounds it (x86-64 SSE,
 * no FMA contraction).  The samplers work in double like PHP.  exp_mode 0
 * calls libm exp() (what PHP calls); exp_mode 1 calls the sampling contract's
 * snai_exp() (snai_b200/csrc/snai_exp.h), which the GPU sampler also uses.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "snai_exp.h"

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* Model and per-sequence state                                              */
/* ------------------------------------------------------------------------- */

typedef struct {
  int vocab, dim, ffn, ctx, layers, heads, hs;
  float *emb, *w_out, *rms_final;
  float **rms_att, **rms_ffn, **wq, **wk, **wv, **wo, **wup, **wdown;
} OModel;

typedef struct {
  const OModel *m;
  int cached;
  float **kc, **vc; /* [layers][ctx * dim], as core/cortex.nim:390-391 */
  float *h, *norm, *att, *ffn, *q, *scores, *tmp;
} OSeq;

struct OTrain;

/* The legacy-shaped handle: one model and one sequence (and, once a training
 * call has been made, the gradients, Adam moments and activations). */
typedef struct {
  OModel *m;
  OSeq *s;
  struct OTrain *tr;
} OState;

static void train_free(struct OTrain *t);

static float *zalloc(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

static OModel *model_new(int vocab, int dim, int ctx, int layers, int heads) {
  OModel *m = (OModel *)calloc(1, sizeof(OModel));
  m->vocab = vocab;
  m->dim = dim;
  m->ctx = ctx;
  m->layers = layers;
  m->ffn = dim * 4; /* core/cortex.nim:267: header ffn is ignored */
  m->heads = heads > 1 ? heads : 1;
  m->hs = dim / m->heads; /* :269-271 */
  if (m->hs % 2 != 0) m->hs -= 1;
  if (m->hs < 2) m->hs = 2;
  size_t vd = (size_t)vocab * dim, dd = (size_t)dim * dim, fd = (size_t)m->ffn * dim;
  m->emb = zalloc(vd);
  m->w_out = zalloc(vd);
  m->rms_final = zalloc(dim);
  float ***lists[] = {&m->rms_att, &m->rms_ffn, &m->wq, &m->wk, &m->wv, &m->wo, &m->wup, &m->wdown};
  for (int i = 0; i < 8; i++) *lists[i] = (float **)calloc(layers ? layers : 1, sizeof(float *));
  for (int l = 0; l < layers; l++) {
    m->rms_att[l] = zalloc(dim);
    m->rms_ffn[l] = zalloc(dim);
    m->wq[l] = zalloc(dd);
    m->wk[l] = zalloc(dd);
    m->wv[l] = zalloc(dd);
    m->wo[l] = zalloc(dd);
    m->wup[l] = zalloc(fd);
    m->wdown[l] = zalloc(fd);
    for (int i = 0; i < dim; i++) m->rms_att[l][i] = m->rms_ffn[l][i] = 1.0f; /* :433-435 */
  }
  for (int i = 0; i < dim; i++) m->rms_final[i] = 1.0f; /* :437-438 */
  return m;
}

static void model_free(OModel *m) {
  if (!m) return;
  for (int l = 0; l < m->layers; l++) {
    free(m->rms_att[l]); free(m->rms_ffn[l]); free(m->wq[l]); free(m->wk[l]);
    free(m->wv[l]); free(m->wo[l]); free(m->wup[l]); free(m->wdown[l]);
  }
  free(m->rms_att); free(m->rms_ffn); free(m->wq); free(m->wk); free(m->wv);
  free(m->wo); free(m->wup); free(m->wdown);
  free(m->emb); free(m->w_out); free(m->rms_final);
  free(m);
}

static OSeq *seq_new(const OModel *m) {
  OSeq *s = (OSeq *)calloc(1, sizeof(OSeq));
  s->m = m;
  s->kc = (float **)calloc(m->layers ? m->layers : 1, sizeof(float *));
  s->vc = (float **)calloc(m->layers ? m->layers : 1, sizeof(float *));
  for (int l = 0; l < m->layers; l++) {
    s->kc[l] = zalloc((size_t)m->ctx * m->dim);
    s->vc[l] = zalloc((size_t)m->ctx * m->dim);
  }
  s->h = zalloc(m->dim);
  s->norm = zalloc(m->dim);
  s->att = zalloc(m->dim);
  s->ffn = zalloc(m->ffn);
  s->q = zalloc(m->dim);
  s->scores = zalloc(m->ctx);
  s->tmp = zalloc(m->dim);
  return s;
}

static void seq_free(OSeq *s) {
  if (!s) return;
  for (int l = 0; l < s->m->layers; l++) { free(s->kc[l]); free(s->vc[l]); }
  free(s->kc); free(s->vc); free(s->h); free(s->norm); free(s->att);
  free(s->ffn); free(s->q); free(s->scores); free(s->tmp);
  free(s);
}

/* ------------------------------------------------------------------------- */
/* Math core, core/cortex.nim:74-123                                         */
/* ------------------------------------------------------------------------- */

static void apply_rope(float *vec, int dim, int hs, int pos) {
  int nh = dim / hs;
  for (int h = 0; h < nh; h++) {
    int off = h * hs;
    for (int i = 0; i + 1 <= hs - 1; i += 2) { /* countup(0, hs-1, 2) */
      float freq = 1.0f / powf(10000.0f, (float)i / (float)hs);
      float theta = (float)pos * freq;
      float c = cosf(theta);
      float s = 1.0f * sinf(theta);
      float v0 = vec[off + i], v1 = vec[off + i + 1];
      vec[off + i] = v0 * c - v1 * s;
      vec[off + i + 1] = v0 * s + v1 * c;
    }
  }
}

static void matvec(const float *w, int rows, int cols, const float *x, float *o) {
  for (int r = 0; r < rows; r++) {
    float s = 0.0f;
    const float *row = w + (size_t)r * cols;
    for (int c = 0; c < cols; c++) s += row[c] * x[c];
    o[r] = s;
  }
}

static void rmsnorm(const float *x, float *o, int dim, const float *w) {
  float ss = 0.0f;
  for (int d = 0; d < dim; d++) ss += x[d] * x[d];
  float inv = 1.0f / sqrtf((ss / (float)dim) + 1e-5f);
  for (int d = 0; d < dim; d++) o[d] = x[d] * inv * w[d];
}

/* core/cortex.nim:487-563 */
static void seq_forward(OSeq *st, const int *tokens, int n, float *logits) {
  const OModel *m = st->m;
  const int D = m->dim;
  for (int i = 0; i < n; i++) {
    int tid = tokens[i];
    if (tid < 0 || tid >= m->vocab) tid = 0;
    int pos = st->cached;
    if (pos >= m->ctx) break;
    memcpy(st->h, m->emb + (size_t)tid * D, sizeof(float) * D);
    for (int l = 0; l < m->layers; l++) {
      rmsnorm(st->h, st->norm, D, m->rms_att[l]);
      matvec(m->wq[l], D, D, st->norm, st->q);
      apply_rope(st->q, D, m->hs, pos);
      float *kp = st->kc[l] + (size_t)pos * D;
      float *vp = st->vc[l] + (size_t)pos * D;
      matvec(m->wk[l], D, D, st->norm, kp);
      apply_rope(kp, D, m->hs, pos);
      matvec(m->wv[l], D, D, st->norm, vp);
      for (int d = 0; d < D; d++) st->att[d] = 0.0f;
      for (int hh = 0; hh < m->heads; hh++) {
        int off = hh * m->hs;
        float max_s = -9999.0f;
        for (int t = 0; t <= pos; t++) {
          const float *tk = st->kc[l] + (size_t)t * D;
          float sc = 0.0f;
          for (int d = 0; d < m->hs; d++) sc += st->q[off + d] * tk[off + d];
          sc /= sqrtf((float)m->hs);
          st->scores[t] = sc;
          if (sc > max_s) max_s = sc;
        }
        float sum_e = 0.0f;
        for (int t = 0; t <= pos; t++) {
          st->scores[t] = expf(st->scores[t] - max_s);
          sum_e += st->scores[t];
        }
        for (int t = 0; t <= pos; t++) {
          float w = st->scores[t] / sum_e;
          const float *tv = st->vc[l] + (size_t)t * D;
          for (int d = 0; d < m->hs; d++) st->att[off + d] += tv[off + d] * w;
        }
      }
      matvec(m->wo[l], D, D, st->att, st->tmp);
      for (int d = 0; d < D; d++) st->h[d] += st->tmp[d];
      rmsnorm(st->h, st->norm, D, m->rms_ffn[l]);
      matvec(m->wup[l], m->ffn, D, st->norm, st->ffn);
      for (int d = 0; d < m->ffn; d++) {
        float v = st->ffn[d];
        st->ffn[d] = v * (1.0f / (1.0f + expf(-v)));
      }
      matvec(m->wdown[l], D, m->ffn, st->ffn, st->att);
      for (int d = 0; d < D; d++) st->h[d] += st->att[d];
    }
    rmsnorm(st->h, st->norm, D, m->rms_final);
    if (i == n - 1 && logits) {
      for (int v = 0; v < m->vocab; v++) {
        float s = 0.0f;
        const float *row = m->w_out + (size_t)v * D;
        for (int d = 0; d < D; d++) s += st->norm[d] * row[d];
        logits[v] = s;
      }
    }
    st->cached += 1;
  }
}

/* ------------------------------------------------------------------------- */
/* Legacy-shaped API                                                         */
/* ------------------------------------------------------------------------- */

EXPORT void *oracle_init(int vocab, int dim, int ctx, int layers, int heads) {
  OState *s = (OState *)calloc(1, sizeof(OState));
  s->m = model_new(vocab, dim, ctx, layers, heads);
  s->s = seq_new(s->m);
  return s;
}

/* core/cortex.nim:978-1044: header, magic check, then tensors in file order;
 * NULL on open failure, short read or bad magic. */
EXPORT void *oracle_load_stream(const char *path, int num_heads) {
  FILE *f = fopen(path, "rb");
  if (!f) return NULL;
  unsigned char hdr[28];
  if (fread(hdr, 1, 28, f) != 28) { fclose(f); return NULL; }
  char magic[9] = {0};
  int mi = 0;
  for (int i = 0; i < 8; i++) if (hdr[i] != 0) magic[mi++] = (char)hdr[i];
  if (strcmp(magic, "SNAI_V4") != 0) { fclose(f); return NULL; }
  uint32_t p[5];
  for (int i = 0; i < 5; i++)
    p[i] = (uint32_t)hdr[8 + 4 * i] | ((uint32_t)hdr[9 + 4 * i] << 8) |
           ((uint32_t)hdr[10 + 4 * i] << 16) | ((uint32_t)hdr[11 + 4 * i] << 24);
  uint32_t vocab = p[0], dim = p[1], ffn = p[2], ctx = p[3], layers = p[4];
  if ((uint64_t)ffn > 4ull * dim) { fclose(f); return NULL; } /* would overflow w_up */
  OState *s = (OState *)oracle_init((int)vocab, (int)dim, (int)ctx, (int)layers, num_heads);
  OModel *m = s->m;
#define BLAST(dst, cnt)                                                  \
  do {                                                                   \
    size_t c_ = (size_t)(cnt);                                           \
    if (fread((dst), sizeof(float), c_, f) != c_) {                      \
      fclose(f);                                                         \
      seq_free(s->s); model_free(s->m); free(s);                         \
      return NULL;                                                       \
    }                                                                    \
  } while (0)
  BLAST(m->emb, (size_t)vocab * dim);
  BLAST(m->w_out, (size_t)vocab * dim);
  BLAST(m->rms_final, dim);
  for (uint32_t l = 0; l < layers; l++) {
    BLAST(m->rms_att[l], dim);
    BLAST(m->rms_ffn[l], dim);
    BLAST(m->wq[l], (size_t)dim * dim);
    BLAST(m->wk[l], (size_t)dim * dim);
    BLAST(m->wv[l], (size_t)dim * dim);
    BLAST(m->wo[l], (size_t)dim * dim);
    BLAST(m->wup[l], (size_t)ffn * dim);
    BLAST(m->wdown[l], (size_t)ffn * dim);
  }
#undef BLAST
  fclose(f);
  return s;
}

EXPORT void oracle_forward(void *h, const int *tokens, int n, float *logits) {
  OState *s = (OState *)h;
  seq_forward(s->s, tokens, n, logits);
}

EXPORT void oracle_reset_cache(void *h) { ((OState *)h)->s->cached = 0; }
EXPORT int oracle_get_pos(void *h) { return ((OState *)h)->s->cached; }
EXPORT int oracle_get_heads(void *h) { return ((OState *)h)->m->heads; }
EXPORT int oracle_get_head_size(void *h) { return ((OState *)h)->m->hs; }
EXPORT int oracle_get_vocab(void *h) { return h ? ((OState *)h)->m->vocab : 0; }
EXPORT int oracle_get_ctx(void *h) { return h ? ((OState *)h)->m->ctx : 0; }
EXPORT int oracle_get_dim(void *h) { return h ? ((OState *)h)->m->dim : 0; }
EXPORT int oracle_get_layers(void *h) { return h ? ((OState *)h)->m->layers : 0; }

EXPORT void oracle_free(void *h) {
  OState *s = (OState *)h;
  if (!s) return;
  train_free(s->tr);
  seq_free(s->s);
  model_free(s->m);
  free(s);
}

/* core/cortex.nim:439-462: tensor pointer and expected size per type code. */
static float *tensor_ptr(OModel *m, int layer, int type, size_t *n) {
  size_t vd = (size_t)m->vocab * m->dim, dd = (size_t)m->dim * m->dim, fd = (size_t)m->ffn * m->dim;
  if (layer >= m->layers || layer < -1) return NULL;
  if (layer == -1) {
    if (type == 0) { *n = vd; return m->emb; }
    if (type == 1) { *n = vd; return m->w_out; }
    if (type == 2) { *n = m->dim; return m->rms_final; }
    return NULL;
  }
  switch (type) {
    case 10: *n = m->dim; return m->rms_att[layer];
    case 11: *n = m->dim; return m->rms_ffn[layer];
    case 12: *n = dd; return m->wq[layer];
    case 13: *n = dd; return m->wk[layer];
    case 14: *n = dd; return m->wv[layer];
    case 15: *n = dd; return m->wo[layer];
    case 16: *n = fd; return m->wup[layer];
    case 17: *n = fd; return m->wdown[layer];
  }
  return NULL;
}

EXPORT void oracle_load_layer(void *h, int layer, int type, const float *w, int n) {
  size_t want = 0;
  float *p = tensor_ptr(((OState *)h)->m, layer, type, &want);
  if (p && (size_t)n == want) memcpy(p, w, want * sizeof(float));
}

EXPORT void oracle_extract_layer(void *h, int layer, int type, float *w, int n) {
  size_t want = 0;
  float *p = tensor_ptr(((OState *)h)->m, layer, type, &want);
  if (p && (size_t)n == want) memcpy(w, p, want * sizeof(float));
}

/* ------------------------------------------------------------------------- */
/* Samplers (double precision, as PHP)                                       */
/* ------------------------------------------------------------------------- */

static double ex(double x, int exp_mode) { return exp_mode ? snai_exp(x) : exp(x); }

/*
 * src/snai_inference.php:151-195.  `logits` is modified in place exactly as
 * the PHP loop modifies the FFI float buffer (temperature, then penalty, each
 * result stored back as float).  `u` replaces mt_rand()/mt_getrandmax().
 * Returns the chosen id (0 when nothing is chosen, as `$best_token = 0`).
 */
EXPORT int oracle_sample_a(float *logits, int V, const int *hist, int H, double temperature,
                           double rep, float u, int exp_mode) {
  int best = 0;
  if (V <= 0) return 0;
  for (int v = 0; v < V; v++) logits[v] = (float)((double)logits[v] / temperature);
  /* array_unique($history): each id once; ids outside [0,V) are skipped. */
  unsigned char *seen = (unsigned char *)calloc((size_t)V, 1);
  for (int i = 0; i < H; i++) {
    int t = hist[i];
    if (t < 0 || t >= V || seen[t]) continue;
    seen[t] = 1;
    if ((double)logits[t] > 0)
      logits[t] = (float)((double)logits[t] / rep);
    else
      logits[t] = (float)((double)logits[t] * rep);
  }
  free(seen);
  double max_val = -INFINITY;
  for (int v = 0; v < V; v++) {
    if ((double)logits[v] > max_val) {
      max_val = (double)logits[v];
      if (temperature <= 0.01) best = v;
    }
  }
  if (temperature > 0.01) {
    double *probs = (double *)malloc(sizeof(double) * (size_t)V);
    double sum = 0.0;
    for (int v = 0; v < V; v++) {
      double p = ex((double)logits[v] - max_val, exp_mode);
      probs[v] = p;
      sum += p;
    }
    double r = (double)u * sum;
    double cum = 0.0;
    for (int v = 0; v < V; v++) {
      cum += probs[v];
      if (cum >= r) { best = v; break; }
    }
    free(probs);
  }
  return best;
}

typedef struct { double val; int id; } KV;

/* arsort on doubles is a stable descending sort (PHP >= 8.0), so the order is
 * (value descending, id ascending).  NaN has no place in PHP's order; here it
 * sorts after every number. */
static int kv_cmp(const void *a, const void *b) {
  const KV *x = (const KV *)a, *y = (const KV *)b;
  int xn = x->val != x->val, yn = y->val != y->val;
  if (xn != yn) return xn - yn;
  if (!xn) {
    if (x->val > y->val) return -1;
    if (x->val < y->val) return 1;
  }
  return (x->id > y->id) - (x->id < y->id);
}

/*
 * src/tensor_ffi_adapter.php:168-204.  Returns the chosen id, or -1 when
 * top_k < 1 (the PHP code would return null there and fail its int type).
 * If `out_order` is not NULL it receives the first min(top_k, V) ids in
 * sorted order (for tests of the selection).
 */
EXPORT int oracle_sample_b(const float *logits, int V, const int *in_tokens, int n_in,
                           double temperature, int top_k, double top_p, double rep, float u,
                           int exp_mode, int *out_order) {
  if (top_k < 1 || V <= 0) return -1;
  unsigned char *in_set = (unsigned char *)calloc((size_t)V, 1);
  for (int i = 0; i < n_in; i++)
    if (in_tokens[i] >= 0 && in_tokens[i] < V) in_set[in_tokens[i]] = 1;
  KV *kv = (KV *)malloc(sizeof(KV) * (size_t)V);
  for (int i = 0; i < V; i++) {
    double val = (double)logits[i];
    if (in_set[i]) val -= rep;
    kv[i].val = val;
    kv[i].id = i;
  }
  free(in_set);
  qsort(kv, (size_t)V, sizeof(KV), kv_cmp);
  int k = top_k < V ? top_k : V;
  if (out_order)
    for (int i = 0; i < k; i++) out_order[i] = kv[i].id;
  if (temperature < 0.01) {
    int id = kv[0].id;
    free(kv);
    return id;
  }
  double *probs = (double *)malloc(sizeof(double) * (size_t)k);
  double sum = 0.0;
  for (int i = 0; i < k; i++) {
    double p = ex(kv[i].val / temperature, exp_mode);
    probs[i] = p;
    sum += p;
  }
  double cum = 0.0;
  int nf = 0;
  for (int i = 0; i < k; i++) {
    double pn = probs[i] / sum;
    probs[i] = pn; /* $filtered[$id] = $p_norm */
    nf++;
    cum += pn;
    if (cum >= top_p) break;
  }
  double r = (double)u * cum;
  double cum_check = 0.0;
  int chosen = kv[0].id; /* array_key_first($filtered) */
  for (int i = 0; i < nf; i++) {
    cum_check += probs[i];
    if (r <= cum_check) { chosen = kv[i].id; break; }
  }
  free(probs);
  free(kv);
  return chosen;
}

/* Element-wise check of the contract exponential against libm (for tests). */
EXPORT void oracle_exp_contract(const double *x, double *y, long n) {
  for (long i = 0; i < n; i++) y[i] = snai_exp(x[i]);
}

EXPORT void oracle_exp_libm(const double *x, double *y, long n) {
  for (long i = 0; i < n; i++) y[i] = exp(x[i]);
}

/* ------------------------------------------------------------------------- */
/* Batched drivers over many sequences (threads), for tests and the CPU      */
/* baseline.  Sequences are independent; one worker owns whole sequences.    */
/* ------------------------------------------------------------------------- */

typedef struct {
  const OModel *m;
  int seq_begin, seq_end;
  const int *prompts; /* [nseq][plen] */
  int plen;
  int steps;
  const float *uniforms; /* [nseq][steps] */
  int variant; /* 0: A, 1: B */
  double temperature, rep, top_p;
  int top_k;
  int exp_mode;
  const int *forced; /* [nseq][steps] teacher-forced tokens, or NULL */
  int *out_ids;      /* [nseq][steps] */
  float *out_logits; /* [nseq][steps+1][V] or NULL */
} GenJob;

static void *gen_worker(void *arg) {
  GenJob *j = (GenJob *)arg;
  const OModel *m = j->m;
  int V = m->vocab;
  float *logits = zalloc(V);
  float *work = zalloc(V);
  int cap = j->plen + j->steps + 1;
  int *hist = (int *)malloc(sizeof(int) * (size_t)cap);
  for (int sidx = j->seq_begin; sidx < j->seq_end; sidx++) {
    OSeq *s = seq_new(m);
    const int *prompt = j->prompts + (size_t)sidx * j->plen;
    int hl = 0;
    for (int i = 0; i < j->plen; i++) hist[hl++] = prompt[i];
    seq_forward(s, prompt, j->plen, logits);
    if (j->out_logits) memcpy(j->out_logits + ((size_t)sidx * (j->steps + 1)) * V, logits, sizeof(float) * V);
    for (int st = 0; st < j->steps; st++) {
      float u = j->uniforms ? j->uniforms[(size_t)sidx * j->steps + st] : 0.5f;
      int id;
      if (j->variant == 0) {
        memcpy(work, logits, sizeof(float) * V);
        id = oracle_sample_a(work, V, hist, hl, j->temperature, j->rep, u, j->exp_mode);
      } else {
        id = oracle_sample_b(logits, V, hist, hl, j->temperature, j->top_k, j->top_p, j->rep, u,
                             j->exp_mode, NULL);
      }
      if (j->out_ids) j->out_ids[(size_t)sidx * j->steps + st] = id;
      int next = j->forced ? j->forced[(size_t)sidx * j->steps + st] : id;
      if (hl < cap) hist[hl++] = next;
      seq_forward(s, &next, 1, logits);
      if (j->out_logits)
        memcpy(j->out_logits + ((size_t)sidx * (j->steps + 1) + st + 1) * V, logits, sizeof(float) * V);
    }
    seq_free(s);
  }
  free(hist);
  free(work);
  free(logits);
  return NULL;
}

/*
 * Runs the snai_inference.php loop (src/snai_inference.php:113-215, stop
 * tokens disabled) for nseq independent sequences on nthreads threads:
 * reset, forward the prompt, then `steps` times {sample, forward the token}.
 * With `forced` the fed token is forced (teacher forcing) while out_ids still
 * receives the sampler's choice.  Returns wall seconds.
 */
EXPORT double oracle_generate(void *h, int nseq, const int *prompts, int plen, int steps,
                              const float *uniforms, int variant, double temperature, double rep,
                              int top_k, double top_p, int exp_mode, const int *forced,
                              int *out_ids, float *out_logits, int nthreads) {
  OState *st = (OState *)h;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > nseq) nthreads = nseq;
  pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
  GenJob *jobs = (GenJob *)calloc((size_t)nthreads, sizeof(GenJob));
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (int t = 0; t < nthreads; t++) {
    GenJob *j = &jobs[t];
    j->m = st->m;
    j->seq_begin = (int)((long)nseq * t / nthreads);
    j->seq_end = (int)((long)nseq * (t + 1) / nthreads);
    j->prompts = prompts;
    j->plen = plen;
    j->steps = steps;
    j->uniforms = uniforms;
    j->variant = variant;
    j->temperature = temperature;
    j->rep = rep;
    j->top_k = top_k;
    j->top_p = top_p;
    j->exp_mode = exp_mode;
    j->forced = forced;
    j->out_ids = out_ids;
    j->out_logits = out_logits;
    pthread_create(&th[t], NULL, gen_worker, j);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  clock_gettime(CLOCK_MONOTONIC, &t1);
  free(th);
  free(jobs);
  return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}

/* --- timed decode sample for the CPU baseline ------------------------------ */

typedef struct {
  const OModel *m;
  int seq_begin, seq_end, start_pos, steps, variant, top_k;
  double temperature, rep, top_p;
  unsigned seed;
  long tokens_done;
} BenchJob;

static uint32_t lcg(uint32_t *s) {
  *s = *s * 1664525u + 1013904223u;
  return *s;
}

static void *bench_worker(void *arg) {
  BenchJob *j = (BenchJob *)arg;
  const OModel *m = j->m;
  int V = m->vocab;
  float *logits = zalloc(V), *work = zalloc(V);
  int *hist = (int *)malloc(sizeof(int) * (size_t)(j->start_pos + j->steps + 1));
  for (int sidx = j->seq_begin; sidx < j->seq_end; sidx++) {
    OSeq *s = seq_new(m);
    uint32_t rs = j->seed + 7919u * (uint32_t)sidx;
    /* A cache state standing for a prompt of start_pos tokens: values of the
     * magnitude the projections produce; only the timing is used. */
    for (int l = 0; l < m->layers; l++)
      for (size_t i = 0; i < (size_t)j->start_pos * m->dim; i++) {
        s->kc[l][i] = ((float)(lcg(&rs) >> 8) * (1.0f / 16777216.0f) - 0.5f) * 0.1f;
        s->vc[l][i] = ((float)(lcg(&rs) >> 8) * (1.0f / 16777216.0f) - 0.5f) * 0.1f;
      }
    s->cached = j->start_pos;
    int hl = 0;
    for (int i = 0; i < j->start_pos; i++) hist[hl++] = (int)(lcg(&rs) % (uint32_t)V);
    int tok = (int)(lcg(&rs) % (uint32_t)V);
    for (int st = 0; st < j->steps && s->cached < m->ctx; st++) {
      seq_forward(s, &tok, 1, logits);
      float u = (float)(lcg(&rs) >> 8) * (1.0f / 16777216.0f);
      if (j->variant == 0) {
        memcpy(work, logits, sizeof(float) * V);
        tok = oracle_sample_a(work, V, hist, hl, j->temperature, j->rep, u, 0);
      } else {
        tok = oracle_sample_b(logits, V, hist, hl, j->temperature, j->top_k, j->top_p, j->rep, u, 0, NULL);
      }
      hist[hl++] = tok;
      j->tokens_done++;
    }
    seq_free(s);
  }
  free(hist);
  free(work);
  free(logits);
  return NULL;
}

/*
 * Times `steps` decode steps (forward one token + sample, as one iteration
 * of src/snai_inference.php:139-215) for nseq sequences whose caches stand at
 * start_pos, on nthreads threads.  Returns generated tokens per second.
 */
EXPORT double oracle_bench_decode(void *h, int nseq, int start_pos, int steps, int variant,
                                  double temperature, double rep, int top_k, double top_p,
                                  unsigned seed, int nthreads) {
  OState *st = (OState *)h;
  if (start_pos >= st->m->ctx) start_pos = st->m->ctx - 1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > nseq) nthreads = nseq;
  pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
  BenchJob *jobs = (BenchJob *)calloc((size_t)nthreads, sizeof(BenchJob));
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (int t = 0; t < nthreads; t++) {
    BenchJob *j = &jobs[t];
    j->m = st->m;
    j->seq_begin = (int)((long)nseq * t / nthreads);
    j->seq_end = (int)((long)nseq * (t + 1) / nthreads);
    j->start_pos = start_pos;
    j->steps = steps;
    j->variant = variant;
    j->temperature = temperature;
    j->rep = rep;
    j->top_k = top_k;
    j->top_p = top_p;
    j->seed = seed;
    pthread_create(&th[t], NULL, bench_worker, j);
  }
  long tokens = 0;
  for (int t = 0; t < nthreads; t++) {
    pthread_join(th[t], NULL);
    tokens += jobs[t].tokens_done;
  }
  clock_gettime(CLOCK_MONOTONIC, &t1);
  free(th);
  free(jobs);
  double secs = (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
  return secs > 0 ? (double)tokens / secs : 0.0;
}

/* Times the samplers alone over `rows` rows of [rows, V] logits on nthreads
 * threads (each row is one PHP sampler call).  Returns rows per second. */
typedef struct {
  const float *logits;
  int V, r0, r1, variant, H, top_k, exp_mode;
  const int *hist;
  const float *uniforms;
  double temperature, rep, top_p;
  int *out;
} SampJob;

static void *samp_worker(void *arg) {
  SampJob *j = (SampJob *)arg;
  float *work = zalloc(j->V);
  for (int r = j->r0; r < j->r1; r++) {
    const float *row = j->logits + (size_t)r * j->V;
    const int *hh = j->hist + (size_t)r * j->H;
    int id;
    if (j->variant == 0) {
      memcpy(work, row, sizeof(float) * j->V);
      id = oracle_sample_a(work, j->V, hh, j->H, j->temperature, j->rep, j->uniforms[r], j->exp_mode);
    } else {
      id = oracle_sample_b(row, j->V, hh, j->H, j->temperature, j->top_k, j->top_p, j->rep,
                           j->uniforms[r], j->exp_mode, NULL);
    }
    if (j->out) j->out[r] = id;
  }
  free(work);
  return NULL;
}

EXPORT double oracle_sample_rows(const float *logits, int rows, int V, const int *hist, int H,
                                 const float *uniforms, int variant, double temperature,
                                 double rep, int top_k, double top_p, int exp_mode, int *out,
                                 int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > rows) nthreads = rows;
  pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
  SampJob *jobs = (SampJob *)calloc((size_t)nthreads, sizeof(SampJob));
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (int t = 0; t < nthreads; t++) {
    SampJob *j = &jobs[t];
    j->logits = logits;
    j->V = V;
    j->r0 = (int)((long)rows * t / nthreads);
    j->r1 = (int)((long)rows * (t + 1) / nthreads);
    j->variant = variant;
    j->H = H;
    j->hist = hist;
    j->uniforms = uniforms;
    j->temperature = temperature;
    j->rep = rep;
    j->top_k = top_k;
    j->top_p = top_p;
    j->exp_mode = exp_mode;
    j->out = out;
    pthread_create(&th[t], NULL, samp_worker, j);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  clock_gettime(CLOCK_MONOTONIC, &t1);
  free(th);
  free(jobs);
  double secs = (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
  return secs > 0 ? rows / secs : 0.0;
}

/* --- persistent batch of sequences for step-by-step CPU timing ------------ */

typedef struct {
  const OModel *m;
  int nseq, start_pos;
  OSeq **seqs;
  int **hist;
  int *hlen;
  int *tok;
  float **logits;
  float **work;
  uint32_t *rng;
} OBatch;

/* nseq sequences whose caches stand at start_pos (values standing for a
 * prompt: only the timing of later steps is used), each with a history of
 * start_pos random ids. */
EXPORT void *oracle_batch_new(void *h, int nseq, int start_pos, unsigned seed) {
  OState *st = (OState *)h;
  const OModel *m = st->m;
  if (start_pos >= m->ctx) start_pos = m->ctx - 1;
  if (start_pos < 0) start_pos = 0;
  OBatch *b = (OBatch *)calloc(1, sizeof(OBatch));
  b->m = m;
  b->nseq = nseq;
  b->start_pos = start_pos;
  b->seqs = (OSeq **)calloc((size_t)nseq, sizeof(OSeq *));
  b->hist = (int **)calloc((size_t)nseq, sizeof(int *));
  b->hlen = (int *)calloc((size_t)nseq, sizeof(int));
  b->tok = (int *)calloc((size_t)nseq, sizeof(int));
  b->logits = (float **)calloc((size_t)nseq, sizeof(float *));
  b->work = (float **)calloc((size_t)nseq, sizeof(float *));
  b->rng = (uint32_t *)calloc((size_t)nseq, sizeof(uint32_t));
  for (int s = 0; s < nseq; s++) {
    OSeq *q = seq_new(m);
    uint32_t rs = seed + 7919u * (uint32_t)s;
    for (int l = 0; l < m->layers; l++)
      for (size_t i = 0; i < (size_t)start_pos * m->dim; i++) {
        q->kc[l][i] = ((float)(lcg(&rs) >> 8) * (1.0f / 16777216.0f) - 0.5f) * 0.1f;
        q->vc[l][i] = ((float)(lcg(&rs) >> 8) * (1.0f / 16777216.0f) - 0.5f) * 0.1f;
      }
    q->cached = start_pos;
    b->seqs[s] = q;
    b->hist[s] = (int *)malloc(sizeof(int) * (size_t)(m->ctx + 1));
    for (int i = 0; i < start_pos; i++) b->hist[s][i] = (int)(lcg(&rs) % (uint32_t)m->vocab);
    b->hlen[s] = start_pos;
    b->tok[s] = (int)(lcg(&rs) % (uint32_t)m->vocab);
    b->logits[s] = zalloc(m->vocab);
    b->work[s] = zalloc(m->vocab);
    b->rng[s] = rs;
  }
  return b;
}

EXPORT void oracle_batch_free(void *p) {
  OBatch *b = (OBatch *)p;
  if (!b) return;
  for (int s = 0; s < b->nseq; s++) {
    seq_free(b->seqs[s]);
    free(b->hist[s]);
    free(b->logits[s]);
    free(b->work[s]);
  }
  free(b->seqs); free(b->hist); free(b->hlen); free(b->tok); free(b->logits); free(b->work); free(b->rng);
  free(b);
}

typedef struct {
  OBatch *b;
  int s0, s1, variant, top_k;
  double temperature, rep, top_p;
} StepJob;

static void *step_worker(void *arg) {
  StepJob *j = (StepJob *)arg;
  OBatch *b = j->b;
  const int V = b->m->vocab;
  for (int s = j->s0; s < j->s1; s++) {
    OSeq *q = b->seqs[s];
    if (q->cached >= b->m->ctx) { /* wrap: regenerate from start_pos */
      q->cached = b->start_pos;
      b->hlen[s] = b->start_pos;
    }
    seq_forward(q, &b->tok[s], 1, b->logits[s]);
    b->hist[s][b->hlen[s]++] = b->tok[s];
    float u = (float)(lcg(&b->rng[s]) >> 8) * (1.0f / 16777216.0f);
    if (j->variant == 0) {
      memcpy(b->work[s], b->logits[s], sizeof(float) * V);
      b->tok[s] = oracle_sample_a(b->work[s], V, b->hist[s], b->hlen[s], j->temperature, j->rep, u, 0);
    } else {
      b->tok[s] = oracle_sample_b(b->logits[s], V, b->hist[s], b->hlen[s], j->temperature, j->top_k, j->top_p,
                                  j->rep, u, 0, NULL);
    }
  }
  return NULL;
}

/* One decode step (src/snai_inference.php:139-215: forward one token, then
 * the PHP sampler with libm exp) for every sequence of the batch, spread over
 * nthreads threads.  Returns wall seconds. */
EXPORT double oracle_batch_step(void *p, int variant, double temperature, double rep, int top_k, double top_p,
                                int nthreads) {
  OBatch *b = (OBatch *)p;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > b->nseq) nthreads = b->nseq;
  pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
  StepJob *jobs = (StepJob *)calloc((size_t)nthreads, sizeof(StepJob));
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (int t = 0; t < nthreads; t++) {
    StepJob *j = &jobs[t];
    j->b = b;
    j->s0 = (int)((long)b->nseq * t / nthreads);
    j->s1 = (int)((long)b->nseq * (t + 1) / nthreads);
    j->variant = variant;
    j->top_k = top_k;
    j->temperature = temperature;
    j->rep = rep;
    j->top_p = top_p;
    pthread_create(&th[t], NULL, step_worker, j);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  clock_gettime(CLOCK_MONOTONIC, &t1);
  free(th);
  free(jobs);
  return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}

/* ------------------------------------------------------------------------- */
/* Training step, core/cortex.nim:565-822 (+ Adam :145-207, clip :230-258)   */
/* ------------------------------------------------------------------------- */

/* Gradients and Adam moments have the weights' shapes; activations are kept
 * per layer for ctx positions, as the reference's act_* buffers. */
typedef struct OTrain {
  OModel *g, *mm, *vv;
  int adam_t;
  int ctx, L, D, F, V;
  float **a_hidden, **a_norm_att, **a_q, **a_att, **a_hidden_ffn, **a_norm_ffn, **a_ffn_in, **a_ffn_out;
  float *a_hidden_final, *probs;
  float **dk, **dv; /* d_k_cache, d_v_cache [L][ctx * D] */
  float *d_logits, *d_hidden, *d_norm, *d_att, *d_q, *d_ffn, *scores, *d_w, *norm;
} OTrain;

static void model_zero(OModel *m) {
  size_t vd = (size_t)m->vocab * m->dim, dd = (size_t)m->dim * m->dim, fd = (size_t)m->ffn * m->dim;
  memset(m->emb, 0, vd * 4);
  memset(m->w_out, 0, vd * 4);
  memset(m->rms_final, 0, (size_t)m->dim * 4);
  for (int l = 0; l < m->layers; l++) {
    memset(m->rms_att[l], 0, (size_t)m->dim * 4);
    memset(m->rms_ffn[l], 0, (size_t)m->dim * 4);
    memset(m->wq[l], 0, dd * 4); memset(m->wk[l], 0, dd * 4); memset(m->wv[l], 0, dd * 4);
    memset(m->wo[l], 0, dd * 4); memset(m->wup[l], 0, fd * 4); memset(m->wdown[l], 0, fd * 4);
  }
}

static float **alloc_rows(int L, size_t n) {
  float **p = (float **)calloc(L ? L : 1, sizeof(float *));
  for (int l = 0; l < L; l++) p[l] = zalloc(n);
  return p;
}

static void free_rows(float **p, int L) {
  if (!p) return;
  for (int l = 0; l < L; l++) free(p[l]);
  free(p);
}

static OTrain *train_get(OState *s) {
  if (s->tr) return s->tr;
  const OModel *m = s->m;
  OTrain *t = (OTrain *)calloc(1, sizeof(OTrain));
  t->ctx = m->ctx; t->L = m->layers; t->D = m->dim; t->F = m->ffn; t->V = m->vocab;
  t->g = model_new(m->vocab, m->dim, m->ctx, m->layers, m->heads);
  t->mm = model_new(m->vocab, m->dim, m->ctx, m->layers, m->heads);
  t->vv = model_new(m->vocab, m->dim, m->ctx, m->layers, m->heads);
  model_zero(t->g); model_zero(t->mm); model_zero(t->vv);
  size_t cd = (size_t)m->ctx * m->dim, cf = (size_t)m->ctx * m->ffn;
  t->a_hidden = alloc_rows(t->L, cd); t->a_norm_att = alloc_rows(t->L, cd); t->a_q = alloc_rows(t->L, cd);
  t->a_att = alloc_rows(t->L, cd); t->a_hidden_ffn = alloc_rows(t->L, cd); t->a_norm_ffn = alloc_rows(t->L, cd);
  t->a_ffn_in = alloc_rows(t->L, cf); t->a_ffn_out = alloc_rows(t->L, cf);
  t->dk = alloc_rows(t->L, cd); t->dv = alloc_rows(t->L, cd);
  t->a_hidden_final = zalloc(cd);
  t->probs = zalloc((size_t)m->ctx * m->vocab);
  t->d_logits = zalloc(m->vocab); t->d_hidden = zalloc(m->dim); t->d_norm = zalloc(m->dim);
  t->d_att = zalloc(m->dim); t->d_q = zalloc(m->dim); t->d_ffn = zalloc(m->ffn);
  t->scores = zalloc(m->ctx); t->d_w = zalloc(m->ctx); t->norm = zalloc(m->dim);
  s->tr = t;
  return t;
}

static void train_free(OTrain *t) {
  if (!t) return;
  model_free(t->g); model_free(t->mm); model_free(t->vv);
  free_rows(t->a_hidden, t->L); free_rows(t->a_norm_att, t->L); free_rows(t->a_q, t->L);
  free_rows(t->a_att, t->L); free_rows(t->a_hidden_ffn, t->L); free_rows(t->a_norm_ffn, t->L);
  free_rows(t->a_ffn_in, t->L); free_rows(t->a_ffn_out, t->L); free_rows(t->dk, t->L); free_rows(t->dv, t->L);
  free(t->a_hidden_final); free(t->probs); free(t->d_logits); free(t->d_hidden); free(t->d_norm);
  free(t->d_att); free(t->d_q); free(t->d_ffn); free(t->scores); free(t->d_w); free(t->norm);
  free(t);
}

/* applyRoPE with backward = true: the rotation by -theta (:74-87). */
static void apply_rope_back(float *vec, int dim, int hs, int pos) {
  int nh = dim / hs;
  for (int h = 0; h < nh; h++) {
    int off = h * hs;
    for (int i = 0; i + 1 <= hs - 1; i += 2) {
      float freq = 1.0f / powf(10000.0f, (float)i / (float)hs);
      float theta = (float)pos * freq;
      float c = cosf(theta);
      float s = -1.0f * sinf(theta);
      float v0 = vec[off + i], v1 = vec[off + i + 1];
      vec[off + i] = v0 * c - v1 * s;
      vec[off + i + 1] = v0 * s + v1 * c;
    }
  }
}

/* matVecMulBackwardAcc (:100-115): d_in (= or +=) M^T d_out, gm += d_out x^T. */
static void matvec_back(const float *w, float *gw, int rows, int cols, const float *x, const float *d_out,
                        float *d_in, int accumulate) {
  if (d_in) {
    if (!accumulate)
      for (int c = 0; c < cols; c++) d_in[c] = 0.0f;
    for (int r = 0; r < rows; r++) {
      float dov = d_out[r];
      const float *row = w + (size_t)r * cols;
      for (int c = 0; c < cols; c++) d_in[c] += row[c] * dov;
    }
  }
  for (int r = 0; r < rows; r++) {
    float dov = d_out[r];
    float *grow = gw + (size_t)r * cols;
    for (int c = 0; c < cols; c++) grow[c] += dov * x[c];
  }
}

/* applyRMSNormBackwardAcc (:125-143): d_out becomes the input gradient. */
static void rmsnorm_back(float *d_out, const float *a, int dim, const float *w, float *gw) {
  float ss = 0.0f;
  for (int d = 0; d < dim; d++) ss += a[d] * a[d];
  float inv = 1.0f / sqrtf((ss / (float)dim) + 1e-5f);
  float sum_dy_nx = 0.0f;
  for (int d = 0; d < dim; d++) sum_dy_nx += d_out[d] * w[d] * (a[d] * inv);
  float mean = sum_dy_nx / (float)dim;
  for (int d = 0; d < dim; d++) {
    float nx = a[d] * inv;
    gw[d] += d_out[d] * nx;
    d_out[d] = (d_out[d] * w[d] - nx * mean) * inv;
  }
}

/* Forward with saved activations, loss and BPTT (:565-818).  Gradients are
 * zeroed first and left in t->g.  The sequence's KV cache rows 0..act-1 are
 * overwritten as the reference does; its token count is not touched.
 * Returns total_loss / act, or 0 when act <= 0. */
static float train_grads(OState *st, const int *t_in, const int *t_tg, int num_tok) {
  OModel *m = st->m;
  OSeq *sq = st->s;
  OTrain *t = train_get(st);
  OModel *g = t->g;
  const int D = m->dim, F = m->ffn, V = m->vocab, L = m->layers, hs = m->hs;
  int act = num_tok < m->ctx ? num_tok : m->ctx;
  if (act <= 0) return 0.0f;
  model_zero(g);
  for (int l = 0; l < L; l++) {
    memset(t->dk[l], 0, (size_t)act * D * 4);
    memset(t->dv[l], 0, (size_t)act * D * 4);
  }
  float total_loss = 0.0f;
  float *h = sq->h, *norm = sq->norm, *att = sq->att;
  for (int pos = 0; pos < act; pos++) {
    int tid = t_in[pos], tg = t_tg[pos];
    if (tid < 0 || tid >= V) tid = 0;
    if (tg < 0 || tg >= V) tg = 0;
    const size_t od = (size_t)pos * D, of = (size_t)pos * F;
    memcpy(h, m->emb + (size_t)tid * D, sizeof(float) * D);
    for (int l = 0; l < L; l++) {
      memcpy(t->a_hidden[l] + od, h, sizeof(float) * D);
      rmsnorm(h, norm, D, m->rms_att[l]);
      memcpy(t->a_norm_att[l] + od, norm, sizeof(float) * D);
      float *q = t->a_q[l] + od;
      matvec(m->wq[l], D, D, norm, q);
      apply_rope(q, D, hs, pos);
      float *kp = sq->kc[l] + od, *vp = sq->vc[l] + od;
      matvec(m->wk[l], D, D, norm, kp);
      apply_rope(kp, D, hs, pos);
      matvec(m->wv[l], D, D, norm, vp);
      for (int d = 0; d < D; d++) att[d] = 0.0f;
      for (int hh = 0; hh < m->heads; hh++) {
        int off = hh * hs;
        float max_s = -9999.0f;
        for (int tt = 0; tt <= pos; tt++) {
          const float *tk = sq->kc[l] + (size_t)tt * D;
          float sc = 0.0f;
          for (int d = 0; d < hs; d++) sc += q[off + d] * tk[off + d];
          sc /= sqrtf((float)hs);
          t->scores[tt] = sc;
          if (sc > max_s) max_s = sc;
        }
        float sum_e = 0.0f;
        for (int tt = 0; tt <= pos; tt++) {
          t->scores[tt] = expf(t->scores[tt] - max_s);
          sum_e += t->scores[tt];
        }
        for (int tt = 0; tt <= pos; tt++) {
          float w = t->scores[tt] / sum_e;
          const float *tv = sq->vc[l] + (size_t)tt * D;
          for (int d = 0; d < hs; d++) att[off + d] += tv[off + d] * w;
        }
      }
      memcpy(t->a_att[l] + od, att, sizeof(float) * D);
      matvec(m->wo[l], D, D, att, t->d_norm);
      for (int d = 0; d < D; d++) h[d] += t->d_norm[d];
      memcpy(t->a_hidden_ffn[l] + od, h, sizeof(float) * D);
      rmsnorm(h, norm, D, m->rms_ffn[l]);
      memcpy(t->a_norm_ffn[l] + od, norm, sizeof(float) * D);
      float *fin = t->a_ffn_in[l] + of, *fout = t->a_ffn_out[l] + of;
      matvec(m->wup[l], F, D, norm, fin);
      for (int d = 0; d < F; d++) {
        float v = fin[d];
        fout[d] = v * (1.0f / (1.0f + expf(-v)));
      }
      matvec(m->wdown[l], D, F, fout, att);
      for (int d = 0; d < D; d++) h[d] += att[d];
    }
    memcpy(t->a_hidden_final + od, h, sizeof(float) * D);
    rmsnorm(h, norm, D, m->rms_final);
    float max_l = -9999.0f;
    float *lg = t->probs + (size_t)pos * V;
    for (int v = 0; v < V; v++) {
      float s = 0.0f;
      const float *row = m->w_out + (size_t)v * D;
      for (int d = 0; d < D; d++) s += norm[d] * row[d];
      lg[v] = s;
      if (s > max_l) max_l = s;
    }
    float sum_p = 0.0f;
    for (int v = 0; v < V; v++) {
      lg[v] = expf(lg[v] - max_l);
      sum_p += lg[v];
    }
    for (int v = 0; v < V; v++) lg[v] /= sum_p;
    total_loss += -logf(lg[tg] + 1e-7f);
  }

  for (int pos = act - 1; pos >= 0; pos--) {
    int tid = t_in[pos], tg = t_tg[pos];
    if (tid < 0 || tid >= V) tid = 0;
    if (tg < 0 || tg >= V) tg = 0;
    const size_t od = (size_t)pos * D, of = (size_t)pos * F;
    const float *lg = t->probs + (size_t)pos * V;
    for (int v = 0; v < V; v++) t->d_logits[v] = lg[v] - (v == tg ? 1.0f : 0.0f);
    for (int d = 0; d < D; d++) t->d_hidden[d] = 0.0f;
    const float *fh = t->a_hidden_final + od;
    rmsnorm(fh, t->norm, D, m->rms_final);
    matvec_back(m->w_out, g->w_out, V, D, t->norm, t->d_logits, t->d_norm, 0);
    rmsnorm_back(t->d_norm, fh, D, m->rms_final, g->rms_final);
    for (int d = 0; d < D; d++) t->d_hidden[d] += t->d_norm[d];
    for (int l = L - 1; l >= 0; l--) {
      for (int d = 0; d < D; d++) t->d_norm[d] = t->d_hidden[d];
      matvec_back(m->wdown[l], g->wdown[l], D, F, t->a_ffn_out[l] + of, t->d_norm, t->d_ffn, 0);
      const float *fin = t->a_ffn_in[l] + of;
      for (int d = 0; d < F; d++) {
        float x = fin[d];
        float sig = 1.0f / (1.0f + expf(-x));
        t->d_ffn[d] *= sig * (1.0f + x * (1.0f - sig));
      }
      matvec_back(m->wup[l], g->wup[l], F, D, t->a_norm_ffn[l] + od, t->d_ffn, t->d_norm, 0);
      rmsnorm_back(t->d_norm, t->a_hidden_ffn[l] + od, D, m->rms_ffn[l], g->rms_ffn[l]);
      for (int d = 0; d < D; d++) t->d_hidden[d] += t->d_norm[d];
      for (int d = 0; d < D; d++) t->d_norm[d] = t->d_hidden[d];
      matvec_back(m->wo[l], g->wo[l], D, D, t->a_att[l] + od, t->d_norm, t->d_att, 0);
      const float *q = t->a_q[l] + od;
      for (int d = 0; d < D; d++) t->d_q[d] = 0.0f;
      for (int hh = 0; hh < m->heads; hh++) {
        int off = hh * hs;
        float scale = 1.0f / sqrtf((float)hs);
        float max_s = -9999.0f;
        for (int tt = 0; tt <= pos; tt++) {
          const float *kt = sq->kc[l] + (size_t)tt * D;
          float sc = 0.0f;
          for (int d = 0; d < hs; d++) sc += q[off + d] * kt[off + d];
          sc *= scale;
          t->scores[tt] = sc;
          if (sc > max_s) max_s = sc;
        }
        float sum_e = 0.0f;
        for (int tt = 0; tt <= pos; tt++) {
          t->scores[tt] = expf(t->scores[tt] - max_s);
          sum_e += t->scores[tt];
        }
        float sum_w_dw = 0.0f;
        for (int tt = 0; tt <= pos; tt++) {
          float w = t->scores[tt] / sum_e;
          t->scores[tt] = w;
          const float *vt = sq->vc[l] + (size_t)tt * D;
          float dw = 0.0f;
          for (int d = 0; d < hs; d++) dw += t->d_att[off + d] * vt[off + d];
          float *dvt = t->dv[l] + (size_t)tt * D;
          for (int d = 0; d < hs; d++) dvt[off + d] += t->d_att[off + d] * w;
          t->d_w[tt] = dw;
          sum_w_dw += w * dw;
        }
        for (int tt = 0; tt <= pos; tt++) {
          float w = t->scores[tt];
          float ds = w * (t->d_w[tt] - sum_w_dw) * scale;
          const float *kt = sq->kc[l] + (size_t)tt * D;
          float *dkt = t->dk[l] + (size_t)tt * D;
          for (int d = 0; d < hs; d++) {
            t->d_q[off + d] += ds * kt[off + d];
            dkt[off + d] += ds * q[off + d];
          }
        }
      }
      float *cdk = t->dk[l] + od, *cdv = t->dv[l] + od;
      apply_rope_back(t->d_q, D, hs, pos);
      apply_rope_back(cdk, D, hs, pos);
      const float *na = t->a_norm_att[l] + od;
      matvec_back(m->wq[l], g->wq[l], D, D, na, t->d_q, t->d_norm, 0);
      matvec_back(m->wk[l], g->wk[l], D, D, na, cdk, t->d_norm, 1);
      matvec_back(m->wv[l], g->wv[l], D, D, na, cdv, t->d_norm, 1);
      rmsnorm_back(t->d_norm, t->a_hidden[l] + od, D, m->rms_att[l], g->rms_att[l]);
      for (int d = 0; d < D; d++) t->d_hidden[d] += t->d_norm[d];
    }
    float *ge = g->emb + (size_t)tid * D;
    for (int d = 0; d < D; d++) ge[d] += t->d_hidden[d];
  }
  return total_loss / (float)act;
}

static float l2sq(const float *a, size_t n) {
  float s = 0.0f;
  for (size_t i = 0; i < n; i++) s += a[i] * a[i];
  return s;
}

static void scale_arr(float *a, size_t n, float sc) {
  for (size_t i = 0; i < n; i++) a[i] *= sc;
}

/* adamStep (:145-160). */
static void adam_step(float *w, float *m, float *v, float *g, float lr, float b1, float b2, float b1t, float b2t,
                      float scale, int sparse) {
  if (scale == 0.0f) return;
  float grad = *g / scale;
  if (sparse && grad == 0.0f) return;
  if (grad != grad || grad > 9999.0f || grad < -9999.0f) {
    *g = 0.0f;
    return;
  }
  *m = b1 * *m + (1.0f - b1) * grad;
  *v = b2 * *v + (1.0f - b2) * grad * grad;
  float m_hat = *m / b1t;
  float v_hat = *v / b2t;
  *w -= lr * m_hat / (sqrtf(v_hat) + 1e-8f);
  *g = 0.0f;
}

/* clipGlobalGradientNorm(s, 1.0) (:230-258), then applyGlobalAdamUpdate(lr,
 * scale) (:162-207, CPU branch). */
static void train_apply(OState *st, float lr, float scale) {
  OModel *m = st->m;
  OTrain *t = train_get(st);
  OModel *g = t->g;
  const int L = m->layers;
  const size_t vd = (size_t)m->vocab * m->dim, dd = (size_t)m->dim * m->dim, fd = (size_t)m->ffn * m->dim;
  const size_t D = (size_t)m->dim;
  float total_sq = 0.0f;
  total_sq += l2sq(g->emb, vd);
  total_sq += l2sq(g->w_out, vd);
  total_sq += l2sq(g->rms_final, D);
  for (int l = 0; l < L; l++) {
    total_sq += l2sq(g->wq[l], dd);
    total_sq += l2sq(g->wk[l], dd);
    total_sq += l2sq(g->wv[l], dd);
    total_sq += l2sq(g->wo[l], dd);
    total_sq += l2sq(g->wup[l], fd);
    total_sq += l2sq(g->wdown[l], fd);
    total_sq += l2sq(g->rms_att[l], D);
    total_sq += l2sq(g->rms_ffn[l], D);
  }
  const float max_norm = 1.0f;
  float gn = sqrtf(total_sq);
  if (gn != gn || gn > max_norm) {
    float sc = (gn != gn || gn == 0.0f) ? 0.0f : max_norm / gn;
    scale_arr(g->emb, vd, sc);
    scale_arr(g->w_out, vd, sc);
    scale_arr(g->rms_final, D, sc);
    for (int l = 0; l < L; l++) {
      scale_arr(g->wq[l], dd, sc); scale_arr(g->wk[l], dd, sc); scale_arr(g->wv[l], dd, sc);
      scale_arr(g->wo[l], dd, sc); scale_arr(g->wup[l], fd, sc); scale_arr(g->wdown[l], fd, sc);
      scale_arr(g->rms_att[l], D, sc); scale_arr(g->rms_ffn[l], D, sc);
    }
  }
  t->adam_t += 1;
  const float b1 = 0.9f, b2 = 0.999f;
  const float b1t = 1.0f - powf(b1, (float)t->adam_t);
  const float b2t = 1.0f - powf(b2, (float)t->adam_t);
  OModel *M = t->mm, *Vv = t->vv;
#define UPD(W, MM, VV, G, N, SP) \
  for (size_t i_ = 0; i_ < (N); i_++) adam_step(&(W)[i_], &(MM)[i_], &(VV)[i_], &(G)[i_], lr, b1, b2, b1t, b2t, scale, SP)
  UPD(m->emb, M->emb, Vv->emb, g->emb, vd, 1);
  UPD(m->w_out, M->w_out, Vv->w_out, g->w_out, vd, 0);
  UPD(m->rms_final, M->rms_final, Vv->rms_final, g->rms_final, D, 0);
  for (int l = 0; l < L; l++) {
    UPD(m->rms_att[l], M->rms_att[l], Vv->rms_att[l], g->rms_att[l], D, 0);
    UPD(m->rms_ffn[l], M->rms_ffn[l], Vv->rms_ffn[l], g->rms_ffn[l], D, 0);
    UPD(m->wq[l], M->wq[l], Vv->wq[l], g->wq[l], dd, 0);
    UPD(m->wk[l], M->wk[l], Vv->wk[l], g->wk[l], dd, 0);
    UPD(m->wv[l], M->wv[l], Vv->wv[l], g->wv[l], dd, 0);
    UPD(m->wo[l], M->wo[l], Vv->wo[l], g->wo[l], dd, 0);
    UPD(m->wup[l], M->wup[l], Vv->wup[l], g->wup[l], fd, 0);
    UPD(m->wdown[l], M->wdown[l], Vv->wdown[l], g->wdown[l], fd, 0);
  }
#undef UPD
}

/* cortex_train_step: gradients, clip, Adam; returns the mean loss. */
EXPORT float oracle_train_step(void *h, const int *t_in, const int *t_tg, int num_tok, float lr) {
  OState *st = (OState *)h;
  int act = num_tok < st->m->ctx ? num_tok : st->m->ctx;
  if (act <= 0) return 0.0f;
  float loss = train_grads(st, t_in, t_tg, num_tok);
  train_apply(st, lr, (float)act);
  return loss;
}

/* The two halves of a step, for tests: gradients only (left in place)... */
EXPORT float oracle_train_grads(void *h, const int *t_in, const int *t_tg, int num_tok) {
  return train_grads((OState *)h, t_in, t_tg, num_tok);
}

/* ...and clip + Adam on the gradients in place, with Adam's divisor `scale`
 * (the step's token count). */
EXPORT void oracle_train_apply(void *h, float lr, float scale) { train_apply((OState *)h, lr, scale); }

/* Gradient (which 0) or Adam first / second moment (1 / 2) tensor by type code. */
static float *train_tensor(OState *st, int which, int layer, int type, size_t *n) {
  OTrain *t = train_get(st);
  OModel *src = which == 0 ? t->g : which == 1 ? t->mm : t->vv;
  return tensor_ptr(src, layer, type, n);
}

EXPORT void oracle_train_tensor_get(void *h, int which, int layer, int type, float *out, int n) {
  size_t want = 0;
  float *p = train_tensor((OState *)h, which, layer, type, &want);
  if (p && (size_t)n == want) memcpy(out, p, want * sizeof(float));
}

EXPORT void oracle_train_tensor_set(void *h, int which, int layer, int type, const float *in, int n) {
  size_t want = 0;
  float *p = train_tensor((OState *)h, which, layer, type, &want);
  if (p && (size_t)n == want) memcpy(p, in, want * sizeof(float));
}

EXPORT int oracle_adam_t(void *h) {
  OState *st = (OState *)h;
  return st->tr ? st->tr->adam_t : 0;
}
