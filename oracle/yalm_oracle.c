/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load this file's library, and only as the checker.  The product library
 * (yalm_b200/) never links or calls it and has no CPU fallback.
 *
 * A plain-C restatement of yalm's CPU decode forward pass (`-d cpu`), function by function, with
 * the reference file:line each one follows (paths relative to the yalm repository).  Arithmetic is
 * fp32 with fp16 weights and an fp16 KV cache, in the same order of operations as the reference
 * where that order is observable:
 *   - the fp16 matvec keeps two 8-lane fused-multiply-add accumulators per row and folds them
 *     lo+hi, then 4+4, then (0+1)+(2+3), as the AVX2/F16C loop does (src/infer.cpp:63-100);
 *   - RoPE rotates interleaved pairs with freq = 1/theta^(j/rotary_dim) and angle = pos*freq
 *     (src/infer.cpp:202-215);
 *   - k and v are rounded to fp16 after clip and RoPE, then stored (src/infer.cpp:296-305).
 * The reference itself is built with -ffast-math, so the compiler may reassociate its plain loops
 * (rmsnorm, softmax sums); results then agree to ~1e-6 relative, not bit for bit.  The pin of this
 * restatement against the reference is tests/test_oracle.py (against oracle/_ref and the golden
 * vectors in tests/golden/).
 *
 * KV cache layout follows the reference: K 16-tiled per kv head, k_cache_idx (src/model.h:14-17);
 * V as [kv_head][head_dim][max_seq_len] (src/infer.cpp:304).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KV_SINKS 2 /* src/model.h:12 */

/* ---------- IEEE binary16 <-> binary32, round to nearest even ---------- */
float yo_h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t yo_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
  }
  if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  }
  if (absx < 0x38800000u) { /* below smallest normal half 2^-14: subnormal or zero */
    if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to zero */
    /* value = m * 2^(e-150) with the implicit bit in m; the half subnormal unit is 2^-24 */
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7fffffu) | 0x800000u;
    uint32_t sh = 126u - e;
    uint32_t q = m >> sh;
    uint32_t rem = m & ((1u << sh) - 1u);
    uint32_t halfway = 1u << (sh - 1u);
    if (rem > halfway || (rem == halfway && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 112u;
  uint32_t m = absx & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

/* k_cache_idx, src/model.h:14-17 */
static inline size_t k_idx(int hi, int t, int msl) {
  return (size_t)(hi / 16) * (16 * (size_t)msl) + (size_t)t * 16 + (size_t)(hi % 16);
}

/* fp16 matvec: src/infer.cpp:63-100.  W (d,n) row-major fp16, x (n,), xout (d,).  n % 16 == 0. */
void yo_matmul_f16(float* xout, const float* x, const uint16_t* w, int n, int d) {
  int i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < d; i++) {
    float lo[8] = {0}, hi[8] = {0};
    const uint16_t* row = w + (size_t)i * n;
    for (int j = 0; j < n; j += 16) {
      for (int k = 0; k < 8; ++k) {
        lo[k] = fmaf(yo_h2f(row[j + k]), x[j + k], lo[k]);
        hi[k] = fmaf(yo_h2f(row[j + 8 + k]), x[j + 8 + k], hi[k]);
      }
    }
    float s8[8];
    for (int k = 0; k < 8; ++k) s8[k] = lo[k] + hi[k];
    float s4[4];
    for (int k = 0; k < 4; ++k) s4[k] = s8[k] + s8[k + 4];
    xout[i] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }
}

/* fp32 matvec: src/infer.cpp:48-59 */
void yo_matmul_f32(float* xout, const float* x, const float* w, int n, int d) {
  int i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < d; i++) {
    float val = 0.0f;
    for (int j = 0; j < n; j++) val += w[(size_t)i * n + j] * x[j];
    xout[i] = val;
  }
}

/* rmsnorm: src/infer.cpp:136-146 */
void yo_rmsnorm(float* o, const float* x, const float* weight, int size, float eps) {
  float rms = 0.0f;
  for (int i = 0; i < size; ++i) rms += x[i] * x[i];
  rms = sqrtf(rms / size + eps);
  float scale = 1.0f / rms;
  for (int i = 0; i < size; ++i) o[i] = x[i] * scale * weight[i];
}

/* softmax: src/infer.cpp:172-187 */
static void softmax(float* o, const float* x, int size) {
  float mx = -FLT_MAX;
  for (int i = 0; i < size; ++i)
    if (x[i] > mx) mx = x[i];
  float sum = 0.0f;
  for (int i = 0; i < size; ++i) {
    o[i] = expf(x[i] - mx);
    sum += o[i];
  }
  for (int i = 0; i < size; ++i) o[i] /= sum;
}

/* activations: src/infer.cpp:189-199 */
static inline float gelu(float x) { return 0.5f * x * (1.0f + tanhf(0.797885f * (x + 0.044715f * x * x * x))); }
static inline float silu(float x) { return x / (1.0f + expf(-x)); }
static inline float clipf(float x, float v) { return x < -v ? -v : (x > v ? v : x); }

/* interleaved-pair RoPE: src/infer.cpp:202-215 */
void yo_rope(float* vec, int d, int head_dim, int pos, float theta, int rotary_dim) {
  for (int i = 0; i < d; i += 2) {
    int j_head = i % head_dim;
    float freq = j_head >= rotary_dim ? 0.f : 1.0f / powf(theta, (float)j_head / (float)rotary_dim);
    float val = pos * freq;
    float fcr = cosf(val);
    float fci = sinf(val);
    float v0 = vec[i];
    float v1 = vec[i + 1];
    vec[i] = v0 * fcr - v1 * fci;
    vec[i + 1] = v0 * fci + v1 * fcr;
  }
}

/* one attention head: src/infer.cpp:218-250.  kh: 16-tiled K slice, vh: [head_dim][msl] V slice */
void yo_attn(float* xout, float* atth, const float* qh, const uint16_t* kh, const uint16_t* vh, int head_dim,
             int max_seq_len, int kv_len) {
  for (int t = 0; t < kv_len; ++t) {
    float score = 0.0f;
    for (int i = 0; i < head_dim; ++i) score += qh[i] * yo_h2f(kh[k_idx(i, t, max_seq_len)]);
    score /= sqrtf((float)head_dim);
    atth[t] = score;
  }
  softmax(atth, atth, kv_len);
  for (int i = 0; i < head_dim; ++i) {
    float vi = 0.0f;
    for (int t = 0; t < kv_len; ++t) vi += atth[t] * yo_h2f(vh[(size_t)i * max_seq_len + t]);
    xout[i] = vi;
  }
}

/* all heads with GQA mapping g = h / (n_heads / n_kv_heads): src/infer.cpp:394-415 */
void yo_mha(float* xout, float* att, const uint16_t* kb, const uint16_t* vb, const float* q, int head_dim, int kv_len,
            int max_seq_len, int n_heads, int n_kv_heads) {
  int q_per_kv = n_heads / n_kv_heads;
  int h;
#pragma omp parallel for schedule(static)
  for (h = 0; h < n_heads; h++) {
    int g = h / q_per_kv;
    const uint16_t* kh = kb + (size_t)g * head_dim * max_seq_len;
    const uint16_t* vh = vb + (size_t)g * head_dim * max_seq_len;
    yo_attn(xout + (size_t)head_dim * h, att + (size_t)max_seq_len * h, q + (size_t)head_dim * h, kh, vh, head_dim,
            max_seq_len, kv_len);
  }
}

/* position bookkeeping: src/infer.cpp:489-494 */
void yo_positions(int pos, int max_seq_len, int* kv_sink, int* kv_pos, int* kv_len) {
  *kv_sink = pos >= max_seq_len ? KV_SINKS : 0;
  *kv_pos = *kv_sink + (pos - *kv_sink) % (max_seq_len - *kv_sink);
  *kv_len = pos >= max_seq_len ? max_seq_len : pos + 1;
}

/* ---------------- whole model ---------------- */
typedef struct {
  int dim, hidden_dim, head_dim, n_layers, n_heads, n_kv_heads, vocab_size, max_seq_len, rotary_dim, act_silu;
  float rope_theta, norm_eps, qkv_clip;
  const uint16_t* emb;     /* [vocab, dim] */
  const float* rms_final;  /* [dim] */
  const uint16_t* wcls;    /* [vocab, dim] */
  const float** rms_att;   /* per layer [dim] */
  const float** rms_ffn;
  const uint16_t **wq, **wk, **wv, **wo, **w1, **w2, **w3;
  uint16_t** kcache; /* per layer [n_kv][hd/16][msl][16] */
  uint16_t** vcache; /* per layer [n_kv][hd][msl] */
  float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
} yo_model;

static void* xcalloc(size_t n, size_t s) {
  void* p = calloc(n ? n : 1, s);
  if (!p) abort();
  return p;
}

/* ints: dim hidden head_dim n_layers n_heads n_kv vocab msl rotary act_silu; floats: theta eps clip.
 * Pointer arrays have n_layers entries each and are copied; the weights themselves are borrowed. */
yo_model* yo_model_new(const int* ci, const float* cf, const uint16_t* emb, const float* rms_final, const uint16_t* wcls,
                       const float** rms_att, const float** rms_ffn, const uint16_t** wq, const uint16_t** wk,
                       const uint16_t** wv, const uint16_t** wo, const uint16_t** w1, const uint16_t** w2,
                       const uint16_t** w3) {
  yo_model* m = (yo_model*)xcalloc(1, sizeof(yo_model));
  m->dim = ci[0];
  m->hidden_dim = ci[1];
  m->head_dim = ci[2];
  m->n_layers = ci[3];
  m->n_heads = ci[4];
  m->n_kv_heads = ci[5];
  m->vocab_size = ci[6];
  m->max_seq_len = ci[7];
  m->rotary_dim = ci[8];
  m->act_silu = ci[9];
  m->rope_theta = cf[0];
  m->norm_eps = cf[1];
  m->qkv_clip = cf[2];
  m->emb = emb;
  m->rms_final = rms_final;
  m->wcls = wcls;
  int L = m->n_layers;
#define COPYARR(dst, src, T)                     \
  m->dst = (T*)xcalloc((size_t)L, sizeof(T));    \
  memcpy((void*)m->dst, src, (size_t)L * sizeof(T));
  COPYARR(rms_att, rms_att, const float*)
  COPYARR(rms_ffn, rms_ffn, const float*)
  COPYARR(wq, wq, const uint16_t*)
  COPYARR(wk, wk, const uint16_t*)
  COPYARR(wv, wv, const uint16_t*)
  COPYARR(wo, wo, const uint16_t*)
  COPYARR(w1, w1, const uint16_t*)
  COPYARR(w2, w2, const uint16_t*)
  COPYARR(w3, w3, const uint16_t*)
#undef COPYARR
  size_t kvsz = (size_t)m->max_seq_len * m->n_kv_heads * m->head_dim;
  m->kcache = (uint16_t**)xcalloc((size_t)L, sizeof(uint16_t*));
  m->vcache = (uint16_t**)xcalloc((size_t)L, sizeof(uint16_t*));
  for (int l = 0; l < L; ++l) {
    m->kcache[l] = (uint16_t*)xcalloc(kvsz, 2);
    m->vcache[l] = (uint16_t*)xcalloc(kvsz, 2);
  }
  int q_dim = m->n_heads * m->head_dim, kv_dim = m->n_kv_heads * m->head_dim;
  m->x = (float*)xcalloc((size_t)m->dim, 4);
  m->xb = (float*)xcalloc((size_t)m->dim, 4);
  m->xb2 = (float*)xcalloc((size_t)(m->dim > q_dim ? m->dim : q_dim), 4);
  m->hb = (float*)xcalloc((size_t)(m->hidden_dim > m->dim ? m->hidden_dim : m->dim), 4);
  m->hb2 = (float*)xcalloc((size_t)m->hidden_dim, 4);
  m->q = (float*)xcalloc((size_t)q_dim, 4);
  m->k = (float*)xcalloc((size_t)kv_dim, 4);
  m->v = (float*)xcalloc((size_t)kv_dim, 4);
  m->att = (float*)xcalloc((size_t)m->n_heads * m->max_seq_len, 4);
  m->logits = (float*)xcalloc((size_t)m->vocab_size, 4);
  return m;
}

void yo_model_free(yo_model* m) {
  if (!m) return;
  for (int l = 0; l < m->n_layers; ++l) {
    free(m->kcache[l]);
    free(m->vcache[l]);
  }
  free(m->kcache);
  free(m->vcache);
  free((void*)m->rms_att);
  free((void*)m->rms_ffn);
  free((void*)m->wq);
  free((void*)m->wk);
  free((void*)m->wv);
  free((void*)m->wo);
  free((void*)m->w1);
  free((void*)m->w2);
  free((void*)m->w3);
  free(m->x);
  free(m->xb);
  free(m->xb2);
  free(m->hb);
  free(m->hb2);
  free(m->q);
  free(m->k);
  free(m->v);
  free(m->att);
  free(m->logits);
  free(m);
}

/* one transformer block: Block::_block_cpu, src/infer.cpp:256-392 (dense FFN; no MoE) */
static void block_forward(yo_model* m, int l, int pos, int kv_sink, int kv_pos, int kv_len) {
  int dim = m->dim, hd = m->head_dim, msl = m->max_seq_len;
  int q_dim = m->n_heads * hd, kv_dim = m->n_kv_heads * hd;
  yo_rmsnorm(m->xb, m->x, m->rms_att[l], dim, m->norm_eps);
  yo_matmul_f16(m->q, m->xb, m->wq[l], dim, q_dim);
  yo_matmul_f16(m->k, m->xb, m->wk[l], dim, kv_dim);
  yo_matmul_f16(m->v, m->xb, m->wv[l], dim, kv_dim);
  for (int i = 0; i < q_dim; ++i) m->q[i] = clipf(m->q[i], m->qkv_clip);
  for (int i = 0; i < kv_dim; ++i) {
    m->k[i] = clipf(m->k[i], m->qkv_clip);
    m->v[i] = clipf(m->v[i], m->qkv_clip);
  }
  yo_rope(m->q, q_dim, hd, pos, m->rope_theta, m->rotary_dim);
  yo_rope(m->k, kv_dim, hd, pos, m->rope_theta, m->rotary_dim);
  uint16_t* kb = m->kcache[l];
  uint16_t* vb = m->vcache[l];
  for (int i = 0; i < kv_dim; ++i) { /* src/infer.cpp:300-305 */
    int g = i / hd, j = i % hd;
    kb[(size_t)g * hd * msl + k_idx(j, kv_pos, msl)] = yo_f2h(m->k[i]);
    vb[(size_t)g * hd * msl + (size_t)j * msl + kv_pos] = yo_f2h(m->v[i]);
  }
  for (int r = 0; r < kv_sink; r++) { /* sink re-rotation: src/infer.cpp:311-325 */
    for (int i = 0; i < kv_dim; ++i) {
      int g = i / hd, j = i % hd;
      m->k[i] = yo_h2f(kb[(size_t)g * hd * msl + k_idx(j, r, msl)]);
    }
    yo_rope(m->k, kv_dim, hd, 1, m->rope_theta, m->rotary_dim);
    for (int i = 0; i < kv_dim; ++i) {
      int g = i / hd, j = i % hd;
      kb[(size_t)g * hd * msl + k_idx(j, r, msl)] = yo_f2h(m->k[i]);
    }
  }
  yo_mha(m->xb2, m->att, kb, vb, m->q, hd, kv_len, msl, m->n_heads, m->n_kv_heads);
  yo_matmul_f16(m->hb, m->xb2, m->wo[l], q_dim, dim); /* src/infer.cpp:339-344 */
  for (int i = 0; i < dim; ++i) m->x[i] += m->hb[i];
  yo_rmsnorm(m->xb, m->x, m->rms_ffn[l], dim, m->norm_eps);
  yo_matmul_f16(m->hb, m->xb, m->w1[l], dim, m->hidden_dim); /* src/infer.cpp:367-390 */
  yo_matmul_f16(m->hb2, m->xb, m->w3[l], dim, m->hidden_dim);
  for (int i = 0; i < m->hidden_dim; ++i) m->hb[i] = (m->act_silu ? silu(m->hb[i]) : gelu(m->hb[i])) * m->hb2[i];
  yo_matmul_f16(m->xb2, m->hb, m->w2[l], m->hidden_dim, dim);
  for (int i = 0; i < dim; ++i) m->x[i] += m->xb2[i] * 1.0f;
}

/* Model::_forward_cpu, src/infer.cpp:483-528.  mode 0 = hydrate only, 1 = logits. */
void yo_forward(yo_model* m, int token, int pos, int mode, float* logits_out) {
  for (int i = 0; i < m->dim; ++i) m->x[i] = yo_h2f(m->emb[(size_t)token * m->dim + i]); /* :460-481 */
  int kv_sink, kv_pos, kv_len;
  yo_positions(pos, m->max_seq_len, &kv_sink, &kv_pos, &kv_len);
  for (int l = 0; l < m->n_layers; ++l) block_forward(m, l, pos, kv_sink, kv_pos, kv_len);
  if (!mode) return;
  yo_rmsnorm(m->x, m->x, m->rms_final, m->dim, m->norm_eps);
  yo_matmul_f16(m->logits, m->x, m->wcls, m->dim, m->vocab_size);
  if (logits_out) memcpy(logits_out, m->logits, sizeof(float) * (size_t)m->vocab_size);
}

/* canonical [slot][head_dim] view of one layer / kv head of the cache (fp16 bits) */
void yo_read_kv(const yo_model* m, int layer, int kvh, int pos0, int n, uint16_t* k_out, uint16_t* v_out) {
  int hd = m->head_dim, msl = m->max_seq_len;
  const uint16_t* kb = m->kcache[layer] + (size_t)kvh * hd * msl;
  const uint16_t* vb = m->vcache[layer] + (size_t)kvh * hd * msl;
  for (int t = 0; t < n; ++t)
    for (int j = 0; j < hd; ++j) {
      k_out[(size_t)t * hd + j] = kb[k_idx(j, pos0 + t, msl)];
      v_out[(size_t)t * hd + j] = vb[(size_t)j * msl + pos0 + t];
    }
}

/* the residual stream after the last forward (before the final norm when mode was 0) */
void yo_read_x(const yo_model* m, float* out) { memcpy(out, m->x, sizeof(float) * (size_t)m->dim); }
