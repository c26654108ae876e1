/* oracle.c — CPU restatement of AutoANE's MeZO-LoRA-split projection path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libb2p.so, never part of it.
 * Built with -ffp-contract=off so every product and sum rounds separately, as
 * the reference's scalar C and vDSP element-wise calls do. Matrix products use
 * OpenBLAS cblas_sgemm (the reference uses Accelerate's cblas_sgemm); their
 * internal summation order is BLAS-defined, so agreement with the reference
 * on Apple hardware is at fp32 rounding level, not bit level.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* OpenBLAS CBLAS entry points (declared here: the wheel ships no cblas.h). */
enum { OrRowMajor = 101 };
enum { OrNoTrans = 111, OrTrans = 112 };
extern void cblas_sgemm(int order, int ta, int tb, int M, int N, int K, float alpha, const float* A, int lda,
                        const float* B, int ldb, float beta, float* C, int ldc);
extern void openblas_set_num_threads(int n);
extern int openblas_get_num_threads(void);

static void* xmalloc(size_t n) {
  void* p = malloc(n ? n : 1);
  if (!p) {
    fprintf(stderr, "oracle: malloc(%zu) failed\n", n);
    abort();
  }
  return p;
}

int or_set_threads(int n) {
  if (n > 0) openblas_set_num_threads(n);
  return openblas_get_num_threads();
}

/* ---------------- xoshiro256+ (train_mezo.m:97-119) ---------------- */
static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t or_xo_next(or_xo* st) {
  uint64_t* s = st->s;
  const uint64_t result = s[0] + s[3];
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return result;
}

void or_xo_seed(or_xo* st, uint64_t seed) {
  for (int i = 0; i < 4; i++) {
    seed += 0x9E3779B97F4A7C15ULL;
    uint64_t z = seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    st->s[i] = z ^ (z >> 31);
  }
}

/* perturb_buffer (train_mezo.m:122-136) */
void or_perturb_buffer(or_xo* st, float* buf, size_t n, float scale) {
  const float neg = -scale;
  size_t i = 0;
  for (; i + 3 < n; i += 4) {
    const uint64_t r = or_xo_next(st);
    buf[i + 0] += (r & 1) ? scale : neg;
    buf[i + 1] += (r & 2) ? scale : neg;
    buf[i + 2] += (r & 4) ? scale : neg;
    buf[i + 3] += (r & 8) ? scale : neg;
  }
  for (; i < n; i++) {
    const uint64_t r = or_xo_next(st);
    buf[i] += (r & 1) ? scale : neg;
  }
}

void or_sign_mask(uint64_t seed, const int64_t* sizes, int nbuf, uint32_t* mask) {
  or_xo st;
  or_xo_seed(&st, seed);
  int64_t total = 0;
  for (int b = 0; b < nbuf; b++) total += sizes[b];
  memset(mask, 0, (size_t)((total + 31) / 32) * 4);
  int64_t p = 0;
  for (int b = 0; b < nbuf; b++) {
    const int64_t n = sizes[b];
    int64_t i = 0;
    for (; i + 3 < n; i += 4) {
      const uint64_t r = or_xo_next(&st);
      for (int k = 0; k < 4; k++)
        if (r & (1ull << k)) mask[(p + i + k) >> 5] |= 1u << ((p + i + k) & 31);
    }
    for (; i < n; i++) {
      const uint64_t r = or_xo_next(&st);
      if (r & 1) mask[(p + i) >> 5] |= 1u << ((p + i) & 31);
    }
    p += n;
  }
}

/* ---------------- LoRA-split parameter layout (train_mezo.m:560-588) ---------------- */
or_layout or_lora_layout(int nlayers, int dim, int q_dim, int kv_dim, int rank) {
  or_layout L;
  const int64_t r = rank, D = dim, Q = q_dim, KV = kv_dim;
  int64_t o = 0;
  L.Aq = o; o += r * D;
  L.Bq = o; o += Q * r;
  L.Ak = o; o += r * D;
  L.Bk = o; o += KV * r;
  L.Av = o; o += r * D;
  L.Bv = o; o += KV * r;
  L.Ao = o; o += r * Q;
  L.Bo = o; o += D * r;
  L.rms_att = o; o += D;
  L.rms_ffn = o; o += D;
  L.layer_size = o;
  L.rms_final = (int64_t)nlayers * o;
  L.total = L.rms_final + D;
  return L;
}

int or_lora_buffer_sizes(int nlayers, int dim, int q_dim, int kv_dim, int rank, int64_t* sz) {
  const int64_t r = rank, D = dim, Q = q_dim, KV = kv_dim;
  int n = 0;
  for (int l = 0; l < nlayers; l++) {
    sz[n++] = r * D;   /* Aq */
    sz[n++] = Q * r;   /* Bq */
    sz[n++] = r * D;   /* Ak */
    sz[n++] = KV * r;  /* Bk */
    sz[n++] = r * D;   /* Av */
    sz[n++] = KV * r;  /* Bv */
    sz[n++] = r * Q;   /* Ao */
    sz[n++] = D * r;   /* Bo */
    sz[n++] = D;       /* rms_att */
    sz[n++] = D;       /* rms_ffn */
  }
  sz[n++] = D; /* rms_final */
  return n;
}

void or_perturb_lora(float* theta, int nlayers, int dim, int q_dim, int kv_dim, int rank, uint64_t seed,
                     float scale) {
  int64_t* sz = (int64_t*)xmalloc(sizeof(int64_t) * (size_t)(10 * nlayers + 1));
  const int nb = or_lora_buffer_sizes(nlayers, dim, q_dim, kv_dim, rank, sz);
  or_xo st;
  or_xo_seed(&st, seed);
  int64_t off = 0;
  for (int b = 0; b < nb; b++) {
    or_perturb_buffer(&st, theta + off, (size_t)sz[b], scale);
    off += sz[b];
  }
  free(sz);
}

/* ---------------- ops (training/cpu_ops.h) ---------------- */
void or_sgemm_nn(int M, int N, int K, const float* A, const float* B, float* C, float beta) {
  cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, M, N, K, 1.0f, A, K, B, N, beta, C, N);
}

/* rmsnorm (cpu_ops.h:7-22): ss = Σ_i x_i² in channel order; ss = ss/d + 1e-5;
 * out = (x * rsqrt(ss)) * w. */
void or_rmsnorm(float* out, const float* x, const float* w, int d, int S) {
  float* ss = (float*)calloc((size_t)S, sizeof(float));
  for (int i = 0; i < d; i++)
    for (int t = 0; t < S; t++) {
      const float sq = x[(size_t)i * S + t] * x[(size_t)i * S + t];
      ss[t] = sq + ss[t];
    }
  const float invd = 1.0f / d, eps = 1e-5f;
  for (int t = 0; t < S; t++) {
    const float m = ss[t] * invd;
    ss[t] = 1.0f / sqrtf(m + eps);
  }
  for (int i = 0; i < d; i++)
    for (int t = 0; t < S; t++) {
      const float v = x[(size_t)i * S + t] * ss[t];
      out[(size_t)i * S + t] = v * w[i];
    }
  free(ss);
}

/* rope_forward_inplace (cpu_ops.h:299-315), interleaved pairs (2i, 2i+1) per head */
void or_rope_forward(float* x, int seq, int dim, int hd, float theta) {
  const int nheads = dim / hd;
  for (int h = 0; h < nheads; h++)
    for (int i = 0; i < hd / 2; i++) {
      const float freq = 1.0f / powf(theta, 2.0f * i / (float)hd);
      for (int p = 0; p < seq; p++) {
        const float ang = p * freq;
        const float c = cosf(ang), s = sinf(ang);
        const size_t i0 = (size_t)(h * hd + 2 * i) * seq + p;
        const size_t i1 = (size_t)(h * hd + 2 * i + 1) * seq + p;
        const float v0 = x[i0], v1 = x[i1];
        x[i0] = v0 * c - v1 * s;
        x[i1] = v0 * s + v1 * c;
      }
    }
}

void or_rope_tables(float* cos_out, float* sin_out, int seq, int hd, float theta) {
  for (int i = 0; i < hd / 2; i++) {
    const float freq = 1.0f / powf(theta, 2.0f * i / (float)hd);
    for (int p = 0; p < seq; p++) {
      const float ang = p * freq;
      cos_out[(size_t)p * (hd / 2) + i] = cosf(ang);
      sin_out[(size_t)p * (hd / 2) + i] = sinf(ang);
    }
  }
}

/* cpu_sdpa_forward (cpu_ops.h:321-360): causal softmax(QᵀK/√hd)·V per head, with
 * the reference's 1e-10 in the normaliser and -1e9 masking. */
void or_sdpa_forward(const float* Q, const float* Kt, const float* Vt, float* out, int heads, int hd, int seq) {
  const float scale = 1.0f / sqrtf((float)hd);
  float* sc = (float*)xmalloc(sizeof(float) * (size_t)seq * seq);
  for (int h = 0; h < heads; h++) {
    const float* Qh = Q + (size_t)h * hd * seq;
    const float* Kh = Kt + (size_t)h * hd * seq;
    const float* Vh = Vt + (size_t)h * hd * seq;
    float* oh = out + (size_t)h * hd * seq;
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, seq, seq, hd, scale, Qh, seq, Kh, seq, 0.0f, sc, seq);
    for (int s = 0; s < seq; s++) {
      float* row = sc + (size_t)s * seq;
      for (int j = s + 1; j < seq; j++) row[j] = -1e9f;
      float maxv = -1e30f;
      for (int j = 0; j <= s; j++) maxv = fmaxf(maxv, row[j]);
      float sum = 0;
      for (int j = 0; j <= s; j++) {
        row[j] = expf(row[j] - maxv);
        sum += row[j];
      }
      const float inv = 1.0f / (sum + 1e-10f);
      for (int j = 0; j <= s; j++) row[j] *= inv;
      for (int j = s + 1; j < seq; j++) row[j] = 0.0f;
    }
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, hd, seq, seq, 1.0f, Vh, seq, sc, seq, 0.0f, oh, seq);
  }
  free(sc);
}

/* cross_entropy_loss (cpu_ops.h:108-133), logits token-major [S, V]. */
float or_cross_entropy(const float* logits, const uint16_t* targets, int V, int S) {
  float total = 0;
  float* e = (float*)xmalloc(sizeof(float) * (size_t)V);
  for (int t = 0; t < S; t++) {
    const float* row = logits + (size_t)t * V;
    float maxv = row[0];
    for (int v = 1; v < V; v++) maxv = fmaxf(maxv, row[v]);
    float sum = 0;
    for (int v = 0; v < V; v++) {
      e[v] = expf(row[v] + (-maxv));
      sum += e[v];
    }
    const int tgt = targets[t];
    if (tgt < 0 || tgt >= V) {
      fprintf(stderr, "oracle: target[%d]=%d out of range (vocab %d)\n", t, tgt, V);
      abort();
    }
    total += -(row[tgt] - maxv) + logf(sum);
  }
  free(e);
  return total / S;
}

/* lora_addmm (train_mezo.m:694-703): tmp = A·x; out += B·tmp */
void or_lora_addmm(float* out, const float* A, const float* B, const float* x, float* tmp, int out_dim, int rank,
                   int in_dim, int seq) {
  cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, rank, seq, in_dim, 1.0f, A, in_dim, x, seq, 0.0f, tmp, seq);
  cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, out_dim, seq, rank, 1.0f, B, rank, tmp, seq, 1.0f, out, seq);
}

/* gqa_tile_kv (training/io.h:439-446): KV head kv feeds query heads kv*R .. kv*R+R-1 */
static void gqa_tile(float* out, const float* in, int kv_heads, int ratio, int hd, int seq) {
  for (int kv = 0; kv < kv_heads; kv++)
    for (int r = 0; r < ratio; r++)
      memcpy(out + (size_t)(kv * ratio + r) * hd * seq, in + (size_t)kv * hd * seq, sizeof(float) * hd * seq);
}

/* x += alpha * o  (vDSP_vsma(o, alpha, x) in train_mezo.m:1619, 1692) */
static void resid_add(float* x, const float* o, float alpha, size_t n) {
  for (size_t i = 0; i < n; i++) {
    const float p = o[i] * alpha;
    x[i] = p + x[i];
  }
}

/* ---------------- DO_FORWARD_PASS (train_mezo.m:1528-1699, cpu_only + lora_split) ---------------- */
float or_forward_loss(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                      or_taps* taps) {
  const int D = m->dim, H = m->hidden, S = m->seq, QD = m->heads * m->hd, KVD = m->kv_heads * m->hd;
  const int r = m->rank;
  const or_layout L = or_lora_layout(m->nlayers, D, QD, KVD, r);
  float* x = (float*)xmalloc(sizeof(float) * (size_t)D * S);
  float* xn = (float*)xmalloc(sizeof(float) * (size_t)D * S);
  float* Q = (float*)xmalloc(sizeof(float) * (size_t)QD * S);
  float* K = (float*)xmalloc(sizeof(float) * (size_t)KVD * S);
  float* V = (float*)xmalloc(sizeof(float) * (size_t)KVD * S);
  float* Kt = (float*)xmalloc(sizeof(float) * (size_t)QD * S);
  float* Vt = (float*)xmalloc(sizeof(float) * (size_t)QD * S);
  float* att = (float*)xmalloc(sizeof(float) * (size_t)QD * S);
  float* o = (float*)xmalloc(sizeof(float) * (size_t)D * S);
  float* h1 = (float*)xmalloc(sizeof(float) * (size_t)H * S);
  float* h3 = (float*)xmalloc(sizeof(float) * (size_t)H * S);
  float* tmp = (float*)xmalloc(sizeof(float) * (size_t)r * S);
  float* logits = (float*)xmalloc(sizeof(float) * (size_t)S * m->cv);

  /* embed_lookup (cpu_ops.h:190-197) */
  for (int t = 0; t < S; t++) {
    const int tok = tokens[t];
    if (tok < 0 || tok >= m->vocab) {
      fprintf(stderr, "oracle: token[%d]=%d out of range\n", t, tok);
      abort();
    }
    for (int d = 0; d < D; d++) x[(size_t)d * S + t] = m->embed[(size_t)tok * D + d];
  }
  for (int l = 0; l < m->nlayers; l++) {
    const float* th = theta + (size_t)l * L.layer_size;
    if (taps && taps->layer_x) memcpy(taps->layer_x + (size_t)l * D * S, x, sizeof(float) * (size_t)D * S);
    or_rmsnorm(xn, x, th + L.rms_att, D, S);
    or_sgemm_nn(QD, S, D, m->Wq[l], xn, Q, 0.0f);
    or_sgemm_nn(KVD, S, D, m->Wk[l], xn, K, 0.0f);
    or_sgemm_nn(KVD, S, D, m->Wv[l], xn, V, 0.0f);
    or_lora_addmm(Q, th + L.Aq, th + L.Bq, xn, tmp, QD, r, D, S);
    or_lora_addmm(K, th + L.Ak, th + L.Bk, xn, tmp, KVD, r, D, S);
    or_lora_addmm(V, th + L.Av, th + L.Bv, xn, tmp, KVD, r, D, S);
    or_rope_forward(Q, S, QD, m->hd, m->rope_theta);
    or_rope_forward(K, S, KVD, m->hd, m->rope_theta);
    gqa_tile(Kt, K, m->kv_heads, m->heads / m->kv_heads, m->hd, S);
    gqa_tile(Vt, V, m->kv_heads, m->heads / m->kv_heads, m->hd, S);
    or_sdpa_forward(Q, Kt, Vt, att, m->heads, m->hd, S);
    or_sgemm_nn(D, S, QD, m->Wo[l], att, o, 0.0f);
    or_lora_addmm(o, th + L.Ao, th + L.Bo, att, tmp, D, r, QD, S);
    resid_add(x, o, m->res_alpha, (size_t)D * S);
    or_rmsnorm(xn, x, th + L.rms_ffn, D, S);
    or_sgemm_nn(H, S, D, m->W1[l], xn, h1, 0.0f);
    or_sgemm_nn(H, S, D, m->W3[l], xn, h3, 0.0f);
    for (size_t i = 0; i < (size_t)H * S; i++) {
      const float s = h1[i] / (1.0f + expf(-h1[i]));
      h1[i] = s * h3[i];
    }
    or_sgemm_nn(D, S, H, m->W2[l], h1, o, 0.0f);
    resid_add(x, o, m->res_alpha, (size_t)D * S);
  }
  if (taps && taps->layer_x)
    memcpy(taps->layer_x + (size_t)m->nlayers * D * S, x, sizeof(float) * (size_t)D * S);
  if (taps && taps->x_final) memcpy(taps->x_final, x, sizeof(float) * (size_t)D * S);
  or_rmsnorm(xn, x, theta + L.rms_final, D, S);
  if (taps && taps->xn_final) memcpy(taps->xn_final, xn, sizeof(float) * (size_t)D * S);
  /* logits[S, CV] = xnᵀ · cembedᵀ (train_mezo.m:1696-1697) */
  cblas_sgemm(OrRowMajor, OrTrans, OrTrans, S, m->cv, D, 1.0f, xn, S, m->cembed, D, 0.0f, logits, m->cv);
  if (taps && taps->logits) memcpy(taps->logits, logits, sizeof(float) * (size_t)S * m->cv);
  const float loss = or_cross_entropy(logits, ctargets, m->cv, S);
  free(x); free(xn); free(Q); free(K); free(V); free(Kt); free(Vt); free(att); free(o);
  free(h1); free(h3); free(tmp); free(logits);
  return loss;
}

/* MeZO-LoRA-split step body (train_mezo.m:2938-3012) */
void or_mezo_step(const or_model* m, float* theta, const uint16_t* tokens, const uint16_t* ctargets, uint64_t seed,
                  float eps, float lr, float* loss_plus, float* loss_minus, float* proj_grad) {
  const int QD = m->heads * m->hd, KVD = m->kv_heads * m->hd;
  or_perturb_lora(theta, m->nlayers, m->dim, QD, KVD, m->rank, seed, +eps);
  const float lp = or_forward_loss(m, theta, tokens, ctargets, NULL);
  or_perturb_lora(theta, m->nlayers, m->dim, QD, KVD, m->rank, seed, -2.0f * eps);
  const float lm = or_forward_loss(m, theta, tokens, ctargets, NULL);
  or_perturb_lora(theta, m->nlayers, m->dim, QD, KVD, m->rank, seed, +eps);
  const float g = (lp - lm) / (2.0f * eps);
  const float update_scale = -lr * g;
  or_perturb_lora(theta, m->nlayers, m->dim, QD, KVD, m->rank, seed, update_scale);
  if (loss_plus) *loss_plus = lp;
  if (loss_minus) *loss_minus = lm;
  if (proj_grad) *proj_grad = g;
}
