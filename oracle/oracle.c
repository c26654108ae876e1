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
  return or_lora_layout_ffn(nlayers, dim, q_dim, kv_dim, 0, rank, 0);
}

or_layout or_lora_layout_ffn(int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn) {
  or_layout L;
  const int64_t r = rank, D = dim, Q = q_dim, KV = kv_dim, H = hidden;
  int64_t o = 0;
  L.Aq = o; o += r * D;
  L.Bq = o; o += Q * r;
  L.Ak = o; o += r * D;
  L.Bk = o; o += KV * r;
  L.Av = o; o += r * D;
  L.Bv = o; o += KV * r;
  L.Ao = o; o += r * Q;
  L.Bo = o; o += D * r;
  L.A1 = L.B1 = L.A2 = L.B2 = L.A3 = L.B3 = -1;
  if (ffn) { /* train_mezo.m:575-582 */
    L.A1 = o; o += r * D;
    L.B1 = o; o += H * r;
    L.A2 = o; o += r * H;
    L.B2 = o; o += D * r;
    L.A3 = o; o += r * D;
    L.B3 = o; o += H * r;
  }
  L.rms_att = o; o += D;
  L.rms_ffn = o; o += D;
  L.layer_size = o;
  L.rms_final = (int64_t)nlayers * o;
  L.total = L.rms_final + D;
  return L;
}

int or_lora_buffer_sizes(int nlayers, int dim, int q_dim, int kv_dim, int rank, int64_t* sz) {
  return or_lora_buffer_sizes_ffn(nlayers, dim, q_dim, kv_dim, 0, rank, 0, sz);
}

int or_lora_buffer_sizes_ffn(int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn,
                             int64_t* sz) {
  const int64_t r = rank, D = dim, Q = q_dim, KV = kv_dim, H = hidden;
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
    if (ffn) {
      sz[n++] = r * D; /* A1 */
      sz[n++] = H * r; /* B1 */
      sz[n++] = r * H; /* A2 */
      sz[n++] = D * r; /* B2 */
      sz[n++] = r * D; /* A3 */
      sz[n++] = H * r; /* B3 */
    }
    sz[n++] = D;       /* rms_att */
    sz[n++] = D;       /* rms_ffn */
  }
  sz[n++] = D; /* rms_final */
  return n;
}

void or_perturb_lora(float* theta, int nlayers, int dim, int q_dim, int kv_dim, int rank, uint64_t seed,
                     float scale) {
  or_perturb_lora_ffn(theta, nlayers, dim, q_dim, kv_dim, 0, rank, 0, seed, scale);
}

/* perturb_lora_weights (train_mezo.m:560-588): one xoshiro stream over every buffer in order */
void or_perturb_lora_ffn(float* theta, int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn,
                         uint64_t seed, float scale) {
  int64_t* sz = (int64_t*)xmalloc(sizeof(int64_t) * (size_t)(16 * nlayers + 1));
  const int nb = or_lora_buffer_sizes_ffn(nlayers, dim, q_dim, kv_dim, hidden, rank, ffn, sz);
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
  const or_layout L = or_lora_layout_ffn(m->nlayers, D, QD, KVD, H, r, m->lora_ffn);
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
    if (m->lora_ffn) { /* train_mezo.m:1634-1638 */
      or_lora_addmm(h1, th + L.A1, th + L.B1, xn, tmp, H, r, D, S);
      or_lora_addmm(h3, th + L.A3, th + L.B3, xn, tmp, H, r, D, S);
    }
    for (size_t i = 0; i < (size_t)H * S; i++) {
      const float s = h1[i] / (1.0f + expf(-h1[i]));
      h1[i] = s * h3[i];
    }
    or_sgemm_nn(D, S, H, m->W2[l], h1, o, 0.0f);
    if (m->lora_ffn) or_lora_addmm(o, th + L.A2, th + L.B2, h1, tmp, D, r, H, S); /* train_mezo.m:1658-1661 */
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
  or_perturb_lora_ffn(theta, m->nlayers, m->dim, QD, KVD, m->hidden, m->rank, m->lora_ffn, seed, +eps);
  const float lp = or_forward_loss(m, theta, tokens, ctargets, NULL);
  or_perturb_lora_ffn(theta, m->nlayers, m->dim, QD, KVD, m->hidden, m->rank, m->lora_ffn, seed, -2.0f * eps);
  const float lm = or_forward_loss(m, theta, tokens, ctargets, NULL);
  or_perturb_lora_ffn(theta, m->nlayers, m->dim, QD, KVD, m->hidden, m->rank, m->lora_ffn, seed, +eps);
  const float g = (lp - lm) / (2.0f * eps);
  const float update_scale = -lr * g;
  or_perturb_lora_ffn(theta, m->nlayers, m->dim, QD, KVD, m->hidden, m->rank, m->lora_ffn, seed, update_scale);
  if (loss_plus) *loss_plus = lp;
  if (loss_minus) *loss_minus = lm;
  if (proj_grad) *proj_grad = g;
}

/* ================= backprop-LoRA (P16) ================= */

/* rmsnorm_bwd (cpu_ops.h:24-60): dx = rrms (w dy - x dot rrms^2/d); dw += Σ_s dy x rrms */
void or_rmsnorm_bwd(float* dx, float* dw, const float* dy, const float* x, const float* w, int d, int S) {
  float* ss = (float*)calloc((size_t)S, sizeof(float));
  float* rrms = (float*)xmalloc(sizeof(float) * (size_t)S);
  float* dot = (float*)calloc((size_t)S, sizeof(float));
  for (int i = 0; i < d; i++)
    for (int t = 0; t < S; t++) {
      const float sq = x[(size_t)i * S + t] * x[(size_t)i * S + t];
      ss[t] = sq + ss[t];
    }
  const float invd = 1.0f / d, eps = 1e-5f;
  for (int t = 0; t < S; t++) {
    const float m = ss[t] * invd;
    rrms[t] = 1.0f / sqrtf(m + eps);
  }
  for (int i = 0; i < d; i++)
    for (int t = 0; t < S; t++) {
      const float p = dy[(size_t)i * S + t] * x[(size_t)i * S + t];
      const float q = p * w[i];
      dot[t] = q + dot[t];
    }
  for (int t = 0; t < S; t++) {
    const float r2 = rrms[t] * rrms[t];
    const float r2d = r2 * invd;
    dot[t] = dot[t] * r2d;
  }
  for (int i = 0; i < d; i++) {
    float acc = 0.f;
    for (int t = 0; t < S; t++) {
      const size_t k = (size_t)i * S + t;
      const float xd = x[k] * dot[t];
      const float wd = dy[k] * w[i];
      const float v = wd - xd;
      dx[k] = v * rrms[t];
      const float g = dy[k] * x[k];
      acc += g * rrms[t];
    }
    dw[i] += acc;
  }
  free(ss);
  free(rrms);
  free(dot);
}

/* rope_backward_inplace (cpu_ops.h:377-393): rotate pairs by -angle */
void or_rope_backward(float* dx, int seq, int dim, int hd, float theta) {
  const int nheads = dim / hd;
  for (int h = 0; h < nheads; h++)
    for (int i = 0; i < hd / 2; i++) {
      const float freq = 1.0f / powf(theta, 2.0f * i / (float)hd);
      for (int p = 0; p < seq; p++) {
        const float ang = p * freq;
        const float c = cosf(ang), s = sinf(ang);
        const size_t i0 = (size_t)(h * hd + 2 * i) * seq + p;
        const size_t i1 = (size_t)(h * hd + 2 * i + 1) * seq + p;
        const float v0 = dx[i0], v1 = dx[i1];
        dx[i0] = v0 * c + v1 * s;
        dx[i1] = -v0 * s + v1 * c;
      }
    }
}

/* cpu_sdpa_backward (cpu_ops.h:213-290): recompute causal softmax P per head,
 * dV = dA·P, dP = dAᵀ·V, dS = (dP - rowsum(dP∘P))∘P/√hd, dQ = K·dSᵀ, dK = Q·dS.
 * Inputs at HEADS (K, V already tiled); outputs at HEADS. */
void or_sdpa_backward(const float* Q, const float* Kt, const float* Vt, const float* da, float* dq, float* dk,
                      float* dv, int heads, int hd, int seq) {
  const float scale = 1.0f / sqrtf((float)hd);
  float* P = (float*)xmalloc(sizeof(float) * (size_t)seq * seq);
  float* dS = (float*)xmalloc(sizeof(float) * (size_t)seq * seq);
  for (int h = 0; h < heads; h++) {
    const size_t o = (size_t)h * hd * seq;
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, seq, seq, hd, scale, Q + o, seq, Kt + o, seq, 0.0f, P, seq);
    for (int s = 0; s < seq; s++) {
      float* row = P + (size_t)s * seq;
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
    cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, hd, seq, seq, 1.0f, da + o, seq, P, seq, 0.0f, dv + o, seq);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, seq, seq, hd, 1.0f, da + o, seq, Vt + o, seq, 0.0f, dS, seq);
    for (int s = 0; s < seq; s++) {
      float* dp = dS + (size_t)s * seq;
      const float* pr = P + (size_t)s * seq;
      float dot = 0;
      for (int j = 0; j < seq; j++) dot += dp[j] * pr[j];
      for (int j = 0; j < seq; j++) dp[j] = (dp[j] - dot) * pr[j] * scale;
    }
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, hd, seq, seq, 1.0f, Kt + o, seq, dS, seq, 0.0f, dq + o, seq);
    cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, hd, seq, seq, 1.0f, Q + o, seq, dS, seq, 0.0f, dk + o, seq);
  }
  free(P);
  free(dS);
}

/* gqa_reduce_kv (training/io.h:449-459): sum the query heads sharing a KV head */
static void gqa_reduce(float* out, const float* in, int kv_heads, int ratio, int hd, int seq) {
  memset(out, 0, sizeof(float) * (size_t)kv_heads * hd * seq);
  for (int kv = 0; kv < kv_heads; kv++)
    for (int r = 0; r < ratio; r++) {
      const float* src = in + (size_t)(kv * ratio + r) * hd * seq;
      float* dst = out + (size_t)kv * hd * seq;
      for (size_t i = 0; i < (size_t)hd * seq; i++) dst[i] = src[i] + dst[i];
    }
}

/* W_eff = W + B·A (lora_merge_weight, training/config.h:278-283) */
static float* merged(const float* W, const float* B, const float* A, int out_dim, int rank, int in_dim) {
  float* M = (float*)xmalloc(sizeof(float) * (size_t)out_dim * in_dim);
  memcpy(M, W, sizeof(float) * (size_t)out_dim * in_dim);
  cblas_sgemm(OrRowMajor, OrNoTrans, OrNoTrans, out_dim, in_dim, rank, 1.0f, B, rank, A, in_dim, 1.0f, M, in_dim);
  return M;
}

/* dB += dW·Aᵀ ; dA += Bᵀ·dW (lora_grad_project, training/config.h:286-292) */
static void grad_project(float* dA, float* dB, const float* dW, const float* A, const float* B, int out_dim, int rank,
                         int in_dim) {
  cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, out_dim, rank, in_dim, 1.0f, dW, in_dim, A, in_dim, 1.0f, dB, rank);
  cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, rank, in_dim, out_dim, 1.0f, B, rank, dW, in_dim, 1.0f, dA, in_dim);
}

/* Shared forward-with-saves + backward. grad (theta layout) is overwritten with the
 * LoRA A/B and RMS gradients. With dw != NULL it also receives every projection's
 * dW (train.m:1027-1151; per layer Wq, Wk, Wv, Wo, W1, W2, W3, each [out, in]), and
 * gembed [vocab, dim] the embedding gradient: embed_backward rows, then the
 * classifier gradient scattered through c2f (NULL: identity). Returns the loss. */
static float backprop(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                      float* grad, float* dw, float* gembed, const int32_t* c2f) {
  const int D = m->dim, H = m->hidden, S = m->seq, QD = m->heads * m->hd, KVD = m->kv_heads * m->hd;
  const int r = m->rank, NL = m->nlayers, CV = m->cv, ratio = m->heads / m->kv_heads;
  const or_layout L = or_lora_layout(NL, D, QD, KVD, r);
  const size_t DS = (size_t)D * S, QS = (size_t)QD * S, KS = (size_t)KVD * S, HS = (size_t)H * S;
  /* per-layer saves (BP_LayerActs, backprop_lora.h:15-27) */
  float* x_pre = (float*)xmalloc(sizeof(float) * DS * NL);
  float* xnorm = (float*)xmalloc(sizeof(float) * DS * NL);
  float* Qs = (float*)xmalloc(sizeof(float) * QS * NL);
  float* Ks = (float*)xmalloc(sizeof(float) * KS * NL);
  float* Vs = (float*)xmalloc(sizeof(float) * KS * NL);
  float* att = (float*)xmalloc(sizeof(float) * QS * NL);
  float* x2 = (float*)xmalloc(sizeof(float) * DS * NL);
  float* h1 = (float*)xmalloc(sizeof(float) * HS * NL);
  float* h3 = (float*)xmalloc(sizeof(float) * HS * NL);
  float* x2n = dw ? (float*)xmalloc(sizeof(float) * DS * NL) : NULL;
  float* x = (float*)xmalloc(sizeof(float) * DS);
  float* xn = (float*)xmalloc(sizeof(float) * DS);
  float* Q = (float*)xmalloc(sizeof(float) * QS);
  float* K = (float*)xmalloc(sizeof(float) * KS);
  float* Kt = (float*)xmalloc(sizeof(float) * QS);
  float* Vt = (float*)xmalloc(sizeof(float) * QS);
  float* o = (float*)xmalloc(sizeof(float) * DS);
  float* g = (float*)xmalloc(sizeof(float) * HS);
  float* tmp = (float*)xmalloc(sizeof(float) * (size_t)r * S);
  float* logits = (float*)xmalloc(sizeof(float) * (size_t)S * CV);
  for (int t = 0; t < S; t++) {
    const int tok = tokens[t];
    if (tok < 0 || tok >= m->vocab) {
      fprintf(stderr, "oracle: token[%d]=%d out of range\n", t, tok);
      abort();
    }
    for (int d = 0; d < D; d++) x[(size_t)d * S + t] = m->embed[(size_t)tok * D + d];
  }
  for (int l = 0; l < NL; l++) {
    const float* th = theta + (size_t)l * L.layer_size;
    memcpy(x_pre + DS * l, x, sizeof(float) * DS);
    or_rmsnorm(xnorm + DS * l, x, th + L.rms_att, D, S);
    const float* xnl = xnorm + DS * l;
    float *Ql = Qs + QS * l, *Kl = Ks + KS * l, *Vl = Vs + KS * l;
    or_sgemm_nn(QD, S, D, m->Wq[l], xnl, Ql, 0.0f);
    or_sgemm_nn(KVD, S, D, m->Wk[l], xnl, Kl, 0.0f);
    or_sgemm_nn(KVD, S, D, m->Wv[l], xnl, Vl, 0.0f);
    or_lora_addmm(Ql, th + L.Aq, th + L.Bq, xnl, tmp, QD, r, D, S);
    or_lora_addmm(Kl, th + L.Ak, th + L.Bk, xnl, tmp, KVD, r, D, S);
    or_lora_addmm(Vl, th + L.Av, th + L.Bv, xnl, tmp, KVD, r, D, S);
    memcpy(Q, Ql, sizeof(float) * QS);
    memcpy(K, Kl, sizeof(float) * KS);
    or_rope_forward(Q, S, QD, m->hd, m->rope_theta);
    or_rope_forward(K, S, KVD, m->hd, m->rope_theta);
    gqa_tile(Kt, K, m->kv_heads, ratio, m->hd, S);
    gqa_tile(Vt, Vl, m->kv_heads, ratio, m->hd, S);
    or_sdpa_forward(Q, Kt, Vt, att + QS * l, m->heads, m->hd, S);
    or_sgemm_nn(D, S, QD, m->Wo[l], att + QS * l, o, 0.0f);
    or_lora_addmm(o, th + L.Ao, th + L.Bo, att + QS * l, tmp, D, r, QD, S);
    resid_add(x, o, m->res_alpha, DS);
    memcpy(x2 + DS * l, x, sizeof(float) * DS);
    or_rmsnorm(xn, x, th + L.rms_ffn, D, S);
    if (x2n) memcpy(x2n + DS * l, xn, sizeof(float) * DS);
    or_sgemm_nn(H, S, D, m->W1[l], xn, h1 + HS * l, 0.0f);
    or_sgemm_nn(H, S, D, m->W3[l], xn, h3 + HS * l, 0.0f);
    for (size_t i = 0; i < HS; i++) {
      const float sv = h1[HS * l + i] / (1.0f + expf(-h1[HS * l + i]));
      g[i] = sv * h3[HS * l + i];
    }
    or_sgemm_nn(D, S, H, m->W2[l], g, o, 0.0f);
    resid_add(x, o, m->res_alpha, DS);
  }
  /* x is x_pre_final; logits and dlogits (cross_entropy_loss, cpu_ops.h:108-133) */
  or_rmsnorm(xn, x, theta + L.rms_final, D, S);
  cblas_sgemm(OrRowMajor, OrTrans, OrTrans, S, CV, D, 1.0f, xn, S, m->cembed, D, 0.0f, logits, CV);
  float* xn_final = NULL;
  if (dw) {
    xn_final = (float*)xmalloc(sizeof(float) * DS);
    memcpy(xn_final, xn, sizeof(float) * DS);
  }
  float total = 0;
  const float invS = 1.0f / S;
  for (int t = 0; t < S; t++) {
    float* row = logits + (size_t)t * CV;
    float maxv = row[0];
    for (int v = 1; v < CV; v++) maxv = fmaxf(maxv, row[v]);
    const float tgt_logit = row[ctargets[t]];
    float sum = 0;
    for (int v = 0; v < CV; v++) {
      row[v] = expf(row[v] + (-maxv));
      sum += row[v];
    }
    const float inv = 1.0f / sum;
    for (int v = 0; v < CV; v++) row[v] *= inv;
    total += -(tgt_logit - maxv) + logf(sum);
    row[ctargets[t]] -= 1.0f;
    for (int v = 0; v < CV; v++) row[v] *= invS;
  }
  const float loss = total / S;
  /* ---- backward (bp_lora_backward, backprop_lora.h:147-288) ---- */
  memset(grad, 0, sizeof(float) * (size_t)L.total);
  float* dy = (float*)xmalloc(sizeof(float) * DS);
  float* dxr = (float*)xmalloc(sizeof(float) * DS);
  float* dx2 = (float*)xmalloc(sizeof(float) * DS);
  float* dx2s = (float*)xmalloc(sizeof(float) * DS);
  float* dsl = (float*)xmalloc(sizeof(float) * HS);
  float* dh1 = (float*)xmalloc(sizeof(float) * HS);
  float* dh3 = (float*)xmalloc(sizeof(float) * HS);
  float* da = (float*)xmalloc(sizeof(float) * QS);
  float* dqf = (float*)xmalloc(sizeof(float) * QS);
  float* dkf = (float*)xmalloc(sizeof(float) * QS);
  float* dvf = (float*)xmalloc(sizeof(float) * QS);
  float* dk = (float*)xmalloc(sizeof(float) * KS);
  float* dv = (float*)xmalloc(sizeof(float) * KS);
  float* dW = (float*)xmalloc(sizeof(float) * (size_t)(QD > D ? QD : D) * (QD > D ? QD : D));
  cblas_sgemm(OrRowMajor, OrTrans, OrTrans, D, S, CV, 1.0f, m->cembed, D, logits, CV, 0.0f, dy, S);
  memset(dxr, 0, sizeof(float) * DS);
  or_rmsnorm_bwd(dxr, grad + L.rms_final, dy, x, theta + L.rms_final, D, S);
  memcpy(dy, dxr, sizeof(float) * DS);
  const float alpha = m->res_alpha;
  const size_t per_l = (size_t)QD * D + 2 * (size_t)KVD * D + (size_t)D * QD + 3 * (size_t)H * D;
  float* gate = dw ? (float*)xmalloc(sizeof(float) * HS) : NULL;
  for (int l = NL - 1; l >= 0; l--) {
    const float* th = theta + (size_t)l * L.layer_size;
    float* gl = grad + (size_t)l * L.layer_size;
    float* dWq = dw ? dw + per_l * l : NULL;
    float* dWk = dw ? dWq + (size_t)QD * D : NULL;
    float* dWv = dw ? dWk + (size_t)KVD * D : NULL;
    float* dWo = dw ? dWv + (size_t)KVD * D : NULL;
    float* dW1 = dw ? dWo + (size_t)D * QD : NULL;
    float* dW2 = dw ? dW1 + (size_t)H * D : NULL;
    float* dW3 = dw ? dW2 + (size_t)D * H : NULL;
    for (size_t i = 0; i < DS; i++) dx2s[i] = dy[i] * alpha; /* dffn */
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, H, S, D, 1.0f, m->W2[l], H, dx2s, S, 0.0f, dsl, S);
    for (size_t i = 0; i < HS; i++) {
      const float a1 = h1[HS * l + i], a3 = h3[HS * l + i];
      const float sig = 1.0f / (1.0f + expf(-a1));
      dh3[i] = dsl[i] * (a1 * sig);
      dh1[i] = (dsl[i] * a3) * (sig * (1.0f + a1 * (1.0f - sig)));
    }
    if (dw) {
      /* dW2 = dffn · silu_outᵀ; dW1 = dh1 · x2normᵀ; dW3 = dh3 · x2normᵀ (train.m:1027-1034) */
      for (size_t i = 0; i < HS; i++) {
        const float sv = h1[HS * l + i] / (1.0f + expf(-h1[HS * l + i]));
        gate[i] = sv * h3[HS * l + i];
      }
      cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, D, H, S, 1.0f, dx2s, S, gate, S, 0.0f, dW2, H);
      cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, H, D, S, 1.0f, dh1, S, x2n + DS * l, S, 0.0f, dW1, D);
      cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, H, D, S, 1.0f, dh3, S, x2n + DS * l, S, 0.0f, dW3, D);
    }
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, D, S, H, 1.0f, m->W1[l], D, dh1, S, 0.0f, dxr, S);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, D, S, H, 1.0f, m->W3[l], D, dh3, S, 1.0f, dxr, S);
    memset(dx2, 0, sizeof(float) * DS);
    or_rmsnorm_bwd(dx2, gl + L.rms_ffn, dxr, x2 + DS * l, th + L.rms_ffn, D, S);
    for (size_t i = 0; i < DS; i++) dx2[i] += dy[i];
    for (size_t i = 0; i < DS; i++) dx2s[i] = dx2[i] * alpha;
    float* Wo_e = merged(m->Wo[l], th + L.Bo, th + L.Ao, D, r, QD);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, QD, S, D, 1.0f, Wo_e, QD, dx2s, S, 0.0f, da, S);
    free(Wo_e);
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, D, QD, S, 1.0f, dx2s, S, att + QS * l, S, 0.0f, dW, QD);
    grad_project(gl + L.Ao, gl + L.Bo, dW, th + L.Ao, th + L.Bo, D, r, QD);
    if (dw) memcpy(dWo, dW, sizeof(float) * (size_t)D * QD);
    memcpy(Q, Qs + QS * l, sizeof(float) * QS);
    memcpy(K, Ks + KS * l, sizeof(float) * KS);
    or_rope_forward(Q, S, QD, m->hd, m->rope_theta);
    or_rope_forward(K, S, KVD, m->hd, m->rope_theta);
    gqa_tile(Kt, K, m->kv_heads, ratio, m->hd, S);
    gqa_tile(Vt, Vs + KS * l, m->kv_heads, ratio, m->hd, S);
    or_sdpa_backward(Q, Kt, Vt, da, dqf, dkf, dvf, m->heads, m->hd, S);
    gqa_reduce(dk, dkf, m->kv_heads, ratio, m->hd, S);
    gqa_reduce(dv, dvf, m->kv_heads, ratio, m->hd, S);
    or_rope_backward(dqf, S, QD, m->hd, m->rope_theta);
    or_rope_backward(dk, S, KVD, m->hd, m->rope_theta);
    const float* xnl = xnorm + DS * l;
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, QD, D, S, 1.0f, dqf, S, xnl, S, 0.0f, dW, D);
    grad_project(gl + L.Aq, gl + L.Bq, dW, th + L.Aq, th + L.Bq, QD, r, D);
    if (dw) memcpy(dWq, dW, sizeof(float) * (size_t)QD * D);
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, KVD, D, S, 1.0f, dk, S, xnl, S, 0.0f, dW, D);
    grad_project(gl + L.Ak, gl + L.Bk, dW, th + L.Ak, th + L.Bk, KVD, r, D);
    if (dw) memcpy(dWk, dW, sizeof(float) * (size_t)KVD * D);
    cblas_sgemm(OrRowMajor, OrNoTrans, OrTrans, KVD, D, S, 1.0f, dv, S, xnl, S, 0.0f, dW, D);
    grad_project(gl + L.Av, gl + L.Bv, dW, th + L.Av, th + L.Bv, KVD, r, D);
    if (dw) memcpy(dWv, dW, sizeof(float) * (size_t)KVD * D);
    float* Wq_e = merged(m->Wq[l], th + L.Bq, th + L.Aq, QD, r, D);
    float* Wk_e = merged(m->Wk[l], th + L.Bk, th + L.Ak, KVD, r, D);
    float* Wv_e = merged(m->Wv[l], th + L.Bv, th + L.Av, KVD, r, D);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, D, S, QD, 1.0f, Wq_e, D, dqf, S, 0.0f, dxr, S);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, D, S, KVD, 1.0f, Wk_e, D, dk, S, 1.0f, dxr, S);
    cblas_sgemm(OrRowMajor, OrTrans, OrNoTrans, D, S, KVD, 1.0f, Wv_e, D, dv, S, 1.0f, dxr, S);
    free(Wq_e);
    free(Wk_e);
    free(Wv_e);
    memset(dy, 0, sizeof(float) * DS);
    or_rmsnorm_bwd(dy, gl + L.rms_att, dxr, x_pre + DS * l, th + L.rms_att, D, S);
    for (size_t i = 0; i < DS; i++) dy[i] = dy[i] + dx2[i];
  }
  if (dw) {
    /* embed_backward (cpu_ops.h:199-207) then vocab_scatter_grads (cpu_ops.h:176-182) of
     * gcembed = dlogitsᵀ · x_finalᵀ (train.m:938-941) */
    memset(gembed, 0, sizeof(float) * (size_t)m->vocab * D);
    for (int t = 0; t < S; t++) {
      float* row = gembed + (size_t)tokens[t] * D;
      for (int d = 0; d < D; d++) row[d] = dy[(size_t)d * S + t] + row[d];
    }
    float* gce = (float*)xmalloc(sizeof(float) * (size_t)CV * D);
    cblas_sgemm(OrRowMajor, OrTrans, OrTrans, CV, D, S, 1.0f, logits, CV, xn_final, S, 0.0f, gce, D);
    for (int v = 0; v < CV; v++) {
      float* row = gembed + (size_t)(c2f ? c2f[v] : v) * D;
      for (int d = 0; d < D; d++) row[d] = gce[(size_t)v * D + d] + row[d];
    }
    free(gce);
    free(x2n);
    free(gate);
    free(xn_final);
  }
  free(x_pre); free(xnorm); free(Qs); free(Ks); free(Vs); free(att); free(x2); free(h1); free(h3);
  free(x); free(xn); free(Q); free(K); free(Kt); free(Vt); free(o); free(g); free(tmp); free(logits);
  free(dy); free(dxr); free(dx2); free(dx2s); free(dsl); free(dh1); free(dh3); free(da); free(dqf); free(dkf);
  free(dvf); free(dk); free(dv); free(dW);
  return loss;
}

float or_p16_grad(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                  float* grad) {
  return backprop(m, theta, tokens, ctargets, grad, NULL, NULL, NULL);
}

float or_full_grad(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                   float* grad, float* dw, float* gembed, const int32_t* c2f) {
  return backprop(m, theta, tokens, ctargets, grad, dw, gembed, c2f);
}

/* adam_update (cpu_ops.h:62-104), one rounding per vectorised operation */
void or_adam(float* w, const float* g, float* m, float* v, size_t n, int t, float lr, float b1, float b2, float eps,
             float wd) {
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
  const float bc1 = 1.0f - powf(b1, (float)t), bc2 = 1.0f - powf(b2, (float)t);
  const float ibc1 = 1.0f / bc1, ibc2 = 1.0f / bc2, neg_lr = -lr;
  for (size_t i = 0; i < n; i++) {
    const float m1 = m[i] * b1;
    const float gm = g[i] * omb1;
    m[i] = gm + m1;
    const float g2 = g[i] * g[i];
    const float v1 = v[i] * b2;
    const float gv = g2 * omb2;
    v[i] = gv + v1;
    const float mh = m[i] * ibc1;
    const float vh = v[i] * ibc2;
    const float den = sqrtf(vh) + eps;
    float u = mh / den;
    if (wd > 0.0f) {
      const float ww = w[i] * wd;
      u = ww + u;
    }
    const float step = u * neg_lr;
    w[i] = step + w[i];
  }
}
