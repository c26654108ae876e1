/* ref_driver.c — exports the reference's own CPU code, compiled in place from
 * the AutoANE tree (training/cpu_ops.h, training/backprop_lora.h) against the
 * shim in oracle/shim, so tests can pin the oracle restatement to it.
 * TEST INFRASTRUCTURE ONLY; built into oracle/_ref/ by oracle/build.py and
 * never linked into the product.
 *
 * Model sizes are compile-time, as in the reference: the build passes
 * -include training/models/<model>.h (training/Makefile:15-23).
 */
#include "backprop_lora.h" /* reference header: pulls cpu_ops.h (reference) + shim config.h/io.h */

int ref_dims(float* out) {
  out[0] = DIM; out[1] = HIDDEN; out[2] = HEADS; out[3] = KV_HEADS; out[4] = HD;
  out[5] = SEQ; out[6] = NLAYERS; out[7] = VOCAB; out[8] = ROPE_THETA;
  return 9;
}

void ref_rmsnorm(float* out, const float* x, const float* w, int d, int S) { rmsnorm(out, x, w, d, S); }
void ref_rmsnorm_bwd(float* dx, float* dw, const float* dy, const float* x, const float* w, int d, int S) {
  rmsnorm_bwd(dx, dw, dy, x, w, d, S);
}
void ref_rope_forward(float* x, int seq, int dim, int hd) { rope_forward_inplace(x, seq, dim, hd); }
void ref_rope_backward(float* dx, int seq, int dim, int hd) { rope_backward_inplace(dx, seq, dim, hd); }
void ref_sdpa_forward(const float* Q, const float* K, const float* V, float* out, int heads, int hd, int seq) {
  cpu_sdpa_forward(Q, K, V, out, heads, hd, seq);
}
void ref_sdpa_backward(const float* Q, const float* K, const float* V, const float* da, float* dq, float* dk,
                       float* dv, int heads, int hd, int seq) {
  cpu_sdpa_backward(Q, K, V, da, dq, dk, dv, heads, hd, seq);
}
float ref_cross_entropy(float* dlogits, const float* logits, const uint16_t* targets, int V, int S) {
  return cross_entropy_loss(dlogits, logits, targets, V, S);
}
void ref_adam(float* w, const float* g, float* m, float* v, size_t n, int t, float lr, float b1, float b2, float eps,
              float wd) {
  AdamState s = {m, v, n};
  adam_update(w, g, &s, t, lr, b1, b2, eps, wd);
}
void ref_embed_lookup(float* x, const float* embed, const uint16_t* tokens, int dim, int seq, int vocab) {
  embed_lookup(x, embed, tokens, dim, seq, vocab);
}

/* lora_addmm as written in training/train_mezo.m:694-703 (that file is
 * Objective-C and cannot be compiled here; the two calls are transcribed). */
static void ref_lora_addmm(float* out, const float* A, const float* B, const float* x, float* tmp, int out_dim,
                           int rank, int in_dim) {
  cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, rank, SEQ, in_dim, 1.0f, A, in_dim, x, SEQ, 0.0f, tmp,
              SEQ);
  cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, out_dim, SEQ, rank, 1.0f, B, rank, tmp, SEQ, 1.0f, out,
              SEQ);
}

/* DO_FORWARD_PASS, cpu_only + lora_split branch (training/train_mezo.m:1528-1699),
 * transcribed over the reference's compiled cpu_ops.h functions.
 * lora[l*8 + {0..7}] = Aq,Bq,Ak,Bk,Av,Bv,Ao,Bo of layer l; rms[l*2 + {0,1}] =
 * rms_att, rms_ffn. */
float ref_forward_loss(const float* const* Wq, const float* const* Wk, const float* const* Wv,
                       const float* const* Wo, const float* const* W1, const float* const* W2,
                       const float* const* W3, const float* const* lora, const float* const* rms,
                       const float* rms_final, const float* embed, const float* cembed, int CV, int rank,
                       float res_alpha, const uint16_t* input_toks, const uint16_t* ctargets) {
  float* x_cur = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* xnorm_buf = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* Q = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* K = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* V = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* attn_out = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* o_out = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* h1 = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* h3 = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* silu_out = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* k_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* v_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* logits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* dlogits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* lora_tmp = (float*)safe_malloc((size_t)rank * SEQ * 4);
  float loss;
  embed_lookup(x_cur, embed, input_toks, DIM, SEQ, VOCAB);
  for (int L = 0; L < NLAYERS; L++) {
    const float* const* ll = lora + (size_t)L * 8;
    rmsnorm(xnorm_buf, x_cur, rms[2 * L], DIM, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, Q_DIM, SEQ, DIM, 1.0f, Wq[L], DIM, xnorm_buf, SEQ, 0.0f,
                Q, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wk[L], DIM, xnorm_buf, SEQ,
                0.0f, K, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wv[L], DIM, xnorm_buf, SEQ,
                0.0f, V, SEQ);
    ref_lora_addmm(Q, ll[0], ll[1], xnorm_buf, lora_tmp, Q_DIM, rank, DIM);
    ref_lora_addmm(K, ll[2], ll[3], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    ref_lora_addmm(V, ll[4], ll[5], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    rope_forward_inplace(Q, SEQ, Q_DIM, HD);
    rope_forward_inplace(K, SEQ, KV_DIM, HD);
    gqa_tile_kv(k_tiled, K, SEQ);
    gqa_tile_kv(v_tiled, V, SEQ);
    cpu_sdpa_forward(Q, k_tiled, v_tiled, attn_out, HEADS, HD, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, Q_DIM, 1.0f, Wo[L], Q_DIM, attn_out, SEQ, 0.0f,
                o_out, SEQ);
    ref_lora_addmm(o_out, ll[6], ll[7], attn_out, lora_tmp, DIM, rank, Q_DIM);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
    rmsnorm(xnorm_buf, x_cur, rms[2 * L + 1], DIM, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W1[L], DIM, xnorm_buf, SEQ,
                0.0f, h1, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W3[L], DIM, xnorm_buf, SEQ,
                0.0f, h3, SEQ);
    for (int i = 0; i < HIDDEN * SEQ; i++) {
      float s = h1[i] / (1.0f + expf(-h1[i]));
      silu_out[i] = s * h3[i];
    }
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, HIDDEN, 1.0f, W2[L], HIDDEN, silu_out, SEQ,
                0.0f, o_out, SEQ);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
  }
  rmsnorm(xnorm_buf, x_cur, rms_final, DIM, SEQ);
  cblas_sgemm(CblasRowMajor, CblasTrans, CblasTrans, SEQ, CV, DIM, 1.0f, xnorm_buf, SEQ, cembed, DIM, 0.0f, logits,
              CV);
  loss = cross_entropy_loss(dlogits, logits, ctargets, CV, SEQ);
  free(x_cur); free(xnorm_buf); free(Q); free(K); free(V); free(attn_out); free(o_out);
  free(h1); free(h3); free(silu_out); free(k_tiled); free(v_tiled); free(logits); free(dlogits); free(lora_tmp);
  return loss;
}
